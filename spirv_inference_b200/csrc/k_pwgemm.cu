// Pointwise (1x1) convolution / GEMM with a short reduction and a wide output
// (the inverted-residual expand convolutions on 14x14 and 7x7 maps:
// conv2d.comp through the Conv2d lowering of scheduler.rs:321-427), with the
// activation tile resident: C[M][N] = act(A[M][K] . W[N][K]^T + bias),
// K <= 160, 3xTF32.
//
// The row-tiled GEMM (k_gemm_tc.cu) re-reads and re-splits an A tile for every
// n tile; when N spans several n tiles that split dominates.  Here a
// persistent CTA (one per SM) takes an m tile of 128 rows, loads its whole
// K once (TMA, 128-byte swizzle), has eight warps write the tf32 lo terms
// once, and then sweeps every n tile of BN columns over it:
//   warp 8      TMA producers: lane 0 the A tile (all K blocks) when the
//               previous m tile's MMAs are done; lane 1 the pre-split
//               weights (hi | lo, contiguous: one N = 2 BN operand) per
//               (n tile, K block) into a two-stage ring;
//   warps 0-7   the lo split of the resident A tile;
//   warp 9      MMA issuer: raw x [hi; lo] (N = 2 BN) + lo x hi per k-step
//               into one of two TMEM accumulators per n tile;
//   warps 10-17 two epilogue groups draining alternate n tiles: TMEM ->
//               registers -> bias, activation -> swizzled staging -> TMA store.
// Waits are bounded (2 s) and report a device status like the other
// tensor-core kernels.
#include <cuda.h>

#include <mutex>

#include "sm100_prims.cuh"
#include "spx_internal.cuh"

namespace spx {

__device__ int g_pw_status = 0;

namespace {

using namespace sm100;

constexpr int kBuildWarps = 8;
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kEpiWarp0 = 10;
constexpr int kEpiGroups = 2;
constexpr int kThreads = (kEpiWarp0 + 4 * kEpiGroups) * 32;
constexpr uint32_t kATile = 128 * 32 * 4;   // 128 rows x 32 fp32 (one K block)
constexpr uint32_t kEStage = 128 * 128;     // 128 rows x 32 fp32 staging
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr unsigned long long kDrainNs = 200000000ull;
constexpr int kMaxKb = 5;

struct PwArgs {
  int M, N, K, kb, bn, n_tiles, m_tiles;
  uint32_t b_bytes;      // bn x 128 (one of hi / lo)
  uint32_t idesc, idesc2, tmem_cols;
  const float* bias;
  int act;
};

__device__ __forceinline__ void grp_sync(int g) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory");
}
__device__ __forceinline__ bool grp_all(int g, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\t"
      "setp.ne.u32 a, %1, 0;\n\t"
      "barrier.red.and.pred b, %2, 128, a;\n\t"
      "selp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(1 + g)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    pwgemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBhi,
                  const __grid_constant__ CUtensorMap tmBlo, const __grid_constant__ CUtensorMap tmY,
                  const PwArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* a_raw = smem;                                   // kb x 16 KB
  uint8_t* a_lo = a_raw + (size_t)p.kb * kATile;           // kb x 16 KB
  uint8_t* bst = a_lo + (size_t)p.kb * kATile;             // 2 stages x (hi | lo)
  uint8_t* estage = bst + 2 * 2 * (size_t)p.b_bytes;       // kEpiGroups x 16 KB
  uint64_t* bars = (uint64_t*)(estage + kEpiGroups * (size_t)kEStage);
  uint64_t* araw = bars;        // A tile landed
  uint64_t* alo = bars + 1;     // lo terms written (kBuildWarps arrivals)
  uint64_t* aempty = bars + 2;  // MMAs of the m tile done (A slots free)
  uint64_t* bfull = bars + 3;   // [2]
  uint64_t* bempty = bars + 5;  // [2]
  uint64_t* tfull = bars + 7;   // [2]
  uint64_t* tempty = bars + 9;  // [2]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = (uint32_t*)(bars + 12);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mb_init(araw, 1);
    mb_init(alo, kBuildWarps);
    mb_init(aempty, 1);
    for (int j = 0; j < 2; ++j) {
      mb_init(&bfull[j], 1);
      mb_init(&bempty[j], 1);
      mb_init(&tfull[j], 1);
      mb_init(&tempty[j], 4 * 32);
    }
    mb_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sa(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProdWarp) {
    if (lane == 0) {
      // ---- A producer: one m tile at a time, all K blocks ----
      uint32_t ph = 0;
      bool armed = false;
      for (int mt = blockIdx.x; mt < p.m_tiles; mt += gridDim.x) {
        if (!mb_wait(aempty, ph ^ 1, abort_flag, &g_pw_status, kWaitNs, 64)) break;
        mb_expect_tx(araw, (uint32_t)p.kb * kATile);
        for (int kb = 0; kb < p.kb; ++kb)
          tma_2d(a_raw + (size_t)kb * kATile, &tmA, araw, kb * 32, mt * 128);
        armed = true;
        ph ^= 1;
      }
      if (*abort_flag && armed) {
        volatile int never = 0;
        mb_wait(araw, ph ^ 1, &never, &g_pw_status, kDrainNs, 64);
      }
    } else if (lane == 1) {
      // ---- B producer: (m tile, n tile, K block) ring of two stages ----
      int j = 0;
      uint32_t eph = 0, b_armed = 0, b_par = 0;
      for (int mt = blockIdx.x; mt < p.m_tiles; mt += gridDim.x)
        for (int nt = 0; nt < p.n_tiles; ++nt)
          for (int kb = 0; kb < p.kb; ++kb) {
            if (!mb_wait(&bempty[j], eph ^ 1, abort_flag, &g_pw_status, kWaitNs, 64)) goto b_done;
            uint8_t* st = bst + (size_t)j * 2 * p.b_bytes;
            mb_expect_tx(&bfull[j], 2 * p.b_bytes);
            tma_2d(st, &tmBhi, &bfull[j], kb * 32, nt * p.bn);
            tma_2d(st + p.b_bytes, &tmBlo, &bfull[j], kb * 32, nt * p.bn);
            b_armed |= 1u << j;
            b_par = (b_par & ~(1u << j)) | (eph << j);
            if (++j == 2) {
              j = 0;
              eph ^= 1;
            }
          }
    b_done:
      if (*abort_flag) {
        volatile int never = 0;
        for (int q = 0; q < 2; ++q)
          if (b_armed & (1u << q))
            mb_wait(&bfull[q], (b_par >> q) & 1, &never, &g_pw_status, kDrainNs, 64);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      int j = 0, acc = 0;
      uint32_t ph = 0, aph = 0, aaph = 0;
      bool issued = false, ok = true;
      for (int mt = blockIdx.x; mt < p.m_tiles && ok; mt += gridDim.x) {
        if (!mb_wait(alo, aaph, abort_flag, &g_pw_status, kWaitNs, 64)) break;
        aaph ^= 1;
        for (int nt = 0; nt < p.n_tiles && ok; ++nt) {
          if (!mb_wait(&tempty[acc], aph ^ 1, abort_flag, &g_pw_status, kWaitNs, 64)) {
            ok = false;
            break;
          }
          tc_after();
          const uint32_t d = tmem + (uint32_t)(acc * 2 * p.bn);
          for (int kb = 0; kb < p.kb; ++kb) {
            if (!mb_wait(&bfull[j], ph, abort_flag, &g_pw_status, kWaitNs, 32)) {
              ok = false;
              break;
            }
            tc_after();
            const uint32_t ar = sa(a_raw + (size_t)kb * kATile), al = sa(a_lo + (size_t)kb * kATile);
            const uint32_t bh = sa(bst + (size_t)j * 2 * p.b_bytes);
            const int ksteps = min(4, (p.K - kb * 32 + 7) / 8);
#pragma unroll 1
            for (int k = 0; k < ksteps; ++k) {
              const uint32_t off = k * 32;
              mma_tf32(d, sw128_desc(ar + off), sw128_desc(bh + off), p.idesc2, (kb | k) ? 1u : 0u);
              mma_tf32(d, sw128_desc(al + off), sw128_desc(bh + off), p.idesc, 1u);
            }
            issued = true;
            mma_commit(&bempty[j]);
            if (++j == 2) {
              j = 0;
              ph ^= 1;
            }
          }
          if (!ok) break;
          mma_commit(&tfull[acc]);
          if (++acc == 2) {
            acc = 0;
            aph ^= 1;
          }
        }
        if (ok) mma_commit(aempty);  // the m tile's A slots are free once these MMAs finish
      }
      if (*abort_flag && issued) {
        mma_commit(drain);
        volatile int never = 0;
        mb_wait(drain, 0, &never, &g_pw_status, kDrainNs, 64);
      }
    }
  } else if (warp < kBuildWarps) {
    // ---- lo split of the resident A tile, once per m tile ----
    uint32_t rph = 0;
    for (int mt = blockIdx.x; mt < p.m_tiles; mt += gridDim.x) {
      const bool ok = __all_sync(0xffffffffu,
                                 mb_wait(araw, rph, abort_flag, &g_pw_status, kWaitNs, 64));
      if (!ok) break;
      rph ^= 1;
      const int n16 = p.kb * (int)(kATile / 16);
      for (int i = threadIdx.x; i < n16; i += kBuildWarps * 32) {
        const float4 v = reinterpret_cast<const float4*>(a_raw)[i];
        reinterpret_cast<float4*>(a_lo)[i] =
            make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mb_arrive(alo);
    }
  } else {
    // ---- epilogue: group g drains the n tiles of parity g ----
    const int q = warp & 3;
    const int grp = (warp - kEpiWarp0) / 4;
    const bool issuer = warp == kEpiWarp0 + 4 * grp && lane == 0;
    uint8_t* stg = estage + (size_t)grp * kEStage;
    const int m = q * 32 + lane;
    uint32_t aph = 0;
    int seq = 0;  // tiles in the MMA's order: (m tile, n tile)
    bool ok_all = true;
    for (int mt = blockIdx.x; mt < p.m_tiles && ok_all; mt += gridDim.x) {
      for (int nt = 0; nt < p.n_tiles; ++nt, ++seq) {
        if ((seq & 1) != grp) continue;
        const int acc = grp;
        const bool ok = grp_all(grp, mb_wait(&tfull[acc], aph, abort_flag, &g_pw_status,
                                             kWaitNs, 128));
        if (!ok) {
          ok_all = false;
          break;
        }
        aph ^= 1;
        tc_after();
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 2 * p.bn);
        for (int c0 = 0; c0 < p.bn; c0 += 32) {
          const int n0 = nt * p.bn + c0;
          if (n0 >= p.N) break;
          float v[32];
          tmem_ld_32x32(tbase + (uint32_t)c0, v);
          {
            float v2[32];
            tmem_ld_32x32(tbase + (uint32_t)(p.bn + c0), v2);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] += v2[e];
          }
          if (issuer) bulk_wait_read0();
          grp_sync(grp);
          float4* row = reinterpret_cast<float4*>(stg + m * 128);
          with_act(p.act, [&](auto tag) {
            constexpr int A = decltype(tag)::value;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int ch = n0 + 4 * e;
              const float4 b4 = (p.bias && ch < p.N)
                                    ? __ldg(reinterpret_cast<const float4*>(p.bias + ch))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              float4 o;
              o.x = act_c<A>(v[4 * e + 0] + b4.x);
              o.y = act_c<A>(v[4 * e + 1] + b4.y);
              o.z = act_c<A>(v[4 * e + 2] + b4.z);
              o.w = act_c<A>(v[4 * e + 3] + b4.w);
              row[e ^ (m & 7)] = o;
            }
          });
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          grp_sync(grp);
          if (issuer) {
            tma_store_2d(&tmY, stg, n0, mt * 128);  // clipped at M and N
            bulk_commit();
          }
        }
        tc_before();
        mb_arrive(&tempty[acc]);
      }
    }
    if (issuer) bulk_wait_all();
  }

  tc_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                             const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                             const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) ==
            cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = (EncodeFn)q;
  });
  return fn;
}

int map2d(EncodeFn fn, CUtensorMap* m, const float* t, int rows, int cols, int box_cols,
          int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)t, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : fail(SPX_ERR_CUDA, "pw_gemm: map encode failed (%d)", (int)r);
}

size_t pw_smem(int kb, int bn) {
  return 1024 + 2 * (size_t)kb * kATile + 4 * (size_t)bn * 128 + kEpiGroups * (size_t)kEStage + 128;
}

int sms_count() {
  static int v = 0;
  if (!v) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    if (v <= 0) v = kNumSms;
  }
  return v;
}

}  // namespace

int pw_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_pw_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_pw_status, &zero, sizeof(int));
  }
  return v;
}

// -1: not eligible (caller falls back), else SPX_OK or an error code.
int try_pwgemm(cudaStream_t s, int64_t* cnt, const float* a, const float* w_hi, const float* w_lo,
               const float* bias, const float* res, float* c, int M, int N, int K, int act) {
  if (res || !w_hi || !w_lo || !c || M <= 0 || N < 128 || K <= 0 || K > kMaxKb * 32 || K % 4 ||
      N % 4)
    return -1;
  auto al = [](const void* v) { return ((uintptr_t)v & 15) == 0; };
  if (!al(a) || !al(w_hi) || !al(w_lo) || !al(c) || (bias && !al(bias))) return -1;
  const int kb = (K + 31) / 32;
  const size_t cap = 227 * 1024;
  int bn = 128;
  while (bn > 32 && pw_smem(kb, bn) > cap) bn /= 2;
  if (pw_smem(kb, bn) > cap) return -1;
  PwArgs p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.kb = kb;
  p.bn = bn;
  p.n_tiles = (N + bn - 1) / bn;
  p.m_tiles = (M + 127) / 128;
  p.b_bytes = (uint32_t)bn * 128;
  p.idesc = idesc_tf32(128, bn);
  p.idesc2 = idesc_tf32(128, 2 * bn);
  uint32_t cols = 32;
  while (cols < (uint32_t)(4 * bn)) cols <<= 1;
  p.tmem_cols = cols;
  p.bias = bias;
  p.act = act;
  EncodeFn fn = encoder();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap ma, mh, ml, my;
  int rc;
  if ((rc = map2d(fn, &ma, a, M, K, 32, 128)) || (rc = map2d(fn, &mh, w_hi, N, K, 32, bn)) ||
      (rc = map2d(fn, &ml, w_lo, N, K, 32, bn)) || (rc = map2d(fn, &my, c, M, N, 32, 128)))
    return rc;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(pwgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)cap);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "pw_gemm: smem attribute");
  const int grid = p.m_tiles < sms_count() ? p.m_tiles : sms_count();
  pwgemm_kernel<<<grid, kThreads, pw_smem(kb, bn), s>>>(ma, mh, ml, my, p);
  return after_launch(cnt, "pw_gemm");
}

}  // namespace spx
