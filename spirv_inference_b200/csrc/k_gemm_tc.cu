// Tensor-core GEMM for sm_100a: TMA -> shared memory -> tcgen05.mma (kind::tf32)
// with the accumulator in TMEM, split "3xTF32" so results keep fp32 accuracy.
//
// Serves the dense contractions whose operands are both K-contiguous:
// pointwise (1x1, stride 1) convolutions over NHWC activations with OHWI
// weights (A = x as [M = n*h*w][K = ic], B = w as [N = oc][K]), and
// fully_connected / linear layers (B = W[out][in]).
//
// Precision: every fp32 operand x is split on chip into hi = rna_tf32(x) and
// lo = rna_tf32(x - hi); each k-step issues hi*hi + hi*lo + lo*hi into an fp32
// TMEM accumulator.  Relative error per product is ~2^-21, the neglected
// lo*lo term ~2^-22: fp32-level results, as the reference's fp32 kernels
// (kernels/conv2d/glsl/conv2d.comp, fully_connected.comp) require.
//
// Structure (one CTA per SM, persistent over output tiles, 10 warps):
//   warp 8      TMA producer: A tile 128 x 32 and B tile BN x 32 per k-block
//               into an S-stage ring, 128-byte swizzle, mbarrier transaction
//               counts.
//   warps 4-7   converters: split A and B of a landed stage in place (hi) and
//               into a second buffer (lo), then fence.proxy.async + arrive.
//   warp 9      TMEM owner and MMA issuer (one thread): 12 UMMAs per k-block
//               (4 k-steps x 3 products), commit frees the stage; a commit at
//               the end of a tile hands one of two TMEM accumulators
//               (2 x BN columns) to the epilogue.
//   warps 0-3   epilogue: tcgen05.ld 32 rows x 16 columns per warp, alpha,
//               bias, residual, activation, store; then release the
//               accumulator, so tile i's epilogue overlaps tile i+1's k-loop.
// Every wait is bounded (globaltimer); on timeout the CTA raises an abort flag,
// records a device status, drains its own in-flight copies and MMAs, frees
// TMEM and exits.  The host reads the status at the next sync.
#include <cuda.h>

#include <mutex>

#include "spx_internal.cuh"

namespace spx {

__device__ int g_tc_status = 0;

namespace {

constexpr int kBM = 128;         // UMMA M: output rows per tile
constexpr int kBK = 32;          // fp32 elements per k-block (one 128-byte row)
constexpr int kThreads = 320;    // 10 warps
constexpr int kMaxStages = 6;
constexpr uint32_t kATileBytes = kBM * kBK * 4;       // 16 KB
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr unsigned long long kDrainNs = 200000000ull;     // 0.2 s drain on abort

struct TcArgs {
  int M, N, K, BN, n_tiles, m_tiles, k_blocks, stages;
  uint32_t idesc, tmem_cols, stage_bytes, b_bytes;
  const float* bias;
  const float* res;
  float* c;
  int64_t ldc;
  float alpha;
  int act;
  int vec4;
};

__device__ __forceinline__ uint32_t su32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on the phase with the given parity.  Returns false when the
// CTA is aborting (another role timed out) or this wait itself timed out.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                         unsigned long long limit = kTimeoutNs) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (bar_try(b, parity)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > limit) {
      *abort_flag = 1;
      atomicExch(&g_tc_status, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes grouped in 8-row (1024-byte) atoms.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused, K fits one row)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // swizzle: 128B
  return d;
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return __uint_as_float(h);
}

// In-place hi / separate lo split of n16 16-byte vectors.
__device__ __forceinline__ void split_buffer(float4* hi, float4* lo, int n16, int tid, int nthr) {
  for (int i = tid; i < n16; i += nthr) {
    float4 v = hi[i];
    float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
    float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    l.x = isfinite(l.x) ? tf32_rna(l.x) : 0.0f;
    l.y = isfinite(l.y) ? tf32_rna(l.y) : 0.0f;
    l.z = isfinite(l.z) ? tf32_rna(l.z) : 0.0f;
    l.w = isfinite(l.w) ? tf32_rna(l.w) : 0.0f;
    hi[i] = h;
    lo[i] = l;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const TcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = p.stages;
  uint64_t* full = (uint64_t*)(smem + (size_t)S * p.stage_bytes);
  uint64_t* conv = full + kMaxStages;
  uint64_t* empty = conv + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&conv[s], 128);
      bar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&tfull[a], 1);
      bar_init(&tempty[a], 128);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = p.m_tiles * p.n_tiles;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
      int s = 0;
      uint32_t ph = 0, armed = 0, armed_par = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const int mt = t / p.n_tiles, nt = t % p.n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!bar_wait(&empty[s], ph ^ 1, abort_flag)) goto producer_done;
          uint8_t* st = smem + (size_t)s * p.stage_bytes;
          bar_expect_tx(&full[s], kATileBytes + p.b_bytes);
          tma_load_2d(st, &tmA, &full[s], kb * kBK, mt * kBM);
          tma_load_2d(st + 2 * kATileBytes, &tmB, &full[s], kb * kBK, nt * p.BN);
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_flag) {  // let this CTA's own copies land before it exits
        for (int i = 0; i < S; ++i)
          if (armed & (1u << i)) {
            volatile int never = 0;
            bar_wait(&full[i], (armed_par >> i) & 1, &never, kDrainNs);
          }
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        if (!bar_wait(&tempty[acc], aph ^ 1, abort_flag)) goto mma_done;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * p.BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!bar_wait(&conv[s], ph, abort_flag)) goto mma_done;
          tc_fence_after();
          const uint32_t a_hi = su32(smem + (size_t)s * p.stage_bytes);
          const uint32_t a_lo = a_hi + kATileBytes;
          const uint32_t b_hi = a_hi + 2 * kATileBytes;
          const uint32_t b_lo = b_hi + p.b_bytes;
#pragma unroll
          for (int k = 0; k < kBK / 8; ++k) {
            const uint32_t off = k * 32;  // 8 tf32 = 32 bytes along K
            const uint64_t dah = sdesc(a_hi + off), dal = sdesc(a_lo + off);
            const uint64_t dbh = sdesc(b_hi + off), dbl = sdesc(b_lo + off);
            umma_tf32(d, dal, dbh, p.idesc, (kb | k) ? 1u : 0u);
            umma_tf32(d, dah, dbl, p.idesc, 1u);
            umma_tf32(d, dah, dbh, p.idesc, 1u);
          }
          issued = true;
          umma_commit(&empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (!acc) aph ^= 1;
      }
    mma_done:
      if (*abort_flag && issued) {  // wait for this CTA's MMAs before TMEM is freed
        umma_commit(drain);
        volatile int never = 0;
        bar_wait(drain, 0, &never, kDrainNs);
      }
    }
  } else if (warp >= 4) {
    // ---------------- converters (hi/lo split) ----------------
    const int ct = threadIdx.x - 128;
    int s = 0;
    uint32_t ph = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (!bar_wait(&full[s], ph, abort_flag)) goto conv_done;
        uint8_t* st = smem + (size_t)s * p.stage_bytes;
        split_buffer((float4*)st, (float4*)(st + kATileBytes), kATileBytes / 16, ct, 128);
        split_buffer((float4*)(st + 2 * kATileBytes),
                     (float4*)(st + 2 * kATileBytes + p.b_bytes), p.b_bytes / 16, ct, 128);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        bar_arrive(&conv[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  conv_done:;
  } else {
    // ---------------- epilogue ----------------
    int acc = 0;
    uint32_t aph = 0;
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      if (!bar_wait(&tfull[acc], aph, abort_flag)) goto epi_done;
      tc_fence_after();
      {
        const int64_t m = (int64_t)mt * kBM + row;
        const uint32_t tbase = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * p.BN);
        float* crow = p.c + m * p.ldc;
        const float* rrow = p.res ? p.res + m * p.ldc : nullptr;
        for (int c0 = 0; c0 < p.BN; c0 += 16) {
          float v[16];
          tmem_ld16(tbase + (uint32_t)c0, v);
          const int n0 = nt * p.BN + c0;
          if (m >= p.M || n0 >= p.N) continue;
          if (p.vec4 && n0 + 16 <= p.N) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
              float4 o;
              float* op = &o.x;
              float4 bv = p.bias ? *reinterpret_cast<const float4*>(p.bias + n0 + j)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
              float4 rv = rrow ? *reinterpret_cast<const float4*>(rrow + n0 + j)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
              const float* bp = &bv.x;
              const float* rp = &rv.x;
#pragma unroll
              for (int q = 0; q < 4; ++q) op[q] = apply_act(p.act, v[j + q] * p.alpha + bp[q] + rp[q]);
              *reinterpret_cast<float4*>(crow + n0 + j) = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int n = n0 + j;
              if (n < p.N) {
                float x = v[j] * p.alpha;
                if (p.bias) x += p.bias[n];
                if (rrow) x += rrow[n];
                crow[n] = apply_act(p.act, x);
              }
            }
          }
        }
      }
      tc_fence_before();
      bar_arrive(&tempty[acc]);
      acc ^= 1;
      if (!acc) aph ^= 1;
    }
  epi_done:;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// 2-D fp32 tensor map over rows x cols (cols contiguous, row pitch ld), box
// box_rows x 32 columns, 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
             int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SPX_OK;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = kNumSms;
  }
  return n;
}

}  // namespace

bool gemm_tc_eligible(const float* a, int64_t lda, const float* b, int64_t ldb, int M, int N,
                      int K, const float* c, int64_t ldc) {
  auto al16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
  return M > 0 && N > 0 && K > 0 && K % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 && lda >= K &&
         ldb >= K && al16(a) && al16(b) && ldc >= N && c != nullptr;
}

int launch_gemm_tc(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda, const float* b,
                   int64_t ldb, int M, int N, int K, const float* bias, const float* res, float* c,
                   int64_t ldc, float alpha, int act) {
  TcArgs p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  const int nt = (N + 255) / 256;
  p.BN = ((N + nt - 1) / nt + 15) / 16 * 16;
  p.n_tiles = (N + p.BN - 1) / p.BN;
  p.m_tiles = (M + kBM - 1) / kBM;
  p.k_blocks = (K + kBK - 1) / kBK;
  p.b_bytes = (uint32_t)p.BN * kBK * 4;
  p.stage_bytes = 2 * kATileBytes + 2 * p.b_bytes;
  const int budget = 227 * 1024 - 1024 - 256;
  p.stages = budget / (int)p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  if (p.stages < 2) return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc: tile does not fit");
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * p.BN)) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = (1u << 4)                          // accumulator F32
            | (2u << 7) | (2u << 10)           // A, B: TF32
            | ((uint32_t)(p.BN >> 3) << 17)    // N
            | ((uint32_t)(kBM >> 4) << 24);    // M
  p.bias = bias;
  p.res = res;
  p.c = c;
  p.ldc = ldc;
  p.alpha = alpha;
  p.act = act;
  p.vec4 = (ldc % 4 == 0) && (((uintptr_t)c & 15) == 0) &&
           (!res || ((uintptr_t)res & 15) == 0) && (!bias || ((uintptr_t)bias & 15) == 0);
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_map(&ma, a, M, K, lda, kBM))) return rc;
  if ((rc = make_map(&mb, b, N, K, ldb, p.BN))) return rc;
  const size_t smem = 1024 + (size_t)p.stages * p.stage_bytes + 256;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    227 * 1024);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "gemm_tc: smem attribute");
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  gemm_tc_kernel<<<grid, kThreads, smem, s>>>(ma, mb, p);
  return after_launch(cnt, "gemm_tc");
}

int tc_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
  }
  return v;
}

}  // namespace spx
