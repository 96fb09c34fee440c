// Batched tensor-core GEMM for short reductions (K <= 128): the attention
// products of the HLO graphs (hlo_dot_batched.comp:19-38 as lowered by
// source/xla_hlo/src/compiler.rs:1009-1084: Q.K^T per (batch, head) and P.V),
// where both operands are activations, so each is split into tf32 hi / lo on
// chip and the product is issued as 3xTF32 tcgen05.mma.
//
//   C[b][i][m][n] = alpha * sum_k A[b][i][m][k] * B[b][i / div][k][n]
//
// A must be K-contiguous.  B is either K-contiguous ([n][k] rows, Q.K^T) or
// N-contiguous ([k][n] rows, P.V); the N-contiguous tile arrives as a plain
// TMA box and the split pass writes it transposed into the K-major
// 128-byte-swizzled layout the MMA reads.  One CTA per (batch, head, m tile,
// n tile): thread 0 issues every TMA box of the tile at once (the whole K
// fits shared memory), the 128 threads write the lo terms (and the
// transposed B), one thread issues the MMAs into a TMEM accumulator, and the
// four warps drain their lane quarter to C.  Waits are bounded (2 s) and
// report a device status like the other tensor-core kernels.
#include <cuda.h>

#include <mutex>

#include "sm100_prims.cuh"
#include "spx_internal.cuh"

namespace spx {

__device__ int g_bg_status = 0;

namespace {

using namespace sm100;

constexpr int kThreads = 128;
constexpr uint32_t kATile = 128 * 32 * 4;  // one 128 x 32 fp32 k-block
constexpr unsigned long long kWaitNs = 2000000000ull;

struct BgArgs {
  int m, n, k, inner, div, m_tiles, n_tiles, bn, kblocks, bnmajor;
  int64_t c_bs, c_bis, c_ms;
  float alpha;
  float* c;
  uint32_t idesc, tmem_cols, b_tile;  // b_tile = bn x 32 fp32 bytes
};

__global__ void __launch_bounds__(kThreads, 1)
    bgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const BgArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int KB = p.kblocks;
  uint8_t* a_hi = smem;                                  // KB x 16 KB (TMA, swizzled)
  uint8_t* a_lo = a_hi + (size_t)KB * kATile;            // KB x 16 KB
  uint8_t* b_hi = a_lo + (size_t)KB * kATile;            // KB x b_tile (K-major, swizzled)
  uint8_t* b_lo = b_hi + (size_t)KB * p.b_tile;          // KB x b_tile
  uint8_t* b_st = b_lo + (size_t)KB * p.b_tile;          // N-major staging: KB x 32 x bn
  uint64_t* bars = (uint64_t*)(b_st + (p.bnmajor ? (size_t)KB * p.b_tile : 0));
  uint64_t* full = bars;
  uint64_t* done = bars + 1;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  int t = blockIdx.x;
  const int nt = t % p.n_tiles;
  t /= p.n_tiles;
  const int mt = t % p.m_tiles;
  t /= p.m_tiles;
  const int ii = t % p.inner;
  const int bb = t / p.inner;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mb_init(full, 1);
    mb_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sa(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_slot;

  if (threadIdx.x == 0) {
    mb_expect_tx(full, (uint32_t)KB * (kATile + p.b_tile));
    for (int kb = 0; kb < KB; ++kb) {
      tma_4d(a_hi + (size_t)kb * kATile, &tmA, full, kb * 32, mt * 128, ii, bb);
      if (p.bnmajor)
        tma_4d(b_st + (size_t)kb * p.b_tile, &tmB, full, nt * p.bn, kb * 32, ii / p.div, bb);
      else
        tma_4d(b_hi + (size_t)kb * p.b_tile, &tmB, full, kb * 32, nt * p.bn, ii / p.div, bb);
    }
  }
  bool ok = mb_wait(full, 0, abort_flag, &g_bg_status, kWaitNs, 64);
  ok = __syncthreads_and(ok);
  if (!ok && threadIdx.x == 0) {  // this CTA's copies land before its memory is released
    volatile int never = 0;
    mb_wait(full, 0, &never, &g_bg_status, 200000000ull, 64);
  }
  if (ok) {
    // lo terms in the operand's own swizzled position (A, K-major B)
    const int a16 = KB * (int)(kATile / 16);
    for (int i = threadIdx.x; i < a16; i += kThreads) {
      const float4 v = reinterpret_cast<const float4*>(a_hi)[i];
      reinterpret_cast<float4*>(a_lo)[i] =
          make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
    }
    if (!p.bnmajor) {
      const int b16 = KB * (int)(p.b_tile / 16);
      for (int i = threadIdx.x; i < b16; i += kThreads) {
        const float4 v = reinterpret_cast<const float4*>(b_hi)[i];
        reinterpret_cast<float4*>(b_lo)[i] =
            make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
      }
    } else {
      // Staging row k holds B[k][0..bn); K-major row n, 16-byte chunk k/4,
      // 128-byte swizzle: byte n*128 + ((k/4 ^ n%8) * 16) + (k%4) * 4.
      // A thread takes 4 consecutive k of one n (one 16-byte chunk).
      const int chunks = KB * p.bn * 8;
      for (int i = threadIdx.x; i < chunks; i += kThreads) {
        const int n = i % p.bn;
        const int kc = (i / p.bn) % 8;
        const int kb = i / (p.bn * 8);
        const float* st = reinterpret_cast<const float*>(b_st + (size_t)kb * p.b_tile);
        float4 v;
        v.x = st[(kc * 4 + 0) * p.bn + n];
        v.y = st[(kc * 4 + 1) * p.bn + n];
        v.z = st[(kc * 4 + 2) * p.bn + n];
        v.w = st[(kc * 4 + 3) * p.bn + n];
        const size_t off = (size_t)kb * p.b_tile + (size_t)n * 128 + ((kc ^ (n & 7)) * 16);
        *reinterpret_cast<float4*>(b_hi + off) = v;
        *reinterpret_cast<float4*>(b_lo + off) =
            make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (ok && threadIdx.x == 32) {
    tc_after();
    for (int kb = 0; kb < KB; ++kb) {
      const uint32_t ah = sa(a_hi + (size_t)kb * kATile), al = sa(a_lo + (size_t)kb * kATile);
      const uint32_t bh = sa(b_hi + (size_t)kb * p.b_tile), bl = sa(b_lo + (size_t)kb * p.b_tile);
      const int ksteps = min(4, (p.k - kb * 32 + 7) / 8);
#pragma unroll 1
      for (int k = 0; k < ksteps; ++k) {
        const uint32_t off = k * 32;
        mma_tf32(tmem, sw128_desc(al + off), sw128_desc(bh + off), p.idesc, (kb | k) ? 1u : 0u);
        mma_tf32(tmem, sw128_desc(ah + off), sw128_desc(bl + off), p.idesc, 1u);
        mma_tf32(tmem, sw128_desc(ah + off), sw128_desc(bh + off), p.idesc, 1u);
      }
    }
    mma_commit(done);
  }
  if (ok) ok = mb_wait(done, 0, abort_flag, &g_bg_status, kWaitNs, 128);
  ok = __all_sync(0xffffffffu, ok);
  if (ok) {
    tc_after();
    const int row = mt * 128 + warp * 32 + lane;
    float* crow = p.c + (int64_t)bb * p.c_bs + (int64_t)ii * p.c_bis + (int64_t)row * p.c_ms;
    const bool vec = (p.c_ms % 4 == 0) && (((uintptr_t)p.c & 15) == 0) && (p.c_bs % 4 == 0) &&
                     (p.c_bis % 4 == 0);
    for (int c0 = 0; c0 < p.bn; c0 += 32) {
      float v[32];
      tmem_ld_32x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      const int n0 = nt * p.bn + c0;
      if (row >= p.m) continue;
      if (vec && n0 + 32 <= p.n) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          reinterpret_cast<float4*>(crow + n0)[e] =
              make_float4(v[4 * e] * p.alpha, v[4 * e + 1] * p.alpha, v[4 * e + 2] * p.alpha,
                          v[4 * e + 3] * p.alpha);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (n0 + e < p.n) crow[n0 + e] = v[e] * p.alpha;
      }
    }
  }
  tc_before();
  __syncthreads();
  if (warp == 1) {
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

bool m16(int64_t v) { return v % 4 == 0; }  // a stride of a whole number of 16-byte units

size_t bg_smem(int kb, int bn, bool bnmajor) {
  return 1024 + (size_t)kb * (2 * kATile + (bnmajor ? 3 : 2) * (size_t)bn * 128) + 64;
}

}  // namespace

int bg_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_bg_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_bg_status, &zero, sizeof(int));
  }
  return v;
}

// -1: not eligible (caller falls back), else SPX_OK or an error code.
int try_bgemm_tc(cudaStream_t s, int64_t* cnt, const float* a, const float* b, const float* bias,
                 const float* res, float* c, const spx_gemm_params* q) {
  if (bias || res || q->activation != SPX_ACT_NONE) return -1;
  if (q->k > 128 || q->k < 1 || q->a_ks != 1) return -1;
  const bool bnmajor = q->b_ns == 1 && q->b_ks != 1;
  if (!bnmajor && q->b_ks != 1) return -1;
  const int inner = q->batch_inner > 0 ? q->batch_inner : 1;
  const int div = q->b_inner_div > 0 ? q->b_inner_div : 1;
  if (inner % div) return -1;
  auto al = [](const void* v) { return ((uintptr_t)v & 15) == 0; };
  if (!al(a) || !al(b) || !al(c)) return -1;
  if (!m16(q->a_ms) || !m16(q->a_bs) || !m16(q->a_bis) || !m16(q->b_bs) || !m16(q->b_bis) ||
      !m16(bnmajor ? q->b_ks : q->b_ns))
    return -1;
  if (q->k % 4) return -1;  // K-contiguous rows in whole 16-byte units
  if (bnmajor && q->n % 4) return -1;
  const int kb = (q->k + 31) / 32;
  // n tile: the widest of 256 / 128 / 64 / 32 whose shared memory fits; prefer
  // tiles small enough for two CTAs per SM when the grid is large.
  int bn = 0;
  const int cap = 227 * 1024;
  for (int cand : {256, 128, 64, 32}) {
    if (cand > ((q->n + 31) / 32) * 32) continue;
    if (bg_smem(kb, cand, bnmajor) <= (size_t)cap) {
      bn = cand;
      break;
    }
  }
  if (!bn) return -1;
  BgArgs p{};
  p.m = q->m;
  p.n = q->n;
  p.k = q->k;
  p.inner = inner;
  p.div = div;
  p.m_tiles = (q->m + 127) / 128;
  p.n_tiles = (q->n + bn - 1) / bn;
  p.bn = bn;
  p.kblocks = kb;
  p.bnmajor = bnmajor ? 1 : 0;
  p.c_bs = q->c_bs;
  p.c_bis = q->c_bis;
  p.c_ms = q->c_ms;
  p.alpha = q->alpha;
  p.c = c;
  p.b_tile = (uint32_t)bn * 128;
  p.tmem_cols = (uint32_t)(bn < 32 ? 32 : bn);
  p.idesc = idesc_tf32(128, bn);
  const int64_t grid = (int64_t)q->batch * inner * p.m_tiles * p.n_tiles;
  if (grid > INT32_MAX) return -1;
  EncodeFn fn = encoder();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap ma, mb;
  {
    cuuint64_t dims[4] = {(cuuint64_t)q->k, (cuuint64_t)q->m, (cuuint64_t)inner,
                          (cuuint64_t)q->batch};
    // A batch dimension of extent 1 may carry stride 0; any 16-byte multiple
    // serves the encoder there.
    cuuint64_t str[3] = {(cuuint64_t)q->a_ms * 4, (cuuint64_t)(q->a_bis ? q->a_bis * 4 : 16),
                         (cuuint64_t)(q->a_bs ? q->a_bs * 4 : 16)};
    cuuint32_t box[4] = {32, 128, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)a, dims, str, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -1;
  }
  {
    const int binner = inner / div;
    cuuint64_t dims[4], str[3];
    cuuint32_t box[4];
    if (bnmajor) {
      dims[0] = (cuuint64_t)q->n;
      dims[1] = (cuuint64_t)q->k;
      str[0] = (cuuint64_t)q->b_ks * 4;
      box[0] = (cuuint32_t)bn;
      box[1] = 32;
    } else {
      dims[0] = (cuuint64_t)q->k;
      dims[1] = (cuuint64_t)q->n;
      str[0] = (cuuint64_t)q->b_ns * 4;
      box[0] = 32;
      box[1] = (cuuint32_t)bn;
    }
    dims[2] = (cuuint64_t)binner;
    dims[3] = (cuuint64_t)q->batch;
    str[1] = (cuuint64_t)(q->b_bis ? q->b_bis * 4 : 16);
    str[2] = (cuuint64_t)(q->b_bs ? q->b_bs * 4 : 16);
    box[2] = 1;
    box[3] = 1;
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)b, dims, str, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                    bnmajor ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -1;
  }
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(bgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "bgemm_tc: smem attribute");
  const size_t smem = bg_smem(kb, bn, bnmajor);
  bgemm_tc_kernel<<<(int)grid, kThreads, smem, s>>>(ma, mb, p);
  return after_launch(cnt, "bgemm_tc");
}

}  // namespace spx
