// FP32 SIMT GEMM / implicit-GEMM convolution.
//
// One kernel template covers every dense contraction of the reference's
// kernel set in exact fp32 arithmetic:
//   * conv2d.comp / hlo_conv_nhwc_hwio.comp  -> implicit GEMM over NHWC input
//     (M = n*oh*ow, N = oc, K = kh*kw*ic), OHWI or HWIO weights
//   * fully_connected.comp, hlo_dot_rank2.comp, hlo_dot_batched.comp
//     -> strided batched GEMM (no host transposes)
// with bias, residual and activation fused into the epilogue (the reference
// issues those as separate relu/relu6/add dispatches, scheduler.rs:1146-1197).
//
// This is the exact-fp32 path used for shapes the tensor-core kernel does not
// take (K or N not a multiple of its tile granule, strided batched operands).
// Tiles: BM x BN outputs per 256-thread CTA, TM x TN per thread, BK-deep
// double-buffered shared-memory stages with register prefetch of the next
// stage while the current one is consumed.
#include "spx_internal.cuh"

namespace spx {

namespace {

struct GemmArgs {
  const float* a;
  const float* b;
  const float* bias;
  const float* res;
  float* c;
  int M, N, K;
  int batch_inner, b_inner_div;
  int64_t a_bs, a_ms, a_ks, b_bs, b_ks, b_ns, c_bs, c_ms, a_bis, b_bis, c_bis;
  float alpha;
  int act;
  // implicit convolution (A_MODE == 2)
  int ih, iw, ic, oh, ow, kw, sh, sw, pt, pl, dh, dw;
};

// A_MODE: 0 = strided matrix, k-contiguous mapping; 1 = strided matrix,
// m-contiguous mapping; 2 = implicit convolution gather from NHWC.
// B_KC: B's k index is the contiguous one (b_ks == 1, OHWI / W[n][k]).
template <int BM, int BN, int BK, int TM, int TN, int A_MODE, bool B_KC>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_simt_kernel(const GemmArgs p) {
  constexpr int THREADS = (BM / TM) * (BN / TN);
  constexpr int A_LOADS = BM * BK / THREADS;
  constexpr int B_LOADS = BN * BK / THREADS;
  static_assert(BM * BK % THREADS == 0 && BN * BK % THREADS == 0, "tile");
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];

  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int z = blockIdx.z;
  const int outer = z / p.batch_inner, inner = z % p.batch_inner;
  const float* A = p.a + outer * p.a_bs + inner * p.a_bis;
  const float* B = p.b + outer * p.b_bs + (inner / p.b_inner_div) * p.b_bis;
  float* C = p.c + outer * p.c_bs + inner * p.c_bis;
  const float* R = p.res ? p.res + outer * p.c_bs + inner * p.c_bis : nullptr;

  // Per-slot row bookkeeping for A loads.
  int a_kk[A_LOADS];
  int64_t a_m[A_LOADS];
  int64_t a_base[A_LOADS];  // conv: image base offset; matrix: row offset
  int a_iy[A_LOADS], a_ix[A_LOADS];
#pragma unroll
  for (int i = 0; i < A_LOADS; ++i) {
    int e = tid + i * THREADS;
    int mm, kk;
    if (A_MODE == 1) { mm = e % BM; kk = e / BM; } else { kk = e % BK; mm = e / BK; }
    a_kk[i] = kk;
    int64_t m = m0 + mm;
    a_m[i] = m;
    if (A_MODE == 2) {
      int64_t mc = m < p.M ? m : 0;
      int ox = (int)(mc % p.ow);
      int64_t t = mc / p.ow;
      int oy = (int)(t % p.oh);
      int64_t img = t / p.oh;
      a_base[i] = img * p.ih * p.iw * (int64_t)p.ic;
      a_iy[i] = oy * p.sh - p.pt;
      a_ix[i] = ox * p.sw - p.pl;
    } else {
      a_base[i] = m * p.a_ms;
      a_iy[i] = a_ix[i] = 0;
    }
  }

  float a_reg[A_LOADS], b_reg[B_LOADS];
  auto load_tiles = [&](int k0) {
    if (A_MODE == 2) {
      // All A slots of this thread share kk when THREADS % BK == 0.
#pragma unroll
      for (int i = 0; i < A_LOADS; ++i) {
        int k = k0 + a_kk[i];
        float v = 0.0f;
        if (k < p.K && a_m[i] < p.M) {
          int ci = k % p.ic;
          int t = k / p.ic;
          int kx = t % p.kw;
          int ky = t / p.kw;
          int iy = a_iy[i] + ky * p.dh;
          int ix = a_ix[i] + kx * p.dw;
          if (iy >= 0 && iy < p.ih && ix >= 0 && ix < p.iw)
            v = __ldg(A + a_base[i] + ((int64_t)iy * p.iw + ix) * p.ic + ci);
        }
        a_reg[i] = v;
      }
    } else {
#pragma unroll
      for (int i = 0; i < A_LOADS; ++i) {
        int k = k0 + a_kk[i];
        a_reg[i] = (k < p.K && a_m[i] < p.M) ? __ldg(A + a_base[i] + k * p.a_ks) : 0.0f;
      }
    }
#pragma unroll
    for (int i = 0; i < B_LOADS; ++i) {
      int e = tid + i * THREADS;
      int nn, kk;
      if (B_KC) { kk = e % BK; nn = e / BK; } else { nn = e % BN; kk = e / BN; }
      int k = k0 + kk, n = n0 + nn;
      b_reg[i] = (k < p.K && n < p.N) ? __ldg(B + (int64_t)k * p.b_ks + (int64_t)n * p.b_ns) : 0.0f;
    }
  };
  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int i = 0; i < A_LOADS; ++i) {
      int e = tid + i * THREADS;
      int mm, kk;
      if (A_MODE == 1) { mm = e % BM; kk = e / BM; } else { kk = e % BK; mm = e / BK; }
      As[buf][kk][mm] = a_reg[i];
    }
#pragma unroll
    for (int i = 0; i < B_LOADS; ++i) {
      int e = tid + i * THREADS;
      int nn, kk;
      if (B_KC) { kk = e % BK; nn = e / BK; } else { nn = e % BN; kk = e / BN; }
      Bs[buf][kk][nn] = b_reg[i];
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  const int ktiles = (p.K + BK - 1) / BK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();
  int buf = 0;
  for (int t = 0; t < ktiles; ++t) {
    if (t + 1 < ktiles) load_tiles((t + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float ar[TM], br[TN];
#pragma unroll
      for (int i = 0; i < TM; i += 4) {
        float4 v = *reinterpret_cast<const float4*>(&As[buf][kk][ty * TM + i]);
        ar[i] = v.x; ar[i + 1] = v.y; ar[i + 2] = v.z; ar[i + 3] = v.w;
      }
#pragma unroll
      for (int j = 0; j < TN; j += 4) {
        float4 v = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * TN + j]);
        br[j] = v.x; br[j + 1] = v.y; br[j + 2] = v.z; br[j + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    if (t + 1 < ktiles) store_tiles(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    int64_t m = m0 + ty * TM + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int n = n0 + tx * TN + j;
      if (n >= p.N) continue;
      float v = acc[i][j] * p.alpha;
      if (p.bias) v += __ldg(p.bias + n);
      if (R) v += R[m * p.c_ms + n];
      C[m * p.c_ms + n] = apply_act(p.act, v);
    }
  }
}

template <int BM, int BN, int BK, int TM, int TN>
int dispatch_cfg(cudaStream_t s, const GemmArgs& a, int a_mode, bool b_kc, int batches) {
  constexpr int THREADS = (BM / TM) * (BN / TN);
  dim3 grid((unsigned)ceil_div(a.M, BM), (unsigned)ceil_div(a.N, BN), (unsigned)batches);
#define SPX_GEMM_CASE(AM, BKC) \
  gemm_simt_kernel<BM, BN, BK, TM, TN, AM, BKC><<<grid, THREADS, 0, s>>>(a)
  if (a_mode == 0) { if (b_kc) SPX_GEMM_CASE(0, true); else SPX_GEMM_CASE(0, false); }
  else if (a_mode == 1) { if (b_kc) SPX_GEMM_CASE(1, true); else SPX_GEMM_CASE(1, false); }
  else { if (b_kc) SPX_GEMM_CASE(2, true); else SPX_GEMM_CASE(2, false); }
#undef SPX_GEMM_CASE
  return SPX_OK;
}

int run_simt(cudaStream_t s, int64_t* cnt, const GemmArgs& a, int a_mode, bool b_kc,
             int batches) {
  if (a.M <= 0 || a.N <= 0 || batches <= 0) return SPX_OK;
  if (ceil_div(a.N, 16) > 65535 || batches > 65535)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm: grid too large (N=%d, batches=%d)", a.N, batches);
  if (a.N > 64) dispatch_cfg<128, 128, 16, 8, 8>(s, a, a_mode, b_kc, batches);
  else if (a.N > 32) dispatch_cfg<128, 64, 16, 8, 4>(s, a, a_mode, b_kc, batches);
  else if (a.N > 16) dispatch_cfg<256, 32, 16, 8, 4>(s, a, a_mode, b_kc, batches);
  else dispatch_cfg<256, 16, 16, 4, 4>(s, a, a_mode, b_kc, batches);
  return after_launch(cnt, "gemm_simt");
}

}  // namespace

int launch_gemm_simt(cudaStream_t s, int64_t* cnt, const float* a, const float* b,
                     const float* bias, const float* res, float* c, const spx_gemm_params* p) {
  GemmArgs g = {};
  g.a = a; g.b = b; g.bias = bias; g.res = res; g.c = c;
  g.M = p->m; g.N = p->n; g.K = p->k;
  g.batch_inner = p->batch_inner > 0 ? p->batch_inner : 1;
  g.b_inner_div = p->b_inner_div > 0 ? p->b_inner_div : 1;
  g.a_bs = p->a_bs; g.a_ms = p->a_ms; g.a_ks = p->a_ks;
  g.b_bs = p->b_bs; g.b_ks = p->b_ks; g.b_ns = p->b_ns;
  g.c_bs = p->c_bs; g.c_ms = p->c_ms;
  g.a_bis = p->a_bis; g.b_bis = p->b_bis; g.c_bis = p->c_bis;
  g.alpha = p->alpha; g.act = p->activation;
  int a_mode = (p->a_ks == 1 || p->a_ms != 1) ? 0 : 1;
  bool b_kc = p->b_ks == 1 && p->b_ns != 1;
  return run_simt(s, cnt, g, a_mode, b_kc, p->batch * g.batch_inner);
}

int launch_conv_simt(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                     const float* bias, const float* res, float* y, const spx_conv_params* p) {
  GemmArgs g = {};
  g.a = x; g.b = w; g.bias = bias; g.res = res; g.c = y;
  g.M = p->n * p->oh * p->ow;
  g.N = p->oc;
  g.K = p->kh * p->kw * p->ic;
  g.batch_inner = 1; g.b_inner_div = 1;
  g.c_ms = p->oc;
  g.alpha = 1.0f; g.act = p->activation;
  bool b_kc;
  if (p->weight_layout == SPX_WEIGHT_OHWI) { g.b_ks = 1; g.b_ns = g.K; b_kc = true; }
  else { g.b_ks = p->oc; g.b_ns = 1; b_kc = false; }
  bool pointwise = p->kh == 1 && p->kw == 1 && p->stride_h == 1 && p->stride_w == 1 &&
                   p->pad_top == 0 && p->pad_left == 0 && p->oh == p->ih && p->ow == p->iw;
  if (pointwise) {
    g.a_ms = p->ic; g.a_ks = 1;
    return run_simt(s, cnt, g, 0, b_kc, 1);
  }
  g.ih = p->ih; g.iw = p->iw; g.ic = p->ic; g.oh = p->oh; g.ow = p->ow; g.kw = p->kw;
  g.sh = p->stride_h; g.sw = p->stride_w; g.pt = p->pad_top; g.pl = p->pad_left;
  g.dh = p->dilation_h > 0 ? p->dilation_h : 1;
  g.dw = p->dilation_w > 0 ? p->dilation_w : 1;
  return run_simt(s, cnt, g, 2, b_kc, 1);
}

}  // namespace spx
