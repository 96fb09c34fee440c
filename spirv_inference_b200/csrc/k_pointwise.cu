// Pointwise (1x1, stride 1) convolution on CUDA cores for the short
// reductions of inverted-residual blocks (expand 16 -> 96, project 144 -> 24
// and the like, conv2d.comp:26-50 with kh = kw = 1).  At K or N below ~200
// these layers move far more bytes than they do arithmetic: exact fp32 FMAs
// on CUDA cores keep up with HBM, and a CTA's output is written as whole rows
// without the tensor-core path's TMEM -> register -> shared-memory epilogue
// per 32-column chunk.
//
// A CTA owns a tile of kP = 256 consecutive pixels (rows of the NHWC [M][K]
// input; one contiguous run of memory) and 128 threads; thread t computes
// pixels t and t + 128.  Shared memory holds
//   ws  the weights transposed to [K][N] (read as 16-byte warp broadcasts),
//   bs  the bias,
//   xs  the input tile transposed to [k][pixel] (row pitch kP + 1, so a warp's
//       32 pixels of one channel are 32 banks),
//   ys  one output chunk [pixel][NC] (row pitch NC + 1: conflict-free column
//       writes), written back as 16-byte row vectors with the residual and
//       the activation applied.
// K <= 64: the whole input tile is staged once and the N outputs are produced
// in chunks of NC.  K > 64 (projections): N == NC and the reduction runs over
// 32-channel chunks of the input tile.  Each output is the bias plus the K
// products accumulated in channel order with fmaf.
#include "spx_internal.cuh"

namespace spx {
namespace {

constexpr int kP = 256;        // pixels per CTA tile
constexpr int kT = 128;        // threads per CTA
constexpr int kXPitch = kP + 1;
constexpr int kKSingle = 64;   // K up to this: one staging of the input tile
constexpr int kKChunk = 32;    // otherwise: the reduction in 32-channel chunks

inline bool al16v(const void* p) { return ((uintptr_t)p & 15) == 0; }

// Stages xs[k][p] = x[m0 + p][k0 + k] for k < kc (kc % 4 == 0), p < kP.
__device__ __forceinline__ void stage_x(const float* __restrict__ x, float* xs, int64_t m0,
                                        int64_t M, int K, int k0, int kc) {
  const int q4 = kc >> 2;  // 16-byte vectors per pixel row
  const int dp = kT / q4, dj = kT % q4;
  int p = threadIdx.x / q4, j = threadIdx.x % q4;
  const int rows = (int)(M - m0 < kP ? M - m0 : kP);
  while (p < rows) {
    const float4 v =
        __ldg(reinterpret_cast<const float4*>(x + (m0 + p) * (int64_t)K + k0) + j);
    float* d = xs + (4 * j) * kXPitch + p;
    d[0] = v.x;
    d[kXPitch] = v.y;
    d[2 * kXPitch] = v.z;
    d[3 * kXPitch] = v.w;
    p += dp;
    j += dj;
    if (j >= q4) {
      j -= q4;
      ++p;
    }
  }
}

template <int NC>
__global__ void __launch_bounds__(kT, 3) pw_simt_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    const float* __restrict__ res, float* __restrict__ y, int64_t M, int K, int N, int act) {
  extern __shared__ __align__(16) float smem[];
  float* ws = smem;                    // [K][N]
  float* bs = ws + K * N;              // [N]
  float* xs = bs + ((N + 3) & ~3);     // [kc][kXPitch]
  const int xs_rows = K <= kKSingle ? K : kKChunk;
  float* ys = xs + ((xs_rows * kXPitch + 3) & ~3);  // [kP][NC + 1]
  constexpr int kYPitch = NC + 1;
  const int t = threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.x * kP;

  // OHWI weights w[n][k] -> ws[k][n]: coalesced reads, once per CTA.
  for (int i = t; i < K * N; i += kT) {
    const int n = i / K, k = i - n * K;
    ws[k * N + n] = __ldg(w + i);
  }
  for (int i = t; i < N; i += kT) bs[i] = bias ? __ldg(bias + i) : 0.0f;
  const bool single = K <= kKSingle;
  if (single) stage_x(x, xs, m0, M, K, 0, K);
  __syncthreads();

  for (int nc0 = 0; nc0 < N; nc0 += NC) {
    float a0[NC], a1[NC];
#pragma unroll
    for (int n = 0; n < NC; ++n) a0[n] = a1[n] = bs[nc0 + n];
    for (int k0 = 0; k0 < K; k0 += kKChunk) {
      int kc = K - k0;
      if (single) {
        k0 = 0;
        kc = K;
      } else {
        if (kc > kKChunk) kc = kKChunk;
        if (k0 > 0) __syncthreads();  // every thread done with the previous chunk
        stage_x(x, xs, m0, M, K, k0, kc);
        __syncthreads();
      }
      const float* xr = xs + t;
      const float4* wr = reinterpret_cast<const float4*>(ws + k0 * N + nc0);
      const int wq = N >> 2;  // float4 per ws row
#pragma unroll 2
      for (int k = 0; k < kc; ++k) {
        const float x0 = xr[k * kXPitch], x1 = xr[k * kXPitch + kT];
        const float4* wk = wr + k * wq;
#pragma unroll
        for (int q = 0; q < NC / 4; ++q) {
          const float4 w4 = wk[q];
          a0[4 * q + 0] = fmaf(x0, w4.x, a0[4 * q + 0]);
          a0[4 * q + 1] = fmaf(x0, w4.y, a0[4 * q + 1]);
          a0[4 * q + 2] = fmaf(x0, w4.z, a0[4 * q + 2]);
          a0[4 * q + 3] = fmaf(x0, w4.w, a0[4 * q + 3]);
          a1[4 * q + 0] = fmaf(x1, w4.x, a1[4 * q + 0]);
          a1[4 * q + 1] = fmaf(x1, w4.y, a1[4 * q + 1]);
          a1[4 * q + 2] = fmaf(x1, w4.z, a1[4 * q + 2]);
          a1[4 * q + 3] = fmaf(x1, w4.w, a1[4 * q + 3]);
        }
      }
      if (single) break;
    }
    // Output chunk: registers -> ys -> 16-byte row vectors.
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      ys[t * kYPitch + n] = a0[n];
      ys[(t + kT) * kYPitch + n] = a1[n];
    }
    __syncthreads();
    const int rows = (int)(M - m0 < kP ? M - m0 : kP);
    constexpr int q4 = NC / 4;
    with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
      for (int i = t; i < rows * q4; i += kT) {
        const int p = i / q4, n = 4 * (i - p * q4);
        const float* s = ys + p * kYPitch + n;
        float4 v = make_float4(s[0], s[1], s[2], s[3]);
        const int64_t off = (m0 + p) * (int64_t)N + nc0 + n;
        if (res) {
          const float4 r = __ldg(reinterpret_cast<const float4*>(res + off));
          v.x += r.x;
          v.y += r.y;
          v.z += r.z;
          v.w += r.w;
        }
        v.x = act_c<A>(v.x);
        v.y = act_c<A>(v.y);
        v.z = act_c<A>(v.z);
        v.w = act_c<A>(v.w);
        *reinterpret_cast<float4*>(y + off) = v;
      }
    });
    __syncthreads();  // ys (and, for K > 64, xs) free for the next chunk
  }
}

int pw_chunk(int K, int N) {
  if (K <= kKSingle) {
    for (int nc : {32, 24, 40, 16})
      if (N % nc == 0) return nc;
    return 0;
  }
  return (N == 16 || N == 24 || N == 32 || N == 40) ? N : 0;
}

size_t pw_smem(int K, int N, int nc) {
  const int xs_rows = K <= kKSingle ? K : kKChunk;
  return sizeof(float) * ((size_t)K * N + ((N + 3) & ~3) + ((xs_rows * kXPitch + 3) & ~3) +
                          (size_t)kP * (nc + 1));
}

}  // namespace

bool pw_simt_eligible(const float* x, const float* y, const float* res, int64_t M, int K, int N) {
  if (M <= 0 || K <= 0 || N <= 0 || K % 4 || N % 4) return false;
  if ((int64_t)K * N > 8192) return false;  // weights fit in shared memory with the tiles
  if (!al16v(x) || !al16v(y) || (res && !al16v(res))) return false;
  const int nc = pw_chunk(K, N);
  return nc != 0 && pw_smem(K, N, nc) <= 110 * 1024;
}

int launch_pw_simt(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* bias, const float* res, float* y, int64_t M, int K, int N,
                   int act) {
  const int nc = pw_chunk(K, N);
  if (!nc) return fail(SPX_ERR_UNSUPPORTED, "pointwise: N=%d has no supported chunk", N);
  const size_t smem = pw_smem(K, N, nc);
  const int64_t grid = (M + kP - 1) / kP;
  if (grid > INT32_MAX) return fail(SPX_ERR_INVALID_ARGUMENT, "pointwise: M too large");
#define SPX_PW(NCV)                                                                          \
  case NCV:                                                                                  \
    cudaFuncSetAttribute(pw_simt_kernel<NCV>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                         (int)smem);                                                         \
    pw_simt_kernel<NCV><<<(int)grid, kT, smem, s>>>(x, w, bias, res, y, M, K, N, act);       \
    break;
  switch (nc) {
    SPX_PW(16)
    SPX_PW(24)
    SPX_PW(32)
    SPX_PW(40)
    default: return fail(SPX_ERR_UNSUPPORTED, "pointwise: chunk %d", nc);
  }
#undef SPX_PW
  return after_launch(cnt, "pw_simt");
}

}  // namespace spx
