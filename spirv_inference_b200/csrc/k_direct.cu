// Direct (non-GEMM) kernels for the bandwidth-bound spatial convolutions of
// the CNN graphs, NHWC:
//
//  * conv_smallk: dense conv whose reduction K = kh*kw*ic is small (the
//    3x3x3 stem of MobileNetV2 / EfficientNet-Lite0, conv2d.comp:26-50 as an
//    NHWC kernel).  Weights [K][oc] sit in shared memory and are read as
//    16-byte warp broadcasts; one thread computes all oc outputs of one
//    pixel.  A warp's 32 pixels are consecutive, so their outputs are one
//    contiguous run: it is staged in shared memory and written as whole
//    rows of 16-byte vectors.  Input bytes are read once from HBM (tap
//    overlap is served by L1), outputs written once.
//
//  * dw_rows: depthwise conv (depthwise_conv2d.comp:27-49) with a vertical
//    sliding window: a thread owns 4 channels of one output column and R
//    consecutive output rows, keeps the kh x kw x 4 weights in registers, and
//    reads each input row of its window once instead of kh times.  Channel
//    groups are the fastest-varying thread index so a warp reads contiguous
//    runs of the NHWC rows.  32-bit index arithmetic.
#include "spx_internal.cuh"

namespace spx {
namespace {

// KH / KW / IC > 0 fix the window at compile time (the 3x3x3 stems: the 27
// input loads of a pixel are then issued before its FMAs); 0 = runtime.
template <int OC, int KH = 0, int KW = 0, int IC = 0>
__global__ void __launch_bounds__(128) conv_smallk_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    const float* __restrict__ res, float* __restrict__ y, int n, int ih, int iw, int ic_rt,
    int oh, int ow, int kh_rt, int kw_rt, int sh, int sw, int pt, int pl, int dh, int dw, int act,
    int w_layout) {
  const int kh = KH > 0 ? KH : kh_rt, kw = KW > 0 ? KW : kw_rt, ic = IC > 0 ? IC : ic_rt;
  extern __shared__ float ws[];  // [K][OC], bias[OC], then per-warp output staging
  constexpr int kStride = OC + 4;  // staging row pitch (floats): conflict-free float4 rows
  const int K = kh * kw * ic;
  float* stage = ws + K * OC + OC + (threadIdx.x >> 5) * 32 * kStride;
  for (int i = threadIdx.x; i < K * OC; i += blockDim.x) {
    const int k = i / OC, o = i % OC;
    // OHWI: w[o][k]; HWIO: w[k][o]  (k = (ky*kw + kx)*ic + ci in both)
    ws[i] = w_layout == SPX_WEIGHT_OHWI ? w[(size_t)o * K + k] : w[(size_t)k * OC + o];
  }
  for (int o = threadIdx.x; o < OC; o += blockDim.x) ws[K * OC + o] = bias ? bias[o] : 0.0f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int total = n * oh * ow;
  // Warp-uniform loop: each warp takes 32 consecutive output pixels, whose
  // NHWC outputs are one contiguous 32 * OC run.
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int base = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32; base < total;
       base += warps * 32) {
    const int pix = base + lane;
    float acc[OC];
#pragma unroll
    for (int o = 0; o < OC; ++o) acc[o] = ws[K * OC + o];
    if (pix < total) {
      const int ox = pix % ow;
      const int t = pix / ow;
      const int oy = t % oh;
      const int img = t / oh;
      const float* xi = x + (size_t)img * ih * iw * ic;
      if constexpr (KH > 0 && KW > 0 && IC > 0) {
        float xv[KH * KW * IC];
#pragma unroll
        for (int ky = 0; ky < KH; ++ky)
#pragma unroll
          for (int kx = 0; kx < KW; ++kx) {
            const int iy = oy * sh + ky * dh - pt, ix = ox * sw + kx * dw - pl;
            const bool in = iy >= 0 && iy < ih && ix >= 0 && ix < iw;
            const float* xp = xi + ((size_t)(in ? iy : 0) * iw + (in ? ix : 0)) * IC;
#pragma unroll
            for (int ci = 0; ci < IC; ++ci) xv[(ky * KW + kx) * IC + ci] = in ? __ldg(xp + ci) : 0.0f;
          }
#pragma unroll
        for (int k = 0; k < KH * KW * IC; ++k) {
          const float4* wp = reinterpret_cast<const float4*>(ws + k * OC);
#pragma unroll
          for (int o = 0; o < OC / 4; ++o) {
            const float4 wv = wp[o];
            acc[4 * o + 0] = fmaf(xv[k], wv.x, acc[4 * o + 0]);
            acc[4 * o + 1] = fmaf(xv[k], wv.y, acc[4 * o + 1]);
            acc[4 * o + 2] = fmaf(xv[k], wv.z, acc[4 * o + 2]);
            acc[4 * o + 3] = fmaf(xv[k], wv.w, acc[4 * o + 3]);
          }
        }
      } else
      for (int ky = 0; ky < kh; ++ky) {
        const int iy = oy * sh + ky * dh - pt;
        if (iy < 0 || iy >= ih) continue;
        for (int kx = 0; kx < kw; ++kx) {
          const int ix = ox * sw + kx * dw - pl;
          if (ix < 0 || ix >= iw) continue;
          const float* xp = xi + ((size_t)iy * iw + ix) * ic;
          const float4* wp = reinterpret_cast<const float4*>(ws + ((ky * kw + kx) * ic) * OC);
          for (int ci = 0; ci < ic; ++ci) {
            const float v = __ldg(xp + ci);
#pragma unroll
            for (int o = 0; o < OC / 4; ++o) {
              const float4 wv = wp[ci * (OC / 4) + o];
              acc[4 * o + 0] = fmaf(v, wv.x, acc[4 * o + 0]);
              acc[4 * o + 1] = fmaf(v, wv.y, acc[4 * o + 1]);
              acc[4 * o + 2] = fmaf(v, wv.z, acc[4 * o + 2]);
              acc[4 * o + 3] = fmaf(v, wv.w, acc[4 * o + 3]);
            }
          }
        }
      }
    }
    // Stage the warp's 32 x OC outputs, then write them out as whole rows of
    // 16-byte vectors (coalesced), adding the residual and the activation.
    __syncwarp();
#pragma unroll
    for (int o = 0; o < OC; o += 4)
      *reinterpret_cast<float4*>(stage + lane * kStride + o) =
          make_float4(acc[o], acc[o + 1], acc[o + 2], acc[o + 3]);
    __syncwarp();
    const int valid = min(32, total - base) * OC / 4;  // float4s of this warp's run
    float* yb = y + (size_t)base * OC;
    const float* rb = res ? res + (size_t)base * OC : nullptr;
    with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
#pragma unroll
      for (int i = 0; i < OC / 4; ++i) {
        const int e4 = i * 32 + lane;  // float4 index within the run
        if (e4 < valid) {
          const int px = (e4 * 4) / OC, ch = (e4 * 4) % OC;
          float4 v = *reinterpret_cast<const float4*>(stage + px * kStride + ch);
          if (rb) {
            const float4 r = *reinterpret_cast<const float4*>(rb + (size_t)e4 * 4);
            v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
          }
          v.x = act_c<A>(v.x); v.y = act_c<A>(v.y);
          v.z = act_c<A>(v.z); v.w = act_c<A>(v.w);
          *reinterpret_cast<float4*>(yb + (size_t)e4 * 4) = v;
        }
      }
    });
  }
}

// The 3x3x3 stems (compile-time window, OC outputs): as conv_smallk, but each
// thread computes two pixels (lane and lane + 32 of a warp's 64-pixel run),
// so every 16-byte weight broadcast from shared memory feeds eight FMAs
// instead of four and the kernel runs at the FMA rate rather than the
// shared-memory rate.
template <int OC, int KH, int KW, int IC>
__global__ void __launch_bounds__(128) conv_stem2_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    const float* __restrict__ res, float* __restrict__ y, int n, int ih, int iw, int oh, int ow,
    int sh, int sw, int pt, int pl, int act, int w_layout) {
  constexpr int K = KH * KW * IC;
  constexpr int kStride = OC + 4;
  extern __shared__ float ws[];  // [K][OC], bias[OC], then per-warp 64-row output staging
  float* stage = ws + K * OC + OC + (threadIdx.x >> 5) * 64 * kStride;
  for (int i = threadIdx.x; i < K * OC; i += blockDim.x) {
    const int k = i / OC, o = i % OC;
    ws[i] = w_layout == SPX_WEIGHT_OHWI ? w[(size_t)o * K + k] : w[(size_t)k * OC + o];
  }
  for (int o = threadIdx.x; o < OC; o += blockDim.x) ws[K * OC + o] = bias ? bias[o] : 0.0f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int total = n * oh * ow;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int base = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 64; base < total;
       base += warps * 64) {
    float acc[2][OC];
    const float* xi[2];
    int oy[2], ox[2];
    bool live[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pix = base + h * 32 + lane;
      live[h] = pix < total;
      const int pc = live[h] ? pix : 0;
      ox[h] = pc % ow;
      const int t = pc / ow;
      oy[h] = t % oh;
      xi[h] = x + (size_t)(t / oh) * ih * iw * IC;
#pragma unroll
      for (int o = 0; o < OC; ++o) acc[h][o] = ws[K * OC + o];
    }
#pragma unroll
    for (int ky = 0; ky < KH; ++ky)
#pragma unroll
      for (int kx = 0; kx < KW; ++kx) {
        float xv[2][IC];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int iy = oy[h] * sh + ky - pt, ix = ox[h] * sw + kx - pl;
          const bool in = live[h] && iy >= 0 && iy < ih && ix >= 0 && ix < iw;
          const float* xp = xi[h] + ((size_t)(in ? iy : 0) * iw + (in ? ix : 0)) * IC;
#pragma unroll
          for (int ci = 0; ci < IC; ++ci) xv[h][ci] = in ? __ldg(xp + ci) : 0.0f;
        }
#pragma unroll
        for (int ci = 0; ci < IC; ++ci) {
          const float4* wp = reinterpret_cast<const float4*>(ws + ((ky * KW + kx) * IC + ci) * OC);
#pragma unroll
          for (int o = 0; o < OC / 4; ++o) {
            const float4 wv = wp[o];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              acc[h][4 * o + 0] = fmaf(xv[h][ci], wv.x, acc[h][4 * o + 0]);
              acc[h][4 * o + 1] = fmaf(xv[h][ci], wv.y, acc[h][4 * o + 1]);
              acc[h][4 * o + 2] = fmaf(xv[h][ci], wv.z, acc[h][4 * o + 2]);
              acc[h][4 * o + 3] = fmaf(xv[h][ci], wv.w, acc[h][4 * o + 3]);
            }
          }
        }
      }
    // Stage the warp's 64 x OC outputs, then write them out as whole rows of
    // 16-byte vectors (coalesced), adding the residual and the activation.
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int o = 0; o < OC; o += 4)
        *reinterpret_cast<float4*>(stage + (h * 32 + lane) * kStride + o) =
            make_float4(acc[h][o], acc[h][o + 1], acc[h][o + 2], acc[h][o + 3]);
    __syncwarp();
    const int valid = min(64, total - base) * OC / 4;  // float4s of this warp's run
    float* yb = y + (size_t)base * OC;
    const float* rb = res ? res + (size_t)base * OC : nullptr;
    with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
#pragma unroll
      for (int i = 0; i < 2 * OC / 4; ++i) {
        const int e4 = i * 32 + lane;
        if (e4 < valid) {
          const int px = (e4 * 4) / OC, ch = (e4 * 4) % OC;
          float4 v = *reinterpret_cast<const float4*>(stage + px * kStride + ch);
          if (rb) {
            const float4 r = *reinterpret_cast<const float4*>(rb + (size_t)e4 * 4);
            v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
          }
          v.x = act_c<A>(v.x); v.y = act_c<A>(v.y);
          v.z = act_c<A>(v.z); v.w = act_c<A>(v.w);
          *reinterpret_cast<float4*>(yb + (size_t)e4 * 4) = v;
        }
      }
    });
    __syncwarp();
  }
}

template <int KH, int KW, int SH, int R>
__global__ void __launch_bounds__(256, 2) dw_rows_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
    float* __restrict__ y, int n, int ih, int iw, int c, int oh, int ow, int sw, int pt, int pl,
    int act, int row_blocks) {
  const int cv = c >> 2;
  const int total = n * row_blocks * ow * cv;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int cg = idx % cv;
    int t = idx / cv;
    const int ox = t % ow;
    t /= ow;
    const int rb = t % row_blocks;
    const int img = t / row_blocks;
    const int ch = cg * 4;
    float4 wr[KH][KW];
#pragma unroll
    for (int ky = 0; ky < KH; ++ky)
#pragma unroll
      for (int kx = 0; kx < KW; ++kx)
        wr[ky][kx] = __ldg(reinterpret_cast<const float4*>(w + (ky * KW + kx) * c + ch));
    const float4 b = bias ? __ldg(reinterpret_cast<const float4*>(bias + ch))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = b;
    const int oy0 = rb * R;
    const int iy0 = oy0 * SH - pt;
    const float* xi = x + (size_t)img * ih * iw * c + ch;
    // Input rows iy0 .. iy0 + (R-1)*SH + KH-1 feed output rows oy0 .. oy0+R-1.
#pragma unroll
    for (int j = 0; j < (R - 1) * SH + KH; ++j) {
      const int iy = iy0 + j;
      if (iy < 0 || iy >= ih) continue;
      float4 row[KW];
#pragma unroll
      for (int kx = 0; kx < KW; ++kx) {
        const int ix = ox * sw + kx - pl;
        row[kx] = (ix >= 0 && ix < iw)
                      ? __ldg(reinterpret_cast<const float4*>(xi + ((size_t)iy * iw + ix) * c))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int ky = j - r * SH;
        if (ky < 0 || ky >= KH) continue;
#pragma unroll
        for (int kx = 0; kx < KW; ++kx) {
          acc[r].x = fmaf(row[kx].x, wr[ky][kx].x, acc[r].x);
          acc[r].y = fmaf(row[kx].y, wr[ky][kx].y, acc[r].y);
          acc[r].z = fmaf(row[kx].z, wr[ky][kx].z, acc[r].z);
          acc[r].w = fmaf(row[kx].w, wr[ky][kx].w, acc[r].w);
        }
      }
    }
    with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int oy = oy0 + r;
        if (oy < oh) {
          float4 v = acc[r];
          v.x = act_c<A>(v.x); v.y = act_c<A>(v.y);
          v.z = act_c<A>(v.z); v.w = act_c<A>(v.w);
          *reinterpret_cast<float4*>(y + (((size_t)img * oh + oy) * ow + ox) * c + ch) = v;
        }
      }
    });
  }
}

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int KH, int KW, int SH>
int dw_dispatch_r(cudaStream_t s, const float* x, const float* w, const float* b, float* y,
                  const spx_dw_params* p) {
  constexpr int R = SH == 1 ? 4 : 2;
  const int row_blocks = (p->oh + R - 1) / R;
  const int64_t total = (int64_t)p->n * row_blocks * p->ow * (p->c / 4);
  dw_rows_kernel<KH, KW, SH, R><<<grid_for(total, 256, 16), 256, 0, s>>>(
      x, w, b, y, p->n, p->ih, p->iw, p->c, p->oh, p->ow, p->stride_w, p->pad_top, p->pad_left,
      p->activation, row_blocks);
  return SPX_OK;
}

}  // namespace

// Returns SPX_OK after launching, or -1 when the shape is not covered (the
// caller then uses the generic kernel).
int try_dw_rows(cudaStream_t s, int64_t* cnt, const float* x, const float* w, const float* b,
                float* y, const spx_dw_params* p) {
  const bool dil1 = (p->dilation_h <= 1) && (p->dilation_w <= 1);
  if (!dil1 || p->c % 4 || !al16(x) || !al16(w) || !al16(y) || (b && !al16(b))) return -1;
  if ((int64_t)p->n * p->ih * p->iw * p->c >= INT32_MAX ||
      (int64_t)p->n * p->oh * p->ow * p->c >= INT32_MAX)
    return -1;
  int rc = -1;
  if (p->kh == 3 && p->kw == 3 && p->stride_h == 1) rc = dw_dispatch_r<3, 3, 1>(s, x, w, b, y, p);
  else if (p->kh == 3 && p->kw == 3 && p->stride_h == 2) rc = dw_dispatch_r<3, 3, 2>(s, x, w, b, y, p);
  else if (p->kh == 5 && p->kw == 5 && p->stride_h == 1) rc = dw_dispatch_r<5, 5, 1>(s, x, w, b, y, p);
  else if (p->kh == 5 && p->kw == 5 && p->stride_h == 2) rc = dw_dispatch_r<5, 5, 2>(s, x, w, b, y, p);
  if (rc < 0) return -1;
  return after_launch(cnt, "depthwise_rows");
}

int try_conv_smallk(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                    const float* bias, const float* res, float* y, const spx_conv_params* p) {
  const int K = p->kh * p->kw * p->ic;
  if (K > 64 || (p->oc != 8 && p->oc != 16 && p->oc != 32 && p->oc != 64)) return -1;
  if (!al16(y) || (res && !al16(res))) return -1;
  if ((int64_t)p->n * p->oh * p->ow >= INT32_MAX / 64 ||
      (int64_t)p->n * p->ih * p->iw * p->ic >= INT32_MAX)
    return -1;
  const int total = p->n * p->oh * p->ow;
  // weights + bias, then 4 warps x 32 rows x (oc + 4) floats of output staging
  const size_t smem = ((size_t)K * p->oc + p->oc + 4 * 32 * (p->oc + 4)) * sizeof(float);
  const int grid = grid_for(total, 128, 16);
  const int dh = p->dilation_h > 0 ? p->dilation_h : 1, dw = p->dilation_w > 0 ? p->dilation_w : 1;
#define SPX_SMALLK(...)                                                                        \
  if (smem > 48 * 1024)                                                                        \
    cudaFuncSetAttribute(conv_smallk_kernel<__VA_ARGS__>,                                      \
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);              \
  conv_smallk_kernel<__VA_ARGS__><<<grid, 128, smem, s>>>(x, w, bias, res, y, p->n, p->ih, p->iw,      \
                                                  p->ic, p->oh, p->ow, p->kh, p->kw,           \
                                                  p->stride_h, p->stride_w, p->pad_top,        \
                                                  p->pad_left, dh, dw, p->activation,          \
                                                  p->weight_layout)
  const bool k333 = p->kh == 3 && p->kw == 3 && p->ic == 3;
  if (k333 && p->oc == 32 && dh == 1 && dw == 1) {
    const size_t smem2 = ((size_t)27 * 32 + 32 + 4 * 64 * (32 + 4)) * sizeof(float);
    cudaFuncSetAttribute(conv_stem2_kernel<32, 3, 3, 3>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
    conv_stem2_kernel<32, 3, 3, 3><<<grid_for(total, 256, 16), 128, smem2, s>>>(
        x, w, bias, res, y, p->n, p->ih, p->iw, p->oh, p->ow, p->stride_h, p->stride_w,
        p->pad_top, p->pad_left, p->activation, p->weight_layout);
    return after_launch(cnt, "conv_stem2");
  }
  switch (p->oc) {
    case 8: SPX_SMALLK(8); break;
    case 16: SPX_SMALLK(16); break;
    case 32:
      if (k333) { SPX_SMALLK(32, 3, 3, 3); } else { SPX_SMALLK(32); }
      break;
    default: SPX_SMALLK(64); break;
  }
#undef SPX_SMALLK
  return after_launch(cnt, "conv_smallk");
}

}  // namespace spx
