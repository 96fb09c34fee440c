// Spatial, bandwidth-bound kernels: depthwise convolution, window pooling,
// global average pooling and rank-4 reductions.
//
// NHWC kernels (the device-resident path) vectorise along channels (16-byte
// loads when C % 4 == 0) so a warp reads contiguous 512-byte runs, fuse bias
// and activation, and are grid-stride loops sized in multiples of the SM
// count.  The *_nchw kernels restate the reference shaders one output per
// thread for the drop-in boundary, where the caller's layout is NCHW.
#include "spx_internal.cuh"

namespace spx {

namespace {

struct DwArgs {
  int n, ih, iw, c, oh, ow, kh, kw, sh, sw, pt, pl, dh, dw, act;
};

// depthwise_conv2d.comp:27-49 in NHWC: accumulator starts at the bias, then
// taps in (ky, kx) order, out-of-range taps skipped (implicit zero pad).
template <int VEC>
__global__ void dw_nhwc_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               const float* __restrict__ bias, float* __restrict__ y, DwArgs p,
                               int64_t total) {
  const int cv = p.c / VEC;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int cg = (int)(idx % cv);
    int64_t t = idx / cv;
    int ox = (int)(t % p.ow);
    t /= p.ow;
    int oy = (int)(t % p.oh);
    int64_t n = t / p.oh;
    int c = cg * VEC;
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = bias ? __ldg(bias + c + v) : 0.0f;
    const float* xn = x + n * p.ih * p.iw * (int64_t)p.c + c;
    for (int ky = 0; ky < p.kh; ++ky) {
      int iy = oy * p.sh + ky * p.dh - p.pt;
      if (iy < 0 || iy >= p.ih) continue;
      for (int kx = 0; kx < p.kw; ++kx) {
        int ix = ox * p.sw + kx * p.dw - p.pl;
        if (ix < 0 || ix >= p.iw) continue;
        const float* xp = xn + ((int64_t)iy * p.iw + ix) * p.c;
        const float* wp = w + (ky * p.kw + kx) * p.c + c;
        if (VEC == 4) {
          float4 xv = __ldg(reinterpret_cast<const float4*>(xp));
          float4 wv = __ldg(reinterpret_cast<const float4*>(wp));
          acc[0] = fmaf(xv.x, wv.x, acc[0]);
          acc[1 % VEC] = fmaf(xv.y, wv.y, acc[1 % VEC]);
          acc[2 % VEC] = fmaf(xv.z, wv.z, acc[2 % VEC]);
          acc[3 % VEC] = fmaf(xv.w, wv.w, acc[3 % VEC]);
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[v] = fmaf(__ldg(xp + v), __ldg(wp + v), acc[v]);
        }
      }
    }
    float* yp = y + idx * VEC;
    if (VEC == 4) {
      *reinterpret_cast<float4*>(yp) =
          make_float4(apply_act(p.act, acc[0]), apply_act(p.act, acc[1 % VEC]),
                      apply_act(p.act, acc[2 % VEC]), apply_act(p.act, acc[3 % VEC]));
    } else {
#pragma unroll
      for (int v = 0; v < VEC; ++v) yp[v] = apply_act(p.act, acc[v]);
    }
  }
}

struct PoolArgs {
  int n, ih, iw, c, oh, ow, kh, kw, sh, sw, pt, pl, kind;
};

// hlo_reduce_window_rank4.comp:25-49 (NHWC): max starts at -FLT_MAX, sum at 0;
// out-of-range taps are skipped.  kind 2 (average) divides by the number of
// in-range taps (TFLite AVERAGE_POOL_2D).
template <int VEC>
__global__ void pool_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, PoolArgs p,
                                 int64_t total) {
  const int cv = p.c / VEC;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int cg = (int)(idx % cv);
    int64_t t = idx / cv;
    int ox = (int)(t % p.ow);
    t /= p.ow;
    int oy = (int)(t % p.oh);
    int64_t n = t / p.oh;
    int c = cg * VEC;
    float acc[VEC];
    const float init = p.kind == SPX_POOL_MAX ? -3.4028234663852886e+38f : 0.0f;
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = init;
    int count = 0;
    const float* xn = x + n * p.ih * p.iw * (int64_t)p.c + c;
    for (int ky = 0; ky < p.kh; ++ky) {
      int iy = oy * p.sh + ky - p.pt;
      if (iy < 0 || iy >= p.ih) continue;
      for (int kx = 0; kx < p.kw; ++kx) {
        int ix = ox * p.sw + kx - p.pl;
        if (ix < 0 || ix >= p.iw) continue;
        ++count;
        const float* xp = xn + ((int64_t)iy * p.iw + ix) * p.c;
        float xv[VEC];
        if (VEC == 4) {
          float4 q = __ldg(reinterpret_cast<const float4*>(xp));
          xv[0] = q.x; xv[1 % VEC] = q.y; xv[2 % VEC] = q.z; xv[3 % VEC] = q.w;
        } else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) xv[v] = __ldg(xp + v);
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v)
          acc[v] = p.kind == SPX_POOL_MAX ? fmaxf(acc[v], xv[v]) : acc[v] + xv[v];
      }
    }
    if (p.kind == SPX_POOL_AVG) {
      float d = (float)(count > 0 ? count : 1);
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[v] = acc[v] / d;
    }
    float* yp = y + idx * VEC;
#pragma unroll
    for (int v = 0; v < VEC; ++v) yp[v] = acc[v];
  }
}

// Global average pool NHWC: y[n][c] = (sum over hw of x[n][hw][c]) / hw.
template <int VEC>
__global__ void gap_nhwc_kernel(const float* __restrict__ x, float* __restrict__ y, int n, int hw,
                                int c) {
  const int cv = c / VEC;
  int64_t total = (int64_t)n * cv;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const float inv_div = (float)hw;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int64_t img = idx / cv;
    int ch = (int)(idx % cv) * VEC;
    const float* xp = x + img * hw * (int64_t)c + ch;
    float acc[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[v] = 0.0f;
    // Unrolled so several independent loads are in flight per thread; the
    // additions stay in pixel order.
#pragma unroll 8
    for (int i = 0; i < hw; ++i) {
      if (VEC == 4) {
        float4 q = __ldg(reinterpret_cast<const float4*>(xp + (int64_t)i * c));
        acc[0] += q.x; acc[1 % VEC] += q.y; acc[2 % VEC] += q.z; acc[3 % VEC] += q.w;
      } else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[v] += __ldg(xp + (int64_t)i * c + v);
      }
    }
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[img * c + ch + v] = acc[v] / inv_div;
  }
}

// ---- reference-layout (NCHW) restatements --------------------------------

// depthwise_conv2d.comp:27-49, push layout kernels.rs:155-177; weights
// [c][kh][kw] followed by c biases (scheduler.rs:1364-1400).
__global__ void dw_nchw_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ y, DwArgs p, int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int ow_ = (int)(idx % p.ow);
    int oh_ = (int)((idx / p.ow) % p.oh);
    int c = (int)((idx / ((int64_t)p.ow * p.oh)) % p.c);
    int64_t n = idx / ((int64_t)p.ow * p.oh * p.c);
    float acc = w[(int64_t)p.c * p.kh * p.kw + c];
    for (int ky = 0; ky < p.kh; ++ky) {
      int iy = oh_ * p.sh + ky * p.dh - p.pt;
      if (iy < 0 || iy >= p.ih) continue;
      for (int kx = 0; kx < p.kw; ++kx) {
        int ix = ow_ * p.sw + kx * p.dw - p.pl;
        if (ix < 0 || ix >= p.iw) continue;
        acc = fmaf(x[((n * p.c + c) * p.ih + iy) * p.iw + ix], w[(c * p.kh + ky) * p.kw + kx], acc);
      }
    }
    y[idx] = acc;
  }
}

// max_pool2d.comp:25-44 (NCHW), push layout kernels.rs:184-192.
__global__ void maxpool_nchw_kernel(const float* __restrict__ x, float* __restrict__ y,
                                    PoolArgs p, int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int ow_ = (int)(idx % p.ow);
    int oh_ = (int)((idx / p.ow) % p.oh);
    int c = (int)((idx / ((int64_t)p.ow * p.oh)) % p.c);
    int64_t n = idx / ((int64_t)p.ow * p.oh * p.c);
    float best = -3.402823466e+38f;
    for (int ky = 0; ky < p.kh; ++ky) {
      int iy = oh_ * p.sh + ky - p.pt;
      if (iy < 0 || iy >= p.ih) continue;
      for (int kx = 0; kx < p.kw; ++kx) {
        int ix = ow_ * p.sw + kx - p.pl;
        if (ix < 0 || ix >= p.iw) continue;
        best = fmaxf(best, x[((n * p.c + c) * p.ih + iy) * p.iw + ix]);
      }
    }
    y[idx] = best;
  }
}

// global_avg_pool_sum.comp:15-28: one thread per (n, c) walks h*w in order.
__global__ void gap_sum_nchw_kernel(const float* __restrict__ x, float* __restrict__ y, int n,
                                    int c, int h, int w) {
  int64_t total = (int64_t)n * c;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const float* xp = x + idx * h * (int64_t)w;
    float acc = 0.0f;
    for (int i = 0; i < h * w; ++i) acc += xp[i];
    y[idx] = acc;
  }
}

// global_avg_pool_finalize.comp:15-19.
__global__ void gap_finalize_kernel(const float* __restrict__ x, float* __restrict__ y, int n,
                                    int c, int h, int w) {
  int64_t total = (int64_t)n * c;
  float d = (float)(h * w);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride)
    y[idx] = x[idx] / d;
}

// resize_bilinear.comp (NCHW): source coordinate by align_corners /
// half_pixel_centers, clamped, then two horizontal lerps and a vertical one
// (GLSL mix(a, b, t) = a * (1 - t) + b * t).
__device__ __forceinline__ float glsl_mix(float a, float b, float t) {
  return a * (1.0f - t) + b * t;
}
__device__ __forceinline__ float src_coord(int o, int in_size, int out_size, int ac, int hp) {
  if (ac != 0 && out_size > 1) return (float)o * (float)(in_size - 1) / (float)(out_size - 1);
  if (hp != 0) return ((float)o + 0.5f) * (float)in_size / (float)out_size - 0.5f;
  return (float)o * (float)in_size / (float)out_size;
}
__global__ void resize_bilinear_kernel(const float* __restrict__ x, float* __restrict__ y, int n,
                                       int c, int ih, int iw, int oh, int ow, int ac, int hp,
                                       int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int ox = (int)(idx % ow);
    int oy = (int)((idx / ow) % oh);
    int64_t nc = idx / ((int64_t)ow * oh);
    float in_y = fminf(fmaxf(src_coord(oy, ih, oh, ac, hp), 0.0f), (float)(ih - 1));
    float in_x = fminf(fmaxf(src_coord(ox, iw, ow, ac, hp), 0.0f), (float)(iw - 1));
    int y0 = (int)floorf(in_y), x0 = (int)floorf(in_x);
    int y1 = min(y0 + 1, ih - 1), x1 = min(x0 + 1, iw - 1);
    float yl = in_y - (float)y0, xl = in_x - (float)x0;
    const float* base = x + nc * ih * (int64_t)iw;
    float top = glsl_mix(base[y0 * iw + x0], base[y0 * iw + x1], xl);
    float bot = glsl_mix(base[y1 * iw + x0], base[y1 * iw + x1], xl);
    y[idx] = glsl_mix(top, bot, yl);
  }
}

// hlo_reduce_rank4.comp:44-79.  Output coordinates are decoded from the
// non-reduced axes (innermost first); the reduced box is walked in row-major
// order.  Small boxes: one thread per output, same order as the reference.
// Large boxes: one warp per output, lanes stride the flattened box, then a
// shuffle tree (max is order-independent; sums differ only by rounding).
struct RedArgs {
  int rank, d[4], od[4], r[4], kind;
  int64_t total;
  int64_t box;  // number of reduced elements per output
  int bd[4];    // box extents (d[a] if reduced else 1)
};

__device__ __forceinline__ void red_out_coord(const RedArgs& p, int64_t idx, int oc[4]) {
  oc[0] = oc[1] = oc[2] = oc[3] = 0;
  int64_t tmp = idx;
  for (int axis = p.rank - 1; axis >= 0; --axis) {
    if (p.r[axis] == 0) {
      int dim = max(p.od[axis], 1);
      oc[axis] = (int)(tmp % dim);
      tmp /= dim;
    }
  }
}

__global__ void reduce_rank4_thread(const float* __restrict__ x, float* __restrict__ y, RedArgs p) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < p.total; idx += stride) {
    int oc[4];
    red_out_coord(p, idx, oc);
    float acc = p.kind == 1 ? -3.4028234663852886e+38f : 0.0f;
    for (int a0 = 0; a0 < p.bd[0]; ++a0)
      for (int a1 = 0; a1 < p.bd[1]; ++a1)
        for (int a2 = 0; a2 < p.bd[2]; ++a2)
          for (int a3 = 0; a3 < p.bd[3]; ++a3) {
            int c0 = p.r[0] ? a0 : oc[0], c1 = p.r[1] ? a1 : oc[1];
            int c2 = p.r[2] ? a2 : oc[2], c3 = p.r[3] ? a3 : oc[3];
            float v = x[(((int64_t)c0 * p.d[1] + c1) * p.d[2] + c2) * p.d[3] + c3];
            acc = p.kind == 1 ? fmaxf(acc, v) : acc + v;
          }
    y[idx] = acc;
  }
}

__global__ void reduce_rank4_warp(const float* __restrict__ x, float* __restrict__ y, RedArgs p) {
  const int lane = threadIdx.x & 31;
  int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t idx = warp; idx < p.total; idx += nwarps) {
    int oc[4];
    red_out_coord(p, idx, oc);
    float acc = p.kind == 1 ? -3.4028234663852886e+38f : 0.0f;
    for (int64_t e = lane; e < p.box; e += 32) {
      int64_t t = e;
      int a3 = (int)(t % p.bd[3]); t /= p.bd[3];
      int a2 = (int)(t % p.bd[2]); t /= p.bd[2];
      int a1 = (int)(t % p.bd[1]); t /= p.bd[1];
      int a0 = (int)t;
      int c0 = p.r[0] ? a0 : oc[0], c1 = p.r[1] ? a1 : oc[1];
      int c2 = p.r[2] ? a2 : oc[2], c3 = p.r[3] ? a3 : oc[3];
      float v = x[(((int64_t)c0 * p.d[1] + c1) * p.d[2] + c2) * p.d[3] + c3];
      acc = p.kind == 1 ? fmaxf(acc, v) : acc + v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float other = __shfl_xor_sync(0xffffffffu, acc, o);
      acc = p.kind == 1 ? fmaxf(acc, other) : acc + other;
    }
    if (lane == 0) y[idx] = acc;
  }
}

bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

int launch_dw_nhwc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* bias, float* y, const spx_dw_params* q) {
  DwArgs p = {q->n, q->ih, q->iw, q->c, q->oh, q->ow, q->kh, q->kw, q->stride_h, q->stride_w,
              q->pad_top, q->pad_left, q->dilation_h > 0 ? q->dilation_h : 1,
              q->dilation_w > 0 ? q->dilation_w : 1, q->activation};
  if (p.n <= 0 || p.c <= 0 || p.oh <= 0 || p.ow <= 0 || p.kh <= 0 || p.kw <= 0 || p.sh <= 0 ||
      p.sw <= 0 || p.ih <= 0 || p.iw <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "depthwise: bad shape");
  {
    int rc = g_dw_path != 1 ? try_dw_tma(s, cnt, x, w, bias, y, q) : -1;
    if (rc != -1) return rc;
    rc = try_dw_rows(s, cnt, x, w, bias, y, q);
    if (rc != -1) return rc;
  }
  int64_t pix = (int64_t)p.n * p.oh * p.ow;
  if (p.c % 4 == 0 && al16(x) && al16(w) && al16(y)) {
    int64_t total = pix * (p.c / 4);
    dw_nhwc_kernel<4><<<grid_for(total, 256), 256, 0, s>>>(x, w, bias, y, p, total);
  } else {
    int64_t total = pix * p.c;
    dw_nhwc_kernel<1><<<grid_for(total, 256), 256, 0, s>>>(x, w, bias, y, p, total);
  }
  return after_launch(cnt, "depthwise_nhwc");
}

int launch_pool_nhwc(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                     const spx_pool_params* q) {
  PoolArgs p = {q->n, q->ih, q->iw, q->c, q->oh, q->ow, q->kh, q->kw, q->stride_h, q->stride_w,
                q->pad_top, q->pad_left, q->kind};
  if (p.n <= 0 || p.c <= 0 || p.oh <= 0 || p.ow <= 0 || p.kh <= 0 || p.kw <= 0 || p.sh <= 0 ||
      p.sw <= 0 || (p.kind != SPX_POOL_MAX && p.kind != SPX_POOL_SUM && p.kind != SPX_POOL_AVG))
    return fail(SPX_ERR_INVALID_ARGUMENT, "pool: bad parameters");
  int64_t pix = (int64_t)p.n * p.oh * p.ow;
  if (p.c % 4 == 0 && al16(x) && al16(y)) {
    int64_t total = pix * (p.c / 4);
    pool_nhwc_kernel<4><<<grid_for(total, 256), 256, 0, s>>>(x, y, p, total);
  } else {
    int64_t total = pix * p.c;
    pool_nhwc_kernel<1><<<grid_for(total, 256), 256, 0, s>>>(x, y, p, total);
  }
  return after_launch(cnt, "pool_nhwc");
}

int launch_gap_nhwc(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n, int hw,
                    int c) {
  if (n <= 0 || hw <= 0 || c <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "gap: bad shape");
  if (c % 4 == 0 && al16(x) && al16(y))
    gap_nhwc_kernel<4><<<grid_for((int64_t)n * c / 4, 128), 128, 0, s>>>(x, y, n, hw, c);
  else
    gap_nhwc_kernel<1><<<grid_for((int64_t)n * c, 128), 128, 0, s>>>(x, y, n, hw, c);
  return after_launch(cnt, "gap_nhwc");
}

int launch_compat_dw_nchw(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                          float* y, const int32_t* q) {
  // n,c,ih,iw,oh,ow,kh,kw,stride_h,stride_w,same,pad_top,pad_left,dil_h,dil_w,total
  DwArgs p = {q[0], q[2], q[3], q[1], q[4], q[5], q[6], q[7], q[8], q[9], q[11], q[12],
              q[13], q[14], 0};
  int64_t total = (int64_t)p.n * p.c * p.oh * p.ow;
  if (total != q[15] || total <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "depthwise_conv2d: total %d != n*c*oh*ow", q[15]);
  dw_nchw_kernel<<<grid_for(total, 64), 64, 0, s>>>(x, w, y, p, total);
  return after_launch(cnt, "depthwise_conv2d_nchw");
}

int launch_compat_maxpool_nchw(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                               const int32_t* q) {
  // n,c,ih,iw,oh,ow,kh,kw,stride_h,stride_w,same,pad_top,pad_left,total
  PoolArgs p = {q[0], q[2], q[3], q[1], q[4], q[5], q[6], q[7], q[8], q[9], q[11], q[12],
                SPX_POOL_MAX};
  int64_t total = (int64_t)p.n * p.c * p.oh * p.ow;
  if (total != q[13] || total <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "max_pool2d: total %d != n*c*oh*ow", q[13]);
  maxpool_nchw_kernel<<<grid_for(total, 64), 64, 0, s>>>(x, y, p, total);
  return after_launch(cnt, "max_pool2d_nchw");
}

int launch_compat_gap_sum_nchw(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n,
                               int c, int h, int w) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "gap_sum: shape");
  gap_sum_nchw_kernel<<<grid_for((int64_t)n * c, 64), 64, 0, s>>>(x, y, n, c, h, w);
  return after_launch(cnt, "global_avg_pool_sum");
}

int launch_compat_gap_finalize(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n,
                               int c, int h, int w) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "gap_fin: shape");
  gap_finalize_kernel<<<grid_for((int64_t)n * c, 64), 64, 0, s>>>(x, y, n, c, h, w);
  return after_launch(cnt, "global_avg_pool_finalize");
}

int launch_compat_resize_bilinear(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                                  const int32_t* q) {
  // n,c,ih,iw,oh,ow,align_corners,half_pixel_centers,total
  int64_t total = (int64_t)q[0] * q[1] * q[4] * q[5];
  if (total != q[8] || total <= 0 || q[2] <= 0 || q[3] <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "resize_bilinear: bad push constants");
  resize_bilinear_kernel<<<grid_for(total, 64), 64, 0, s>>>(x, y, q[0], q[1], q[2], q[3], q[4],
                                                            q[5], q[6], q[7], total);
  return after_launch(cnt, "resize_bilinear");
}

int launch_reduce_rank4(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                        const int32_t* q) {
  RedArgs p;
  p.rank = q[0];
  if (p.rank < 1 || p.rank > 4) return fail(SPX_ERR_INVALID_ARGUMENT, "reduce: rank %d", p.rank);
  p.box = 1;
  for (int i = 0; i < 4; ++i) {
    p.d[i] = q[1 + i];
    p.od[i] = q[5 + i];
    p.r[i] = q[9 + i];
    if (p.d[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "reduce: bad dim");
    p.bd[i] = p.r[i] ? p.d[i] : 1;
    p.box *= p.bd[i];
  }
  p.kind = q[13];
  p.total = q[14];
  int64_t expect = 1;
  for (int i = 0; i < p.rank; ++i)
    if (!p.r[i]) expect *= p.od[i] > 0 ? p.od[i] : 1;
  if (p.total != expect || p.total <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "reduce: total %lld != %lld", (long long)p.total,
                (long long)expect);
  if (p.box >= 64)
    reduce_rank4_warp<<<grid_for(p.total * 32, 256), 256, 0, s>>>(x, y, p);
  else
    reduce_rank4_thread<<<grid_for(p.total, 64), 64, 0, s>>>(x, y, p);
  return after_launch(cnt, "reduce_rank4");
}

}  // namespace spx
