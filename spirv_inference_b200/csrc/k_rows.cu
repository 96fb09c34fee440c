// Row-wise kernels: softmax (softmax10.comp / softmax1000.comp generalised
// to batched rows, plus the scaled + causal form used by attention),
// LayerNorm, RMSNorm, rotary embedding and argmax.
//
// One warp per row for rows up to a few thousand columns: a row is read once
// for the max, once for the sum and once for the output; the second and
// third passes hit L1/L2.  Bandwidth-bound; grid sized to the SM count.
#include "spx_internal.cuh"

namespace spx {
namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// softmax1000.comp:10-22 per row: m = max_j x_j; s = sum_j exp(x_j - m);
// y_i = exp(x_i - m) / s.  With scale / causal masking for attention.
__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y, int rows,
                                    int cols, float scale, int causal, int q_len, int q_offset) {
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x >> 5;
  for (int r = blockIdx.x * warps_per_block + (threadIdx.x >> 5); r < rows;
       r += gridDim.x * warps_per_block) {
    const float* xr = x + (int64_t)r * cols;
    float* yr = y + (int64_t)r * cols;
    int limit = cols;
    if (causal) {
      int q = q_offset + (q_len > 0 ? r % q_len : 0);
      limit = min(cols, q + 1);
    }
    float m = -3.4028234663852886e+38f;
    for (int j = lane; j < limit; j += 32) m = fmaxf(m, xr[j] * scale);
    m = warp_max(m);
    float s = 0.0f;
    for (int j = lane; j < limit; j += 32) s += expf(xr[j] * scale - m);
    s = warp_sum(s);
    for (int j = lane; j < cols; j += 32) yr[j] = j < limit ? expf(xr[j] * scale - m) / s : 0.0f;
  }
}

// Row LayerNorm (TF semantics): mean, biased variance, (x-mean)/sqrt(var+eps).
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ res,
                                 float* __restrict__ x_out, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, float* __restrict__ y, int rows,
                                 int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
    const float* xr = x + (int64_t)r * cols;
    const float* rr = res ? res + (int64_t)r * cols : nullptr;
    float s = 0.0f;
    for (int j = lane; j < cols; j += 32) {
      float v = xr[j] + (rr ? rr[j] : 0.0f);
      if (x_out) x_out[(int64_t)r * cols + j] = v;
      s += v;
    }
    float mean = warp_sum(s) / (float)cols;
    float q = 0.0f;
    for (int j = lane; j < cols; j += 32) {
      float d = xr[j] + (rr ? rr[j] : 0.0f) - mean;
      q += d * d;
    }
    float var = warp_sum(q) / (float)cols;
    float inv = 1.0f / sqrtf(var + eps);
    for (int j = lane; j < cols; j += 32) {
      float v = xr[j] + (rr ? rr[j] : 0.0f);
      y[(int64_t)r * cols + j] = (v - mean) * inv * gamma[j] + beta[j];
    }
  }
}

// RMSNorm (Llama): x / sqrt(mean(x^2) + eps) * gamma (gamma optional).
// One 256-thread block per row; 16-byte accesses when the row allows.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x,
                                                      const float* __restrict__ gamma,
                                                      float* __restrict__ y, int rows, int cols,
                                                      float eps) {
  __shared__ float part[8];
  const bool vec = (cols & 3) == 0 && (((uintptr_t)x | (uintptr_t)y |
                                        (gamma ? (uintptr_t)gamma : 0)) & 15) == 0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + (int64_t)r * cols;
    float* yr = y + (int64_t)r * cols;
    float q = 0.0f;
    if (vec) {
      for (int j = threadIdx.x; j < cols / 4; j += blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(xr)[j];
        q += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
    } else {
      for (int j = threadIdx.x; j < cols; j += blockDim.x) q += xr[j] * xr[j];
    }
    q = warp_sum(q);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = q;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += part[w];
    const float inv = 1.0f / sqrtf(tot / (float)cols + eps);
    if (vec) {
      for (int j = threadIdx.x; j < cols / 4; j += blockDim.x) {
        float4 v = reinterpret_cast<const float4*>(xr)[j];
        v.x *= inv; v.y *= inv; v.z *= inv; v.w *= inv;
        if (gamma) {
          const float4 gv = reinterpret_cast<const float4*>(gamma)[j];
          v.x = gv.x * v.x; v.y = gv.y * v.y; v.z = gv.z * v.z; v.w = gv.w * v.w;
        }
        reinterpret_cast<float4*>(yr)[j] = v;
      }
    } else {
      for (int j = threadIdx.x; j < cols; j += blockDim.x)
        yr[j] = gamma ? gamma[j] * (xr[j] * inv) : xr[j] * inv;
    }
    __syncthreads();
  }
}

// Rotate-half RoPE on [tokens][heads][head_dim]:
//   inv_freq_i = 1 / theta^(2i/d), angle = pos * inv_freq_i,
//   out_i = x_i cos - x_{i+d/2} sin, out_{i+d/2} = x_{i+d/2} cos + x_i sin.
__global__ void rope_kernel(float* __restrict__ x, const int32_t* __restrict__ pos, int tokens,
                            int heads, int head_dim, float theta) {
  const int half = head_dim / 2;
  int64_t total = (int64_t)tokens * heads * half;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int i = (int)(idx % half);
    int64_t th = idx / half;
    int t = (int)(th / heads);
    float inv_freq = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    float ang = (float)pos[t] * inv_freq;
    float c = cosf(ang), s = sinf(ang);
    float* base = x + th * head_dim;
    float a = base[i], b = base[i + half];
    base[i] = a * c - b * s;
    base[i + half] = b * c + a * s;
  }
}

// Row argmax, first maximum wins (numpy semantics).
__global__ void argmax_rows_kernel(const float* __restrict__ x, int32_t* __restrict__ idx,
                                   float* __restrict__ val, int rows, int cols) {
  __shared__ float sv[32];
  __shared__ int si[32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + (int64_t)r * cols;
    float best = -3.4028234663852886e+38f;
    int bi = 0x7fffffff;
    if ((cols & 3) == 0 && ((uintptr_t)x & 15) == 0) {
      // 16-byte loads, four in flight per thread; a thread's columns rise
      // within each vector, so strict > keeps the first maximum.
      const float4* xv = reinterpret_cast<const float4*>(xr);
      const int nv = cols >> 2;
#pragma unroll 4
      for (int j = threadIdx.x; j < nv; j += blockDim.x) {
        const float4 v = xv[j];
        if (v.x > best || (v.x == best && 4 * j < bi)) { best = v.x; bi = 4 * j; }
        if (v.y > best) { best = v.y; bi = 4 * j + 1; }
        if (v.z > best) { best = v.z; bi = 4 * j + 2; }
        if (v.w > best) { best = v.w; bi = 4 * j + 3; }
      }
    } else {
      for (int j = threadIdx.x; j < cols; j += blockDim.x) {
        float v = xr[j];
        if (v > best || (v == best && j < bi)) { best = v; bi = j; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[w] = best; si[w] = bi; }
    __syncthreads();
    if (w == 0) {
      int nw = blockDim.x >> 5;
      best = lane < nw ? sv[lane] : -3.4028234663852886e+38f;
      bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
      }
      if (lane == 0) {
        idx[r] = bi;
        if (val) val[r] = best;
      }
    }
    __syncthreads();
  }
}

}  // namespace

int launch_softmax_rows(cudaStream_t s, int64_t* cnt, const float* x, float* y, int rows,
                        int cols, float scale, int causal, int q_len, int q_offset) {
  if (rows <= 0 || cols <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "softmax: bad shape");
  softmax_rows_kernel<<<grid_for((int64_t)rows * 32, 256), 256, 0, s>>>(x, y, rows, cols, scale,
                                                                     causal, q_len, q_offset);
  return after_launch(cnt, "softmax_rows");
}

int launch_layernorm(cudaStream_t s, int64_t* cnt, const float* x, const float* res,
                     float* x_out, const float* gamma, const float* beta, float* y, int rows,
                     int cols, float eps) {
  if (rows <= 0 || cols <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "layernorm: bad shape");
  layernorm_kernel<<<grid_for((int64_t)rows * 32, 256), 256, 0, s>>>(x, res, x_out, gamma, beta,
                                                                  y, rows, cols, eps);
  return after_launch(cnt, "layernorm");
}

int launch_rmsnorm(cudaStream_t s, int64_t* cnt, const float* x, const float* gamma, float* y,
                   int rows, int cols, float eps) {
  if (rows <= 0 || cols <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "rmsnorm: bad shape");
  rmsnorm_kernel<<<grid_for(rows, 1, 8), 256, 0, s>>>(x, gamma, y, rows, cols, eps);
  return after_launch(cnt, "rmsnorm");
}

int launch_rope(cudaStream_t s, int64_t* cnt, float* x, const int32_t* pos, int tokens,
                int heads, int head_dim, float theta) {
  if (tokens <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 2)
    return fail(SPX_ERR_INVALID_ARGUMENT, "rope: bad shape");
  rope_kernel<<<grid_for((int64_t)tokens * heads * head_dim / 2, 256), 256, 0, s>>>(
      x, pos, tokens, heads, head_dim, theta);
  return after_launch(cnt, "rope");
}

int launch_argmax_rows(cudaStream_t s, int64_t* cnt, const float* x, int32_t* idx, float* val,
                       int rows, int cols) {
  if (rows <= 0 || cols <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "argmax: bad shape");
  argmax_rows_kernel<<<grid_for(rows, 1, 8), 1024, 0, s>>>(x, idx, val, rows, cols);
  return after_launch(cnt, "argmax_rows");
}

}  // namespace spx
