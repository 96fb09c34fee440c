// Elementwise and data-movement kernels: the reference's unary / binary
// shader set (kernels/{abs,exp,log,neg,sqrt,rsqrt,sigmoid,tanh,relu,relu6,
// leaky_relu,sine,reshape,add,sub,mul,div,pow,min,max}/glsl/*.comp), pad.comp,
// transpose.comp, concat.comp, l2norm.comp, plus the embedding gather and the
// SwiGLU product used by the decoder graphs.
//
// All of these are HBM-bound: one read (two for binary) and one write per
// element.  Kernels are grid-stride loops sized to a multiple of the SM count
// and use 16-byte vector accesses whenever the pointers and length allow it.
#include "spx_internal.cuh"

namespace spx {
namespace {

// Scalar unary op.  Formulas follow the GLSL bodies exactly where they are
// not plain library calls: relu is `x > 0 ? x : 0` (relu.comp; -0.0 maps to
// +0.0 as tests/parity_test/generate_fixtures.py:21-25 requires), relu6 clamps
// to [0, 6] (relu6.comp:15), leaky_relu is max(alpha*x, x) (leaky_relu.comp),
// tanh clamps to [-20, 20] and uses (e^x - e^-x)/(e^x + e^-x) (tanh.comp),
// sigmoid is 1/(1+e^-x) (sigmoid.comp), rsqrt is 1/sqrt(x) (inversesqrt).
__device__ __forceinline__ float unary_op(int op, float x, float alpha) {
  switch (op) {
    case SPX_UN_ABS: return fabsf(x);
    case SPX_UN_EXP: return expf(x);
    case SPX_UN_LOG: return logf(x);
    case SPX_UN_NEG: return -x;
    case SPX_UN_SQRT: return sqrtf(x);
    case SPX_UN_RSQRT: return 1.0f / sqrtf(x);
    case SPX_UN_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case SPX_UN_TANH: {
      float c = fminf(fmaxf(x, -20.0f), 20.0f);
      float ex = expf(c), enx = expf(-c);
      return (ex - enx) / (ex + enx);
    }
    case SPX_UN_RELU: return x > 0.0f ? x : 0.0f;
    case SPX_UN_RELU6: return fminf(x > 0.0f ? x : 0.0f, 6.0f);
    case SPX_UN_LEAKY_RELU: return fmaxf(alpha * x, x);
    case SPX_UN_SIN: return sinf(x);
    case SPX_UN_GELU_ERF: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
    case SPX_UN_SILU: return x / (1.0f + expf(-x));
    default: return x;  // SPX_UN_COPY
  }
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ y,
                             int64_t n, float alpha) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = unary_op(op, x[i], alpha);
}

__global__ void unary_kernel_v4(int op, const float4* __restrict__ x, float4* __restrict__ y,
                                int64_t n4, float alpha) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = x[i];
    v.x = unary_op(op, v.x, alpha);
    v.y = unary_op(op, v.y, alpha);
    v.z = unary_op(op, v.z, alpha);
    v.w = unary_op(op, v.w, alpha);
    y[i] = v;
  }
}

__device__ __forceinline__ float binary_op(int op, float a, float b) {
  switch (op) {
    case SPX_BIN_ADD: return a + b;
    case SPX_BIN_SUB: return a - b;
    case SPX_BIN_MUL: return a * b;
    case SPX_BIN_DIV: return a / b;
    case SPX_BIN_POW: return powf(a, b);
    case SPX_BIN_MIN: return fminf(a, b);
    case SPX_BIN_MAX: return fmaxf(a, b);
    case SPX_BIN_GT: return a > b ? 1.0f : 0.0f;
    case SPX_BIN_GE: return a >= b ? 1.0f : 0.0f;
    case SPX_BIN_LT: return a < b ? 1.0f : 0.0f;
    case SPX_BIN_LE: return a <= b ? 1.0f : 0.0f;
    case SPX_BIN_EQ: return a == b ? 1.0f : 0.0f;
    default: return a != b ? 1.0f : 0.0f;  // SPX_BIN_NE
  }
}

__global__ void binary_flat_v4(int op, const float4* __restrict__ a, const float4* __restrict__ b,
                               float4* __restrict__ y, int64_t n4) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 u = a[i], v = b[i];
    y[i] = make_float4(binary_op(op, u.x, v.x), binary_op(op, u.y, v.y),
                       binary_op(op, u.z, v.z), binary_op(op, u.w, v.w));
  }
}

struct Bcast {
  int32_t d[4];
  int64_t as[4], bs[4];
};

__global__ void binary_bcast(int op, const float* __restrict__ a, const float* __restrict__ b,
                             float* __restrict__ y, Bcast p, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t t = i;
    int64_t c3 = t % p.d[3]; t /= p.d[3];
    int64_t c2 = t % p.d[2]; t /= p.d[2];
    int64_t c1 = t % p.d[1]; t /= p.d[1];
    int64_t c0 = t;
    int64_t ia = c0 * p.as[0] + c1 * p.as[1] + c2 * p.as[2] + c3 * p.as[3];
    int64_t ib = c0 * p.bs[0] + c1 * p.bs[1] + c2 * p.bs[2] + c3 * p.bs[3];
    y[i] = binary_op(op, a[ia], b[ib]);
  }
}

struct Sel {
  int32_t d[4];
  int64_t ps[4], as[4], bs[4];
};

__global__ void select_kernel(const float* __restrict__ pr, const float* __restrict__ a,
                              const float* __restrict__ b, float* __restrict__ y, Sel p,
                              int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t t = i;
    int64_t c3 = t % p.d[3]; t /= p.d[3];
    int64_t c2 = t % p.d[2]; t /= p.d[2];
    int64_t c1 = t % p.d[1]; t /= p.d[1];
    int64_t c0 = t;
    int64_t ip = c0 * p.ps[0] + c1 * p.ps[1] + c2 * p.ps[2] + c3 * p.ps[3];
    int64_t ia = c0 * p.as[0] + c1 * p.as[1] + c2 * p.as[2] + c3 * p.as[3];
    int64_t ib = c0 * p.bs[0] + c1 * p.bs[1] + c2 * p.bs[2] + c3 * p.bs[3];
    y[i] = pr[ip] != 0.0f ? a[ia] : b[ib];
  }
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u,
                              float* __restrict__ y, int64_t n) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = g[i];
    y[i] = x / (1.0f + expf(-x)) * u[i];
  }
}

// pad.comp: rank-4 constant pad, low-side offsets pl0..pl3.
__global__ void pad4_kernel(const float* __restrict__ x, float* __restrict__ y, float pv,
                            int od0, int od1, int od2, int od3, int id0, int id1, int id2,
                            int id3, int pl0, int pl1, int pl2, int pl3, int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t t = i;
    int c3 = (int)(t % od3); t /= od3;
    int c2 = (int)(t % od2); t /= od2;
    int c1 = (int)(t % od1); t /= od1;
    int c0 = (int)t;
    int s0 = c0 - pl0, s1 = c1 - pl1, s2 = c2 - pl2, s3 = c3 - pl3;
    float v = pv;
    if (s0 >= 0 && s0 < id0 && s1 >= 0 && s1 < id1 && s2 >= 0 && s2 < id2 && s3 >= 0 &&
        s3 < id3)
      v = x[(((int64_t)s0 * id1 + s1) * id2 + s2) * id3 + s3];
    y[i] = v;
  }
}

// transpose.comp: output axis k takes input axis p[k].
__global__ void transpose4_kernel(const float* __restrict__ x, float* __restrict__ y, int in1,
                                  int in2, int in3, int o1, int o2, int o3, int p0, int p1,
                                  int p2, int p3, int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t in_str[4] = {(int64_t)in1 * in2 * in3, (int64_t)in2 * in3, in3, 1};
  int64_t s0 = in_str[p0], s1 = in_str[p1], s2 = in_str[p2], s3 = in_str[p3];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t t = i;
    int64_t c3 = t % o3; t /= o3;
    int64_t c2 = t % o2; t /= o2;
    int64_t c1 = t % o1; t /= o1;
    int64_t c0 = t;
    y[i] = x[c0 * s0 + c1 * s1 + c2 * s2 + c3 * s3];
  }
}

__global__ void concat_kernel(const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ y, int64_t a_total, int64_t total) {
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride)
    y[i] = i < a_total ? a[i] : b[i - a_total];
}

// l2norm.comp: divide by a host-computed norm, floored at 1e-12.
__global__ void l2norm_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                              float norm) {
  float d = fmaxf(norm, 1.0e-12f);
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = x[i] / d;
}

__global__ void embedding_kernel(const float* __restrict__ table, const int32_t* __restrict__ ids,
                                 float* __restrict__ y, int tokens, int dim) {
  for (int t = blockIdx.x; t < tokens; t += gridDim.x) {
    const float* row = table + (int64_t)ids[t] * dim;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) y[(int64_t)t * dim + j] = row[j];
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

int launch_unary(cudaStream_t s, int64_t* cnt, int op, const float* x, float* y, int64_t n,
                 float alpha) {
  if (op < 0 || op > SPX_UN_SILU) return fail(SPX_ERR_UNSUPPORTED, "unary op %d unknown", op);
  if (n < 0) return fail(SPX_ERR_INVALID_ARGUMENT, "unary: negative length");
  if (n == 0) return SPX_OK;
  if (n % 4 == 0 && aligned16(x) && aligned16(y)) {
    unary_kernel_v4<<<grid_for(n / 4, 256), 256, 0, s>>>(op, (const float4*)x, (float4*)y, n / 4,
                                                         alpha);
  } else {
    unary_kernel<<<grid_for(n, 256), 256, 0, s>>>(op, x, y, n, alpha);
  }
  return after_launch(cnt, "unary");
}

int launch_binary(cudaStream_t s, int64_t* cnt, int op, const float* a, const float* b,
                  float* y, const spx_bcast_params* p) {
  if (op < 0 || op > SPX_BIN_NE) return fail(SPX_ERR_UNSUPPORTED, "binary op %d unknown", op);
  int64_t n = 1;
  for (int i = 0; i < 4; ++i) {
    if (p->d[i] < 0) return fail(SPX_ERR_INVALID_ARGUMENT, "binary: negative dim");
    n *= p->d[i];
  }
  if (n == 0) return SPX_OK;
  // Contiguous same-shape fast path.
  int64_t cs[4] = {(int64_t)p->d[1] * p->d[2] * p->d[3], (int64_t)p->d[2] * p->d[3], p->d[3], 1};
  bool contig = true;
  for (int i = 0; i < 4; ++i)
    if (p->d[i] > 1 && (p->a_stride[i] != cs[i] || p->b_stride[i] != cs[i])) contig = false;
  if (contig && n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(y)) {
    binary_flat_v4<<<grid_for(n / 4, 256), 256, 0, s>>>(op, (const float4*)a, (const float4*)b,
                                                        (float4*)y, n / 4);
  } else {
    Bcast q;
    for (int i = 0; i < 4; ++i) {
      q.d[i] = p->d[i] > 0 ? p->d[i] : 1;
      q.as[i] = p->a_stride[i];
      q.bs[i] = p->b_stride[i];
    }
    binary_bcast<<<grid_for(n, 256), 256, 0, s>>>(op, a, b, y, q, n);
  }
  return after_launch(cnt, "binary");
}

int launch_select(cudaStream_t s, int64_t* cnt, const float* pr, const float* a, const float* b,
                  float* y, const spx_select_params* p) {
  int64_t n = 1;
  Sel q;
  for (int i = 0; i < 4; ++i) {
    if (p->d[i] < 0) return fail(SPX_ERR_INVALID_ARGUMENT, "select: negative dim");
    n *= p->d[i];
    q.d[i] = p->d[i] > 0 ? p->d[i] : 1;
    q.ps[i] = p->p_stride[i];
    q.as[i] = p->a_stride[i];
    q.bs[i] = p->b_stride[i];
  }
  if (n == 0) return SPX_OK;
  select_kernel<<<grid_for(n, 256), 256, 0, s>>>(pr, a, b, y, q, n);
  return after_launch(cnt, "select");
}

int launch_swiglu(cudaStream_t s, int64_t* cnt, const float* gate, const float* up, float* y,
                  int64_t n) {
  if (n <= 0) return n == 0 ? SPX_OK : fail(SPX_ERR_INVALID_ARGUMENT, "swiglu: bad length");
  swiglu_kernel<<<grid_for(n, 256), 256, 0, s>>>(gate, up, y, n);
  return after_launch(cnt, "swiglu");
}

int launch_pad4(cudaStream_t s, int64_t* cnt, const float* x, float* y, float pv,
                const int32_t* q) {
  int64_t total = (int64_t)q[0] * q[1] * q[2] * q[3];
  for (int i = 0; i < 12; ++i)
    if (q[i] < 0 || (i < 8 && q[i] == 0)) return fail(SPX_ERR_INVALID_ARGUMENT, "pad: bad dims");
  if (q[12] != total) return fail(SPX_ERR_INVALID_ARGUMENT, "pad: total %d != product", q[12]);
  pad4_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, y, pv, q[0], q[1], q[2], q[3], q[4], q[5],
                                                   q[6], q[7], q[8], q[9], q[10], q[11], total);
  return after_launch(cnt, "pad4");
}

int launch_transpose4(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                      const int32_t* q) {
  int seen = 0;
  for (int k = 0; k < 4; ++k) {
    if (q[8 + k] < 0 || q[8 + k] > 3) return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: bad perm");
    seen |= 1 << q[8 + k];
    if (q[k] <= 0 || q[4 + k] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: bad dims");
  }
  if (seen != 15) return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: perm is not a permutation");
  for (int k = 0; k < 4; ++k)
    if (q[4 + k] != q[q[8 + k]])
      return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: out dim %d != in dim %d", k, q[8 + k]);
  int64_t total = (int64_t)q[4] * q[5] * q[6] * q[7];
  if (q[12] != total) return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: total mismatch");
  transpose4_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, y, q[1], q[2], q[3], q[5], q[6], q[7],
                                                         q[8], q[9], q[10], q[11], total);
  return after_launch(cnt, "transpose4");
}

int launch_compat_concat(cudaStream_t s, int64_t* cnt, const float* a, const float* b, float* y,
                         int a_total, int total) {
  if (a_total < 0 || total < a_total) return fail(SPX_ERR_INVALID_ARGUMENT, "concat: bad sizes");
  if (total == 0) return SPX_OK;
  concat_kernel<<<grid_for(total, 256), 256, 0, s>>>(a, b, y, a_total, total);
  return after_launch(cnt, "concat");
}

int launch_compat_l2norm(cudaStream_t s, int64_t* cnt, const float* x, float* y, int total,
                         float norm) {
  if (total <= 0) return total == 0 ? SPX_OK : fail(SPX_ERR_INVALID_ARGUMENT, "l2norm: total");
  l2norm_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, y, total, norm);
  return after_launch(cnt, "l2norm");
}

int launch_embedding(cudaStream_t s, int64_t* cnt, const float* table, const int32_t* ids,
                     float* y, int tokens, int dim) {
  if (tokens <= 0 || dim <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "embedding: bad sizes");
  embedding_kernel<<<grid_for(tokens, 1, 64), 256, 0, s>>>(table, ids, y, tokens, dim);
  return after_launch(cnt, "embedding");
}

}  // namespace spx

// Compute capability the loaded device code was compiled for (major * 10 +
// minor, from cudaFuncGetAttributes on one of the library's kernels): 100 for
// the sm_100a build.  Lets a test confirm the architecture without any binary
// tool.
extern "C" int spx_binary_version(int device, int* version) {
  using namespace spx;
  if (!version) return fail(SPX_ERR_INVALID_ARGUMENT, "binary_version: null version");
  int rc;
  if ((rc = check_cuda(cudaSetDevice(device), "cudaSetDevice"))) return rc;
  cudaFuncAttributes a{};
  if ((rc = check_cuda(cudaFuncGetAttributes(&a, unary_kernel), "cudaFuncGetAttributes")))
    return rc;
  *version = a.binaryVersion;
  return SPX_OK;
}
