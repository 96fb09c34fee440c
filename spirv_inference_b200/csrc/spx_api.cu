// libspx C ABI: error reporting, kernel registry, the drop-in dispatch
// boundary (spx_run_kernel) and the device-resident graph API.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "spx_internal.cuh"

namespace spx {

static thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SPX_OK;
  int code = e == cudaErrorMemoryAllocation ? SPX_ERR_OUT_OF_MEMORY
             : (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice) ? SPX_ERR_NO_DEVICE
                                                                        : SPX_ERR_CUDA;
  return fail(code, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int after_launch(int64_t* counter, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, what);
  if (counter) ++*counter;
  return SPX_OK;
}

int g_gemm_path = 0;
int64_t g_ar_wait_limit_us = 2000000;
int g_dw_path = 0;
int g_pw_path = 0;
int g_pw_gemm = 0;
int g_dwp_groups = 47;
int g_dwp_stages = 4;
int g_dwp_accs = 4;
int g_dwp_epi1 = 62;
int g_pdl = 1;

// ---- algorithm selection for dense contractions ---------------------------
int launch_conv_nhwc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                     const float* w_hi, const float* w_lo, const float* bias, const float* res,
                     float* y, const spx_conv_params* p) {
  if (p->n <= 0 || p->ih <= 0 || p->iw <= 0 || p->ic <= 0 || p->oc <= 0 || p->oh <= 0 ||
      p->ow <= 0 || p->kh <= 0 || p->kw <= 0 || p->stride_h <= 0 || p->stride_w <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_nhwc: non-positive shape parameter");
  if (p->weight_layout != SPX_WEIGHT_OHWI && p->weight_layout != SPX_WEIGHT_HWIO)
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_nhwc: weight_layout %d", p->weight_layout);
  if ((int64_t)p->n * p->oh * p->ow > INT32_MAX || (int64_t)p->kh * p->kw * p->ic > INT32_MAX)
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_nhwc: GEMM extent exceeds int32");
  const bool pointwise = p->kh == 1 && p->kw == 1 && p->stride_h == 1 && p->stride_w == 1 &&
                         p->pad_top == 0 && p->pad_left == 0 && p->oh == p->ih && p->ow == p->iw;
  if (g_gemm_path != 1 && pointwise && p->weight_layout == SPX_WEIGHT_OHWI) {
    const int M = p->n * p->oh * p->ow;
    const bool split = w_hi && w_lo;
    const float* wb = split ? w_hi : w;
    // A 1x1-conv classifier over pooled features (1 x 1 maps, few images):
    // weights as the UMMA M side, split-k over a cluster.  Larger maps keep
    // the row-tiled GEMM whatever the batch, so an image's result does not
    // depend on how many images share the launch.
    if (p->oh == 1 && p->ow == 1 && M <= 256 && y && gemm_tc_skinny_eligible(x, p->ic, wb, p->ic, M, p->oc, p->ic) &&
        (!split || ((uintptr_t)w_lo & 15) == 0))
      return launch_gemm_tc_skinny(s, cnt, x, p->ic, wb, split ? w_lo : nullptr, p->ic, M, p->oc,
                                   p->ic, bias, res, y, p->oc, 1.0f, p->activation);
    // Opt-in: short reductions (inverted-residual expand / project layers)
    // in exact fp32 on CUDA cores.  Measured slower than the tensor-core
    // GEMM on every MobileNetV2 layer, so off by default.
    if (g_gemm_path == 0 && g_pw_path == 1 && pw_simt_eligible(x, y, res, M, p->ic, p->oc))
      return launch_pw_simt(s, cnt, x, w, bias, res, y, M, p->ic, p->oc, p->activation);
    // Wide outputs over short reductions: the activation tile stays resident
    // and is split once for all n tiles.
    if (g_pw_gemm && split) {
      const int rc = try_pwgemm(s, cnt, x, w_hi, w_lo, bias, res, y, M, p->oc, p->ic,
                                p->activation);
      if (rc != -1) return rc;
    }
    if (gemm_tc_eligible(x, p->ic, wb, p->ic, M, p->oc, p->ic, y, p->oc) &&
        (!split || ((uintptr_t)w_lo & 15) == 0))
      return launch_gemm_tc(s, cnt, x, p->ic, wb, split ? w_lo : nullptr, p->ic, M, p->oc, p->ic,
                            bias, res, y, p->oc, 1.0f, p->activation);
  }
  if (g_gemm_path != 1 && !pointwise) {
    const bool split = w_hi && w_lo;
    const float* wb = split ? w_hi : w;
    if (conv_tc_eligible(x, wb, y, p) && (!split || ((uintptr_t)w_lo & 15) == 0))
      return launch_conv_tc(s, cnt, x, wb, split ? w_lo : nullptr, bias, res, y, p);
  }
  if (g_gemm_path == 2)
    return fail(SPX_ERR_UNSUPPORTED, "conv2d_nhwc: shape not eligible for the tensor-core path");
  if (!pointwise) {
    int rc = try_conv_smallk(s, cnt, x, w, bias, res, y, p);
    if (rc != -1) return rc;
  }
  return launch_conv_simt(s, cnt, x, w, bias, res, y, p);
}

int launch_gemm(cudaStream_t s, int64_t* cnt, const float* a, const float* b, const float* b_hi,
                const float* b_lo, const float* bias, const float* res, float* c,
                const spx_gemm_params* p) {
  if (p->batch <= 0 || p->m <= 0 || p->n <= 0 || p->k <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm: non-positive extent");
  const bool single = p->batch == 1 && (p->batch_inner <= 1);
  const bool split = b_hi && b_lo;
  const float* bb = split ? b_hi : b;
  // A handful of rows (decode, small-batch FC): stream the fp32 weights once
  // on CUDA cores; a 128-row tensor-core tile would be almost all padding.
  if (g_gemm_path == 0 && single && b && p->a_ks == 1 && p->b_ks == 1 && c &&
      p->c_ms >= p->n && gemm_rows_eligible(a, p->a_ms, b, p->b_ns, p->m, p->k))
    return launch_gemm_rows(s, cnt, a, p->a_ms, b, p->b_ns, p->m, p->n, p->k, bias, res, c,
                            p->c_ms, p->alpha, p->activation, 0);
  // Up to 256 rows: weights as the UMMA M side, split-k over a cluster; with
  // pre-split weights the tiles arrive as hi / lo and only the rows are split.
  if (g_gemm_path != 1 && single && bb && p->a_ks == 1 && p->b_ks == 1 && c &&
      p->c_ms >= p->n && gemm_tc_skinny_eligible(a, p->a_ms, bb, p->b_ns, p->m, p->n, p->k))
    return launch_gemm_tc_skinny(s, cnt, a, p->a_ms, bb, split ? b_lo : nullptr, p->b_ns, p->m,
                                 p->n, p->k, bias, res, c, p->c_ms, p->alpha, p->activation);
  if (g_gemm_path != 1 && single && p->a_ks == 1 && p->b_ks == 1 &&
      gemm_tc_eligible(a, p->a_ms, bb, p->b_ns, p->m, p->n, p->k, c, p->c_ms) &&
      (!split || ((uintptr_t)b_lo & 15) == 0))
    return launch_gemm_tc(s, cnt, a, p->a_ms, bb, split ? b_lo : nullptr, p->b_ns, p->m, p->n,
                          p->k, bias, res, c, p->c_ms, p->alpha, p->activation);
  // Batched products with a short reduction (attention Q.K^T and P.V).
  if (g_gemm_path != 1 && !single && b) {
    const int rc = try_bgemm_tc(s, cnt, a, b, bias, res, c, p);
    if (rc != -1) return rc;
  }
  if (g_gemm_path == 2)
    return fail(SPX_ERR_UNSUPPORTED, "gemm: operands not eligible for the tensor-core path");
  return launch_gemm_simt(s, cnt, a, b, bias, res, c, p);
}

}  // namespace spx

using namespace spx;

// ===========================================================================
// Registry: names, push-constant counts and work-group sizes of the
// reference kernels (source/tflite_loader/src/kernels.rs:12-238; HLO kernels
// from source/xla_hlo/src/compiler.rs:768-1135 and 1155-1228).
// ===========================================================================
namespace {
struct KernelEntry {
  const char* name;
  int push;   // expected push-constant count
  int local;  // reference work-group size
};
const KernelEntry kKernels[] = {
    {"add", 1, 128}, {"sub", 1, 128}, {"mul", 1, 128}, {"div", 1, 128}, {"pow", 1, 128},
    {"min", 1, 128}, {"max", 1, 128}, {"exp", 1, 128}, {"neg", 1, 128}, {"abs", 1, 128},
    {"sqrt", 1, 128}, {"rsqrt", 1, 128}, {"log", 1, 128}, {"leaky_relu", 2, 128},
    {"logistic", 1, 128}, {"sigmoid", 1, 128}, {"tanh", 1, 128}, {"relu6", 1, 128},
    {"relu", 1, 128}, {"sine", 1, 128}, {"reshape", 1, 128}, {"concat", 2, 128},
    {"transpose", 13, 128}, {"conv2d", 15, 64}, {"depthwise_conv2d", 16, 64},
    {"global_avg_pool_sum", 4, 64}, {"max_pool2d", 14, 64}, {"l2norm", 2, 128},
    {"resize_bilinear", 9, 64}, {"global_avg_pool_finalize", 4, 64},
    {"fully_connected", 4, 64}, {"softmax10", 0, 10}, {"softmax1000", 1, 256},
    {"hlo_conv_nhwc_hwio", 14, 64}, {"hlo_dot_rank2", 4, 64}, {"hlo_dot_batched", 5, 64},
    {"hlo_reduce_rank4", 15, 64}, {"hlo_reduce_window_rank4", 14, 64}, {"pad", 13, 128},
};
constexpr int kNumKernels = sizeof(kKernels) / sizeof(kKernels[0]);

std::string canonical_name(const char* kernel) {
  std::string s = kernel ? kernel : "";
  const std::string suffix = ".spv";
  if (s.size() > suffix.size() && s.compare(s.size() - suffix.size(), suffix.size(), suffix) == 0)
    s.resize(s.size() - suffix.size());
  // kernels.rs:244-257 resolves spv stems onto kernel directories; the stem
  // is the kernel identity.
  return s;
}

const KernelEntry* find_kernel(const std::string& name) {
  for (int i = 0; i < kNumKernels; ++i)
    if (name == kKernels[i].name) return &kKernels[i];
  return nullptr;
}

// ---- per-device state of the drop-in boundary ------------------------------
struct DeviceCache {
  std::mutex mu;
  bool init = false;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float* buf[6] = {nullptr};
  size_t cap[6] = {0};
  cudaDeviceProp prop;
};
DeviceCache g_cache[64];

int ensure_buf(DeviceCache& c, int i, size_t elems) {
  size_t bytes = std::max<size_t>(elems, 1) * sizeof(float);
  if (c.cap[i] >= bytes) return SPX_OK;
  size_t want = std::max(bytes, c.cap[i] * 2);
  if (c.buf[i]) cudaFree(c.buf[i]);
  c.buf[i] = nullptr;
  c.cap[i] = 0;
  int rc = check_cuda(cudaMalloc(&c.buf[i], want), "cudaMalloc (run_kernel buffer)");
  if (rc) return rc;
  c.cap[i] = want;
  return SPX_OK;
}

int need(bool ok, const char* kernel, const char* what) {
  return ok ? SPX_OK : fail(SPX_ERR_INVALID_ARGUMENT, "%s: %s", kernel, what);
}

int unary_code(const std::string& n) {
  if (n == "abs") return SPX_UN_ABS;
  if (n == "exp") return SPX_UN_EXP;
  if (n == "log") return SPX_UN_LOG;
  if (n == "neg") return SPX_UN_NEG;
  if (n == "sqrt") return SPX_UN_SQRT;
  if (n == "rsqrt") return SPX_UN_RSQRT;
  if (n == "sigmoid" || n == "logistic") return SPX_UN_SIGMOID;
  if (n == "tanh") return SPX_UN_TANH;
  if (n == "relu") return SPX_UN_RELU;
  if (n == "relu6") return SPX_UN_RELU6;
  if (n == "leaky_relu") return SPX_UN_LEAKY_RELU;
  if (n == "sine") return SPX_UN_SIN;
  if (n == "reshape") return SPX_UN_COPY;
  return -1;
}
int binary_code(const std::string& n) {
  if (n == "add") return SPX_BIN_ADD;
  if (n == "sub") return SPX_BIN_SUB;
  if (n == "mul") return SPX_BIN_MUL;
  if (n == "div") return SPX_BIN_DIV;
  if (n == "pow") return SPX_BIN_POW;
  if (n == "min") return SPX_BIN_MIN;
  if (n == "max") return SPX_BIN_MAX;
  return -1;
}

// Issues the device work of one reference dispatch.  in0/in1/out are device
// buffers holding the caller's bindings; sizes were validated against the
// push constants.  scratch buffers 3..5 are available.
int dispatch_compat(DeviceCache& c, const std::string& k, const float* in0, size_t n0,
                    const float* in1, size_t n1, float* out, size_t nout, const int32_t* q,
                    size_t nq, float in1_first, int64_t* cnt) {
  cudaStream_t s = c.stream;
  const char* kn = k.c_str();
  int rc;
  int u = unary_code(k);
  if (u >= 0) {
    int64_t total = q[0];
    if ((rc = need(total >= 0 && (size_t)total <= n0 && (size_t)total <= nout, kn,
                   "total exceeds input or output length")))
      return rc;
    float alpha = 0.0f;
    if (u == SPX_UN_LEAKY_RELU) memcpy(&alpha, &q[1], sizeof(float));
    return launch_unary(s, cnt, u, in0, out, total, alpha);
  }
  int b = binary_code(k);
  if (b >= 0) {
    int64_t total = q[0];
    if ((rc = need(total >= 0 && (size_t)total <= n0 && (size_t)total <= n1 &&
                       (size_t)total <= nout,
                   kn, "total exceeds an input or the output length (equal sizes required)")))
      return rc;
    spx_bcast_params p = {{1, 1, 1, (int32_t)total}, {0, 0, 0, 1}, {0, 0, 0, 1}};
    if (total == 0) return SPX_OK;
    return launch_binary(s, cnt, b, in0, in1, out, &p);
  }
  if (k == "concat") {
    if ((rc = need(q[0] >= 0 && q[1] >= q[0] && (size_t)q[0] <= n0 &&
                       (size_t)(q[1] - q[0]) <= n1 && (size_t)q[1] <= nout,
                   kn, "a_total/total inconsistent with buffer lengths")))
      return rc;
    return launch_compat_concat(s, cnt, in0, in1, out, q[0], q[1]);
  }
  if (k == "transpose") {
    int64_t in_total = (int64_t)q[0] * q[1] * q[2] * q[3];
    if ((rc = need(in_total >= 0 && (size_t)in_total <= n0 && q[12] >= 0 &&
                       (size_t)q[12] <= nout,
                   kn, "dims exceed buffer lengths")))
      return rc;
    return launch_transpose4(s, cnt, in0, out, q);
  }
  if (k == "conv2d") {
    // n,ic,ih,iw,oc,oh,ow,kh,kw,stride_h,stride_w,same,pad_top,pad_left,total
    int N = q[0], IC = q[1], IH = q[2], IW = q[3], OC = q[4], OH = q[5], OW = q[6], KH = q[7],
        KW = q[8];
    for (int i = 0; i < 11; ++i)
      if (q[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d: push[%d] <= 0", i);
    int64_t in_el = (int64_t)N * IC * IH * IW, w_el = (int64_t)OC * IC * KH * KW;
    int64_t total = (int64_t)N * OC * OH * OW;
    if ((rc = need(total == q[14], kn, "total != n*oc*oh*ow"))) return rc;
    if ((rc = need((size_t)in_el <= n0 && (size_t)(w_el + OC) <= n1 && (size_t)total <= nout, kn,
                   "buffers shorter than the shape implies")))
      return rc;
    // NCHW -> NHWC input, OIHW -> OHWI weights, NHWC conv with bias, NHWC -> NCHW.
    if ((rc = ensure_buf(c, 3, in_el)) || (rc = ensure_buf(c, 4, w_el)) ||
        (rc = ensure_buf(c, 5, total)))
      return rc;
    int32_t t_in[13] = {N, IC, IH, IW, N, IH, IW, IC, 0, 2, 3, 1, (int32_t)in_el};
    int32_t t_w[13] = {OC, IC, KH, KW, OC, KH, KW, IC, 0, 2, 3, 1, (int32_t)w_el};
    int32_t t_out[13] = {N, OH, OW, OC, N, OC, OH, OW, 0, 3, 1, 2, (int32_t)total};
    if ((rc = launch_transpose4(s, cnt, in0, c.buf[3], t_in))) return rc;
    if ((rc = launch_transpose4(s, cnt, in1, c.buf[4], t_w))) return rc;
    spx_conv_params p = {N, IH, IW, IC, OC, OH, OW, KH, KW, q[9], q[10], q[12], q[13], 1, 1,
                         SPX_WEIGHT_OHWI, SPX_ACT_NONE};
    if ((rc = launch_conv_nhwc(s, cnt, c.buf[3], c.buf[4], nullptr, nullptr, in1 + w_el, nullptr,
                               c.buf[5], &p)))
      return rc;
    return launch_transpose4(s, cnt, c.buf[5], out, t_out);
  }
  if (k == "depthwise_conv2d") {
    for (int i = 0; i < 10; ++i)
      if (q[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "depthwise_conv2d: push[%d] <= 0", i);
    int64_t in_el = (int64_t)q[0] * q[1] * q[2] * q[3];
    int64_t w_el = (int64_t)q[1] * q[6] * q[7] + q[1];
    int64_t total = (int64_t)q[0] * q[1] * q[4] * q[5];
    if ((rc = need((size_t)in_el <= n0 && (size_t)w_el <= n1 && (size_t)total <= nout, kn,
                   "buffers shorter than the shape implies")))
      return rc;
    if (q[13] <= 0 || q[14] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "depthwise: dilation");
    return launch_compat_dw_nchw(s, cnt, in0, in1, out, q);
  }
  if (k == "max_pool2d") {
    for (int i = 0; i < 10; ++i)
      if (q[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "max_pool2d: push[%d] <= 0", i);
    int64_t in_el = (int64_t)q[0] * q[1] * q[2] * q[3];
    int64_t total = (int64_t)q[0] * q[1] * q[4] * q[5];
    if ((rc = need((size_t)in_el <= n0 && (size_t)total <= nout, kn, "buffers too short")))
      return rc;
    return launch_compat_maxpool_nchw(s, cnt, in0, out, q);
  }
  if (k == "global_avg_pool_sum" || k == "global_avg_pool_finalize") {
    int64_t nc = (int64_t)q[0] * q[1];
    bool sum = k == "global_avg_pool_sum";
    int64_t in_el = sum ? nc * q[2] * q[3] : nc;
    if ((rc = need(q[0] > 0 && q[1] > 0 && q[2] > 0 && q[3] > 0 && (size_t)in_el <= n0 &&
                       (size_t)nc <= nout,
                   kn, "bad shape or buffers too short")))
      return rc;
    return sum ? launch_compat_gap_sum_nchw(s, cnt, in0, out, q[0], q[1], q[2], q[3])
               : launch_compat_gap_finalize(s, cnt, in0, out, q[0], q[1], q[2], q[3]);
  }
  if (k == "l2norm") {
    float norm;
    memcpy(&norm, &q[1], sizeof(float));
    if ((rc = need(q[0] >= 0 && (size_t)q[0] <= n0 && (size_t)q[0] <= nout, kn, "total")))
      return rc;
    return launch_compat_l2norm(s, cnt, in0, out, q[0], norm);
  }
  if (k == "resize_bilinear") {
    int64_t in_el = (int64_t)q[0] * q[1] * q[2] * q[3];
    if ((rc = need((size_t)in_el <= n0 && q[8] >= 0 && (size_t)q[8] <= nout, kn, "buffers")))
      return rc;
    return launch_compat_resize_bilinear(s, cnt, in0, out, q);
  }
  if (k == "fully_connected") {
    int B = q[0], I = q[1], O = q[2];
    if ((rc = need(B > 0 && I > 0 && O > 0 && (int64_t)B * O == q[3], kn, "bad shape"))) return rc;
    if ((rc = need((size_t)B * I <= n0 && (size_t)O * I + O <= n1 && (size_t)B * O <= nout, kn,
                   "buffers too short")))
      return rc;
    spx_gemm_params p = {};
    p.batch = 1; p.m = B; p.n = O; p.k = I; p.batch_inner = 1; p.b_inner_div = 1;
    p.a_ms = I; p.a_ks = 1; p.b_ks = 1; p.b_ns = I; p.c_ms = O; p.alpha = 1.0f;
    return launch_gemm(s, cnt, in0, in1, nullptr, nullptr, in1 + (int64_t)O * I, nullptr, out, &p);
  }
  if (k == "softmax10" || k == "softmax1000") {
    int classes = k == "softmax10" ? 10 : q[0];
    if (k == "softmax10" && nq >= 1) classes = 10;  // registry lists "classes"; shader fixes 10
    if ((rc = need(classes > 0 && (size_t)classes <= n0 && (size_t)classes <= nout, kn,
                   "class count exceeds buffers")))
      return rc;
    return launch_softmax_rows(s, cnt, in0, out, 1, classes, 1.0f, 0, 0, 0);
  }
  if (k == "hlo_conv_nhwc_hwio") {
    // n,ih,iw,ic,kh,kw,oc,oh,ow,stride_h,stride_w,pad_top,pad_left,total
    for (int i = 0; i < 11; ++i)
      if (q[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "hlo_conv: push[%d] <= 0", i);
    int64_t in_el = (int64_t)q[0] * q[1] * q[2] * q[3];
    int64_t w_el = (int64_t)q[4] * q[5] * q[3] * q[6];
    int64_t total = (int64_t)q[0] * q[7] * q[8] * q[6];
    if ((rc = need(total == q[13], kn, "total != n*oh*ow*oc"))) return rc;
    if ((rc = need((size_t)in_el <= n0 && (size_t)w_el <= n1 && (size_t)total <= nout, kn,
                   "buffers too short")))
      return rc;
    spx_conv_params p = {q[0], q[1], q[2], q[3], q[6], q[7], q[8], q[4], q[5], q[9], q[10],
                         q[11], q[12], 1, 1, SPX_WEIGHT_HWIO, SPX_ACT_NONE};
    return launch_conv_nhwc(s, cnt, in0, in1, nullptr, nullptr, nullptr, nullptr, out, &p);
  }
  if (k == "hlo_dot_rank2" || k == "hlo_dot_batched") {
    bool batched = k == "hlo_dot_batched";
    int B = batched ? q[0] : 1, M = q[batched], K = q[batched + 1], N = q[batched + 2];
    int64_t total = (int64_t)B * M * N;
    if ((rc = need(B > 0 && M > 0 && K > 0 && N > 0 && total == q[batched + 3], kn,
                   "bad shape or total")))
      return rc;
    if ((rc = need((size_t)B * M * K <= n0 && (size_t)B * K * N <= n1 && (size_t)total <= nout,
                   kn, "buffers too short")))
      return rc;
    spx_gemm_params p = {};
    p.batch = B; p.m = M; p.n = N; p.k = K; p.batch_inner = 1; p.b_inner_div = 1;
    p.a_bs = (int64_t)M * K; p.a_ms = K; p.a_ks = 1;
    p.b_bs = (int64_t)K * N; p.b_ks = N; p.b_ns = 1;
    p.c_bs = (int64_t)M * N; p.c_ms = N; p.alpha = 1.0f;
    return launch_gemm(s, cnt, in0, in1, nullptr, nullptr, nullptr, nullptr, out, &p);
  }
  if (k == "hlo_reduce_rank4") {
    int64_t in_el = (int64_t)q[1] * q[2] * q[3] * q[4];
    if ((rc = need(in_el > 0 && (size_t)in_el <= n0 && q[14] > 0 && (size_t)q[14] <= nout, kn,
                   "buffers too short")))
      return rc;
    return launch_reduce_rank4(s, cnt, in0, out, q);
  }
  if (k == "hlo_reduce_window_rank4") {
    // n,ih,iw,c,oh,ow,wh,ww,stride_h,stride_w,pad_top,pad_left,kind,total
    int64_t in_el = (int64_t)q[0] * q[1] * q[2] * q[3];
    int64_t total = (int64_t)q[0] * q[4] * q[5] * q[3];
    if ((rc = need(total == q[13] && (size_t)in_el <= n0 && (size_t)total <= nout, kn,
                   "total or buffer mismatch")))
      return rc;
    spx_pool_params p = {q[0], q[1], q[2], q[3], q[4], q[5], q[6], q[7], q[8], q[9], q[10], q[11],
                         q[12] == 1 ? SPX_POOL_MAX : SPX_POOL_SUM};
    return launch_pool_nhwc(s, cnt, in0, out, &p);
  }
  if (k == "pad") {
    int64_t in_el = (int64_t)q[4] * q[5] * q[6] * q[7];
    if ((rc = need(n1 >= 1 && in_el > 0 && (size_t)in_el <= n0 && q[12] >= 0 &&
                       (size_t)q[12] <= nout,
                   kn, "buffers too short (binding 1 must hold the pad value)")))
      return rc;
    return launch_pad4(s, cnt, in0, out, in1_first, q);
  }
  return fail(SPX_ERR_UNSUPPORTED, "kernel '%s' has no lowering", kn);
}

}  // namespace

// ===========================================================================
extern "C" {

const char* spx_last_error(void) { return g_error.c_str(); }
const char* spx_version(void) { return "spx 0.1.0 (sm_100a)"; }

int spx_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int spx_select_device(const char* selector, int* ordinal) {
  if (!ordinal) return fail(SPX_ERR_INVALID_ARGUMENT, "select_device: null ordinal");
  std::string s = selector ? selector : "any";
  int n = spx_device_count();
  if (s == "intel") return fail(SPX_ERR_NO_DEVICE, "no Intel device is reachable through CUDA");
  if (s == "any" || s == "nvidia" || s.empty()) {
    if (n == 0) return fail(SPX_ERR_NO_DEVICE, "no CUDA device");
    *ordinal = 0;
    return SPX_OK;
  }
  char* end = nullptr;
  long v = strtol(s.c_str(), &end, 10);
  if (!end || *end != '\0') return fail(SPX_ERR_INVALID_ARGUMENT, "bad device selector '%s'", s.c_str());
  if (v < 0 || v >= n) return fail(SPX_ERR_NO_DEVICE, "device %ld not present (%d devices)", v, n);
  *ordinal = (int)v;
  return SPX_OK;
}

int spx_set_option(const char* name, int64_t value) {
  std::string n = name ? name : "";
  if (n == "dw_path") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "dw_path must be 0..1");
    g_dw_path = (int)value;
    return SPX_OK;
  }
  if (n == "tc_wide_epilogue") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "tc_wide_epilogue must be 0..1");
    g_tc_epi12 = (int)value;
    return SPX_OK;
  }
  if (n == "tc_cat") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "tc_cat must be 0..1");
    g_tc_cat = (int)value;
    return SPX_OK;
  }
  if (n == "tc_lo_tmem") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "tc_lo_tmem must be 0..1");
    g_tc_lo_tmem = (int)value;
    return SPX_OK;
  }
  if (n == "tc_conv_groups") {
    if (value < 1 || value > 2) return fail(SPX_ERR_INVALID_ARGUMENT, "tc_conv_groups must be 1..2");
    g_tc_conv2 = value == 2;
    return SPX_OK;
  }
  if (n == "pw_path") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "pw_path must be 0..1");
    g_pw_path = (int)value;
    return SPX_OK;
  }
  if (n == "pw_gemm") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "pw_gemm must be 0..1");
    g_pw_gemm = (int)value;
    return SPX_OK;
  }
  if (n == "pdl") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "pdl must be 0..1");
    g_pdl = (int)value;
    return SPX_OK;
  }
  if (n == "dwp_stages") {
    if (value < 2 || value > 4) return fail(SPX_ERR_INVALID_ARGUMENT, "dwp_stages must be 2..4");
    g_dwp_stages = (int)value;
    return SPX_OK;
  }
  if (n == "tc_acc4") {
    if (value < 0 || value > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "tc_acc4 must be 0..1");
    g_tc_acc4 = (int)value;
    return SPX_OK;
  }
  if (n == "dwp_epi1") {
    if (value < 0 || value > 63) return fail(SPX_ERR_INVALID_ARGUMENT, "dwp_epi1 must be 0..63");
    g_dwp_epi1 = (int)value;
    return SPX_OK;
  }
  if (n == "dwp_accs") {
    if (value != 2 && value != 4) return fail(SPX_ERR_INVALID_ARGUMENT, "dwp_accs must be 2 or 4");
    g_dwp_accs = (int)value;
    return SPX_OK;
  }
  if (n == "dwp_groups") {
    if (value < 0 || value > 63) return fail(SPX_ERR_INVALID_ARGUMENT, "dwp_groups must be 0..63");
    g_dwp_groups = (int)value;
    return SPX_OK;
  }
  if (n == "ar_wait_limit_us") {
    if (value < 1000 || value > 60000000)
      return fail(SPX_ERR_INVALID_ARGUMENT, "ar_wait_limit_us must be 1000..60000000");
    g_ar_wait_limit_us = value;
    return SPX_OK;
  }
  if (n == "gemm_path") {
    if (value < 0 || value > 2) return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_path must be 0..2");
    g_gemm_path = (int)value;
    return SPX_OK;
  }
  return fail(SPX_ERR_INVALID_ARGUMENT, "unknown option '%s'", n.c_str());
}

int64_t spx_get_option(const char* name) {
  std::string n = name ? name : "";
  if (n == "gemm_path") return g_gemm_path;
  if (n == "dw_path") return g_dw_path;
  if (n == "pw_path") return g_pw_path;
  if (n == "tc_wide_epilogue") return g_tc_epi12;
  if (n == "tc_conv_groups") return g_tc_conv2 ? 2 : 1;
  if (n == "tc_lo_tmem") return g_tc_lo_tmem;
  if (n == "tc_cat") return g_tc_cat;
  if (n == "tc_acc4") return g_tc_acc4;
  if (n == "ar_wait_limit_us") return g_ar_wait_limit_us;
  if (n == "pw_gemm") return g_pw_gemm;
  if (n == "dwp_groups") return g_dwp_groups;
  if (n == "dwp_stages") return g_dwp_stages;
  if (n == "dwp_accs") return g_dwp_accs;
  if (n == "dwp_epi1") return g_dwp_epi1;
  if (n == "pdl") return g_pdl;
  return -1;
}

static int device_status(const char* what) {
  if (dw_take_status())
    return fail(SPX_ERR_CUDA, "%s: a depthwise tile load wait timed out", what);
  if (pw_take_status())
    return fail(SPX_ERR_CUDA, "%s: a resident-tile pointwise GEMM wait timed out", what);
  if (bg_take_status())
    return fail(SPX_ERR_CUDA, "%s: a batched tensor-core GEMM wait timed out", what);
  if (dwp_take_status())
    return fail(SPX_ERR_CUDA, "%s: a fused depthwise-projection pipeline wait timed out", what);
  if (tc_take_status())
    return fail(SPX_ERR_CUDA, "%s: a tensor-core pipeline wait timed out; tiles were abandoned",
                what);
  if (ar_take_status())
    return fail(SPX_ERR_CUDA,
                "%s: an all-reduce waited %lld us for a peer rank and gave up; reset the "
                "communicator on every rank (spx_ar_reset) before its next use",
                what, (long long)g_ar_wait_limit_us);
  return SPX_OK;
}

int spx_device_status(void) { return device_status("device status"); }

int spx_kernel_count(void) { return kNumKernels; }
const char* spx_kernel_name(int i) { return i >= 0 && i < kNumKernels ? kKernels[i].name : nullptr; }
int spx_kernel_push_count(const char* name) {
  const KernelEntry* e = find_kernel(canonical_name(name));
  return e ? e->push : -1;
}
int spx_kernel_local_size(const char* name) {
  const KernelEntry* e = find_kernel(canonical_name(name));
  return e ? e->local : -1;
}

int spx_run_kernel(const char* kernel, const float* input0, size_t input0_len,
                   const float* input1, size_t input1_len, float* output, size_t output_elements,
                   const int32_t* push, size_t push_len, int device, spx_kernel_output_info* info) {
  std::string k = canonical_name(kernel);
  const KernelEntry* e = find_kernel(k);
  if (!e) return fail(SPX_ERR_UNSUPPORTED, "unknown kernel '%s'", kernel ? kernel : "(null)");
  if ((int)push_len != e->push && !(k == "softmax10" && push_len <= 1))
    return fail(SPX_ERR_INVALID_ARGUMENT, "%s expects %d push constants, got %zu", k.c_str(),
                e->push, push_len);
  if (push_len && !push) return fail(SPX_ERR_INVALID_ARGUMENT, "null push constants");
  if ((input0_len && !input0) || (input1_len && !input1) || (output_elements && !output))
    return fail(SPX_ERR_INVALID_ARGUMENT, "null buffer with non-zero length");
  int n = spx_device_count();
  if (n == 0) return fail(SPX_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n || device >= 64)
    return fail(SPX_ERR_NO_DEVICE, "device %d not present", device);
  DeviceCache& c = g_cache[device];
  std::lock_guard<std::mutex> lock(c.mu);
  int rc;
  if ((rc = check_cuda(cudaSetDevice(device), "cudaSetDevice"))) return rc;
  if (!c.init) {
    if ((rc = check_cuda(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking), "stream")))
      return rc;
    if ((rc = check_cuda(cudaEventCreate(&c.ev0), "event")) ||
        (rc = check_cuda(cudaEventCreate(&c.ev1), "event")))
      return rc;
    if ((rc = check_cuda(cudaGetDeviceProperties(&c.prop, device), "properties"))) return rc;
    c.init = true;
  }
  if ((rc = ensure_buf(c, 0, input0_len)) || (rc = ensure_buf(c, 1, input1_len)) ||
      (rc = ensure_buf(c, 2, output_elements)))
    return rc;
  if (input0_len &&
      (rc = check_cuda(cudaMemcpyAsync(c.buf[0], input0, input0_len * 4, cudaMemcpyHostToDevice,
                                       c.stream), "upload input0")))
    return rc;
  if (input1_len &&
      (rc = check_cuda(cudaMemcpyAsync(c.buf[1], input1, input1_len * 4, cudaMemcpyHostToDevice,
                                       c.stream), "upload input1")))
    return rc;
  int32_t q[16] = {0};
  for (size_t i = 0; i < push_len && i < 16; ++i) q[i] = push[i];
  float in1_first = input1_len ? input1[0] : 0.0f;
  cudaEventRecord(c.ev0, c.stream);
  int64_t launched = 0;
  rc = dispatch_compat(c, k, c.buf[0], input0_len, c.buf[1], input1_len, c.buf[2],
                       output_elements, q, push_len, in1_first, &launched);
  if (rc) {
    cudaStreamSynchronize(c.stream);
    return rc;
  }
  cudaEventRecord(c.ev1, c.stream);
  if (output_elements &&
      (rc = check_cuda(cudaMemcpyAsync(output, c.buf[2], output_elements * 4,
                                       cudaMemcpyDeviceToHost, c.stream), "download output")))
    return rc;
  if ((rc = check_cuda(cudaStreamSynchronize(c.stream), "kernel execution"))) return rc;
  if ((rc = device_status(k.c_str()))) return rc;
  if (info) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, c.ev0, c.ev1);
    info->elapsed_ms = ms;
    snprintf(info->device_name, sizeof(info->device_name), "%s", c.prop.name);
    info->vendor_id = 0x10de;
    info->device_id = (uint32_t)c.prop.pciDeviceID;
  }
  return SPX_OK;
}

// ---- graph API --------------------------------------------------------------
static int graph_create(int device, void* stream, spx_graph** out) {
  if (!out) return fail(SPX_ERR_INVALID_ARGUMENT, "graph_create: null out");
  *out = nullptr;
  int n = spx_device_count();
  if (n == 0) return fail(SPX_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n) return fail(SPX_ERR_NO_DEVICE, "device %d not present", device);
  int rc;
  if ((rc = check_cuda(cudaSetDevice(device), "cudaSetDevice"))) return rc;
  spx_graph* g = new spx_graph();
  g->device = device;
  if (stream) {
    g->stream = (cudaStream_t)stream;
  } else {
    if ((rc = check_cuda(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking),
                         "cudaStreamCreate"))) {
      delete g;
      return rc;
    }
    g->own_stream = true;
  }
  *out = g;
  return SPX_OK;
}

int spx_graph_create(int device, spx_graph** out) { return graph_create(device, nullptr, out); }
int spx_graph_create_on_stream(int device, void* s, spx_graph** out) {
  if (!s) return fail(SPX_ERR_INVALID_ARGUMENT, "graph_create_on_stream: null stream");
  return graph_create(device, s, out);
}

int spx_graph_destroy(spx_graph* g) {
  if (!g) return SPX_OK;
  cudaSetDevice(g->device);
  cudaStreamSynchronize(g->stream);
  for (void* p : g->buffers) cudaFree(p);
  if (g->cuda_exec) cudaGraphExecDestroy(g->cuda_exec);
  if (g->cuda_graph) cudaGraphDestroy(g->cuda_graph);
  if (g->own_stream) cudaStreamDestroy(g->stream);
  delete g;
  return SPX_OK;
}

void* spx_graph_stream(spx_graph* g) { return g ? (void*)g->stream : nullptr; }
int spx_graph_device(spx_graph* g) { return g ? g->device : -1; }
int64_t spx_graph_launch_count(spx_graph* g) { return g ? g->launches : 0; }
void spx_graph_reset_launch_count(spx_graph* g) {
  if (g) g->launches = 0;
}

#define SPX_G(g)                                                              \
  do {                                                                        \
    if (!(g)) return fail(SPX_ERR_INVALID_ARGUMENT, "null graph");            \
    int _rc = check_cuda(cudaSetDevice((g)->device), "cudaSetDevice");        \
    if (_rc) return _rc;                                                      \
  } while (0)

int spx_graph_sync(spx_graph* g) {
  SPX_G(g);
  int rc = check_cuda(cudaStreamSynchronize(g->stream), "graph execution");
  if (rc) return rc;
  return device_status("graph execution");
}

int spx_graph_capture_begin(spx_graph* g) {
  SPX_G(g);
  if (g->capturing) return fail(SPX_ERR_INVALID_ARGUMENT, "capture already in progress");
  int rc = check_cuda(cudaStreamBeginCapture(g->stream, cudaStreamCaptureModeThreadLocal),
                      "cudaStreamBeginCapture");
  if (rc) return rc;
  g->capturing = true;
  g->capture_start = g->launches;
  return SPX_OK;
}

int spx_graph_capture_end(spx_graph* g) {
  SPX_G(g);
  if (!g->capturing) return fail(SPX_ERR_INVALID_ARGUMENT, "no capture in progress");
  g->capturing = false;
  cudaGraph_t graph = nullptr;
  int rc = check_cuda(cudaStreamEndCapture(g->stream, &graph), "cudaStreamEndCapture");
  if (rc) return rc;
  if (g->cuda_exec) cudaGraphExecDestroy(g->cuda_exec);
  if (g->cuda_graph) cudaGraphDestroy(g->cuda_graph);
  g->cuda_graph = graph;
  g->cuda_exec = nullptr;
  rc = check_cuda(cudaGraphInstantiate(&g->cuda_exec, graph, 0), "cudaGraphInstantiate");
  g->captured_launches = g->launches - g->capture_start;
  g->launches = g->capture_start;  // captured work has not run yet
  return rc;
}

int spx_graph_replay(spx_graph* g) {
  SPX_G(g);
  if (!g->cuda_exec) return fail(SPX_ERR_INVALID_ARGUMENT, "no captured graph");
  int rc = check_cuda(cudaGraphLaunch(g->cuda_exec, g->stream), "cudaGraphLaunch");
  if (!rc) g->launches += g->captured_launches;
  return rc;
}

int spx_buf_alloc(spx_graph* g, size_t bytes, void** dptr) {
  SPX_G(g);
  if (!dptr) return fail(SPX_ERR_INVALID_ARGUMENT, "buf_alloc: null out");
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
  if (rc) return rc;
  g->buffers.push_back(p);
  *dptr = p;
  return SPX_OK;
}

int spx_buf_free(spx_graph* g, void* dptr) {
  SPX_G(g);
  auto it = std::find(g->buffers.begin(), g->buffers.end(), dptr);
  if (it == g->buffers.end()) return fail(SPX_ERR_INVALID_ARGUMENT, "buf_free: not owned");
  g->buffers.erase(it);
  cudaStreamSynchronize(g->stream);
  return check_cuda(cudaFree(dptr), "cudaFree");
}

int spx_buf_upload(spx_graph* g, void* dst, const void* src, size_t bytes) {
  SPX_G(g);
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g->stream), "upload");
}
int spx_buf_download(spx_graph* g, void* dst, const void* src, size_t bytes) {
  SPX_G(g);
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, g->stream),
                    "download");
}
int spx_buf_zero(spx_graph* g, void* dst, size_t bytes) {
  SPX_G(g);
  return check_cuda(cudaMemsetAsync(dst, 0, bytes, g->stream), "memset");
}
int spx_buf_copy(spx_graph* g, void* dst, const void* src, size_t bytes) {
  SPX_G(g);
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, g->stream),
                    "device copy");
}
int spx_host_alloc_pinned(size_t bytes, void** ptr) {
  if (!ptr) return fail(SPX_ERR_INVALID_ARGUMENT, "host_alloc: null out");
  if (spx_device_count() == 0) return fail(SPX_ERR_NO_DEVICE, "no CUDA device");
  return check_cuda(cudaMallocHost(ptr, bytes ? bytes : 16), "cudaMallocHost");
}
int spx_host_free_pinned(void* ptr) { return check_cuda(cudaFreeHost(ptr), "cudaFreeHost"); }

// ---- ops ----------------------------------------------------------------------
int spx_op_conv2d_nhwc(spx_graph* g, const float* x, const float* w, const float* bias,
                       const float* residual, float* y, const spx_conv_params* p) {
  SPX_G(g);
  if (!x || !w || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_nhwc: null argument");
  return launch_conv_nhwc(g->stream, &g->launches, x, w, nullptr, nullptr, bias, residual, y, p);
}

int spx_op_conv2d_nhwc_split(spx_graph* g, const float* x, const float* w, const float* w_hi,
                             const float* w_lo, const float* bias, const float* residual, float* y,
                             const spx_conv_params* p) {
  SPX_G(g);
  if (!x || !w || !w_hi || !w_lo || !y || !p)
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_nhwc_split: null argument");
  return launch_conv_nhwc(g->stream, &g->launches, x, w, w_hi, w_lo, bias, residual, y, p);
}

int spx_weights_split(spx_graph* g, const float* w, float* w_hi, float* w_lo, int64_t n) {
  SPX_G(g);
  if (!w || !w_hi || !w_lo) return fail(SPX_ERR_INVALID_ARGUMENT, "weights_split: null argument");
  return launch_weights_split(g->stream, &g->launches, w, w_hi, w_lo, n);
}

int spx_op_depthwise_conv2d_nhwc(spx_graph* g, const float* x, const float* w, const float* bias,
                                 float* y, const spx_dw_params* p) {
  SPX_G(g);
  if (!x || !w || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "depthwise: null argument");
  return launch_dw_nhwc(g->stream, &g->launches, x, w, bias, y, p);
}

int spx_op_gemm(spx_graph* g, const float* a, const float* b, const float* bias,
                const float* residual, float* c, const spx_gemm_params* p) {
  SPX_G(g);
  if (!a || !b || !c || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "gemm: null argument");
  return launch_gemm(g->stream, &g->launches, a, b, nullptr, nullptr, bias, residual, c, p);
}

int spx_op_gemm_split(spx_graph* g, const float* a, const float* b, const float* b_hi,
                      const float* b_lo, const float* bias, const float* residual, float* c,
                      const spx_gemm_params* p) {
  SPX_G(g);
  if (!a || !b || !b_hi || !b_lo || !c || !p)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_split: null argument");
  return launch_gemm(g->stream, &g->launches, a, b, b_hi, b_lo, bias, residual, c, p);
}

int spx_op_pool2d_nhwc(spx_graph* g, const float* x, float* y, const spx_pool_params* p) {
  SPX_G(g);
  if (!x || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "pool: null argument");
  return launch_pool_nhwc(g->stream, &g->launches, x, y, p);
}

int spx_op_global_avg_pool_nhwc(spx_graph* g, const float* x, float* y, int32_t n, int32_t hw,
                                int32_t c) {
  SPX_G(g);
  if (!x || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "gap: null argument");
  return launch_gap_nhwc(g->stream, &g->launches, x, y, n, hw, c);
}

int spx_op_softmax_rows(spx_graph* g, const float* x, float* y, int32_t rows, int32_t cols) {
  SPX_G(g);
  if (!x || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "softmax: null argument");
  return launch_softmax_rows(g->stream, &g->launches, x, y, rows, cols, 1.0f, 0, 0, 0);
}

int spx_op_attention_softmax(spx_graph* g, const float* x, float* y, int32_t rows, int32_t cols,
                             float scale, int32_t causal, int32_t q_len, int32_t q_offset) {
  SPX_G(g);
  if (!x || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "attention_softmax: null argument");
  return launch_softmax_rows(g->stream, &g->launches, x, y, rows, cols, scale, causal, q_len,
                             q_offset);
}

int spx_op_unary(spx_graph* g, int32_t op, const float* x, float* y, int64_t n, float alpha) {
  SPX_G(g);
  if (!x || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "unary: null argument");
  return launch_unary(g->stream, &g->launches, op, x, y, n, alpha);
}

int spx_op_binary(spx_graph* g, int32_t op, const float* a, const float* b, float* y,
                  const spx_bcast_params* p) {
  SPX_G(g);
  if (!a || !b || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "binary: null argument");
  return launch_binary(g->stream, &g->launches, op, a, b, y, p);
}

int spx_op_dw_project_nhwc(spx_graph* g, const float* x, const float* w_dw, const float* b_dw,
                           const float* w_proj_hi, const float* w_proj_lo, const float* b_proj,
                           const float* residual, float* y, const spx_dwproj_params* p) {
  SPX_G(g);
  return launch_dw_project(g->stream, &g->launches, x, w_dw, b_dw, w_proj_hi, w_proj_lo, b_proj,
                           residual, y, p, false);
}

int spx_op_stem_conv_nhwc(spx_graph* g, const float* x, const float* w_hi, const float* w_lo,
                          const float* bias, float* y, const spx_conv_params* p) {
  SPX_G(g);
  return launch_stem_tc(g->stream, &g->launches, x, w_hi, w_lo, bias, y, p, false);
}

int spx_stem_conv_supported(const spx_conv_params* p) {
  return launch_stem_tc(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, p, true) ==
                 SPX_OK
             ? 1
             : 0;
}

int spx_dw_project_supported(const spx_dwproj_params* p) {
  return launch_dw_project(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                           nullptr, nullptr, nullptr, p, true) == SPX_OK
             ? 1
             : 0;
}

int spx_op_select(spx_graph* g, const float* pred, const float* a, const float* b, float* y,
                  const spx_select_params* p) {
  SPX_G(g);
  if (!pred || !a || !b || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "select: null argument");
  return launch_select(g->stream, &g->launches, pred, a, b, y, p);
}

int spx_op_reduce_rank4(spx_graph* g, const float* x, float* y, const int32_t push[15]) {
  SPX_G(g);
  if (!x || !y || !push) return fail(SPX_ERR_INVALID_ARGUMENT, "reduce: null argument");
  return launch_reduce_rank4(g->stream, &g->launches, x, y, push);
}

int spx_op_layernorm(spx_graph* g, const float* x, const float* residual, float* x_out,
                     const float* gamma, const float* beta, float* y, int32_t rows, int32_t cols,
                     float eps) {
  SPX_G(g);
  if (!x || !gamma || !beta || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "layernorm: null");
  return launch_layernorm(g->stream, &g->launches, x, residual, x_out, gamma, beta, y, rows, cols,
                          eps);
}

int spx_op_rmsnorm(spx_graph* g, const float* x, const float* gamma, float* y, int32_t rows,
                   int32_t cols, float eps) {
  SPX_G(g);
  if (!x || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "rmsnorm: null");
  return launch_rmsnorm(g->stream, &g->launches, x, gamma, y, rows, cols, eps);
}

int spx_op_rope(spx_graph* g, float* x, const int32_t* positions, int32_t tokens, int32_t heads,
                int32_t head_dim, float theta) {
  SPX_G(g);
  if (!x || !positions) return fail(SPX_ERR_INVALID_ARGUMENT, "rope: null");
  return launch_rope(g->stream, &g->launches, x, positions, tokens, heads, head_dim, theta);
}

int spx_op_embedding(spx_graph* g, const float* table, const int32_t* ids, float* y,
                     int32_t tokens, int32_t dim) {
  SPX_G(g);
  if (!table || !ids || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "embedding: null");
  return launch_embedding(g->stream, &g->launches, table, ids, y, tokens, dim);
}

int spx_op_argmax_rows(spx_graph* g, const float* x, int32_t* idx, float* val, int32_t rows,
                       int32_t cols) {
  SPX_G(g);
  if (!x || !idx) return fail(SPX_ERR_INVALID_ARGUMENT, "argmax: null");
  return launch_argmax_rows(g->stream, &g->launches, x, idx, val, rows, cols);
}

int spx_op_rope_kv_append(spx_graph* g, const float* qkv, int64_t ld_qkv, const float* cos_table,
                          const float* sin_table, const int32_t* state, float* q_out,
                          float* k_cache, float* v_cache, const spx_kv_params* p) {
  SPX_G(g);
  if (!qkv || !cos_table || !sin_table || !state || !q_out || !k_cache || !v_cache || !p)
    return fail(SPX_ERR_INVALID_ARGUMENT, "rope_kv_append: null");
  return launch_rope_kv_append(g->stream, &g->launches, qkv, ld_qkv, cos_table, sin_table, state,
                               q_out, k_cache, v_cache, p->batch, p->q_len, p->q_heads,
                               p->kv_heads, p->head_dim, p->max_seq);
}

int spx_op_attention_kv(spx_graph* g, const float* q, const float* k_cache, const float* v_cache,
                        float* out, const int32_t* state, const spx_kv_params* p, float scale) {
  SPX_G(g);
  if (!q || !k_cache || !v_cache || !out || !state || !p)
    return fail(SPX_ERR_INVALID_ARGUMENT, "attention_kv: null");
  return launch_attention_kv(g->stream, &g->launches, q, k_cache, v_cache, out, state, p->batch,
                             p->q_len, p->q_heads, p->kv_heads, p->head_dim, p->max_seq, scale);
}

int spx_op_swiglu_linear(spx_graph* g, const float* a, int64_t lda, const float* w, int64_t ldw,
                         int32_t m, int32_t f, int32_t k, float rms_eps, float* c, int64_t ldc) {
  SPX_G(g);
  if (!a || !w || !c) return fail(SPX_ERR_INVALID_ARGUMENT, "swiglu_linear: null");
  if (f <= 0 || ldc < f) return fail(SPX_ERR_INVALID_ARGUMENT, "swiglu_linear: bad shape");
  return launch_gemm_rows(g->stream, &g->launches, a, lda, w, ldw, m, f, k, nullptr, nullptr, c,
                          ldc, 1.0f, SPX_ACT_NONE, (int64_t)f, rms_eps < 0 ? -1.0f : rms_eps);
}

int spx_op_rms_linear(spx_graph* g, const float* x, int64_t ldx, const float* w, int64_t ldw,
                      int32_t m, int32_t n, int32_t k, float rms_eps, const float* residual,
                      float* c, int64_t ldc, uint64_t* argmax_keys) {
  SPX_G(g);
  if (!x || !w || !c) return fail(SPX_ERR_INVALID_ARGUMENT, "rms_linear: null");
  if (n <= 0 || ldc < n) return fail(SPX_ERR_INVALID_ARGUMENT, "rms_linear: bad shape");
  return launch_gemm_rows(g->stream, &g->launches, x, ldx, w, ldw, m, n, k, nullptr, residual, c,
                          ldc, 1.0f, SPX_ACT_NONE, 0, rms_eps < 0 ? -1.0f : rms_eps,
                          reinterpret_cast<unsigned long long*>(argmax_keys));
}

int spx_op_swiglu_rows(spx_graph* g, const float* gu, int64_t ld, float* y, int64_t ldy,
                       int32_t rows, int32_t f) {
  SPX_G(g);
  if (!gu || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "swiglu_rows: null");
  return launch_swiglu_rows(g->stream, &g->launches, gu, ld, y, ldy, rows, f);
}

int spx_op_token_commit(spx_graph* g, int32_t* ids, int32_t* hist, int32_t* state,
                        int32_t batch, int32_t advance, int32_t hist_cap, uint64_t* argmax_keys) {
  SPX_G(g);
  if (!ids || !hist || !state) return fail(SPX_ERR_INVALID_ARGUMENT, "token_commit: null");
  return launch_token_commit(g->stream, &g->launches, ids, hist, state, batch, advance, hist_cap,
                             reinterpret_cast<unsigned long long*>(argmax_keys));
}

int spx_op_argmax_partial(spx_graph* g, const float* x, int64_t ldx, int32_t rows, int32_t cols,
                          int32_t col_offset, float* packed) {
  SPX_G(g);
  if (!x || !packed) return fail(SPX_ERR_INVALID_ARGUMENT, "argmax_partial: null");
  return launch_argmax_partial(g->stream, &g->launches, x, ldx, rows, cols, col_offset, packed);
}

int spx_op_argmax_merge(spx_graph* g, const float* packed, int32_t parts, int32_t rows,
                        int32_t* ids) {
  SPX_G(g);
  if (!packed || !ids) return fail(SPX_ERR_INVALID_ARGUMENT, "argmax_merge: null");
  return launch_argmax_merge(g->stream, &g->launches, packed, parts, rows, ids);
}

int spx_op_expand_dw_nhwc(spx_graph* g, const float* x, const float* w_expand,
                          const float* b_expand, const float* w_dw, const float* b_dw, float* y,
                          const spx_expand_dw_params* p) {
  SPX_G(g);
  return launch_expand_dw(g->stream, &g->launches, x, w_expand, b_expand, w_dw, b_dw, y, p);
}

int spx_op_expand_dw_nhwc_split(spx_graph* g, const float* x, const float* w_expand,
                                const float* w_expand_hi, const float* w_expand_lo,
                                const float* b_expand, const float* w_dw, const float* b_dw,
                                float* y, const spx_expand_dw_params* p) {
  SPX_G(g);
  if (g_gemm_path != 1) {
    const int rc = launch_expand_dw_tc(g->stream, &g->launches, x, w_expand_hi, w_expand_lo,
                                       b_expand, w_dw, b_dw, y, p);
    if (rc != -1) return rc;
  }
  if (!w_expand) return fail(SPX_ERR_UNSUPPORTED, "expand_dw: shape not covered by the tensor-core path");
  return launch_expand_dw(g->stream, &g->launches, x, w_expand, b_expand, w_dw, b_dw, y, p);
}

int spx_op_swiglu(spx_graph* g, const float* gate, const float* up, float* y, int64_t n) {
  SPX_G(g);
  if (!gate || !up || !y) return fail(SPX_ERR_INVALID_ARGUMENT, "swiglu: null");
  return launch_swiglu(g->stream, &g->launches, gate, up, y, n);
}

int spx_op_pad4(spx_graph* g, const float* x, float* y, float pad_value, const int32_t push[13]) {
  SPX_G(g);
  if (!x || !y || !push) return fail(SPX_ERR_INVALID_ARGUMENT, "pad: null");
  return launch_pad4(g->stream, &g->launches, x, y, pad_value, push);
}

int spx_op_transpose4(spx_graph* g, const float* x, float* y, const int32_t push[13]) {
  SPX_G(g);
  if (!x || !y || !push) return fail(SPX_ERR_INVALID_ARGUMENT, "transpose: null");
  return launch_transpose4(g->stream, &g->launches, x, y, push);
}

}  // extern "C"
