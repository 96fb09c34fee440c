// ORACLE — test infrastructure only.  Nothing in the product library links,
// loads or calls this file; only tests/, __graft_entry__.smoke() and the
// bench's CPU-baseline leg use it, as the checker.
//
// A plain C++ restatement of the reference's per-op kernels
// (kernels/<name>/glsl/<name>.comp of agkdc1/SPIRV_INFERENCE) for the CPU.
// Each GLSL `main()` becomes a loop over the invocation index `idx` with the
// same per-output loop order and fp32 accumulation; push constants are read
// in the registry order of source/tflite_loader/src/kernels.rs:12-238 and the
// HLO lowerings of source/xla_hlo/src/compiler.rs:768-1135.  The entry point
// has the same shape as the device boundary (spx_run_kernel) so tests run the
// same dispatch sequence on both.
//
// Parallelism: OpenMP over output elements (each output is computed by one
// iteration exactly as one GLSL invocation would, so results do not depend
// on the thread count).  Built with -ffp-contract=off so every `acc += a*b`
// rounds the product and the sum separately.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <string>

extern "C" {

static inline float glsl_max(float a, float b) { return fmaxf(a, b); }
static inline float glsl_min(float a, float b) { return fminf(a, b); }

// ---- unary / binary (kernels/<op>/glsl/<op>.comp) --------------------------
static float unary(const std::string& k, float x, float alpha) {
  if (k == "abs") return fabsf(x);                                  // abs.comp
  if (k == "exp") return expf(x);                                   // exp.comp
  if (k == "log") return logf(x);                                   // log.comp
  if (k == "neg") return -x;                                        // neg.comp
  if (k == "sqrt") return sqrtf(x);                                 // sqrt.comp
  if (k == "rsqrt") return 1.0f / sqrtf(x);                         // rsqrt.comp (inversesqrt)
  if (k == "sigmoid" || k == "logistic") return 1.0f / (1.0f + expf(-x));  // sigmoid.comp
  if (k == "tanh") {                                                // tanh.comp
    float c = fminf(fmaxf(x, -20.0f), 20.0f);
    float ex = expf(c), enx = expf(-c);
    return (ex - enx) / (ex + enx);
  }
  if (k == "relu") return x > 0.0f ? x : 0.0f;                      // relu.comp max(x, 0.0)
  if (k == "relu6") return glsl_min(x > 0.0f ? x : 0.0f, 6.0f);     // relu6.comp:15
  if (k == "leaky_relu") return glsl_max(alpha * x, x);             // leaky_relu.comp
  if (k == "sine") return sinf(x);                                  // sine.comp
  return x;                                                         // reshape.comp (copy)
}

static int binary_kind(const std::string& k) {
  if (k == "add") return 0;
  if (k == "sub") return 1;
  if (k == "mul") return 2;
  if (k == "div") return 3;
  if (k == "pow") return 4;
  if (k == "min") return 5;
  if (k == "max") return 6;
  return -1;
}
static float binary(int op, float a, float b) {
  switch (op) {
    case 0: return a + b;        // add.comp:15
    case 1: return a - b;        // sub.comp
    case 2: return a * b;        // mul.comp
    case 3: return a / b;        // div.comp
    case 4: return powf(a, b);   // pow.comp
    case 5: return glsl_min(a, b);
    default: return glsl_max(a, b);
  }
}

static bool is_unary(const std::string& k) {
  static const char* names[] = {"abs", "exp", "log", "neg", "sqrt", "rsqrt", "sigmoid",
                                "logistic", "tanh", "relu", "relu6", "leaky_relu", "sine",
                                "reshape"};
  for (const char* n : names)
    if (k == n) return true;
  return false;
}

// conv2d.comp:26-50 (NCHW, OIHW weights followed by oc biases).
static void conv2d(const float* in, const float* w, float* out, const int32_t* q) {
  const int n_ = q[0], IC = q[1], IH = q[2], IW = q[3], OC = q[4], OH = q[5], OW = q[6],
            KH = q[7], KW = q[8], SH = q[9], SW = q[10], PT = q[12], PL = q[13];
  const int64_t total = q[14];
  (void)n_;
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int w_ = (int)(idx % OW);
    int h = (int)((idx / OW) % OH);
    int oc = (int)((idx / ((int64_t)OW * OH)) % OC);
    int64_t n = idx / ((int64_t)OW * OH * OC);
    float acc = w[(int64_t)OC * IC * KH * KW + oc];
    for (int ic = 0; ic < IC; ++ic)
      for (int kh = 0; kh < KH; ++kh) {
        int ih = h * SH + kh - PT;
        if (ih < 0 || ih >= IH) continue;
        for (int kw = 0; kw < KW; ++kw) {
          int iw = w_ * SW + kw - PL;
          if (iw < 0 || iw >= IW) continue;
          acc += in[((n * IC + ic) * IH + ih) * IW + iw] * w[(((int64_t)oc * IC + ic) * KH + kh) * KW + kw];
        }
      }
    out[idx] = acc;
  }
}

// depthwise_conv2d.comp:27-49 (NCHW, [c][kh][kw] weights then c biases).
static void depthwise(const float* in, const float* w, float* out, const int32_t* q) {
  const int C = q[1], IH = q[2], IW = q[3], OH = q[4], OW = q[5], KH = q[6], KW = q[7],
            SH = q[8], SW = q[9], PT = q[11], PL = q[12], DH = q[13], DW = q[14];
  const int64_t total = q[15];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int w_ = (int)(idx % OW);
    int h = (int)((idx / OW) % OH);
    int c = (int)((idx / ((int64_t)OW * OH)) % C);
    int64_t n = idx / ((int64_t)OW * OH * C);
    float acc = w[(int64_t)C * KH * KW + c];
    for (int kh = 0; kh < KH; ++kh) {
      int ih = h * SH + kh * DH - PT;
      if (ih < 0 || ih >= IH) continue;
      for (int kw = 0; kw < KW; ++kw) {
        int iw = w_ * SW + kw * DW - PL;
        if (iw < 0 || iw >= IW) continue;
        acc += in[((n * C + c) * IH + ih) * IW + iw] * w[((int64_t)c * KH + kh) * KW + kw];
      }
    }
    out[idx] = acc;
  }
}

// fully_connected.comp:15-28 ([out][in] weights then out biases).
static void fully_connected(const float* in, const float* w, float* out, const int32_t* q) {
  const int I = q[1], O = q[2];
  const int64_t total = q[3];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int oc = (int)(idx % O);
    int64_t b = idx / O;
    float acc = w[(int64_t)O * I + oc];
    for (int i = 0; i < I; ++i) acc += in[b * I + i] * w[(int64_t)oc * I + i];
    out[idx] = acc;
  }
}

// hlo_conv_nhwc_hwio.comp:25-49 (no bias; loop order ky, kx, ic).
static void hlo_conv(const float* in, const float* w, float* out, const int32_t* q) {
  const int IH = q[1], IW = q[2], IC = q[3], KH = q[4], KW = q[5], OC = q[6], OH = q[7],
            OW = q[8], SH = q[9], SW = q[10], PT = q[11], PL = q[12];
  const int64_t total = q[13];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int oc = (int)(idx % OC);
    int x = (int)((idx / OC) % OW);
    int y = (int)((idx / ((int64_t)OC * OW)) % OH);
    int64_t b = idx / ((int64_t)OC * OW * OH);
    float acc = 0.0f;
    for (int ky = 0; ky < KH; ++ky) {
      int iy = y * SH + ky - PT;
      if (iy < 0 || iy >= IH) continue;
      for (int kx = 0; kx < KW; ++kx) {
        int ix = x * SW + kx - PL;
        if (ix < 0 || ix >= IW) continue;
        const float* ip = in + ((b * IH + iy) * IW + ix) * IC;
        const float* wp = w + ((int64_t)(ky * KW + kx) * IC) * OC + oc;
        for (int ic = 0; ic < IC; ++ic) acc += ip[ic] * wp[(int64_t)ic * OC];
      }
    }
    out[idx] = acc;
  }
}

// hlo_dot_rank2.comp:15-26 and hlo_dot_batched.comp:19-38.
static void dot_batched(const float* a, const float* b, float* out, int B, int M, int K, int N) {
  const int64_t total = (int64_t)B * M * N;
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int64_t mn = (int64_t)M * N;
    int64_t bb = idx / mn, rem = idx % mn;
    int64_t row = rem / N, col = rem % N;
    const float* lp = a + bb * M * K + row * K;
    const float* rp = b + bb * (int64_t)K * N + col;
    float acc = 0.0f;
    for (int kk = 0; kk < K; ++kk) acc += lp[kk] * rp[(int64_t)kk * N];
    out[idx] = acc;
  }
}

// hlo_reduce_rank4.comp:44-79.
static void reduce_rank4(const float* in, float* out, const int32_t* q) {
  const int rank = q[0];
  const int d[4] = {q[1], q[2], q[3], q[4]};
  const int od[4] = {q[5], q[6], q[7], q[8]};
  const int r[4] = {q[9], q[10], q[11], q[12]};
  const int kind = q[13];
  const int64_t total = q[14];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int oc[4] = {0, 0, 0, 0};
    int64_t tmp = idx;
    for (int axis = rank - 1; axis >= 0; --axis)
      if (r[axis] == 0) {
        int dim = od[axis] > 1 ? od[axis] : 1;
        oc[axis] = (int)(tmp % dim);
        tmp /= dim;
      }
    float acc = kind == 1 ? -3.4028234663852886e+38f : 0.0f;
    for (int a0 = 0; a0 < (r[0] ? d[0] : 1); ++a0)
      for (int a1 = 0; a1 < (r[1] ? d[1] : 1); ++a1)
        for (int a2 = 0; a2 < (r[2] ? d[2] : 1); ++a2)
          for (int a3 = 0; a3 < (r[3] ? d[3] : 1); ++a3) {
            int c0 = r[0] ? a0 : oc[0], c1 = r[1] ? a1 : oc[1];
            int c2 = r[2] ? a2 : oc[2], c3 = r[3] ? a3 : oc[3];
            float v = in[(((int64_t)c0 * d[1] + c1) * d[2] + c2) * d[3] + c3];
            acc = kind == 1 ? glsl_max(acc, v) : acc + v;
          }
    out[idx] = acc;
  }
}

// hlo_reduce_window_rank4.comp:25-49 (NHWC).
static void reduce_window(const float* in, float* out, const int32_t* q) {
  const int IH = q[1], IW = q[2], C = q[3], OH = q[4], OW = q[5], WH = q[6], WW = q[7],
            SH = q[8], SW = q[9], PT = q[10], PL = q[11], kind = q[12];
  const int64_t total = q[13];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int ch = (int)(idx % C);
    int ox = (int)((idx / C) % OW);
    int oy = (int)((idx / ((int64_t)C * OW)) % OH);
    int64_t b = idx / ((int64_t)C * OW * OH);
    float acc = kind == 1 ? -3.4028234663852886e+38f : 0.0f;
    for (int ky = 0; ky < WH; ++ky) {
      int iy = oy * SH + ky - PT;
      if (iy < 0 || iy >= IH) continue;
      for (int kx = 0; kx < WW; ++kx) {
        int ix = ox * SW + kx - PL;
        if (ix < 0 || ix >= IW) continue;
        float v = in[((b * IH + iy) * IW + ix) * C + ch];
        acc = kind == 1 ? glsl_max(acc, v) : acc + v;
      }
    }
    out[idx] = acc;
  }
}

// max_pool2d.comp:25-44 (NCHW).
static void max_pool2d(const float* in, float* out, const int32_t* q) {
  const int C = q[1], IH = q[2], IW = q[3], OH = q[4], OW = q[5], KH = q[6], KW = q[7],
            SH = q[8], SW = q[9], PT = q[11], PL = q[12];
  const int64_t total = q[13];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int ow = (int)(idx % OW);
    int oh = (int)((idx / OW) % OH);
    int c = (int)((idx / ((int64_t)OW * OH)) % C);
    int64_t n = idx / ((int64_t)OW * OH * C);
    float best = -3.402823466e+38f;
    for (int kh = 0; kh < KH; ++kh) {
      int ih = oh * SH + kh - PT;
      if (ih < 0 || ih >= IH) continue;
      for (int kw = 0; kw < KW; ++kw) {
        int iw = ow * SW + kw - PL;
        if (iw < 0 || iw >= IW) continue;
        best = glsl_max(best, in[((n * C + c) * IH + ih) * IW + iw]);
      }
    }
    out[idx] = best;
  }
}

// softmax10.comp:8-20 / softmax1000.comp:10-22 (row 0 only, like the shaders).
static void softmax_row(const float* in, float* out, int classes) {
  float m = in[0];
  for (int j = 1; j < classes; ++j) m = glsl_max(m, in[j]);
  float sum = 0.0f;
  for (int j = 0; j < classes; ++j) sum += expf(in[j] - m);
  for (int i = 0; i < classes; ++i) out[i] = expf(in[i] - m) / sum;
}

// pad.comp (rank 4, binding 1 holds the pad value).
static void pad4(const float* in, float pv, float* out, const int32_t* q) {
  const int od1 = q[1], od2 = q[2], od3 = q[3];
  const int id0 = q[4], id1 = q[5], id2 = q[6], id3 = q[7];
  const int pl0 = q[8], pl1 = q[9], pl2 = q[10], pl3 = q[11];
  const int64_t total = q[12];
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < total; ++i) {
    int64_t os1 = (int64_t)od2 * od3, os0 = od1 * os1;
    int c0 = (int)(i / os0), c1 = (int)((i / os1) % od1), c2 = (int)((i / od3) % od2),
        c3 = (int)(i % od3);
    int s0 = c0 - pl0, s1 = c1 - pl1, s2 = c2 - pl2, s3 = c3 - pl3;
    if (s0 >= 0 && s0 < id0 && s1 >= 0 && s1 < id1 && s2 >= 0 && s2 < id2 && s3 >= 0 && s3 < id3)
      out[i] = in[(int64_t)s0 * id1 * id2 * id3 + (int64_t)s1 * id2 * id3 + (int64_t)s2 * id3 + s3];
    else
      out[i] = pv;
  }
}

// transpose.comp (13 push constants; output axis k takes input axis p_k).
static void transpose4(const float* in, float* out, const int32_t* q) {
  const int in1 = q[1], in2 = q[2], in3 = q[3], o1 = q[5], o2 = q[6], o3 = q[7];
  const int axes[4] = {q[8], q[9], q[10], q[11]};
  const int64_t total = q[12];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int v3 = (int)(idx % o3), v2 = (int)((idx / o3) % o2), v1 = (int)((idx / ((int64_t)o3 * o2)) % o1);
    int v0 = (int)(idx / ((int64_t)o3 * o2 * o1));
    int vals[4] = {v0, v1, v2, v3};
    int i[4] = {0, 0, 0, 0};
    for (int k = 0; k < 4; ++k) i[axes[k]] = vals[k];
    out[idx] = in[(((int64_t)i[0] * in1 + i[1]) * in2 + i[2]) * in3 + i[3]];
  }
}

// resize_bilinear.comp (NCHW).
static float src_coord(int o, int in_size, int out_size, int ac, int hp) {
  if (ac != 0 && out_size > 1) return (float)o * (float)(in_size - 1) / (float)(out_size - 1);
  if (hp != 0) return ((float)o + 0.5f) * (float)in_size / (float)out_size - 0.5f;
  return (float)o * (float)in_size / (float)out_size;
}
static float mix(float a, float b, float t) { return a * (1.0f - t) + b * t; }
static void resize_bilinear(const float* in, float* out, const int32_t* q) {
  const int IH = q[2], IW = q[3], OH = q[4], OW = q[5], ac = q[6], hp = q[7];
  const int64_t total = q[8];
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; ++idx) {
    int ow = (int)(idx % OW), oh = (int)((idx / OW) % OH);
    int64_t nc = idx / ((int64_t)OW * OH);
    float iy = fminf(fmaxf(src_coord(oh, IH, OH, ac, hp), 0.0f), (float)(IH - 1));
    float ix = fminf(fmaxf(src_coord(ow, IW, OW, ac, hp), 0.0f), (float)(IW - 1));
    int y0 = (int)floorf(iy), x0 = (int)floorf(ix);
    int y1 = y0 + 1 < IH - 1 ? y0 + 1 : IH - 1, x1 = x0 + 1 < IW - 1 ? x0 + 1 : IW - 1;
    float yl = iy - (float)y0, xl = ix - (float)x0;
    const float* base = in + nc * IH * IW;
    float top = mix(base[y0 * IW + x0], base[y0 * IW + x1], xl);
    float bot = mix(base[y1 * IW + x0], base[y1 * IW + x1], xl);
    out[idx] = mix(top, bot, yl);
  }
}

// Returns 0 on success, 2 for an unknown kernel, 1 for inconsistent sizes.
int oracle_run_kernel(const char* kernel, const float* in0, size_t n0, const float* in1,
                      size_t n1, float* out, size_t nout, const int32_t* push, size_t npush) {
  std::string k = kernel ? kernel : "";
  if (k.size() > 4 && k.compare(k.size() - 4, 4, ".spv") == 0) k.resize(k.size() - 4);
  (void)n0;
  (void)n1;
  const int32_t* q = push;
  if (is_unary(k)) {
    if (npush < 1 || (size_t)q[0] > nout || (size_t)q[0] > n0) return 1;
    float alpha = 0.0f;
    if (k == "leaky_relu") memcpy(&alpha, &q[1], 4);
    const int64_t total = q[0];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) out[i] = unary(k, in0[i], alpha);
    return 0;
  }
  int b = binary_kind(k);
  if (b >= 0) {
    if (npush < 1 || (size_t)q[0] > nout || (size_t)q[0] > n0 || (size_t)q[0] > n1) return 1;
    const int64_t total = q[0];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) out[i] = binary(b, in0[i], in1[i]);
    return 0;
  }
  if (k == "concat") {  // concat.comp
    for (int64_t i = 0; i < q[1]; ++i) out[i] = i < q[0] ? in0[i] : in1[i - q[0]];
    return 0;
  }
  if (k == "conv2d") { conv2d(in0, in1, out, q); return 0; }
  if (k == "depthwise_conv2d") { depthwise(in0, in1, out, q); return 0; }
  if (k == "fully_connected") { fully_connected(in0, in1, out, q); return 0; }
  if (k == "hlo_conv_nhwc_hwio") { hlo_conv(in0, in1, out, q); return 0; }
  if (k == "hlo_dot_rank2") { dot_batched(in0, in1, out, 1, q[0], q[1], q[2]); return 0; }
  if (k == "hlo_dot_batched") { dot_batched(in0, in1, out, q[0], q[1], q[2], q[3]); return 0; }
  if (k == "hlo_reduce_rank4") { reduce_rank4(in0, out, q); return 0; }
  if (k == "hlo_reduce_window_rank4") { reduce_window(in0, out, q); return 0; }
  if (k == "max_pool2d") { max_pool2d(in0, out, q); return 0; }
  if (k == "global_avg_pool_sum") {  // global_avg_pool_sum.comp:15-28
    const int64_t nc = (int64_t)q[0] * q[1];
    const int hw = q[2] * q[3];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nc; ++i) {
      float acc = 0.0f;
      for (int j = 0; j < hw; ++j) acc += in0[i * hw + j];
      out[i] = acc;
    }
    return 0;
  }
  if (k == "global_avg_pool_finalize") {  // global_avg_pool_finalize.comp:15-19
    const int64_t nc = (int64_t)q[0] * q[1];
    for (int64_t i = 0; i < nc; ++i) out[i] = in0[i] / (float)(q[2] * q[3]);
    return 0;
  }
  if (k == "softmax10") { softmax_row(in0, out, 10); return 0; }
  if (k == "softmax1000") { softmax_row(in0, out, q[0]); return 0; }
  if (k == "pad") { pad4(in0, n1 ? in1[0] : 0.0f, out, q); return 0; }
  if (k == "transpose") { transpose4(in0, out, q); return 0; }
  if (k == "l2norm") {  // l2norm.comp
    float norm;
    memcpy(&norm, &q[1], 4);
    float d = fmaxf(norm, 1.0e-12f);
    for (int64_t i = 0; i < q[0]; ++i) out[i] = in0[i] / d;
    return 0;
  }
  if (k == "resize_bilinear") { resize_bilinear(in0, out, q); return 0; }
  return 2;
}

int oracle_num_threads(void);
}

#ifdef _OPENMP
#include <omp.h>
int oracle_num_threads(void) { return omp_get_max_threads(); }
extern "C" void oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
#else
extern "C" void oracle_set_threads(int n) { (void)n; }
int oracle_num_threads(void) { return 1; }
#endif
