// Internal declarations shared by the libspx translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <vector>

#include "spx.h"

// Graph object behind the opaque `spx_graph*` handle.
struct spx_graph {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  std::vector<void*> buffers;
  cudaGraph_t cuda_graph = nullptr;
  cudaGraphExec_t cuda_exec = nullptr;
  bool capturing = false;
  int64_t launches = 0;          // kernels launched (or replayed)
  int64_t captured_launches = 0; // kernels inside the captured CUDA graph
  int64_t capture_start = 0;
};

namespace spx {

constexpr int kNumSms = 148;  // B200: 2 dies x 74 SMs

// Thread-local error reporting.  `fail` records a message and returns code.
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
// Checks the launch that was just issued and bumps the launch counter.
int after_launch(int64_t* counter, const char* what);

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the previous kernel on the stream is still running (on SMs that
// kernel has left); it must call pdl_wait() before its first access to global
// memory that an earlier kernel writes or reads (the wait returns once every
// earlier kernel has completed and its writes are visible).  pdl_trigger()
// lets the next PDL launch begin as soon as every CTA of this grid has
// called it.  Option "pdl" (default 1); 0 = plain launches.
extern int g_pdl;
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int grid_for(int64_t work, int threads, int per_sm = 8) {
  int64_t g = ceil_div(work, threads);
  int64_t cap = (int64_t)kNumSms * per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

// Epilogue activation (SPX_ACT_* codes), shared by every fused epilogue.
__device__ __forceinline__ float apply_act(int act, float v) {
  switch (act) {
    case SPX_ACT_RELU: return v > 0.0f ? v : 0.0f;
    case SPX_ACT_RELU6: return fminf(v > 0.0f ? v : 0.0f, 6.0f);
    case SPX_ACT_RELU_N1_TO_1: return fminf(fmaxf(v, -1.0f), 1.0f);
    case SPX_ACT_TANH: return tanhf(v);
    case SPX_ACT_GELU_ERF: return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    case SPX_ACT_GELU_TANH: {
      float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
      return 0.5f * v * (1.0f + tanhf(u));
    }
    case SPX_ACT_SILU: return v / (1.0f + expf(-v));
    default: return v;
  }
}

// Compile-time activation: epilogues dispatch on the runtime code once per
// tile or chunk (with_act) so the per-element code is a single specialised
// expression instead of a multi-way branch over every activation.
template <int A>
__device__ __forceinline__ float act_c(float v) {
  if constexpr (A == SPX_ACT_RELU) return v > 0.0f ? v : 0.0f;
  else if constexpr (A == SPX_ACT_RELU6) return fminf(v > 0.0f ? v : 0.0f, 6.0f);
  else if constexpr (A == SPX_ACT_RELU_N1_TO_1) return fminf(fmaxf(v, -1.0f), 1.0f);
  else if constexpr (A == SPX_ACT_TANH) return tanhf(v);
  else if constexpr (A == SPX_ACT_GELU_ERF) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  else if constexpr (A == SPX_ACT_GELU_TANH) {
    float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(u));
  } else if constexpr (A == SPX_ACT_SILU) return v / (1.0f + expf(-v));
  else return v;
}
template <int A>
struct ActTag {
  static constexpr int value = A;
};
template <class F>
__device__ __forceinline__ void with_act(int act, F&& f) {
  switch (act) {
    case SPX_ACT_RELU: f(ActTag<SPX_ACT_RELU>{}); break;
    case SPX_ACT_RELU6: f(ActTag<SPX_ACT_RELU6>{}); break;
    case SPX_ACT_RELU_N1_TO_1: f(ActTag<SPX_ACT_RELU_N1_TO_1>{}); break;
    case SPX_ACT_TANH: f(ActTag<SPX_ACT_TANH>{}); break;
    case SPX_ACT_GELU_ERF: f(ActTag<SPX_ACT_GELU_ERF>{}); break;
    case SPX_ACT_GELU_TANH: f(ActTag<SPX_ACT_GELU_TANH>{}); break;
    case SPX_ACT_SILU: f(ActTag<SPX_ACT_SILU>{}); break;
    default: f(ActTag<SPX_ACT_NONE>{}); break;
  }
}
// Activation groups: a kernel instantiated once per group holds only its
// group's specialised epilogues (less code in the instruction cache).  Group
// 0: none and the clamps (ReLU, ReLU6, ReLU(-1, 1)); group 1: the
// transcendental ones (tanh, GELU, SiLU).
__host__ __device__ constexpr int act_group(int act) {
  return (act == SPX_ACT_TANH || act == SPX_ACT_GELU_ERF || act == SPX_ACT_GELU_TANH ||
          act == SPX_ACT_SILU)
             ? 1
             : 0;
}
template <int G, class F>
__device__ __forceinline__ void with_act_group(int act, F&& f) {
  if constexpr (G == 0) {
    switch (act) {
      case SPX_ACT_RELU: f(ActTag<SPX_ACT_RELU>{}); break;
      case SPX_ACT_RELU6: f(ActTag<SPX_ACT_RELU6>{}); break;
      case SPX_ACT_RELU_N1_TO_1: f(ActTag<SPX_ACT_RELU_N1_TO_1>{}); break;
      default: f(ActTag<SPX_ACT_NONE>{}); break;
    }
  } else {
    switch (act) {
      case SPX_ACT_TANH: f(ActTag<SPX_ACT_TANH>{}); break;
      case SPX_ACT_GELU_ERF: f(ActTag<SPX_ACT_GELU_ERF>{}); break;
      case SPX_ACT_GELU_TANH: f(ActTag<SPX_ACT_GELU_TANH>{}); break;
      default: f(ActTag<SPX_ACT_SILU>{}); break;
    }
  }
}
// Host-side twin: picks the kernel instantiation for a runtime code.
template <class F>
inline void host_with_act(int act, F&& f) {
  switch (act) {
    case SPX_ACT_RELU: f(ActTag<SPX_ACT_RELU>{}); break;
    case SPX_ACT_RELU6: f(ActTag<SPX_ACT_RELU6>{}); break;
    case SPX_ACT_RELU_N1_TO_1: f(ActTag<SPX_ACT_RELU_N1_TO_1>{}); break;
    case SPX_ACT_TANH: f(ActTag<SPX_ACT_TANH>{}); break;
    case SPX_ACT_GELU_ERF: f(ActTag<SPX_ACT_GELU_ERF>{}); break;
    case SPX_ACT_GELU_TANH: f(ActTag<SPX_ACT_GELU_TANH>{}); break;
    case SPX_ACT_SILU: f(ActTag<SPX_ACT_SILU>{}); break;
    default: f(ActTag<SPX_ACT_NONE>{}); break;
  }
}

// ---- launchers (each returns SPX_OK or an error code) -------------------
// All take the stream to record on and a launch counter (may be null).
int launch_unary(cudaStream_t s, int64_t* cnt, int op, const float* x, float* y, int64_t n,
                 float alpha);
int launch_binary(cudaStream_t s, int64_t* cnt, int op, const float* a, const float* b,
                  float* y, const spx_bcast_params* p);
int launch_select(cudaStream_t s, int64_t* cnt, const float* pr, const float* a, const float* b,
                  float* y, const spx_select_params* p);
// w_hi / w_lo (both or neither): the weights pre-split by launch_weights_split,
// used when the tensor-core path runs; w itself feeds every other path.
int launch_conv_nhwc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                     const float* w_hi, const float* w_lo, const float* bias, const float* res,
                     float* y, const spx_conv_params* p);
int launch_gemm(cudaStream_t s, int64_t* cnt, const float* a, const float* b, const float* b_hi,
                const float* b_lo, const float* bias, const float* res, float* c,
                const spx_gemm_params* p);
int launch_dw_nhwc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* bias, float* y, const spx_dw_params* p);
int launch_pool_nhwc(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                     const spx_pool_params* p);
int launch_gap_nhwc(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n, int hw,
                    int c);
int launch_softmax_rows(cudaStream_t s, int64_t* cnt, const float* x, float* y, int rows,
                        int cols, float scale, int causal, int q_len, int q_offset);
int launch_reduce_rank4(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                        const int32_t* push);
int launch_layernorm(cudaStream_t s, int64_t* cnt, const float* x, const float* res,
                     float* x_out, const float* gamma, const float* beta, float* y, int rows,
                     int cols, float eps);
int launch_rmsnorm(cudaStream_t s, int64_t* cnt, const float* x, const float* gamma, float* y,
                   int rows, int cols, float eps);
int launch_rope(cudaStream_t s, int64_t* cnt, float* x, const int32_t* pos, int tokens,
                int heads, int head_dim, float theta);
int launch_embedding(cudaStream_t s, int64_t* cnt, const float* table, const int32_t* ids,
                     float* y, int tokens, int dim);
int launch_argmax_rows(cudaStream_t s, int64_t* cnt, const float* x, int32_t* idx, float* val,
                       int rows, int cols);
int launch_swiglu(cudaStream_t s, int64_t* cnt, const float* gate, const float* up, float* y,
                  int64_t n);
// Decode path (k_decode.cu).
bool gemm_rows_eligible(const float* a, int64_t lda, const float* w, int64_t ldw, int M, int K);
int launch_gemm_rows(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda, const float* w,
                     int64_t ldw, int M, int N, int K, const float* bias, const float* res,
                     float* c, int64_t ldc, float alpha, int act, int64_t pair_off,
                     float rms_eps = -1.0f, unsigned long long* amax = nullptr);
int launch_rope_kv_append(cudaStream_t s, int64_t* cnt, const float* qkv, int64_t ld_qkv,
                          const float* cos_t, const float* sin_t, const int32_t* pos,
                          float* q_out, float* kc, float* vc, int B, int T, int Hq, int Hkv,
                          int D, int max_seq);
int launch_attention_kv(cudaStream_t s, int64_t* cnt, const float* q, const float* kc,
                        const float* vc, float* out, const int32_t* pos, int B, int T, int Hq,
                        int Hkv, int D, int max_seq, float scale);
int launch_token_commit(cudaStream_t s, int64_t* cnt, int32_t* ids, int32_t* hist,
                        int32_t* state, int B, int advance, int hist_cap,
                        unsigned long long* keys = nullptr);
int launch_argmax_partial(cudaStream_t s, int64_t* cnt, const float* x, int64_t ldx, int rows,
                          int cols, int col_offset, float* packed);
int launch_argmax_merge(cudaStream_t s, int64_t* cnt, const float* packed, int parts, int rows,
                        int32_t* ids);
int launch_swiglu_rows(cudaStream_t s, int64_t* cnt, const float* gu, int64_t ld, float* y,
                       int64_t ldy, int rows, int f);
int launch_pad4(cudaStream_t s, int64_t* cnt, const float* x, float* y, float pad_value,
                const int32_t* push);
int launch_transpose4(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                      const int32_t* push);

// Exact-fp32 SIMT implementations (k_gemm_simt.cu).
int launch_gemm_simt(cudaStream_t s, int64_t* cnt, const float* a, const float* b,
                     const float* bias, const float* res, float* c, const spx_gemm_params* p);
bool pw_simt_eligible(const float* x, const float* y, const float* res, int64_t M, int K, int N);
int launch_pw_simt(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* bias, const float* res, float* y, int64_t M, int K, int N,
                   int act);
int launch_conv_simt(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                     const float* bias, const float* res, float* y, const spx_conv_params* p);

// Direct kernels (k_direct.cu).  Return -1 when the shape is not covered.
int try_dw_rows(cudaStream_t s, int64_t* cnt, const float* x, const float* w, const float* b,
                float* y, const spx_dw_params* p);
int try_conv_smallk(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                    const float* bias, const float* res, float* y, const spx_conv_params* p);

// TMA-tiled depthwise (k_dw_tma.cu); -1 when the shape is not covered.
int try_dw_tma(cudaStream_t s, int64_t* cnt, const float* x, const float* w, const float* b,
               float* y, const spx_dw_params* p);
// Returns and clears the depthwise kernel's device status (1 = a wait timed out).
int dw_take_status();
// Tensor-core variant (k_gemm_tc.cu): -1 when the shape is not covered.
int launch_expand_dw_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* we_hi,
                        const float* we_lo, const float* be, const float* wd, const float* bd,
                        float* y, const spx_expand_dw_params* q);
int launch_expand_dw(cudaStream_t s, int64_t* cnt, const float* x, const float* we,
                     const float* be, const float* wd, const float* bd, float* y,
                     const spx_expand_dw_params* p);

// tcgen05 3xTF32 GEMM (k_gemm_tc.cu): both operands K-contiguous.
bool gemm_tc_eligible(const float* a, int64_t lda, const float* b, int64_t ldb, int M, int N,
                      int K, const float* c, int64_t ldc);
// b_lo != nullptr: B is given pre-split (b = tf32 hi terms, b_lo = lo terms,
// from launch_weights_split); otherwise B is split on chip.
// Implicit-GEMM convolution geometry for launch_gemm_tc (k_gemm_tc.cu).
struct ConvGeom {
  int oh, ow, ic_blocks, kw, sh, pt, pl, th, tw, tn, tiles_h, tiles_w;
};
int launch_gemm_tc(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda, const float* b,
                   const float* b_lo, int64_t ldb, int M, int N, int K, const float* bias,
                   const float* res, float* c, int64_t ldc, float alpha, int act,
                   const ConvGeom* conv = nullptr, const void* conv_map = nullptr,
                   int conv_img_groups = 0);
// KxK / strided convolutions on tensor cores: NHWC input, OHWI weights
// (w_lo non-null: w is the pre-split hi part), ic a multiple of 32.
bool conv_tc_eligible(const float* x, const float* w, const float* y, const spx_conv_params* q);
int launch_conv_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* w_lo, const float* bias, const float* res, float* y,
                   const spx_conv_params* q);
bool gemm_tc_skinny_eligible(const float* a, int64_t lda, const float* w, int64_t ldw, int M,
                             int N, int K);
// w_lo non-null: w is the pre-split hi part (spx_weights_split) and w_lo the lo part.
int launch_gemm_tc_skinny(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda,
                          const float* w, const float* w_lo, int64_t ldw, int M, int N, int K,
                          const float* bias, const float* res, float* c, int64_t ldc,
                          float alpha, int act);
int launch_weights_split(cudaStream_t s, int64_t* cnt, const float* w, float* hi, float* lo,
                         int64_t n);
// Returns and clears the device status of the tensor-core pipeline (0 = ok,
// 1 = a pipeline wait timed out and the kernel aborted its tiles).
int tc_take_status();
int dwp_take_status();
int bg_take_status();
int pw_take_status();
// 1x1 conv / GEMM with a resident activation tile (k_pwgemm.cu): K <= 160,
// N >= 128, pre-split weights, no residual.  -1 when not eligible.
int try_pwgemm(cudaStream_t s, int64_t* cnt, const float* a, const float* w_hi, const float* w_lo,
               const float* bias, const float* res, float* c, int M, int N, int K, int act);
// 1: pointwise convolutions that try_pwgemm takes run there (default 0).
extern int g_pw_gemm;
// Batched 3xTF32 tensor-core GEMM for K <= 128 (k_bgemm.cu): -1 when the
// operands are not eligible (caller falls back), else SPX_OK or an error.
int try_bgemm_tc(cudaStream_t s, int64_t* cnt, const float* a, const float* b, const float* bias,
                 const float* res, float* c, const spx_gemm_params* q);
// Fused depthwise 3x3 -> 1x1 projection (k_dwproj.cu).  dry_run: eligibility
// check only (SPX_OK or SPX_ERR_UNSUPPORTED), nothing launched.
int launch_stem_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* w_hi,
                   const float* w_lo, const float* bias, float* y, const spx_conv_params* q,
                   bool dry_run);
int launch_dw_project(cudaStream_t s, int64_t* cnt, const float* x, const float* wd,
                      const float* bd, const float* w_hi, const float* w_lo, const float* bp,
                      const float* res, float* y, const spx_dwproj_params* q, bool dry_run);
int ar_take_status();

// Process-wide dense-contraction path: 0 auto, 1 SIMT only, 2 tensor cores
// required (ineligible shapes fail with SPX_ERR_UNSUPPORTED).
extern int g_gemm_path;
// Bound of the peer all-reduce's wait for the other ranks, microseconds.
extern int64_t g_ar_wait_limit_us;
extern int g_tc_epi12;
extern int g_dwp_groups;
extern int g_dwp_epi1;    // dw_project tile classes with one epilogue group (bit mask)
extern int g_dwp_accs;    // dw_project / stem TMEM accumulators (2 or 4)
extern int g_dwp_stages;  // dw_project A/B stage count cap (2..4)  // dw_project builder groups per tile class (bit mask)
extern int g_tc_conv2;
extern int g_tc_lo_tmem;
extern int g_tc_cat;  // tensor-core GEMM: concatenated hi/lo weight product for N tiles <= 128
extern int g_tc_acc4; // tensor-core GEMM: four accumulators for one-k-block tiles
// Depthwise path: 0 automatic (TMA tiles where the shape allows), 1 register
// sliding-window kernel only.
extern int g_dw_path;

// ---- reference-layout kernels used only by the drop-in boundary ---------
// (NCHW layouts of the TFLite shader set, one output element per thread.)
int launch_compat_dw_nchw(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                          float* y, const int32_t* push);
int launch_compat_maxpool_nchw(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                               const int32_t* push);
int launch_compat_gap_sum_nchw(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n,
                               int c, int h, int w);
int launch_compat_gap_finalize(cudaStream_t s, int64_t* cnt, const float* x, float* y, int n,
                               int c, int h, int w);
int launch_compat_resize_bilinear(cudaStream_t s, int64_t* cnt, const float* x, float* y,
                                  const int32_t* push);
int launch_compat_l2norm(cudaStream_t s, int64_t* cnt, const float* x, float* y, int total,
                         float norm);
int launch_compat_concat(cudaStream_t s, int64_t* cnt, const float* a, const float* b, float* y,
                         int a_total, int total);

}  // namespace spx
