/*
 * spx.h — C ABI of libspx, the B200 (sm_100a) operator backend for
 * SPIRV_INFERENCE-style graphs.
 *
 * Two layers are exported:
 *
 *  1. The drop-in dispatch boundary, `spx_run_kernel`.  It replaces
 *     `tflite_loader::vulkan::run_kernel(device_selector, &KernelRun) ->
 *     KernelOutput` (source/tflite_loader/src/vulkan.rs:18-44).  Kernels are
 *     named exactly as in the reference registry (source/tflite_loader/src/
 *     kernels.rs:12-238, plus the HLO kernels of source/xla_hlo/src/
 *     compiler.rs:1155-1228: hlo_conv_nhwc_hwio, hlo_dot_rank2,
 *     hlo_dot_batched, hlo_reduce_rank4, hlo_reduce_window_rank4, pad), take
 *     the same two f32 inputs, the same i32 push constants in the same order,
 *     and produce the same output layout.  A ".spv" suffix on the name is
 *     accepted and ignored, so the reference's `dispatch(…, "conv2d.spv", …)`
 *     call sites (source/tflite_loader/src/scheduler.rs:1096-1144) map 1:1.
 *     Host buffers in, host buffer out, synchronous, like the reference.
 *
 *  2. The device-resident graph API (`spx_graph_*`, `spx_buf_*`, `spx_op_*`).
 *     It generalises the create-once / record / submit pattern of
 *     runtime/chained_graph_runtime/src/main.rs:298-547: one CUDA stream per
 *     graph, device allocations made once, ops recorded back to back on the
 *     stream (optionally captured into a CUDA graph and replayed).  Activations
 *     are NHWC; conv weights are OHWI (TFLite's own order, so no repack) or
 *     HWIO (the HLO path's order).
 *
 * Every call returns SPX_OK (0) or an error code; `spx_last_error()` returns a
 * thread-local message for the last failure on the calling thread.  There is
 * no CPU fallback: without a CUDA device every compute call fails with
 * SPX_ERR_NO_DEVICE.
 */
#ifndef SPX_H_
#define SPX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define SPX_OK 0
#define SPX_ERR_INVALID_ARGUMENT 1 /* bad sizes / push constants / null ptr  */
#define SPX_ERR_UNSUPPORTED 2      /* unknown kernel or unsupported feature;
                                      the reference maps this case to
                                      "blocked_unsupported_feature"
                                      (source/tflite_loader/src/main.rs:66-76) */
#define SPX_ERR_CUDA 3             /* a CUDA runtime call failed             */
#define SPX_ERR_OUT_OF_MEMORY 4
#define SPX_ERR_NO_DEVICE 5        /* no CUDA device / bad ordinal           */

/* ---- activations fused into epilogues ---------------------------------- */
/* Numbering follows TFLite's ActivationFunctionType as decoded by
 * source/tflite_loader/src/op_decoder.rs:21-44 (None=0, Relu=1, Relu6=3);
 * values above 15 are spx extensions for the HLO / transformer graphs. */
#define SPX_ACT_NONE 0
#define SPX_ACT_RELU 1
#define SPX_ACT_RELU_N1_TO_1 2
#define SPX_ACT_RELU6 3
#define SPX_ACT_TANH 4
#define SPX_ACT_GELU_ERF 16  /* x * 0.5 * (1 + erf(x / sqrt 2))           */
#define SPX_ACT_GELU_TANH 17 /* tanh approximation of GELU                 */
#define SPX_ACT_SILU 18      /* x * sigmoid(x)                             */

/* ---- library / device info --------------------------------------------- */
const char* spx_last_error(void);
const char* spx_version(void);
/* Number of CUDA devices (0 when none; never fails). */
int spx_device_count(void);
/* Maps the reference's device selector ("any" | "nvidia" | "intel",
 * source/tflite_loader/src/vulkan.rs:204-231) or a decimal ordinal to a CUDA
 * ordinal.  "intel" has no CUDA device and fails with SPX_ERR_NO_DEVICE. */
int spx_select_device(const char* selector, int* ordinal);
/* Compute capability (major * 10 + minor) the library's device code was built
 * for, read through cudaFuncGetAttributes on `device`: 100 for this sm_100a
 * build.  No counterpart in the reference (a build check). */
int spx_binary_version(int device, int* version);
/* Device-side error status of this process's libspx kernels: SPX_OK, or
 * SPX_ERR_CUDA with spx_last_error() naming the wait that ran out (a pipeline
 * or peer wait past its bound).  Reading clears it.  spx_graph_sync and
 * spx_run_kernel check it themselves; callers that enqueue on their own
 * streams (spx_conv2d_nchw_noalloc) call it after synchronising.
 * libspx keeps per-device state (cached buffers, the no-alloc scratch
 * address): do not cudaDeviceReset a device while the library is in use on
 * it. */
int spx_device_status(void);

/* Process-wide options.  "gemm_path": 0 = automatic (tensor cores where the
 * operands allow, exact-fp32 SIMT otherwise), 1 = SIMT only, 2 = tensor cores
 * required (shapes they cannot take fail with SPX_ERR_UNSUPPORTED).
 * "dw_path": 0 = automatic (TMA-tiled depthwise where the shape allows),
 * 1 = the register sliding-window depthwise kernel only.
 * "pw_path": 0 (default) = 1x1 convolutions on the tensor-core GEMM,
 * 1 = short-reduction 1x1 convolutions (K * N <= 8192) on the CUDA-core
 * pointwise kernel instead (exact fp32; slower on B200, kept for checking).
 * "tc_wide_epilogue": 1 (default) = tensor-core GEMMs with one k-block per
 * tile give four converter warps to the epilogue where that saves a round of
 * output chunks, and for N <= 32 split the epilogue into two groups draining
 * alternate tiles; 0 = never.
 * "tc_conv_groups": 2 (default) = tensor-core GEMMs with several k-blocks per
 * tile split two stages at once (two converter groups), 1 = one at a time.
 * "pw_gemm": 1 = pointwise convolutions with pre-split weights, a reduction of
 * at most 160 and at least 128 outputs keep each 128-row activation tile
 * resident (split once for every n tile); 0 (default) = the row-tiled
 * tensor-core GEMM, measured faster on every MobileNetV2 expand layer.
 * "dwp_groups": bit mask over the fused depthwise -> projection kernel's
 * tile classes (bit 0: stride 1, output width <= 8; bit 1: stride 1, wider,
 * more than 32 channels; bit 4: stride 1, wider, at most 32 channels (one K
 * block); bit 2: stride 2, width <= 8; bit 3: stride 2, wider, at most 160
 * channels; bit 5: stride 2, wider, more than 160 channels); a set bit
 * builds the class's depthwise tiles with two builder groups taking
 * alternate K blocks, a clear bit with one group over each K block.  Results
 * are identical either way; default 47 (measured on the MobileNetV2 layers at
 * batch 256: two groups faster everywhere but on the single-K-block layer).
 * "dwp_stages": most A/B operand stages the fused depthwise -> projection
 * kernel uses (2..4, default 4; fewer where shared memory is short).  More
 * stages let the depthwise builders run ahead of the tensor core.  Results
 * are identical for every value.
 * "dwp_accs": 4 (default) = the fused depthwise -> projection kernel and the
 * tensor-core stem keep four TMEM accumulators where they fit (projection
 * width <= 64), so the tensor core can run two tiles ahead of each epilogue
 * group; 2 = two.  Results are identical either way.
 * "dwp_epi1": bit mask over the same tile classes as "dwp_groups"; a set bit
 * runs the class with one epilogue group of four warps (448 threads, up to
 * 128 registers a thread: the depthwise builders keep everything in
 * registers), a clear bit with two groups draining alternate tiles (576
 * threads, 96 registers).  Default 62 (bits 1-5; measured at batch 256 on
 * the MobileNetV2 layers: 56x56x144 -> 24 262 -> 230 us, 112x112x96 stride 2
 * 273 -> 268 us with one group; the 7x7-map class, bit 0, is level or slower
 * with one).  Results are identical either way.
 * "pdl": 1 (default) = the tensor-core GEMM and fused depthwise kernels are
 * launched with programmatic stream serialisation: a launch may start its
 * set-up (barriers, tensor memory, staged bias) on SMs the previous kernel
 * has left and waits for that kernel's completion before touching any
 * activation; 0 = plain launches.  Results are identical either way.
 * "ar_wait_limit_us": bound of the peer all-reduce's wait for the other ranks
 * (default 2,000,000; 1,000 .. 60,000,000).
 * "tc_acc4": 1 (default) = tensor-core GEMM tiles with one k-block (short
 * reductions such as the 1x1 expand convolutions) keep three or four TMEM
 * accumulators (as many as fit, tiles up to 170 columns wide) and issue the
 * three products separately, so the tensor core can run ahead of the
 * epilogue; 0 = two accumulators.
 * "tc_cat": 1 (default) = tensor-core GEMM tiles up to 128 columns wide issue
 * raw A x [B hi; B lo] as one product of twice the width plus lo A x hi B
 * (two wide MMAs instead of three narrow ones per k-step; the epilogue adds
 * the accumulator's two halves); 0 = three products into one accumulator.
 * "tc_lo_tmem": 1 = with pre-split weights and several k-blocks the
 * activations' tf32 lo terms are written to tensor memory and the lo*hi MMA
 * reads its A operand from there; 0 (default) = lo terms in shared memory. */
int spx_set_option(const char* name, int64_t value);
int64_t spx_get_option(const char* name);

/* Diagnostics: the tensor-core GEMM's launch plan for an M x N x K product
 * (no device work; `conv` = implicit-GEMM conv mode, `vec4` = C / residual /
 * bias allow 16-byte access).  out[0..15] = N tile, n tiles, k-blocks,
 * k-steps of the last k-block, ring stages, stage bytes, epilogue warps,
 * converter groups, epilogue groups, TMEM accumulators, TMEM columns,
 * resident weights, dynamic shared memory bytes, m tiles, converter threads,
 * grid, lo terms in tensor memory.  n_out >= 17. */
int spx_gemm_tc_plan(int32_t M, int32_t N, int32_t K, int32_t presplit, int32_t conv,
                     int32_t vec4, int32_t* out, int32_t n_out);

/* ---- kernel registry (mirror of kernels.rs:12-238 + HLO kernels) ------- */
int spx_kernel_count(void);
/* Name of registry entry i (0 <= i < spx_kernel_count()), NULL if out of range. */
const char* spx_kernel_name(int i);
/* Number of i32 push constants kernel `name` expects, or -1 if unknown. */
int spx_kernel_push_count(const char* name);
/* Work-group size the reference dispatches this kernel with (64 or 128). */
int spx_kernel_local_size(const char* name);

/* ---- 1. drop-in dispatch boundary -------------------------------------- */
/* Mirrors `KernelOutput { values, device_name, vendor_id, device_id,
 * elapsed_ms }` (vulkan.rs:18-25) minus `values`, which go to `output`. */
typedef struct spx_kernel_output_info {
  double elapsed_ms;     /* device time of the kernel(s), CUDA events     */
  char device_name[256];
  uint32_t vendor_id;    /* 0x10de                                        */
  uint32_t device_id;    /* PCI device id                                 */
} spx_kernel_output_info;

/* Replaces vulkan::run_kernel (vulkan.rs:42-185).  `kernel` is a registry
 * name or spv file name.  input0/input1 are the reference's bindings 0 and 1,
 * output is binding 2 with `output_elements` floats.  `push` holds the i32
 * push constants in the registry order (floats as bit patterns, e.g.
 * leaky_relu alpha_bits, kernels.rs:92-97).  `info` may be NULL.
 * Device buffers are cached per device and reused between calls (the
 * reference creates and destroys every Vulkan object per call). */
int spx_run_kernel(const char* kernel, const float* input0, size_t input0_len,
                   const float* input1, size_t input1_len, float* output,
                   size_t output_elements, const int32_t* push, size_t push_len,
                   int device, spx_kernel_output_info* info);

/* Allocation-free form of the "conv2d" dispatch above.  No counterpart in
 * the reference: it exists for callers that cannot let a library allocate
 * device memory (hosts whose own pool allocator owns the whole GPU, or
 * latency-critical loops where cudaMalloc's implicit device synchronisation is
 * not acceptable).  x, w and y are caller-owned DEVICE buffers with the
 * reference layouts (x NCHW, w OIHW followed by oc biases, y NCHW); push holds
 * the same 15 push constants as "conv2d".  Work is recorded on `stream`
 * (a cudaStream_t; NULL = legacy default stream) and the call returns without
 * waiting.  The NHWC / OHWI staging lives in one fixed 16 MiB device array
 * inside the library (every GPU that loads libspx holds it until exit);
 * convolutions whose input + weights + output exceed 4 Mi floats are rejected
 * with SPX_ERR_INVALID_ARGUMENT.  The first call on each device looks up the
 * array's device address; make that first call before any stream capture.
 * That address (like the regular dispatch's per-device buffers) is cached
 * for the life of the process: do not reset the device (cudaDeviceReset)
 * while libspx is loaded.
 * All calls share the array: calls that can overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * No cudaMalloc, cudaFree or allocating library routine is called.
 * pad_top / pad_left must lie in [0, kernel extent).  The call only enqueues
 * work: a bounded pipeline wait that ran out inside it is reported by
 * spx_device_status() once the caller has synchronised `stream`. */
int spx_conv2d_nchw_noalloc(const float* x, const float* w, float* y, const int32_t* push,
                            size_t push_len, void* stream);

/* ---- 2. device-resident graph API -------------------------------------- */
typedef struct spx_graph spx_graph;

/* Creates a graph on `device` with its own non-blocking stream. */
int spx_graph_create(int device, spx_graph** out);
/* Same, but records onto a caller-owned cudaStream_t (passed as void*). */
int spx_graph_create_on_stream(int device, void* cuda_stream, spx_graph** out);
int spx_graph_destroy(spx_graph* g);
void* spx_graph_stream(spx_graph* g);
int spx_graph_device(spx_graph* g);
/* Blocks until all work recorded so far has finished; reports async errors. */
int spx_graph_sync(spx_graph* g);
/* Number of spx kernel launches recorded on this graph since creation or the
 * last reset (replays of a captured CUDA graph count their kernels too). */
int64_t spx_graph_launch_count(spx_graph* g);
void spx_graph_reset_launch_count(spx_graph* g);

/* CUDA-graph capture of everything recorded between begin and end. */
int spx_graph_capture_begin(spx_graph* g);
int spx_graph_capture_end(spx_graph* g);
int spx_graph_replay(spx_graph* g);

/* Device buffers owned by the graph (freed by spx_graph_destroy). */
int spx_buf_alloc(spx_graph* g, size_t bytes, void** dptr);
int spx_buf_free(spx_graph* g, void* dptr);
/* Stream-ordered copies; host buffers should be pinned for overlap. */
int spx_buf_upload(spx_graph* g, void* dst_device, const void* src_host, size_t bytes);
int spx_buf_download(spx_graph* g, void* dst_host, const void* src_device, size_t bytes);
int spx_buf_zero(spx_graph* g, void* dst_device, size_t bytes);
/* Stream-ordered device-to-device copy. */
int spx_buf_copy(spx_graph* g, void* dst_device, const void* src_device, size_t bytes);
int spx_host_alloc_pinned(size_t bytes, void** ptr);
int spx_host_free_pinned(void* ptr);

/* -- ops (all pointers are device pointers, NHWC activations) ------------ */

/* Dense convolution, NHWC in and out, as implicit GEMM
 * (M = n*oh*ow, N = oc, K = kh*kw*ic).  Covers the TFLite Conv2D lowering
 * (scheduler.rs:321-427 + conv2d.comp) and the HLO convolution lowering
 * (compiler.rs:768-855 + hlo_conv_nhwc_hwio.comp).  y = act(conv(x, w) +
 * bias + residual); bias and residual may be NULL. */
#define SPX_WEIGHT_OHWI 0 /* [oc][kh][kw][ic]  (TFLite Conv2D)          */
#define SPX_WEIGHT_HWIO 1 /* [kh][kw][ic][oc]  (HLO b01f_01io->b01f)    */
typedef struct spx_conv_params {
  int32_t n, ih, iw, ic, oc, oh, ow, kh, kw;
  int32_t stride_h, stride_w, pad_top, pad_left, dilation_h, dilation_w;
  int32_t weight_layout; /* SPX_WEIGHT_*                                  */
  int32_t activation;    /* SPX_ACT_*                                     */
} spx_conv_params;
int spx_op_conv2d_nhwc(spx_graph* g, const float* x, const float* w,
                       const float* bias, const float* residual, float* y,
                       const spx_conv_params* p);

/* Weights prepared once for the tensor-core path, which multiplies fp32 data
 * as two tf32 terms (3xTF32): w_hi = tf32 round-to-nearest of w,
 * w_lo = tf32(w - w_hi); n floats each, device buffers.  The *_split ops take
 * w (used by every non-tensor-core path) plus w_hi / w_lo, so the weight
 * split is not repeated for every output tile. */
int spx_weights_split(spx_graph* g, const float* w, float* w_hi, float* w_lo, int64_t n);
int spx_op_conv2d_nhwc_split(spx_graph* g, const float* x, const float* w, const float* w_hi,
                             const float* w_lo, const float* bias, const float* residual, float* y,
                             const spx_conv_params* p);

/* Depthwise convolution (depth_multiplier 1), NHWC, weights [kh][kw][c]
 * (TFLite's [1,kh,kw,c]).  Follows depthwise_conv2d.comp:27-49 and the
 * lowering at scheduler.rs:428-548, with the activation fused. */
typedef struct spx_dw_params {
  int32_t n, ih, iw, c, oh, ow, kh, kw;
  int32_t stride_h, stride_w, pad_top, pad_left, dilation_h, dilation_w;
  int32_t activation;
} spx_dw_params;
int spx_op_depthwise_conv2d_nhwc(spx_graph* g, const float* x, const float* w,
                                 const float* bias, float* y, const spx_dw_params* p);

/* Fused back half of an inverted-residual block: 3x3 depthwise conv (stride
 * 1 or 2, bias b_dw, activation act_dw) followed by the 1x1 projection to
 * `cout` channels (pre-split tf32 hi / lo weights [cout][c] from
 * spx_weights_split, bias b_proj, activation act_proj) and, when `residual`
 * is non-null, the residual add; the depthwise output stays on chip.
 * Replaces the DepthwiseConv2d + Conv2d (+ Add) dispatches of
 * source/tflite_loader/src/scheduler.rs:321-548 and :144-211.  x is NHWC
 * [n][ih][iw][c], w_dw [3][3][c], y and residual NHWC [n][oh][ow][cout].
 * c and cout must be multiples of 4, cout <= 512, every tensor 16-byte
 * aligned; other shapes fail with SPX_ERR_UNSUPPORTED (nothing launched). */
typedef struct spx_dwproj_params {
  int32_t n, ih, iw, c, oh, ow;
  int32_t kernel, stride, pad_top, pad_left;
  int32_t act_dw, cout, act_proj;
} spx_dwproj_params;
int spx_op_dw_project_nhwc(spx_graph* g, const float* x, const float* w_dw, const float* b_dw,
                           const float* w_proj_hi, const float* w_proj_lo, const float* b_proj,
                           const float* residual, float* y, const spx_dwproj_params* p);
/* 3x3 or 7x7 stride-2 convolution over 3-channel NHWC input (the MobileNetV2
 * / EfficientNet-Lite0 stems, conv2d.comp through the Conv2d lowering of
 * scheduler.rs:321-427; ResNet-50's 7x7 stem, hlo_conv_nhwc_hwio through
 * compiler.rs) on the tensor cores: each output pixel's k*k*3 taps are
 * gathered into a GEMM row on chip, 32 taps per K block, and multiplied with
 * the weights in 3xTF32.  w_hi / w_lo: [oc][kpad] tf32 hi / lo of the OHWI
 * weights flattened to k*k*3 taps and zero-padded to kpad = 32 (3x3) or 160
 * (7x7) (spx_weights_split of the padded copy).  p->ic must be 3, the kernel
 * square 3x3 or 7x7 with stride 2 and pads below the kernel size, oc <= 128
 * and a multiple of 4, iw a multiple of 4; bias and activation are fused.
 * Other shapes: SPX_ERR_UNSUPPORTED. */
int spx_op_stem_conv_nhwc(spx_graph* g, const float* x, const float* w_hi, const float* w_lo,
                          const float* bias, float* y, const spx_conv_params* p);
int spx_stem_conv_supported(const spx_conv_params* p);
/* 1 when spx_op_dw_project_nhwc takes this shape, 0 otherwise (no device work). */
int spx_dw_project_supported(const spx_dwproj_params* p);

/* Fused MobileNet block front half (no counterpart op in the reference,
 * which dispatches conv2d.comp then depthwise_conv2d.comp with the expanded
 * tensor in memory between them, scheduler.rs:321-548):
 *   e = act_expand(x . W_e^T + b_e)   (1x1 conv, x [n][ih][iw][cin],
 *                                      W_e OHWI [ce][1][1][cin])
 *   y = act_dw(depthwise3x3(e, W_d, stride, SAME) + b_d)
 *                                     (W_d [3][3][ce], y [n][oh][ow][ce])
 * The expanded tensor never leaves the chip.  cin must be 16, 24 or 32,
 * ce a multiple of 4, stride 1 or 2 with oh = ceil(ih / stride); pads are
 * the SAME offsets (pad_top / pad_left = floor(total / 2)). */
typedef struct spx_expand_dw_params {
  int32_t n, ih, iw, cin, ce, oh, ow, stride, pad_top, pad_left;
  int32_t act_expand, act_dw;
} spx_expand_dw_params;
int spx_op_expand_dw_nhwc(spx_graph* g, const float* x, const float* w_expand,
                          const float* b_expand, const float* w_dw, const float* b_dw, float* y,
                          const spx_expand_dw_params* p);
/* The same with the expand weights also pre-split (spx_weights_split): the
 * expand runs as 3xTF32 tensor-core MMAs into TMEM (both activations ReLU6
 * or both none, ce <= 256); other shapes fall back to spx_op_expand_dw_nhwc
 * (w_expand needed then). */
int spx_op_expand_dw_nhwc_split(spx_graph* g, const float* x, const float* w_expand,
                                const float* w_expand_hi, const float* w_expand_lo,
                                const float* b_expand, const float* w_dw, const float* b_dw,
                                float* y, const spx_expand_dw_params* p);

/* Batched strided GEMM: C[b][m][n] = act(alpha * sum_k A[b,m,k] B[b,k,n]
 * + bias[n] + R[b][m][n]).  Element strides let one entry cover
 * fully_connected (B = W^T), hlo_dot_rank2, hlo_dot_batched with any
 * contracting/batch dims (compiler.rs:1009-1084, without the host
 * transposes) and attention QK^T / PV.  C is row-major with row stride c_ms;
 * R (optional) shares C's strides. */
typedef struct spx_gemm_params {
  int32_t batch, m, n, k; /* batch = number of outer batches (>= 1)      */
  int32_t batch_inner;    /* inner batches per outer batch (>= 1)        */
  int32_t b_inner_div;    /* B uses inner index / b_inner_div (>= 1):
                             grouped-query attention shares one K/V head
                             among b_inner_div query heads               */
  int64_t a_bs, a_ms, a_ks;  /* A strides: outer batch, row, k           */
  int64_t b_bs, b_ks, b_ns;  /* B strides: outer batch, k, column        */
  int64_t c_bs, c_ms;        /* C strides: outer batch, row (column = 1) */
  int64_t a_bis, b_bis, c_bis; /* inner-batch strides                    */
  float alpha;
  int32_t activation;
} spx_gemm_params;
int spx_op_gemm(spx_graph* g, const float* a, const float* b, const float* bias,
                const float* residual, float* c, const spx_gemm_params* p);
/* spx_op_gemm with B also given pre-split (spx_weights_split). */
int spx_op_gemm_split(spx_graph* g, const float* a, const float* b, const float* b_hi,
                      const float* b_lo, const float* bias, const float* residual, float* c,
                      const spx_gemm_params* p);

/* Window pooling NHWC (max / sum / average), reduce_window semantics of
 * hlo_reduce_window_rank4.comp:25-49 and max_pool2d.comp:25-44.
 * Average divides by the number of in-bounds taps. */
#define SPX_POOL_MAX 1
#define SPX_POOL_SUM 0
#define SPX_POOL_AVG 2
typedef struct spx_pool_params {
  int32_t n, ih, iw, c, oh, ow, kh, kw, stride_h, stride_w, pad_top, pad_left;
  int32_t kind;
} spx_pool_params;
int spx_op_pool2d_nhwc(spx_graph* g, const float* x, float* y, const spx_pool_params* p);

/* Global average pool NHWC [n][hw][c] -> [n][c] (global_avg_pool_sum.comp +
 * _finalize.comp in one pass). */
int spx_op_global_avg_pool_nhwc(spx_graph* g, const float* x, float* y,
                                int32_t n, int32_t hw, int32_t c);

/* Row softmax over `cols`, for `rows` rows (softmax10/softmax1000.comp,
 * generalised to batches).  Optional additive mask row-broadcast is not
 * applied here; see spx_op_attention_softmax. */
int spx_op_softmax_rows(spx_graph* g, const float* x, float* y, int32_t rows, int32_t cols);

/* Scaled, masked softmax for attention scores [rows][cols]:
 * y = softmax(scale * x + mask), causal when `causal` != 0 (column j is
 * masked for j > q_offset + row % q_len).  mask may be NULL. */
int spx_op_attention_softmax(spx_graph* g, const float* x, float* y, int32_t rows,
                             int32_t cols, float scale, int32_t causal, int32_t q_len,
                             int32_t q_offset);

/* Elementwise ops.  Unary codes mirror the reference shader set. */
#define SPX_UN_ABS 0
#define SPX_UN_EXP 1
#define SPX_UN_LOG 2
#define SPX_UN_NEG 3
#define SPX_UN_SQRT 4
#define SPX_UN_RSQRT 5
#define SPX_UN_SIGMOID 6
#define SPX_UN_TANH 7
#define SPX_UN_RELU 8
#define SPX_UN_RELU6 9
#define SPX_UN_LEAKY_RELU 10
#define SPX_UN_SIN 11
#define SPX_UN_COPY 12
#define SPX_UN_GELU_ERF 13
#define SPX_UN_SILU 14
int spx_op_unary(spx_graph* g, int32_t op, const float* x, float* y, int64_t n, float alpha);

#define SPX_BIN_ADD 0
#define SPX_BIN_SUB 1
#define SPX_BIN_MUL 2
#define SPX_BIN_DIV 3
#define SPX_BIN_POW 4
#define SPX_BIN_MIN 5
#define SPX_BIN_MAX 6
/* HLO `compare` (compiler.rs runs it on the host): 1.0f where the relation
 * holds, 0.0f elsewhere (NaN compares false except NE). */
#define SPX_BIN_GT 7
#define SPX_BIN_GE 8
#define SPX_BIN_LT 9
#define SPX_BIN_LE 10
#define SPX_BIN_EQ 11
#define SPX_BIN_NE 12
/* y[i0,i1,i2,i3] = a[.] op b[.] over a rank-4 output with element strides
 * for a and b (0 = broadcast along that axis), replacing the reference's CPU
 * broadcast before every HLO elementwise dispatch (compiler.rs:705-729). */
typedef struct spx_bcast_params {
  int32_t d[4];
  int64_t a_stride[4];
  int64_t b_stride[4];
} spx_bcast_params;
int spx_op_binary(spx_graph* g, int32_t op, const float* a, const float* b, float* y,
                  const spx_bcast_params* p);
/* HLO `select` (host-side in the reference, compiler.rs CPU ops): y = pred != 0
 * ? a : b elementwise over the rank-4 output p->d; pred, a and b each have
 * their own element strides (0 = broadcast).  Exact: the branch not taken is
 * never combined arithmetically, so inf / NaN there do not leak. */
typedef struct spx_select_params {
  int32_t d[4];
  int64_t p_stride[4];
  int64_t a_stride[4];
  int64_t b_stride[4];
} spx_select_params;
int spx_op_select(spx_graph* g, const float* pred, const float* a, const float* b, float* y,
                  const spx_select_params* p);

/* hlo_reduce_rank4 with the reference's 15 push constants
 * (compiler.rs:975-991): rank,d0..d3,od0..od3,r0..r3,kind,total. */
int spx_op_reduce_rank4(spx_graph* g, const float* x, float* y, const int32_t push[15]);

/* Row LayerNorm: y = (x - mean) / sqrt(var + eps) * gamma + beta (+ the
 * optional residual added to x first, written to x_out when non-NULL). */
int spx_op_layernorm(spx_graph* g, const float* x, const float* residual, float* x_out,
                     const float* gamma, const float* beta, float* y, int32_t rows,
                     int32_t cols, float eps);
/* Row RMSNorm: y = x / sqrt(mean(x^2) + eps) * gamma (gamma may be NULL:
 * no gain). */
int spx_op_rmsnorm(spx_graph* g, const float* x, const float* gamma, float* y, int32_t rows,
                   int32_t cols, float eps);
/* Rotary embedding (rotate-half form) in place on [tokens][heads][head_dim];
 * positions[t] gives each token's position. */
int spx_op_rope(spx_graph* g, float* x, const int32_t* positions, int32_t tokens,
                int32_t heads, int32_t head_dim, float theta);
/* Embedding gather: y[t][:] = table[ids[t]][:]. */
int spx_op_embedding(spx_graph* g, const float* table, const int32_t* ids, float* y,
                     int32_t tokens, int32_t dim);
/* Row argmax (first maximum wins): idx[r] = argmax_c x[r][c]. */
int spx_op_argmax_rows(spx_graph* g, const float* x, int32_t* idx, float* val, int32_t rows,
                       int32_t cols);
/* y = silu(gate) * up, elementwise over n values. */
int spx_op_swiglu(spx_graph* g, const float* gate, const float* up, float* y, int64_t n);

/* ---- TinyLlama decode with a KV cache -------------------------------------
 * The reference runs every decode step as a full forward pass over a padded
 * 64-token window with a causal mask (source/xla_hlo/tools/export_llama.py:
 * 269-365, run_llama_spirv.py:190-260, one hlo_dot_batched dispatch per
 * matmul).  These entries replace those dispatches with a cached decode:
 * new tokens' K/V are appended to a per-layer cache and attention reads the
 * cache.  Positions live in device memory (`state`) so a whole decode step
 * can be captured once and replayed.
 *
 * Shapes: qkv rows are [q heads | k heads | v heads] x head_dim; the caches
 * are [batch][kv_heads][max_seq][head_dim]; q / attention output are
 * [batch * q_len][q_heads][head_dim].  state[0] is the number of tokens
 * already in the cache (the position of the first new token), state[1] the
 * number of generated tokens. */
typedef struct spx_kv_params {
  int32_t batch, q_len, q_heads, kv_heads, head_dim, max_seq;
} spx_kv_params;
/* RoPE (rotate-half, x * cos + rotate_half(x) * sin with the reference's
 * [max_seq][head_dim] cos / sin tables, run_llama_spirv.py:87-97) on q and k,
 * q written to q_out, k and v appended at positions state[0] + t. */
int spx_op_rope_kv_append(spx_graph* g, const float* qkv, int64_t ld_qkv, const float* cos_table,
                          const float* sin_table, const int32_t* state, float* q_out,
                          float* k_cache, float* v_cache, const spx_kv_params* p);
/* Causal grouped-query attention of the q_len new tokens over the cache
 * (key j visible to the token at position state[0] + t when j <= that
 * position); softmax(q k^T * scale) v per head.  head_dim must be 64. */
int spx_op_attention_kv(spx_graph* g, const float* q, const float* k_cache, const float* v_cache,
                        float* out, const int32_t* state, const spx_kv_params* p, float scale);
/* Fused SwiGLU projection for m <= 8 rows: c[r][j] = silu(a'[r] . w[j]) *
 * (a'[r] . w[j + f]) for j < f, w = [gate rows | up rows] x k (row stride
 * ldw).  a' = a, or with rms_eps >= 0 the gain-free RMSNorm of a
 * (a / sqrt(mean(a^2) + rms_eps); fold the norm's gain into w).  Returns
 * SPX_ERR_INVALID_ARGUMENT for m > 8 (use spx_op_rmsnorm + spx_op_gemm +
 * spx_op_swiglu_rows there). */
int spx_op_swiglu_linear(spx_graph* g, const float* a, int64_t lda, const float* w, int64_t ldw,
                         int32_t m, int32_t f, int32_t k, float rms_eps, float* c, int64_t ldc);
/* c[r][j] = x'[r] . w[j] (+ residual[r][j]) for m <= 8 rows, x' the
 * gain-free RMSNorm of x when rms_eps >= 0 (x itself otherwise).  With
 * argmax_keys (m zero-initialised 64-bit keys) each row's greedy argmax is
 * folded in: keys[r] = max over j of (order-preserving bits of c[r][j],
 * ~j), so the largest value wins and ties go to the smallest j;
 * spx_op_token_commit decodes and resets them. */
int spx_op_rms_linear(spx_graph* g, const float* x, int64_t ldx, const float* w, int64_t ldw,
                      int32_t m, int32_t n, int32_t k, float rms_eps, const float* residual,
                      float* c, int64_t ldc, uint64_t* argmax_keys);
/* y[r][j] = silu(gu[r][j]) * gu[r][j + f], gu row stride ld. */
int spx_op_swiglu_rows(spx_graph* g, const float* gu, int64_t ld, float* y, int64_t ldy,
                       int32_t rows, int32_t f);
/* Greedy bookkeeping: (with argmax_keys: ids[b] = the column of keys[b],
 * keys[b] = 0), hist[state[1]][b] = ids[b] (when state[1] < hist_cap),
 * then state[0] += advance and state[1] += 1. */
int spx_op_token_commit(spx_graph* g, int32_t* ids, int32_t* hist, int32_t* state,
                        int32_t batch, int32_t advance, int32_t hist_cap, uint64_t* argmax_keys);
/* Vocab-parallel argmax: packed[r] = (max value, index + col_offset) of row
 * r (first maximum wins), as two floats, the index as its int32 bits.
 * argmax_merge picks, per row, the largest value over `parts` such arrays
 * laid out [parts][rows] (ties: smallest index) into ids. */
int spx_op_argmax_partial(spx_graph* g, const float* x, int64_t ldx, int32_t rows, int32_t cols,
                          int32_t col_offset, float* packed);
int spx_op_argmax_merge(spx_graph* g, const float* packed, int32_t parts, int32_t rows,
                        int32_t* ids);

/* ---- one-shot all-reduce over peer memory (tensor-parallel decode) ------
 * No counterpart in the reference (its TP plan names an NCCL all-reduce,
 * which this replaces for small messages).  Each rank creates a
 * communicator with two data slots of max_bytes, exports its handle
 * (spx_ar_handle, spx_ar_handle_size() bytes), gathers every rank's handle
 * (rank order) and opens them (spx_ar_open).  A producer writes this rank's
 * partial sum into spx_ar_slot(a, s); spx_op_allreduce sums slot s of all
 * ranks into out (out must not alias a slot).  Consecutive all-reduces must
 * alternate slots 0 / 1 and be issued in the same order on every rank.
 * Waits for peers are bounded (2 s, or the "ar_wait_limit_us" option,
 * 1 ms .. 60 s); a timeout is reported as SPX_ERR_CUDA at the next graph sync
 * and leaves that all-reduce's output untouched.  The communicators are then
 * out of step: every rank calls spx_ar_reset (zeroes its own flags and
 * epochs, synchronous) between two host-side barriers before the next
 * all-reduce. */
typedef struct spx_ar spx_ar;
int spx_ar_create(int32_t device, int32_t rank, int32_t world, size_t max_bytes, spx_ar** out);
size_t spx_ar_handle_size(void);
int spx_ar_handle(spx_ar* a, void* handle, size_t handle_bytes);
int spx_ar_open(spx_ar* a, const void* handles);
float* spx_ar_slot(spx_ar* a, int32_t slot);
int spx_op_allreduce(spx_graph* g, spx_ar* a, int32_t slot, float* out, int64_t n);
int spx_ar_reset(spx_ar* a);
int spx_ar_destroy(spx_ar* a);

/* Rank-4 constant pad (pad.comp with the reference's 13 push constants
 * od0..3, id0..3, pl0..3, total) and rank-4 permutation (transpose.comp's
 * 13 push constants in0..3, out0..3, p0..3, total). */
int spx_op_pad4(spx_graph* g, const float* x, float* y, float pad_value, const int32_t push[13]);
int spx_op_transpose4(spx_graph* g, const float* x, float* y, const int32_t push[13]);

#ifdef __cplusplus
}
#endif
#endif /* SPX_H_ */
