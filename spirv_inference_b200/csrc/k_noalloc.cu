// Allocation-free variant of the drop-in NCHW conv2d dispatch.
//
// The regular path (spx_run_kernel "conv2d") stages the NHWC copy of the
// input, the OHWI copy of the weights and the NHWC result in device buffers
// it obtains with cudaMalloc.  Some callers cannot let a library allocate:
// hosts that hand the whole device memory to their own pool allocator, and
// latency-critical loops where cudaMalloc's implicit device synchronisation
// is not acceptable.  This entry point takes caller-owned device buffers for
// input, weights and output and keeps its staging in one fixed,
// library-owned __device__ array instead.
#include <mutex>

#include "spx_internal.cuh"

namespace spx {
namespace {

// Staging capacity in floats: NHWC input + OHWI weights + NHWC output of one
// call must fit.  16 MiB per GPU that loads the library, held until exit.
constexpr size_t kNoAllocFloats = (size_t)4 << 20;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

struct ScratchAddr {
  bool ready = false;
  float* ptr = nullptr;
};
ScratchAddr g_scratch_addr[64];
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device.  The host-side
// symbol is only a stand-in; its device address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
int scratch_address(float** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(SPX_ERR_NO_DEVICE, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& s = g_scratch_addr[dev];
  if (!s.ready) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                    "cudaGetSymbolAddress(no-alloc scratch)");
    if (rc) return rc;
    s.ptr = (float*)p;
    s.ready = true;
  }
  *out = s.ptr;
  return SPX_OK;
}

}  // namespace
}  // namespace spx

using namespace spx;

extern "C" int spx_conv2d_nchw_noalloc(const float* x, const float* w, float* y,
                                       const int32_t* push, size_t push_len, void* stream) {
  if (!x || !w || !y || !push) return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_noalloc: null argument");
  if (push_len != 15)
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_noalloc expects 15 push constants, got %zu",
                push_len);
  // n,ic,ih,iw,oc,oh,ow,kh,kw,stride_h,stride_w,same,pad_top,pad_left,total
  const int32_t* q = push;
  for (int i = 0; i < 11; ++i)
    if (q[i] <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_noalloc: push[%d] <= 0", i);
  const int N = q[0], IC = q[1], IH = q[2], IW = q[3], OC = q[4], OH = q[5], OW = q[6],
            KH = q[7], KW = q[8];
  const int PT = q[12], PL = q[13];
  if (PT < 0 || PT >= KH || PL < 0 || PL >= KW)
    return fail(SPX_ERR_INVALID_ARGUMENT,
                "conv2d_noalloc: pad_top %d / pad_left %d outside [0, kernel extent %d x %d)", PT,
                PL, KH, KW);
  if ((int64_t)(OH - 1) * q[9] - PT >= IH || (int64_t)(OW - 1) * q[10] - PL >= IW)
    return fail(SPX_ERR_INVALID_ARGUMENT,
                "conv2d_noalloc: output %d x %d with stride %d x %d and pads %d, %d reads past "
                "the %d x %d input", OH, OW, q[9], q[10], PT, PL, IH, IW);
  const int64_t in_el = (int64_t)N * IC * IH * IW, w_el = (int64_t)OC * IC * KH * KW;
  const int64_t total = (int64_t)N * OC * OH * OW;
  if (total != q[14])
    return fail(SPX_ERR_INVALID_ARGUMENT, "conv2d_noalloc: total %d != n*oc*oh*ow", q[14]);
  // Each region starts on a 256-byte boundary inside the scratch array.
  auto round64 = [](int64_t v) { return (v + 63) / 64 * 64; };
  const int64_t need = round64(in_el) + round64(w_el) + round64(total);
  if (need > (int64_t)kNoAllocFloats)
    return fail(SPX_ERR_INVALID_ARGUMENT,
                "conv2d_noalloc: staging needs %lld floats, the fixed scratch holds %lld "
                "(use spx_run_kernel for larger convolutions)",
                (long long)need, (long long)kNoAllocFloats);
  if (spx_device_count() == 0) return fail(SPX_ERR_NO_DEVICE, "no CUDA device");
  float* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  float* x_nhwc = base;
  float* w_ohwi = base + round64(in_el);
  float* y_nhwc = w_ohwi + round64(w_el);
  cudaStream_t s = (cudaStream_t)stream;
  // Every scratch element read below is written earlier in this same call,
  // so nothing needs clearing between calls.
  int32_t t_in[13] = {N, IC, IH, IW, N, IH, IW, IC, 0, 2, 3, 1, (int32_t)in_el};
  int32_t t_w[13] = {OC, IC, KH, KW, OC, KH, KW, IC, 0, 2, 3, 1, (int32_t)w_el};
  int32_t t_out[13] = {N, OH, OW, OC, N, OC, OH, OW, 0, 3, 1, 2, (int32_t)total};
  if ((rc = launch_transpose4(s, nullptr, x, x_nhwc, t_in))) return rc;
  if ((rc = launch_transpose4(s, nullptr, w, w_ohwi, t_w))) return rc;
  spx_conv_params p = {N, IH, IW, IC, OC, OH, OW, KH, KW, q[9], q[10], PT, PL, 1, 1,
                       SPX_WEIGHT_OHWI, SPX_ACT_NONE};
  if ((rc = launch_conv_nhwc(s, nullptr, x_nhwc, w_ohwi, nullptr, nullptr, w + w_el, nullptr,
                             y_nhwc, &p)))
    return rc;
  return launch_transpose4(s, nullptr, y_nhwc, y, t_out);
}
