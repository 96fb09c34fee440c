// Depthwise convolution (depthwise_conv2d.comp:27-49, NHWC, depth multiplier 1)
// with TMA-fed shared-memory tiles.
//
// A persistent CTA walks output tiles of TH x TW pixels x CB channels.  For
// each tile one thread issues a 4-D TMA load (dims C, W, H, N) of the input
// halo box ((TH-1)*S+KH) x ((TW-1)*S+KW) x CB into one of two shared-memory
// buffers; the tensor map's out-of-bounds zero fill supplies the convolution
// padding, including boxes that start at negative coordinates.  While the
// next tile's box is in flight, 256 threads compute the current one: a thread
// owns 4 channels of R consecutive output rows in one column, keeps the
// KH x KW x 4 weights in registers and reads each input row of its window
// once from shared memory.  Bias and activation are fused; outputs leave as
// 16-byte stores, a warp writing whole 128-byte channel runs.
//
// Every mbarrier wait is bounded (globaltimer); on timeout the kernel records
// a device status, waits briefly for its own copy and returns.
#include <cuda.h>

#include <mutex>

#include "spx_internal.cuh"

namespace spx {

__device__ int g_dw_status = 0;

namespace {

constexpr unsigned long long kDwTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t s32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mb_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(s32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mb_wait(uint64_t* b, uint32_t parity) {
  if (mb_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (;;) {
    for (int i = 0; i < 16; ++i)
      if (mb_try(b, parity)) return true;
    if (now_ns() - t0 > kDwTimeoutNs) {
      atomicExch(&g_dw_status, 1);
      return false;
    }
  }
}

template <int KH, int KW, int S, int TH, int TW, int R, int CB>
__global__ void __launch_bounds__(256, KH == 3 ? 2 : 1)
    dw_tma_kernel(const __grid_constant__ CUtensorMap tmX, const float* __restrict__ w,
                  const float* __restrict__ bias, float* __restrict__ y, int n, int c, int oh,
                  int ow, int pt, int pl, int act, int tiles_h, int tiles_w, int c_chunks) {
  constexpr int IH = (TH - 1) * S + KH, IW = (TW - 1) * S + KW;
  constexpr int CG = CB / 4;                   // channel groups of 4 per tile
  constexpr uint32_t kBoxBytes = IH * IW * CB * 4;
  constexpr uint32_t kBufBytes = (kBoxBytes + 127) / 128 * 128;
  static_assert((TH / R) * TW * CG == 256, "one thread per (row block, column, group)");
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* smem_raw = (uint8_t*)(((uintptr_t)smem_dyn + 127) & ~(uintptr_t)127);
  float* buf[2] = {(float*)smem_raw, (float*)(smem_raw + kBufBytes)};
  uint64_t* full = (uint64_t*)(smem_raw + 2 * kBufBytes);
  __shared__ int s_abort;

  const int tid = threadIdx.x;
  const int cg = tid % CG;
  const int ox_l = (tid / CG) % TW;
  const int rb = tid / (CG * TW);
  const int total = n * tiles_h * tiles_w * c_chunks;

  auto tile_coords = [&](int t, int& img, int& ty, int& tx, int& cc) {
    cc = t % c_chunks;
    int r = t / c_chunks;
    tx = r % tiles_w;
    r /= tiles_w;
    ty = r % tiles_h;
    img = r / tiles_h;
  };
  auto issue = [&](int t, int b) {
    int img, ty, tx, cc;
    tile_coords(t, img, ty, tx, cc);
    const int x0 = cc * CB, x1 = tx * TW * S - pl, x2 = ty * TH * S - pt;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(&full[b])),
                 "r"(kBoxBytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(s32(buf[b])),
        "l"(reinterpret_cast<uint64_t>(&tmX)), "r"(x0), "r"(x1), "r"(x2), "r"(img),
        "r"(s32(&full[b]))
        : "memory");
  };

  if (tid == 0) {
    for (int b = 0; b < 2; ++b)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(s32(&full[b])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  __syncthreads();
  if (tid == 0) {
    if ((int)blockIdx.x < total) issue(blockIdx.x, 0);
    if ((int)(blockIdx.x + gridDim.x) < total) issue(blockIdx.x + gridDim.x, 1);
  }
  uint32_t phase = 0;  // bit b: parity to wait for on full[b]
  int b = 0;
  int cc_prev = -1;
  float4 wr[KH][KW];
  float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    int img, ty, tx, cc;
    tile_coords(t, img, ty, tx, cc);
    const int ch = cc * CB + cg * 4;
    const bool live = ch < c;  // the last chunk may run past c (TMA fills zeros there)
    if (cc != cc_prev) {  // weights of this channel chunk, kept in registers
#pragma unroll
      for (int ky = 0; ky < KH; ++ky)
#pragma unroll
        for (int kx = 0; kx < KW; ++kx)
          wr[ky][kx] = live ? __ldg(reinterpret_cast<const float4*>(w + (ky * KW + kx) * c + ch))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      if (bias && live) bv = __ldg(reinterpret_cast<const float4*>(bias + ch));
      cc_prev = cc;
    }
    if (!mb_wait(&full[b], (phase >> b) & 1)) s_abort = 1;
    phase ^= 1u << b;
    __syncthreads();
    if (s_abort) break;
    const float* in = buf[b];
    float4 acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = bv;
#pragma unroll
    for (int j = 0; j < (R - 1) * S + KH; ++j) {
      const int iy = rb * R * S + j;
      float4 row[KW];
#pragma unroll
      for (int kx = 0; kx < KW; ++kx)
        row[kx] = *reinterpret_cast<const float4*>(in + ((iy * IW) + ox_l * S + kx) * CB + cg * 4);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int ky = j - r * S;
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
    __syncthreads();  // every thread is done reading buf[b]
    if (tid == 0 && t + 2 * (int)gridDim.x < total) issue(t + 2 * gridDim.x, b);
    const int ox = tx * TW + ox_l;
    with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int oy = ty * TH + rb * R + r;
        if (oy < oh && ox < ow && live) {
          float4 v = acc[r];
          v.x = act_c<A>(v.x);
          v.y = act_c<A>(v.y);
          v.z = act_c<A>(v.z);
          v.w = act_c<A>(v.w);
          *reinterpret_cast<float4*>(y + (((size_t)img * oh + oy) * ow + ox) * c + ch) = v;
        }
      }
    });
    b ^= 1;
  }
  if (s_abort && tid == 0) {  // let this CTA's own copies land before it exits
    for (int q = 0; q < 2; ++q) {
      const unsigned long long t0 = now_ns();
      while (!mb_try(&full[q], (phase >> q) & 1) && now_ns() - t0 < 200000000ull) {
      }
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

int sms() {
  static int v = 0;
  if (!v) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    if (v <= 0) v = kNumSms;
  }
  return v;
}

template <int KH, int KW, int S, int TH, int TW, int R, int CB>
int launch_cfg(cudaStream_t s, const float* x, const float* w, const float* b, float* y,
               const spx_dw_params* p) {
  constexpr int IH = (TH - 1) * S + KH, IW = (TW - 1) * S + KW;
  constexpr uint32_t kBoxBytes = IH * IW * CB * 4;
  constexpr uint32_t kBufBytes = (kBoxBytes + 127) / 128 * 128;
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)p->c, (cuuint64_t)p->iw, (cuuint64_t)p->ih, (cuuint64_t)p->n};
  cuuint64_t strides[3] = {(cuuint64_t)p->c * 4, (cuuint64_t)p->iw * p->c * 4,
                           (cuuint64_t)p->ih * p->iw * p->c * 4};
  cuuint32_t box[4] = {(cuuint32_t)CB, (cuuint32_t)IW, (cuuint32_t)IH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "dw tensor map encode failed (%d)", (int)r);
  const int tiles_h = (p->oh + TH - 1) / TH, tiles_w = (p->ow + TW - 1) / TW;
  const int c_chunks = (p->c + CB - 1) / CB;
  const int64_t total = (int64_t)p->n * tiles_h * tiles_w * c_chunks;
  const size_t smem = 2 * kBufBytes + 128 + 64;
  auto kern = dw_tma_kernel<KH, KW, S, TH, TW, R, CB>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "dw_tma: smem attribute");
  // Two or more resident CTAs per SM overlap one CTA's compute with another's loads.
  const int per_sm = smem <= 56 * 1024 ? 4 : (smem <= 110 * 1024 ? 2 : 1);
  const int64_t cap = (int64_t)sms() * per_sm;
  const int grid = (int)(total < cap ? total : cap);
  kern<<<grid, 256, smem, s>>>(map, w, b, y, p->n, p->c, p->oh, p->ow, p->pad_top, p->pad_left,
                               p->activation, tiles_h, tiles_w, c_chunks);
  return SPX_OK;
}

bool a16(const void* q) { return ((uintptr_t)q & 15) == 0; }

}  // namespace

int try_dw_tma(cudaStream_t s, int64_t* cnt, const float* x, const float* w, const float* b,
               float* y, const spx_dw_params* p) {
  if (p->dilation_h > 1 || p->dilation_w > 1 || p->stride_h != p->stride_w) return -1;
  // Tiles: 3x3 stride 1 as 14 x 16 outputs (7 rows per thread), 7 x 8 x 128
  // channels on 7x7 maps; stride 2 and 5x5 as 4 x 16 / 8 x 16.  Channel
  // chunks are 32 wide for c >= 32 (a partial last chunk reads the tensor
  // map's zero fill and stores nothing), 16 wide below.  Under 14 x 14
  // (except 7x7 stride 1) most of a tile would be padding: the register
  // kernel serves those.
  const bool m7 = p->oh == 7 && p->ow == 7 && p->stride_h == 1;
  if ((p->oh < 14 || p->ow < 14) && !m7) return -1;
  if (p->c % 4 || !a16(x) || !a16(w) || !a16(y) || (b && !a16(b))) return -1;
  if ((int64_t)p->n * p->oh * p->ow * p->c >= INT32_MAX) return -1;
  if ((int64_t)p->n * (p->oh / 4 + 1) * (p->ow / 8 + 1) * (p->c / 4 + 1) >= INT32_MAX) return -1;
  const int k = p->kh == p->kw ? p->kh : 0, st = p->stride_h;
  int rc = -1;
  if (p->c >= 32) {
    if (m7) {
      if (k == 3) rc = launch_cfg<3, 3, 1, 7, 8, 7, 128>(s, x, w, b, y, p);
    } else if (k == 3 && st == 1) rc = launch_cfg<3, 3, 1, 14, 16, 7, 32>(s, x, w, b, y, p);
    else if (k == 3 && st == 2) rc = launch_cfg<3, 3, 2, 4, 16, 2, 32>(s, x, w, b, y, p);
    else if (k == 5 && st == 1) rc = launch_cfg<5, 5, 1, 8, 16, 4, 32>(s, x, w, b, y, p);
    else if (k == 5 && st == 2) rc = launch_cfg<5, 5, 2, 4, 16, 2, 32>(s, x, w, b, y, p);
  } else if (p->c % 16 == 0 && !m7) {
    if (k == 3 && st == 1) rc = launch_cfg<3, 3, 1, 8, 32, 4, 16>(s, x, w, b, y, p);
    else if (k == 3 && st == 2) rc = launch_cfg<3, 3, 2, 4, 32, 2, 16>(s, x, w, b, y, p);
    else if (k == 5 && st == 1) rc = launch_cfg<5, 5, 1, 8, 32, 4, 16>(s, x, w, b, y, p);
    else if (k == 5 && st == 2) rc = launch_cfg<5, 5, 2, 4, 32, 2, 16>(s, x, w, b, y, p);
  }
  if (rc == -1) return -1;
  if (rc != SPX_OK) return rc;
  return after_launch(cnt, "depthwise_tma");
}

int dw_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dw_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_dw_status, &zero, sizeof(int));
  }
  return v;
}

}  // namespace spx
