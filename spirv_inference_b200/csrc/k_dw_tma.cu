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

// ---------------------------------------------------------------------------
// Fused inverted-residual front half: 1x1 expand conv (+ bias, activation)
// followed by the 3x3 depthwise conv (+ bias, activation), without the
// expanded tensor ever reaching HBM.  Same persistent tile walk as
// dw_tma_kernel, but the TMA halo box is the block's narrow input x
// (CIN <= 32 channels); per tile and 32-channel chunk of the expanded width
// the CTA first computes the expanded halo e = act_e(x . We + be) on CUDA
// cores into shared memory (zero outside the map: the depthwise padding
// applies to e), then runs the depthwise rows of dw_tma_kernel on it.
// Exact fp32 FMAs throughout.
constexpr int kXdCB = 32;  // expanded channels per tile

template <int S, int TH, int TW, int R, int CIN, int ACT>
__global__ void __launch_bounds__(256, 2)
    expand_dw_kernel(const __grid_constant__ CUtensorMap tmX, const float* __restrict__ we,
                     const float* __restrict__ be, const float* __restrict__ wd,
                     const float* __restrict__ bd, float* __restrict__ y, int n, int ih, int iw,
                     int ce, int oh, int ow, int pt, int pl, int act_e, int act_d, int tiles_h,
                     int tiles_w, int c_chunks) {
  constexpr int KH = 3, KW = 3;
  constexpr int IH = (TH - 1) * S + KH, IW = (TW - 1) * S + KW;
  constexpr int NPIX = IH * IW;
  constexpr int CG = kXdCB / 4;
  constexpr uint32_t kBoxBytes = NPIX * CIN * 4;
  constexpr uint32_t kXBuf = (kBoxBytes + 127) / 128 * 128;
  static_assert((TH / R) * TW * CG == 256, "one thread per (row block, column, group)");
  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = (uint8_t*)(((uintptr_t)smem_dyn + 127) & ~(uintptr_t)127);
  float* xbuf[2] = {(float*)base, (float*)(base + kXBuf)};
  float* es = (float*)(base + 2 * kXBuf);            // expanded halo [NPIX][32]
  float* wes = es + NPIX * kXdCB;                    // We chunk [CIN][32]
  float* wds = wes + CIN * kXdCB;                    // depthwise weights chunk [9][32]
  uint64_t* full = (uint64_t*)(wds + 9 * kXdCB + 32);
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
    const int x1 = tx * TW * S - pl, x2 = ty * TH * S - pt;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(&full[b])),
                 "r"(kBoxBytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(s32(xbuf[b])),
        "l"(reinterpret_cast<uint64_t>(&tmX)), "r"(0), "r"(x1), "r"(x2), "r"(img),
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
  uint32_t phase = 0;
  int b = 0;
  int cc_prev = -1;
  float4 bdv = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 bev = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    int img, ty, tx, cc;
    tile_coords(t, img, ty, tx, cc);
    const int ch = cc * kXdCB + cg * 4;
    const bool live = ch < ce;
    if (cc != cc_prev) {
      __syncthreads();  // previous tile's readers of wes are done
      for (int i = tid; i < CIN * kXdCB; i += blockDim.x) {
        const int k = i / kXdCB, c = cc * kXdCB + i % kXdCB;
        wes[i] = c < ce ? we[(size_t)c * CIN + k] : 0.0f;  // We OHWI [ce][cin] -> [cin][32]
      }
      for (int i = tid; i < 9 * kXdCB; i += blockDim.x) {
        const int k = i / kXdCB, c = cc * kXdCB + i % kXdCB;
        wds[i] = c < ce ? wd[(size_t)k * ce + c] : 0.0f;
      }
      bdv = (bd && live) ? __ldg(reinterpret_cast<const float4*>(bd + ch))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
      // The expand step's channel group is tid & 7 (it equals cg only
      // because CG == 8; kept separate for clarity).
      const int ech = cc * kXdCB + (tid & 7) * 4;
      bev = (be && ech < ce) ? __ldg(reinterpret_cast<const float4*>(be + ech))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      cc_prev = cc;
    }
    if (!mb_wait(&full[b], (phase >> b) & 1)) s_abort = 1;
    phase ^= 1u << b;
    __syncthreads();
    if (s_abort) break;
    __syncthreads();  // the x box is ready for every thread
    // Expand: thread = (pixel group pg, channel group cg); pixels pg + 32 i.
    // Per 8-wide k chunk a thread loads its 8 x 4 weights once and reuses
    // them over its pixels; the 8 threads of a pixel group read the same x
    // row (shared-memory broadcast).
    {
      constexpr int NP = (NPIX + 31) / 32;
      const int xcg = tid & 7, pg = tid >> 3;
      const float* xb = xbuf[b];
      float4 acc[NP];
#pragma unroll
      for (int i = 0; i < NP; ++i) acc[i] = bev;
#pragma unroll
      for (int k0 = 0; k0 < CIN; k0 += 4) {
        float4 wv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          wv[q] = *reinterpret_cast<const float4*>(wes + (k0 + q) * kXdCB + xcg * 4);
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const int p = pg + 32 * i;
          if (p < NPIX) {
            const float4 u0 = *reinterpret_cast<const float4*>(xb + p * CIN + k0);
            const float u[4] = {u0.x, u0.y, u0.z, u0.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc[i].x = fmaf(u[q], wv[q].x, acc[i].x);
              acc[i].y = fmaf(u[q], wv[q].y, acc[i].y);
              acc[i].z = fmaf(u[q], wv[q].z, acc[i].z);
              acc[i].w = fmaf(u[q], wv[q].w, acc[i].w);
            }
          }
        }
      }
      const int y0 = ty * TH * S - pt, x0 = tx * TW * S - pl;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int p = pg + 32 * i;
        if (p < NPIX) {
          const int py = y0 + p / IW, px = x0 + p % IW;
          const bool in = py >= 0 && py < ih && px >= 0 && px < iw;
          const float4 e = in ? make_float4(act_c<ACT>(acc[i].x), act_c<ACT>(acc[i].y),
                                            act_c<ACT>(acc[i].z), act_c<ACT>(acc[i].w))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(es + p * kXdCB + xcg * 4) = e;
        }
      }
    }
    __syncthreads();  // xbuf[b] consumed, es ready
    if (tid == 0 && t + 2 * (int)gridDim.x < total) issue(t + 2 * gridDim.x, b);
    // Depthwise on the expanded halo (dw_tma_kernel's row walk).
    float4 wr[KH][KW];
#pragma unroll
    for (int k = 0; k < KH * KW; ++k)
      wr[k / KW][k % KW] = *reinterpret_cast<const float4*>(wds + k * kXdCB + cg * 4);
    float4 acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = bdv;
#pragma unroll
    for (int j = 0; j < (R - 1) * S + KH; ++j) {
      const int iy = rb * R * S + j;
      float4 row[KW];
#pragma unroll
      for (int kx = 0; kx < KW; ++kx)
        row[kx] = *reinterpret_cast<const float4*>(es + ((iy * IW) + ox_l * S + kx) * kXdCB + cg * 4);
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
    const int ox = tx * TW + ox_l;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int oy = ty * TH + rb * R + r;
      if (oy < oh && ox < ow && live) {
        float4 v = acc[r];
        v.x = act_c<ACT>(v.x);
        v.y = act_c<ACT>(v.y);
        v.z = act_c<ACT>(v.z);
        v.w = act_c<ACT>(v.w);
        *reinterpret_cast<float4*>(y + (((size_t)img * oh + oy) * ow + ox) * ce + ch) = v;
      }
    }
    __syncthreads();  // es / xs reused by the next tile
    b ^= 1;
  }
  if (s_abort && tid == 0) {
    for (int q = 0; q < 2; ++q) {
      const unsigned long long t0 = now_ns();
      while (!mb_try(&full[q], (phase >> q) & 1) && now_ns() - t0 < 200000000ull) {
      }
    }
  }
}

template <int S, int TH, int TW, int R, int CIN, int ACT>
int launch_xd(cudaStream_t s, const float* x, const float* we, const float* be, const float* wd,
              const float* bd, float* y, const spx_expand_dw_params* p) {
  constexpr int IH = (TH - 1) * S + 3, IW = (TW - 1) * S + 3;
  constexpr int NPIX = IH * IW;
  constexpr uint32_t kBoxBytes = NPIX * CIN * 4;
  constexpr uint32_t kXBuf = (kBoxBytes + 127) / 128 * 128;
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  cuuint64_t dims[4] = {(cuuint64_t)CIN, (cuuint64_t)p->iw, (cuuint64_t)p->ih, (cuuint64_t)p->n};
  cuuint64_t strides[3] = {(cuuint64_t)CIN * 4, (cuuint64_t)p->iw * CIN * 4,
                           (cuuint64_t)p->ih * p->iw * CIN * 4};
  cuuint32_t box[4] = {(cuuint32_t)CIN, (cuuint32_t)IW, (cuuint32_t)IH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "expand_dw tensor map encode failed (%d)", (int)r);
  const int tiles_h = (p->oh + TH - 1) / TH, tiles_w = (p->ow + TW - 1) / TW;
  const int c_chunks = (p->ce + kXdCB - 1) / kXdCB;
  const int64_t total = (int64_t)p->n * tiles_h * tiles_w * c_chunks;
  const size_t smem = 128 + 2 * kXBuf + (size_t)NPIX * kXdCB * 4 + (size_t)CIN * kXdCB * 4 +
                      9 * kXdCB * 4 + 128 + 64;
  auto kern = expand_dw_kernel<S, TH, TW, R, CIN, ACT>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "expand_dw: smem attribute");
  if (smem > 200 * 1024) return fail(SPX_ERR_UNSUPPORTED, "expand_dw: tile does not fit");
  const int per_sm = smem <= 110 * 1024 ? 2 : 1;
  const int64_t cap = (int64_t)sms() * per_sm;
  const int grid = (int)(total < cap ? total : cap);
  kern<<<grid, 256, smem, s>>>(map, we, be, wd, bd, y, p->n, p->ih, p->iw, p->ce, p->oh, p->ow,
                               p->pad_top, p->pad_left, p->act_expand, p->act_dw, tiles_h,
                               tiles_w, c_chunks);
  return SPX_OK;
}

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

int launch_expand_dw(cudaStream_t s, int64_t* cnt, const float* x, const float* we,
                     const float* be, const float* wd, const float* bd, float* y,
                     const spx_expand_dw_params* p) {
  if (!x || !we || !wd || !y || !p) return fail(SPX_ERR_INVALID_ARGUMENT, "expand_dw: null");
  if (p->n <= 0 || p->ih <= 0 || p->iw <= 0 || p->ce <= 0 || p->ce % 4 || p->oh <= 0 ||
      p->ow <= 0 || (p->stride != 1 && p->stride != 2))
    return fail(SPX_ERR_INVALID_ARGUMENT, "expand_dw: bad shape");
  if (p->oh != (p->ih + p->stride - 1) / p->stride || p->ow != (p->iw + p->stride - 1) / p->stride)
    return fail(SPX_ERR_INVALID_ARGUMENT, "expand_dw: output must be the SAME-padded size");
  if (!a16(x) || !a16(we) || !a16(wd) || !a16(y) || (be && !a16(be)) || (bd && !a16(bd)))
    return fail(SPX_ERR_INVALID_ARGUMENT, "expand_dw: pointers must be 16-byte aligned");
  if ((int64_t)p->n * p->oh * p->ow * p->ce >= INT32_MAX)
    return fail(SPX_ERR_INVALID_ARGUMENT, "expand_dw: tensor too large");
  int rc = -1;
  // Both activations the same, ReLU6 or none (the MobileNet / EfficientNet-Lite
  // blocks), compiled into the kernel.
  if (p->act_expand != p->act_dw ||
      (p->act_expand != SPX_ACT_RELU6 && p->act_expand != SPX_ACT_NONE))
    return fail(SPX_ERR_UNSUPPORTED, "expand_dw: activations must both be ReLU6 or both none");
  const bool r6 = p->act_expand == SPX_ACT_RELU6;
#define SPX_XD(CI)                                                                             \
  if (r6)                                                                                      \
    rc = p->stride == 1 ? launch_xd<1, 14, 16, 7, CI, SPX_ACT_RELU6>(s, x, we, be, wd, bd, y, p) \
                        : launch_xd<2, 4, 16, 2, CI, SPX_ACT_RELU6>(s, x, we, be, wd, bd, y, p); \
  else                                                                                         \
    rc = p->stride == 1 ? launch_xd<1, 14, 16, 7, CI, SPX_ACT_NONE>(s, x, we, be, wd, bd, y, p)  \
                        : launch_xd<2, 4, 16, 2, CI, SPX_ACT_NONE>(s, x, we, be, wd, bd, y, p)
  switch (p->cin) {
    case 16: SPX_XD(16); break;
    case 24: SPX_XD(24); break;
    case 32: SPX_XD(32); break;
    default:
      return fail(SPX_ERR_UNSUPPORTED, "expand_dw: input channels must be 16, 24 or 32");
  }
#undef SPX_XD
  if (rc != SPX_OK) return rc;
  return after_launch(cnt, "expand_dw");
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
