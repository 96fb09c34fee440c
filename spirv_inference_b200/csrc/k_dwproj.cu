// Fused depthwise 3x3 -> pointwise projection (the back half of an inverted
// residual block: depthwise_conv2d.comp followed by the 1x1 conv2d.comp
// projection and, where the block has one, the residual add.comp), with the
// depthwise output never leaving the SM.
//
// Reference ops fused: the DepthwiseConv2d and Conv2d lowerings and the Add
// of source/tflite_loader/src/scheduler.rs:321-548 and :144-211, each a
// separate dispatch with a full HBM round trip of the 6x-expanded tensor.
//
// A persistent CTA (one per SM) walks output tiles of TH x TW pixels of one
// image (128 GEMM rows) and, for each, every 32-channel block of the
// depthwise width (the GEMM's K):
//   warp 8      TMA producers: per K block the pre-split projection weights
//               (hi and lo, NP x 32, 128-byte swizzle) into the A/B stages
//               (lane 1), and per CB-channel sub-block the input halo box
//               ((TH-1)*S+3) x ((TW-1)*S+3) x CB into a ring (lane 0; the
//               tensor map's zero fill is the depthwise padding);
//   warps 0-7   builders: the depthwise conv of the sub-block on CUDA cores
//               (exact fp32 FMAs, bias and activation fused; a thread owns 2
//               channels of R rows x 2 columns and reads each input row of its
//               window once), written straight into the stage's A tile in
//               the UMMA K-major 128-byte-swizzled layout: the raw value (the
//               MMA's tf32 hi) and its tf32 lo term.  The depthwise taps and
//               bias of the sub-block arrive in the same halo slot (TMA).
//               Each builder warp hands a slot back after its lanes' reads
//               (__syncwarp, then one elected proxy fence + arrive), so the
//               TMA refill cannot overtake a slow lane;
//   warp 9      MMA issuer: 3xTF32 (lo*hi + hi*lo + hi*hi) tcgen05.mma into one
//               of two TMEM accumulators (NP columns each), a commit per K
//               block frees the stage, a commit per tile hands the
//               accumulator to the epilogue;
//   warps 10-17 epilogue (two groups of four, alternate tiles): TMEM lane quarter -> registers (a lane = an output
//               pixel, 32 channels) -> projection bias, residual, activation
//               -> one contiguous 128-byte channel run of the NHWC output.
// HBM traffic per tile: the halo (interior read once; the overlap between
// neighbouring tiles mostly hits L2), the output, and the residual.
//
// Every wait is bounded (globaltimer, 2 s); on timeout the CTA raises an
// abort flag, records a device status, drains its own copies and MMAs, frees
// TMEM and exits.  The host reads the status at the next sync.
#include <cuda.h>

#include <mutex>

#include "sm100_prims.cuh"
#include "spx_internal.cuh"

namespace spx {

__device__ int g_dwp_status = 0;

#ifdef SPX_DWP_TRACE
// Development-only timeline of CTA 0 (not compiled into the library).
__device__ unsigned long long g_dwp_trace[16][256];
#define DWP_TRACE(ev, i)                                                         \
  do {                                                                           \
    if (blockIdx.x == 0 && (i) < 256) g_dwp_trace[ev][i] = sm100::gtime();      \
  } while (0)
#else
#define DWP_TRACE(ev, i) \
  do {                   \
  } while (0)
#endif

namespace {

using namespace sm100;

// AG = 0: both activations in group 0 (none / clamps), only those epilogues
// are instantiated; AG = 1: any activation.
template <int AG, class F>
__device__ __forceinline__ void with_act_sel(int act, F&& f) {
  if constexpr (AG == 0) with_act_group<0>(act, static_cast<F&&>(f));
  else with_act(act, static_cast<F&&>(f));
}

constexpr int kBuildWarps = 8;
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kEpiWarp0 = 10;
// Epilogue groups of 4 warps draining alternate tiles: EG = 2 (576 threads,
// 96 registers a thread) for one-K-block tiles, whose epilogue sets the pace;
// EG = 1 (448 threads, 128 registers) where the builders' depthwise does.
__host__ __device__ constexpr int threads_for(int eg) { return (kEpiWarp0 + 4 * eg) * 32; }
constexpr int kMaxEpiGroups = 2;
constexpr uint32_t kEWarp = 32 * 128;                     // one warp's 32 rows x 32 fp32
constexpr uint32_t kEStage = 4 * kEWarp;                   // a group's staging (16 KB)
constexpr uint32_t kAHalf = 128 * 32 * 4;        // one 128 x 32 fp32 A tile: 16 KB
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr unsigned long long kDrainNs = 200000000ull;
constexpr int kMaxHalo = 4;
constexpr int kMaxStages = 4;        // A/B stages (runtime count nst, 2..4)
constexpr uint32_t kBarBytes = 512;  // mbarriers, TMEM slot, abort flag
constexpr int kMaxBias = 512;        // projection bias staged in shared memory
constexpr uint32_t kBiasBytes = kMaxBias * 4;

struct DwpArgs {
  int n, ih, iw, ce, oh, ow, cout, np, n_ntiles, pt, pl, tiles_h, tiles_w, kblocks, total;
  int hst;                 // halo ring depth
  int nst;                 // A/B stages
  uint32_t halo_buf;       // bytes per halo slot (1024-aligned)
  uint32_t stage_bytes;    // A raw | A lo | B hi | B lo
  uint32_t b_bytes;        // NP x 128
  uint32_t idesc, tmem_cols;
  uint32_t idesc2;         // N = 2 NP (hi and lo weight tiles as one operand)
  int cat;                 // 1: raw*[hi;lo] + lo*hi (two MMAs per k-step), acc stride 2 NP
  int nacc;                // TMEM accumulators (2 or 4; epilogue group g drains g, g + 2)
  const float* wd;         // depthwise weights [3][3][ce]
  const float* bd;         // depthwise bias [ce] or null
  int act_d;
  const float* bp;         // projection bias [cout] or null
  const float* res;        // residual [n][oh][ow][cout] or null
  float* y;                // output [n][oh][ow][cout]
  int act_p;
};

// STEM = true: the same pipeline with an im2col builder for a 3x3 stride-2
// convolution over 3-channel NHWC input (the CNN stems, K = 27 padded to
// one 32-wide K block): the halo slot is a 3-D box of whole input rows
// (W * 3 floats), the builders gather each pixel's 27 taps into its A row.
template <int KS, int S, int TH, int TW, int CB, int R, bool STEM = false, int TN = 1, int NG = 1,
          int CW = 2, int AG = 0, int EG = 2>
__global__ void __launch_bounds__(threads_for(EG), 1)
    dwproj_kernel(const __grid_constant__ CUtensorMap tmX,
                  const __grid_constant__ CUtensorMap tmBhi,
                  const __grid_constant__ CUtensorMap tmBlo,
                  const __grid_constant__ CUtensorMap tmWd,
                  const __grid_constant__ CUtensorMap tmBd,
                  const __grid_constant__ CUtensorMap tmY,
                  const __grid_constant__ CUtensorMap tmR, const DwpArgs p) {
  constexpr int IH = (TH - 1) * S + KS, IW = (TW - 1) * S + KS;
  constexpr int CG = CB / 2;  // channel pairs per sub-block
  constexpr int SUBS = STEM ? 1 : 32 / CB;
  // CW: output columns per builder thread (adjacent; 1 or 2)
  constexpr int WIN = (CW - 1) * S + KS;  // input columns a thread's window spans
  // Stem rows: IW pixels x 3 channels, plus up to 3 floats of 16-byte alignment
  // shift, rounded to whole 16-byte units.
  constexpr int kStemRow = (IW * 3 + 3 + 3) / 4 * 4;
  constexpr uint32_t kHaloBytes = STEM ? IH * kStemRow * 4 : TN * IH * IW * CB * 4;
  constexpr int kTilePx = TN * TH * TW;  // GEMM rows of a tile (TN images of TH x TW)
  // A halo slot: the input box, then the sub-block's depthwise taps [KS*KS][CB]
  // and its bias [CB] (TMA boxes of the weight tensors; zero past c).
  constexpr uint32_t kWOff = (kHaloBytes + 127) / 128 * 128;
  constexpr uint32_t kWBytes = KS * KS * CB * 4;
  constexpr uint32_t kBOff = kWOff + (kWBytes + 127) / 128 * 128;  // TMA: 128-byte aligned
  const uint32_t slot_tx = STEM ? kHaloBytes : kHaloBytes + kWBytes + (p.bd ? CB * 4 : 0);
  // NG builder groups: with NG = 2 the two groups of four warps take
  // alternate K-block steps (a group's stage is the step parity), so two K
  // blocks are built at once; each group covers the whole tile.
  constexpr int kGroupThreads = kBuildWarps * 32 / NG;
  constexpr int kArrive = kBuildWarps / NG;  // warp arrivals per stage / halo phase
  static_assert(NG == 1 || NG == 2, "one or two builder groups");
  static_assert(!STEM || NG == 1, "the stem builder is one group");
  static_assert(STEM || TN * CG * (TW / CW) * (TH / R) == kGroupThreads,
                "one builder thread per (image, rows, column pair, channel pair)");
  static_assert(!STEM || (TH * TW == 128 && S == 2 && (KS == 3 || KS == 7)), "stem tile");
  static_assert(TN * TH * TW <= 128, "a tile is at most 128 GEMM rows");
  static_assert(!STEM || TN == 1, "stem tiles hold one image");
  static_assert(TH % R == 0 && 32 % CB == 0, "tile shape");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* halo = smem;
  uint8_t* stages = halo + (size_t)p.hst * p.halo_buf;
  // Epilogue staging: one 128-row x 32-channel tile per group, 128-byte
  // swizzled (the TMA store / residual load box layout).
  uint8_t* estage = stages + (size_t)p.nst * p.stage_bytes;
  uint64_t* hfull = (uint64_t*)(estage + EG * (size_t)kEStage);
  uint64_t* hempty = hfull + kMaxHalo;
  uint64_t* afull = hempty + kMaxHalo;
  uint64_t* bfull = afull + kMaxStages;
  uint64_t* empty = bfull + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 4;
  uint64_t* drain = tempty + 4;
  uint64_t* rfull = drain + 1;  // [4 * EG]: a warp's residual box landed
  uint32_t* tmem_slot = (uint32_t*)(rfull + 4 * EG);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // Projection bias of every n tile, zero past cout (or without a bias): the
  // epilogue reads it as shared-memory broadcasts instead of global loads.
  float* bias_s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(hfull) + kBarBytes);
  for (int i = threadIdx.x; i < p.n_ntiles * p.np && i < kMaxBias; i += threads_for(EG))
    bias_s[i] = (p.bp && i < p.cout) ? __ldg(p.bp + i) : 0.f;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int h = 0; h < p.hst; ++h) {
      mb_init(&hfull[h], 1);
      mb_init(&hempty[h], kArrive);
    }
    for (int j = 0; j < p.nst; ++j) {
      mb_init(&afull[j], kArrive);
      mb_init(&bfull[j], 1);
      mb_init(&empty[j], 1);
    }
    for (int j = 0; j < 4; ++j) {
      mb_init(&tfull[j], 1);
      mb_init(&tempty[j], 4 * 32);
    }
    mb_init(drain, 1);
    for (int w2 = 0; w2 < 4 * EG; ++w2) mb_init(&rfull[w2], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     sa(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tmem_slot;
  // Set-up above touched only this launch's constants: from here on the
  // previous kernel's output is read and buffers it may still read are written.
  pdl_trigger();
  pdl_wait();

  auto decode = [&](int t, int& nt, int& img, int& ty, int& tx) {
    nt = t % p.n_ntiles;
    int r = t / p.n_ntiles;
    tx = r % p.tiles_w;
    r /= p.tiles_w;
    ty = r % p.tiles_h;
    img = (r / p.tiles_h) * TN;  // first image of the tile
  };

  if (warp == kProdWarp) {
    // ---------------- TMA producers ----------------
    // Lane 0 streams the halo slots (input box + depthwise taps + bias) as far
    // ahead as the ring allows; lane 1 streams the projection weights into
    // the A/B stages as they free up.  Independent lanes, so a stage still
    // under the MMA never holds back the next halo prefetch.
    if (lane == 0) {
      int h = 0;
      uint32_t hph = 0, h_armed = 0, h_par = 0;
      for (int t = blockIdx.x; t < p.total; t += gridDim.x) {
        int nt, img, ty, tx;
        decode(t, nt, img, ty, tx);
        const int x0 = tx * TW * S - p.pl, y0 = ty * TH * S - p.pt;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          for (int sub = 0; sub < SUBS; ++sub) {
            if (!mb_wait(&hempty[h], hph ^ 1, abort_flag, &g_dwp_status, kWaitNs, 64))
              goto halo_done;
            if (sub == 0) DWP_TRACE(0, ((t - (int)blockIdx.x) / (int)gridDim.x) * p.kblocks + kb);
            uint8_t* slot = halo + (size_t)h * p.halo_buf;
            const int c0 = kb * 32 + sub * CB;
            mb_expect_tx(&hfull[h], slot_tx);
            if constexpr (STEM) {
              // whole rows of W * 3 floats; the start rounded down to 16 bytes
              tma_3d(slot, &tmX, &hfull[h], (x0 * 3) & ~3, y0, img);
            } else {
              tma_4d(slot, &tmX, &hfull[h], c0, x0, y0, img);
              tma_2d(slot + kWOff, &tmWd, &hfull[h], c0, 0);
              if (p.bd) tma_2d(slot + kBOff, &tmBd, &hfull[h], c0, 0);
            }
            h_armed |= 1u << h;
            h_par = (h_par & ~(1u << h)) | (hph << h);
            if (++h == p.hst) {
              h = 0;
              hph ^= 1;
            }
          }
        }
      }
    halo_done:
      if (*abort_flag) {  // let this CTA's own copies land before it exits
        volatile int never = 0;
        for (int q = 0; q < p.hst; ++q)
          if (h_armed & (1u << q))
            mb_wait(&hfull[q], (h_par >> q) & 1, &never, &g_dwp_status, kDrainNs, 64);
      }
    } else if (lane == 1) {
      int j = 0;
      uint32_t eph = 0, b_armed = 0, b_par = 0;
      for (int t = blockIdx.x; t < p.total; t += gridDim.x) {
        const int nt = t % p.n_ntiles;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mb_wait(&empty[j], eph ^ 1, abort_flag, &g_dwp_status, kWaitNs, 64))
            goto b_done;
          uint8_t* st = stages + (size_t)j * p.stage_bytes;
          mb_expect_tx(&bfull[j], 2 * p.b_bytes);
          tma_2d(st + 2 * kAHalf, &tmBhi, &bfull[j], kb * 32, nt * p.np);
          tma_2d(st + 2 * kAHalf + p.b_bytes, &tmBlo, &bfull[j], kb * 32, nt * p.np);
          b_armed |= 1u << j;
          b_par = (b_par & ~(1u << j)) | (eph << j);
          if (++j == p.nst) {
            j = 0;
            eph ^= 1;
          }
        }
      }
    b_done:
      if (*abort_flag) {
        volatile int never = 0;
        for (int q = 0; q < p.nst; ++q)
          if (b_armed & (1u << q))
            mb_wait(&bfull[q], (b_par >> q) & 1, &never, &g_dwp_status, kDrainNs, 64);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int j = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < p.total; t += gridDim.x) {
        if (!mb_wait(&tempty[acc], aph ^ 1, abort_flag, &g_dwp_status, kWaitNs, 64)) break;
        tc_after();
        const uint32_t d = tmem + (uint32_t)(acc * p.np * (1 + p.cat));
        bool ok = true;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mb_wait(&afull[j], ph, abort_flag, &g_dwp_status, kWaitNs, 32) ||
              !mb_wait(&bfull[j], ph, abort_flag, &g_dwp_status, kWaitNs, 32)) {
            ok = false;
            break;
          }
          tc_after();
          DWP_TRACE(5, ((t - (int)blockIdx.x) / (int)gridDim.x) * p.kblocks + kb);
          const uint32_t a_raw = sa(stages + (size_t)j * p.stage_bytes);
          const uint32_t a_lo = a_raw + kAHalf;
          const uint32_t b_hi = a_raw + 2 * kAHalf;
          const uint32_t b_lo = b_hi + p.b_bytes;
          if (p.cat) {
            // The hi and lo weight tiles are contiguous 128-byte rows: one
            // N = 2 NP operand.  Columns [0, NP) collect raw*hi + lo*hi,
            // columns [NP, 2 NP) raw*lo; the epilogue adds the two halves.
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t off = k * 32;  // 8 tf32 along K
              mma_tf32(d, sw128_desc(a_raw + off), sw128_desc(b_hi + off), p.idesc2,
                       (kb | k) ? 1u : 0u);
              mma_tf32(d, sw128_desc(a_lo + off), sw128_desc(b_hi + off), p.idesc, 1u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t off = k * 32;  // 8 tf32 along K
              mma_tf32(d, sw128_desc(a_lo + off), sw128_desc(b_hi + off), p.idesc,
                       (kb | k) ? 1u : 0u);
              mma_tf32(d, sw128_desc(a_raw + off), sw128_desc(b_lo + off), p.idesc, 1u);
              mma_tf32(d, sw128_desc(a_raw + off), sw128_desc(b_hi + off), p.idesc, 1u);
            }
          }
          issued = true;
          mma_commit(&empty[j]);
          if (++j == p.nst) {
            j = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == p.nacc) {
          acc = 0;
          aph ^= 1;
        }
      }
      if (*abort_flag && issued) {  // this CTA's MMAs finish before TMEM is freed
        mma_commit(drain);
        volatile int never = 0;
        mb_wait(drain, 0, &never, &g_dwp_status, kDrainNs, 64);
      }
    }
  } else if (STEM && warp < kBuildWarps) {
    // ---------------- builders (stem): im2col -> A tile (raw, lo) ----------------
    // Thread: GEMM row m (pixel) and half of the 32 K columns of each K block;
    // k = (ky*KS+kx)*3+c (OHWI weight order), zero for k >= KS*KS*3.  The
    // producer streams the tile's input box once per K block.
    constexpr int kTaps = KS * KS * 3;
    constexpr int kKB = (kTaps + 31) / 32;  // K blocks (p.kblocks); unrolled so every tap's
                                            // halo offset is a compile-time constant
    const int tid = threadIdx.x;
    const int m = tid & 127, khalf = tid >> 7;
    const int oy_l = m / TW, ox_l = m % TW;
    int j = 0, h = 0;
    uint32_t eph = 0, hph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total && ok; t += gridDim.x) {
      int nt, img, ty, tx;
      decode(t, nt, img, ty, tx);
      const int shift = (tx * TW * S - p.pl) * 3 - (((tx * TW * S - p.pl) * 3) & ~3);
      const int st_i = (t - (int)blockIdx.x) / (int)gridDim.x;
      const float* const base = reinterpret_cast<const float*>(halo) + oy_l * S * kStemRow +
                                shift + ox_l * S * 3;
#pragma unroll
      for (int kb = 0; kb < kKB; ++kb) {
        ok = __all_sync(0xffffffffu,
                        mb_wait(&empty[j], eph ^ 1, abort_flag, &g_dwp_status, kWaitNs, 64));
        if (!ok) break;
        if (tid == 0 && kb == 0) DWP_TRACE(1, st_i);
        ok = __all_sync(0xffffffffu,
                        mb_wait(&hfull[h], hph, abort_flag, &g_dwp_status, kWaitNs, 32));
        if (!ok) break;
        if (tid == 0 && kb == 0) DWP_TRACE(2, st_i);
        const float* in = base + (size_t)h * (p.halo_buf / 4);
        float vals[16];
        // khalf is warp-uniform: each branch's 16 offsets are constants.
        auto gather = [&](auto half) {
          constexpr int kh = decltype(half)::value;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int k = kb * 32 + kh * 16 + e;
            const int ky = k / (KS * 3), kx = (k / 3) % KS, c = k % 3;
            vals[e] = k < kTaps ? in[ky * kStemRow + kx * 3 + c] : 0.f;
          }
        };
        if (khalf) gather(std::integral_constant<int, 1>{});
        else gather(std::integral_constant<int, 0>{});
        __syncwarp();
        if (lane == 0) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mb_arrive(&hempty[h]);
        }
        if (++h == p.hst) {
          h = 0;
          hph ^= 1;
        }
        uint8_t* a_raw = stages + (size_t)j * p.stage_bytes;
        uint8_t* a_lo = a_raw + kAHalf;
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int c16 = khalf * 4 + qd;
          const uint32_t off = (uint32_t)m * 128u + (uint32_t)((c16 ^ (m & 7)) * 16);
          const float4 v = make_float4(vals[4 * qd], vals[4 * qd + 1], vals[4 * qd + 2],
                                       vals[4 * qd + 3]);
          *reinterpret_cast<float4*>(a_raw + off) = v;
          *reinterpret_cast<float4*>(a_lo + off) =
              make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mb_arrive(&afull[j]);
        if (tid == 0 && kb == 0) DWP_TRACE(4, st_i);
        if (++j == p.nst) {
          j = 0;
          eph ^= 1;
        }
      }
    }
  } else if (!STEM && warp < kBuildWarps) {
    // ---------------- builders: depthwise conv -> A tile (raw, lo) ----------------
    // Warps run independently; each hands a halo slot back after its lanes'
    // reads (__syncwarp, then one elected proxy fence + arrive: the TMA
    // refill cannot overtake a slow lane) and marks its part of the A tile
    // written the same way.  Wait results are voted per warp, so a wait that
    // gave up makes the whole warp leave together.
    const int tid = threadIdx.x;
    const int bgrp = tid / kGroupThreads;  // builder group: steps with step % NG == bgrp
    const int gtid = tid % kGroupThreads;
    const int cg = gtid % CG;
    // First of this thread's columns.  With one column per thread and
    // 16-channel blocks (64 bytes a pixel), a warp's four lane groups take
    // columns {0, 1, 4, 5} or {2, 3, 6, 7}: their halo pixels then alternate
    // between the two 64-byte bank halves, and so do their A-tile rows
    // after the 128-byte swizzle (adjacent even columns would put all four
    // on the same 16 banks).
    const int colg = (gtid / CG) % (TW / CW);
    const int ox_l = CW == 1 ? ((colg & 1) | ((colg & 2) << 1) | ((colg & 4) >> 1) | (colg & ~7))
                             : colg * CW;
    const int rg = (gtid / (CG * (TW / CW))) % (TH / R);
    const int im = gtid / (CG * (TW / CW) * (TH / R));  // image of the tile
    int step = 0;
    for (int t = blockIdx.x; t < p.total; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < p.kblocks && ok; ++kb, ++step) {
        if (NG == 2 && (step & 1) != bgrp) continue;
        // The stage's previous MMAs are done before its A tile is rewritten
        // (stage j = step mod nst; this is its (step / nst)-th use).  With two
        // groups and three stages a stage's uses alternate between the
        // groups, but a group at step s has built s - 2, which needed the MMA
        // of s - 5 (so of s - 6) done: the stage is never two phases behind.
        const int j = step % p.nst;
        ok = __all_sync(0xffffffffu, mb_wait(&empty[j], ((uint32_t)(step / p.nst) & 1u) ^ 1u,
                                             abort_flag, &g_dwp_status, kWaitNs, 64));
        if (!ok) break;
        uint8_t* a_raw = stages + (size_t)j * p.stage_bytes;
        uint8_t* a_lo = a_raw + kAHalf;
        for (int sub = 0; sub < SUBS; ++sub) {
          const int cl = sub * CB + cg * 2;  // channel within the 32-channel K block
          // Halo slots are filled in sub-block order over all steps.
          const int seq = step * SUBS + sub;
          const int h = seq % p.hst;
          const uint32_t hph = (uint32_t)(seq / p.hst) & 1u;
          if (gtid == 0 && sub == 0) DWP_TRACE(1, step);
          // With two groups the slot's previous fill (sequence seq - hst) may
          // belong to the other group, which can lag a step behind; until it
          // has released that fill, this fill's parity would also match the
          // phase before (the fill two back).  So first wait for that release
          // on the slot's empty barrier (its phase count is unambiguous here:
          // this group has not released seq yet), then for this fill.
          bool wok = true;
          if (NG == 2 && seq >= p.hst)
            wok = mb_wait(&hempty[h], hph ^ 1u, abort_flag, &g_dwp_status, kWaitNs, 32);
          if (wok) wok = mb_wait(&hfull[h], hph, abort_flag, &g_dwp_status, kWaitNs, 32);
          ok = __all_sync(0xffffffffu, wok);
          if (!ok) break;
          if (gtid == 0 && sub == 0) DWP_TRACE(2, step);
          const uint8_t* slot = halo + (size_t)h * p.halo_buf;
          const float* in = reinterpret_cast<const float*>(slot) + im * (IH * IW * CB);
          const float* wsm = reinterpret_cast<const float*>(slot + kWOff);
          float2 wr[KS][KS];
#pragma unroll
          for (int ky = 0; ky < KS; ++ky)
#pragma unroll
            for (int kx = 0; kx < KS; ++kx)
              wr[ky][kx] = *reinterpret_cast<const float2*>(wsm + (ky * KS + kx) * CB + cg * 2);
          const float2 bv = p.bd ? *reinterpret_cast<const float2*>(slot + kBOff + cg * 8)
                                 : make_float2(0.f, 0.f);
          float2 acc[R][CW];
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < CW; ++c) acc[r][c] = bv;
#pragma unroll
          for (int jj = 0; jj < (R - 1) * S + KS; ++jj) {
            const int iy = rg * R * S + jj;
            float2 row[WIN];
#pragma unroll
            for (int ix = 0; ix < WIN; ++ix)
              row[ix] = *reinterpret_cast<const float2*>(in + ((iy * IW) + ox_l * S + ix) * CB +
                                                         cg * 2);
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const int ky = jj - r * S;
              if (ky < 0 || ky >= KS) continue;
#pragma unroll
              for (int c = 0; c < CW; ++c)
#pragma unroll
                for (int kx = 0; kx < KS; ++kx)
                  acc[r][c] = ffma2(row[c * S + kx], wr[ky][kx], acc[r][c]);
            }
          }
          if (gtid == 0 && sub == 0) DWP_TRACE(3, step);
          __syncwarp();
          if (gtid == 0 && sub == 0) DWP_TRACE(10, step);
          if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mb_arrive(&hempty[h]);
          }
          // GEMM row m = (rg*R + r)*TW + ox_l + c; TW is a multiple of 8, so the
          // 128-byte swizzle phase m & 7 = (ox_l + c) & 7 does not depend on r.
          const uint32_t c16s = (uint32_t)(cl >> 2) << 4;  // 16-byte chunk, in bytes
          const uint32_t in16 = (uint32_t)(cl & 3) * 4;    // byte offset inside the chunk
          const uint32_t row0 = (uint32_t)((im * TH * TW + rg * R * TW + ox_l) * 128) + in16;
          with_act_sel<AG>(p.act_d, [&](auto tag) {
            constexpr int A = decltype(tag)::value;
            // Clamped activations cannot produce inf: the lo term needs no
            // special-value check there.
            constexpr bool kFinite = A == SPX_ACT_RELU6 || A == SPX_ACT_RELU_N1_TO_1;
#pragma unroll
            for (int c = 0; c < CW; ++c) {
              const uint32_t colo = row0 + (uint32_t)(c * 128) +
                                    (c16s ^ ((uint32_t)((ox_l + c) & 7) << 4));
#pragma unroll
              for (int r = 0; r < R; ++r) {
                float2 v = acc[r][c];
                v.x = act_c<A>(v.x);
                v.y = act_c<A>(v.y);
                const uint32_t off = colo + (uint32_t)(r * TW * 128);
                *reinterpret_cast<float2*>(a_raw + off) = v;
                *reinterpret_cast<float2*>(a_lo + off) =
                    kFinite ? make_float2(tf32_lo_finite(v.x), tf32_lo_finite(v.y))
                            : make_float2(tf32_lo(v.x), tf32_lo(v.y));
              }
            }
          });
        }
        if (!ok) break;
        if (gtid == 0) DWP_TRACE(8, step);
        // Generic-proxy writes of the A tile become visible to the tensor core.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (gtid == 0) DWP_TRACE(9, step);
        __syncwarp();
        if (lane == 0) mb_arrive(&afull[j]);
        if (gtid == 0) DWP_TRACE(4, step);
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue (warps 10-17) ----------------
    // A lane owns one GEMM row (one output pixel): tcgen05.ld gives it 32
    // consecutive output channels, which it writes (with bias, residual and
    // activation) as one contiguous 128-byte run of the NHWC output.
    // Group g (warps 10+4g .. 13+4g) drains the CTA's tiles of parity g, which
    // the MMA issuer puts in accumulator g: two tiles drain at once.  Each
    // warp owns its 32 rows end to end: its own 4 KB staging tile, its own
    // residual box and TMA store (32 channels x TW x 32/TW rows), so warps
    // never wait on one another.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int grp = (warp - kEpiWarp0) / 4;
    int acc = grp;  // accumulators grp, grp + 2, ... (tiles of this group's parity)
    uint8_t* stg = estage + (size_t)(warp - kEpiWarp0) * kEWarp;
    uint64_t* rbar = &rfull[warp - kEpiWarp0];
    const int row0 = q * 32;                     // first GEMM row of this warp
    const int w_im = row0 / (TH * TW);           // image of the tile these rows are in
    const int w_oy = (row0 % (TH * TW)) / TW;    // their first output row in the tile
    const bool w_live = row0 < kTilePx;          // rows past a 64-row tile are padding
    uint32_t aph = 0, rph = 0;
    bool ok_all = true;
    for (int t = blockIdx.x + grp * gridDim.x; t < p.total; t += EG * gridDim.x) {
      int nt, img, ty, tx;
      decode(t, nt, img, ty, tx);
      const bool ok = __all_sync(0xffffffffu, mb_wait(&tfull[acc], aph, abort_flag,
                                                      &g_dwp_status, kWaitNs, 128));
      if (!ok) break;
      tc_after();
      if (warp == kEpiWarp0 + 2 && lane == 0) DWP_TRACE(6, (t - (int)blockIdx.x) / (int)gridDim.x);
      const uint32_t tbase =
          tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * p.np * (1 + p.cat));
      const int ox0 = tx * TW, oy0 = ty * TH + w_oy, im = img + w_im;
      for (int c0 = 0; c0 < p.np; c0 += 32) {
        const int n0 = nt * p.np + c0;
        if (n0 >= p.cout) break;  // uniform
        float v[32];
        tmem_ld_32x32(tbase + (uint32_t)c0, v);
        if (warp == kEpiWarp0 + 2 && lane == 0 && c0 == 0)
          DWP_TRACE(12, (t - (int)blockIdx.x) / (int)gridDim.x);
        if (p.cat) {
          float v2[32];
          tmem_ld_32x32(tbase + (uint32_t)(p.np + c0), v2);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] += v2[e];
        }
        if (warp == kEpiWarp0 + 2 && lane == 0 && c0 == 0)
          DWP_TRACE(13, (t - (int)blockIdx.x) / (int)gridDim.x);
        if (lane == 0 && w_live) {
          bulk_wait_read0();  // this warp's previous store has read the staging tile
          if (p.res) {
            mb_expect_tx(rbar, kEWarp);
            tma_4d(stg, &tmR, rbar, n0, ox0, oy0, im);
          }
        }
        __syncwarp();
        if (warp == kEpiWarp0 + 2 && lane == 0 && c0 == 0)
          DWP_TRACE(11, (t - (int)blockIdx.x) / (int)gridDim.x);
        if (p.res && w_live) {
          const bool rok = __all_sync(0xffffffffu, mb_wait(rbar, rph, abort_flag, &g_dwp_status,
                                                           kWaitNs, 64));
          rph ^= 1;
          if (!rok) {
            ok_all = false;
            break;
          }
        }
        float4* row = reinterpret_cast<float4*>(stg + lane * 128);
        with_act_sel<AG>(p.act_p, [&](auto tag) {
          constexpr int A = decltype(tag)::value;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 b4 = reinterpret_cast<const float4*>(bias_s + n0)[e];
            const float4 r4 = p.res ? row[e ^ (lane & 7)] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 o;
            o.x = act_c<A>(v[4 * e + 0] + b4.x + r4.x);
            o.y = act_c<A>(v[4 * e + 1] + b4.y + r4.y);
            o.z = act_c<A>(v[4 * e + 2] + b4.z + r4.z);
            o.w = act_c<A>(v[4 * e + 3] + b4.w + r4.w);
            row[e ^ (lane & 7)] = o;
          }
        });
        if (warp == kEpiWarp0 + 2 && lane == 0 && c0 == 0)
          DWP_TRACE(14, (t - (int)blockIdx.x) / (int)gridDim.x);
        // Generic-proxy writes of the tile become visible to the TMA store.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && w_live) {
          tma_store_4d(&tmY, stg, n0, ox0, oy0, im);  // clipped at the map edges and cout
          bulk_commit();
        }
      }
      if (!ok_all) break;
      tc_before();
      mb_arrive(&tempty[acc]);
      if (warp == kEpiWarp0 + 2 && lane == 0) DWP_TRACE(7, (t - (int)blockIdx.x) / (int)gridDim.x);
      acc += EG;
      if (acc >= p.nacc) {
        acc -= p.nacc;
        aph ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's stores have completed
  }

  tc_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                             const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                             const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) ==
            cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = (EncodeFn)q;
  });
  return fn;
}

// Output (and residual) NHWC [n][oh][ow][cout]: 32-channel x TW x 32/TW-row
// boxes (one epilogue warp's rows), 128-byte swizzle (its staging layout).  Boxes past the map or past
// cout are clipped on store and zero-filled on load.
int out_map(EncodeFn fn, CUtensorMap* m, const float* t, int n, int oh, int ow, int cout, int th,
            int tw, int tn = 1) {
  cuuint64_t dims[4] = {(cuuint64_t)cout, (cuuint64_t)ow, (cuuint64_t)oh, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)cout * 4, (cuuint64_t)ow * cout * 4,
                           (cuuint64_t)oh * ow * cout * 4};
  // one epilogue warp's 32 rows: TW columns x 32 / TW rows of one image
  (void)th;
  (void)tn;
  cuuint32_t box[4] = {32, (cuuint32_t)tw, (cuuint32_t)(32 / tw), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)t, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SPX_OK : fail(SPX_ERR_CUDA, "output map encode failed (%d)", (int)r);
}

int num_sms() {
  static int v = 0;
  if (!v) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    if (v <= 0) v = kNumSms;
  }
  return v;
}

// Tile configuration of one instantiation.
struct DwpCfg {
  int th, tw, cb;
};

template <int KS, int S, int TH, int TW, int CB, int R, int TN = 1, int NG = 1, int CW = 2,
          int EG = 2>
int launch_cfg(cudaStream_t s, int64_t* cnt, const float* x, const float* wd, const float* bd,
               const float* w_hi, const float* w_lo, const float* bp, const float* res, float* y,
               const spx_dwproj_params* q, bool dry_run, uint32_t* smem_out) {
  constexpr int IH = (TH - 1) * S + KS, IW = (TW - 1) * S + KS;
  constexpr uint32_t kHaloBytes = TN * IH * IW * CB * 4;
  DwpArgs p{};
  p.n = q->n;
  p.ih = q->ih;
  p.iw = q->iw;
  p.ce = q->c;
  p.oh = q->oh;
  p.ow = q->ow;
  p.cout = q->cout;
  p.n_ntiles = q->cout <= 256 ? 1 : (int)ceil_div(q->cout, 256);
  const int per = (int)ceil_div(q->cout, p.n_ntiles);
  p.np = (int)ceil_div(per, 32) * 32;
  p.pt = q->pad_top;
  p.pl = q->pad_left;
  p.tiles_h = (int)ceil_div(q->oh, TH);
  p.tiles_w = (int)ceil_div(q->ow, TW);
  p.kblocks = (int)ceil_div(q->c, 32);
  const int64_t total = (int64_t)p.n_ntiles * ceil_div(q->n, TN) * p.tiles_h * p.tiles_w;
  if (total > INT32_MAX) return fail(SPX_ERR_UNSUPPORTED, "dw_project: too many tiles");
  p.total = (int)total;
  constexpr uint32_t kSlotBytes =
      (kHaloBytes + 127) / 128 * 128 + (KS * KS * CB * 4 + 127) / 128 * 128 + CB * 4;
  p.halo_buf = (kSlotBytes + 1023) / 1024 * 1024;
  p.b_bytes = (uint32_t)p.np * 128;
  p.stage_bytes = 2 * kAHalf + 2 * p.b_bytes;
  p.cat = p.np <= 128 ? 1 : 0;
  // Four accumulators where tensor memory holds them: the MMA can then run
  // up to two tiles ahead of an epilogue group (short K loops).
  p.nacc = (g_dwp_accs == 4 && 4 * p.np * (1 + p.cat) <= 512) ? 4 : 2;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.nacc * p.np * (1 + p.cat))) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = idesc_tf32(128, p.np);
  p.idesc2 = idesc_tf32(128, 2 * p.np);
  p.wd = wd;
  p.bd = bd;
  p.act_d = q->act_dw;
  p.bp = bp;
  p.res = res;
  p.y = y;
  p.act_p = q->act_proj;
  const uint32_t cap = 227 * 1024;
  // Shared memory: as many A/B stages as fit (up to the "dwp_stages"
  // option) with at least two halo slots, then a third halo slot if it fits.
  auto need = [&](int nst, int hst) {
    return 1024 + (uint32_t)nst * p.stage_bytes + EG * kEStage + kBarBytes + kBiasBytes +
           (uint32_t)hst * p.halo_buf;
  };
  // Half-width halo blocks (CB = 16: two fills per K block) need the third
  // halo slot more than a third A/B stage; full-width ones the other way
  // round.
  p.nst = 0;
  if (CB < 32) {
    for (int hst = 3; hst >= 2 && !p.nst; --hst)
      for (int nst = g_dwp_stages; nst >= 2; --nst)
        if (need(nst, hst) <= cap) {
          p.nst = nst;
          p.hst = hst;
          break;
        }
  } else {
    for (int nst = g_dwp_stages; nst >= 2 && !p.nst; --nst)
      for (int hst = 3; hst >= 2; --hst)
        if (need(nst, hst) <= cap) {
          p.nst = nst;
          p.hst = hst;
          break;
        }
  }
  if (!p.nst) return fail(SPX_ERR_UNSUPPORTED, "dw_project: tile buffers exceed shared memory");
  const uint32_t smem = need(p.nst, p.hst);
  if (smem_out) *smem_out = smem;
  if (dry_run) return SPX_OK;

  EncodeFn fn = encoder();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap mx, mh, ml, mw, mb, my, mr;
  if (int rc = out_map(fn, &my, y, q->n, q->oh, q->ow, q->cout, TH, TW, TN)) return rc;
  mr = my;
  if (res) {
    if (int rc = out_map(fn, &mr, res, q->n, q->oh, q->ow, q->cout, TH, TW, TN)) return rc;
  }
  {
    cuuint64_t dims[4] = {(cuuint64_t)q->c, (cuuint64_t)q->iw, (cuuint64_t)q->ih,
                          (cuuint64_t)q->n};
    cuuint64_t strides[3] = {(cuuint64_t)q->c * 4, (cuuint64_t)q->iw * q->c * 4,
                             (cuuint64_t)q->ih * q->iw * q->c * 4};
    cuuint32_t box[4] = {(cuuint32_t)CB, (cuuint32_t)IW, (cuuint32_t)IH, (cuuint32_t)TN};
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "dw_project: halo map encode failed (%d)", (int)r);
  }
  for (int b = 0; b < 2; ++b) {
    cuuint64_t dims[2] = {(cuuint64_t)q->c, (cuuint64_t)q->cout};
    cuuint64_t strides[1] = {(cuuint64_t)q->c * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)p.np};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(b ? &ml : &mh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    (void*)(b ? w_lo : w_hi), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(SPX_ERR_CUDA, "dw_project: weight map encode failed (%d)", (int)r);
  }
  // Depthwise taps [KS*KS][c] and bias [1][c]: CB-channel boxes per sub-block.
  for (int b = 0; b < 2; ++b) {
    if (b == 1 && !bd) {
      mb = mw;  // unused: the kernel loads no bias box without a bias
      break;
    }
    cuuint64_t dims[2] = {(cuuint64_t)q->c, (cuuint64_t)(b ? 1 : KS * KS)};
    cuuint64_t strides[1] = {(cuuint64_t)q->c * 4};
    cuuint32_t box[2] = {(cuuint32_t)CB, (cuuint32_t)(b ? 1 : KS * KS)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(b ? &mb : &mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    (void*)(b ? bd : wd), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(SPX_ERR_CUDA, "dw_project: depthwise weight map encode failed (%d)", (int)r);
  }
  const bool heavy = act_group(p.act_d) || act_group(p.act_p);
  auto kern = heavy ? dwproj_kernel<KS, S, TH, TW, CB, R, false, TN, NG, CW, 1, EG>
                    : dwproj_kernel<KS, S, TH, TW, CB, R, false, TN, NG, CW, 0, EG>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(dwproj_kernel<KS, S, TH, TW, CB, R, false, TN, NG, CW, 0, EG>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
    if (attr == cudaSuccess)
      attr = cudaFuncSetAttribute(dwproj_kernel<KS, S, TH, TW, CB, R, false, TN, NG, CW, 1, EG>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "dw_project: smem attribute");
  const int grid = (int)(p.total < num_sms() ? p.total : num_sms());
  const cudaError_t le = launch_pdl(kern, dim3(grid), dim3(threads_for(EG)), smem, s, mx, mh, ml, mw, mb,
                                    my, mr, p);
  if (le != cudaSuccess) return check_cuda(le, "dw_project launch");
  return after_launch(cnt, "dw_project");
}

bool al16(const void* v) { return ((uintptr_t)v & 15) == 0; }


// The stem instantiation: 8 x 16 output pixels per tile, one 32-wide K block.
constexpr int kStemTH = 8, kStemTW = 16;

template <int KS>
int launch_stem(cudaStream_t s, int64_t* cnt, const float* x, const float* w_hi,
                const float* w_lo, const float* bias, float* y, const spx_conv_params* q) {
  constexpr int IH = (kStemTH - 1) * 2 + KS, IW = (kStemTW - 1) * 2 + KS;
  constexpr int kKPad = (KS * KS * 3 + 31) / 32 * 32;  // weights [oc][kKPad], zero past the taps
  constexpr int kRow = (IW * 3 + 3 + 3) / 4 * 4;
  constexpr uint32_t kHalo = IH * kRow * 4;
  DwpArgs p{};
  p.n = q->n;
  p.ih = q->ih;
  p.iw = q->iw;
  p.ce = kKPad;
  p.oh = q->oh;
  p.ow = q->ow;
  p.cout = q->oc;
  p.n_ntiles = 1;
  p.np = (int)ceil_div(q->oc, 32) * 32;
  p.pt = q->pad_top;
  p.pl = q->pad_left;
  p.tiles_h = (int)ceil_div(q->oh, kStemTH);
  p.tiles_w = (int)ceil_div(q->ow, kStemTW);
  p.kblocks = kKPad / 32;
  const int64_t total = (int64_t)q->n * p.tiles_h * p.tiles_w;
  if (total > INT32_MAX) return fail(SPX_ERR_UNSUPPORTED, "stem: too many tiles");
  p.total = (int)total;
  p.halo_buf = (kHalo + 1023) / 1024 * 1024;
  p.b_bytes = (uint32_t)p.np * 128;
  p.stage_bytes = 2 * kAHalf + 2 * p.b_bytes;
  p.cat = p.np <= 128 ? 1 : 0;
  // Four accumulators where tensor memory holds them: the MMA can then run
  // up to two tiles ahead of an epilogue group (short K loops).
  p.nacc = (g_dwp_accs == 4 && 4 * p.np * (1 + p.cat) <= 512) ? 4 : 2;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.nacc * p.np * (1 + p.cat))) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = idesc_tf32(128, p.np);
  p.idesc2 = idesc_tf32(128, 2 * p.np);
  p.bp = bias;
  p.y = y;
  p.act_p = q->activation;
  // As many A/B stages as fit next to two halo slots (up to "dwp_stages"),
  // then up to four halo slots.
  const uint32_t cap = 227 * 1024;
  auto need = [&](int nst, int hst) {
    return 1024 + (uint32_t)nst * p.stage_bytes + kMaxEpiGroups * kEStage + kBarBytes + kBiasBytes +
           (uint32_t)hst * p.halo_buf;
  };
  p.nst = 2;
  while (p.nst < g_dwp_stages && need(p.nst + 1, 2) <= cap) ++p.nst;
  p.hst = 2;
  while (p.hst < 4 && need(p.nst, p.hst + 1) <= cap) ++p.hst;
  const uint32_t smem = need(p.nst, p.hst);
  EncodeFn fn = encoder();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap mx, mh, ml, my;
  if (int rc = out_map(fn, &my, y, q->n, q->oh, q->ow, q->oc, kStemTH, kStemTW)) return rc;
  {
    cuuint64_t dims[3] = {(cuuint64_t)q->iw * 3, (cuuint64_t)q->ih, (cuuint64_t)q->n};
    cuuint64_t strides[2] = {(cuuint64_t)q->iw * 12, (cuuint64_t)q->ih * q->iw * 12};
    cuuint32_t box[3] = {(cuuint32_t)kRow, (cuuint32_t)IH, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)x, dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "stem: input map encode failed (%d)", (int)r);
  }
  for (int b = 0; b < 2; ++b) {
    cuuint64_t dims[2] = {(cuuint64_t)kKPad, (cuuint64_t)q->oc};
    cuuint64_t strides[1] = {(cuuint64_t)kKPad * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)p.np};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(b ? &ml : &mh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)(b ? w_lo : w_hi),
                    dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "stem: weight map encode failed (%d)", (int)r);
  }
  auto kern = act_group(p.act_p) ? dwproj_kernel<KS, 2, kStemTH, kStemTW, 32, 4, true, 1, 1, 2, 1>
                                 : dwproj_kernel<KS, 2, kStemTH, kStemTW, 32, 4, true, 1, 1, 2, 0>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(dwproj_kernel<KS, 2, kStemTH, kStemTW, 32, 4, true, 1, 1, 2, 0>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
    if (attr == cudaSuccess)
      attr = cudaFuncSetAttribute(dwproj_kernel<KS, 2, kStemTH, kStemTW, 32, 4, true, 1, 1, 2, 1>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "stem: smem attribute");
  const int grid = (int)(p.total < num_sms() ? p.total : num_sms());
  const cudaError_t le = launch_pdl(kern, dim3(grid), dim3(threads_for(kMaxEpiGroups)), smem, s, mx, mh, ml, mx, mx,
                                    my, my, p);
  if (le != cudaSuccess) return check_cuda(le, "stem launch");
  return after_launch(cnt, "stem_tc");
}

}  // namespace

#ifdef SPX_DWP_TRACE
extern "C" int spx_dwp_trace(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_dwp_trace, sizeof(g_dwp_trace)) == cudaSuccess ? 0 : 3;
}
#endif

int dwp_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dwp_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_dwp_status, &zero, sizeof(int));
  }
  return v;
}

// 3x3 stride-2 convolution of 3-channel NHWC input on the tensor cores (the
// CNN stems).  w_hi / w_lo: [oc][32] tf32 split of the OHWI weights flattened
// to 27 taps and zero-padded to 32.  SPX_ERR_UNSUPPORTED for other shapes.
int launch_stem_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* w_hi,
                   const float* w_lo, const float* bias, float* y, const spx_conv_params* q,
                   bool dry_run) {
  if (!q) return fail(SPX_ERR_INVALID_ARGUMENT, "stem: null params");
  if (q->ic != 3 || (q->kh != 3 && q->kh != 7) || q->kw != q->kh || q->stride_h != 2 ||
      q->stride_w != 2 || q->dilation_h != 1 || q->dilation_w != 1 || q->oc <= 0 ||
      q->oc > 128 || q->oc % 4 || q->iw % 4 || q->n <= 0 || q->oh <= 0 || q->ow <= 0 ||
      q->pad_top < 0 || q->pad_left < 0 || q->pad_top >= q->kh || q->pad_left >= q->kw)
    return fail(SPX_ERR_UNSUPPORTED,
                "stem: 3x3 or 7x7 stride-2 over 3 channels (iw % 4 == 0, oc <= 128) only");
  if (dry_run) return SPX_OK;
  if (!x || !w_hi || !w_lo || !y || !al16(x) || !al16(w_hi) || !al16(w_lo) || !al16(y) ||
      (bias && !al16(bias)))
    return fail(SPX_ERR_INVALID_ARGUMENT, "stem: null or unaligned tensor");
  return q->kh == 7 ? launch_stem<7>(s, cnt, x, w_hi, w_lo, bias, y, q)
                    : launch_stem<3>(s, cnt, x, w_hi, w_lo, bias, y, q);
}

// Returns SPX_ERR_UNSUPPORTED (without launching) for shapes the fused kernel
// does not take; `dry_run` only checks eligibility.
int launch_dw_project(cudaStream_t s, int64_t* cnt, const float* x, const float* wd,
                      const float* bd, const float* w_hi, const float* w_lo, const float* bp,
                      const float* res, float* y, const spx_dwproj_params* q, bool dry_run) {
  if (!q) return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: null params");
  if (q->n <= 0 || q->ih <= 0 || q->iw <= 0 || q->c <= 0 || q->oh <= 0 || q->ow <= 0 ||
      q->cout <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: non-positive size");
  if (q->kernel != 3 || (q->stride != 1 && q->stride != 2))
    return fail(SPX_ERR_UNSUPPORTED, "dw_project: 3x3 depthwise with stride 1 or 2 only");
  if (q->c % 4 || q->cout % 4)
    return fail(SPX_ERR_UNSUPPORTED, "dw_project: channel counts must be multiples of 4");
  if (q->cout > 512) return fail(SPX_ERR_UNSUPPORTED, "dw_project: at most 512 outputs");
  if (q->pad_top < 0 || q->pad_left < 0 || q->pad_top > 2 || q->pad_left > 2)
    return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: pads must be 0..2");
  if ((int64_t)(q->oh - 1) * q->stride - q->pad_top + 3 <= 0 ||
      (int64_t)(q->oh - 1) * q->stride - q->pad_top >= q->ih ||
      (int64_t)(q->ow - 1) * q->stride - q->pad_left >= q->iw)
    return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: output size does not match the input");
  if (!dry_run) {
    if (!x || !wd || !w_hi || !w_lo || !y)
      return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: null tensor");
    if (!al16(x) || !al16(wd) || !al16(w_hi) || !al16(w_lo) || !al16(y) || (bd && !al16(bd)) ||
        (bp && !al16(bp)) || (res && !al16(res)))
      return fail(SPX_ERR_INVALID_ARGUMENT, "dw_project: tensors must be 16-byte aligned");
  }
  // Builder groups per tile class (bit set: two groups, each with twice the
  // rows per thread), from the "dwp_groups" option.
  const int g = g_dwp_groups;
  // Tile classes with one epilogue group (and 128 registers a thread), from
  // the "dwp_epi1" option (same bits).
  const int e1 = g_dwp_epi1;
#define SPX_DWP_CFG(bit, S_, TH_, TW_, CB_, R_, TN_, CW_)                                       \
  {                                                                                             \
  if ((e1 >> bit) & 1)                                                                          \
    return (g >> bit) & 1                                                                       \
               ? launch_cfg<3, S_, TH_, TW_, CB_, 2 * R_, TN_, 2, CW_, 1>(                      \
                     s, cnt, x, wd, bd, w_hi, w_lo, bp, res, y, q, dry_run, nullptr)            \
               : launch_cfg<3, S_, TH_, TW_, CB_, R_, TN_, 1, CW_, 1>(                          \
                     s, cnt, x, wd, bd, w_hi, w_lo, bp, res, y, q, dry_run, nullptr);           \
  return (g >> bit) & 1 ? launch_cfg<3, S_, TH_, TW_, CB_, 2 * R_, TN_, 2, CW_, 2>(             \
                              s, cnt, x, wd, bd, w_hi, w_lo, bp, res, y, q, dry_run, nullptr)   \
                        : launch_cfg<3, S_, TH_, TW_, CB_, R_, TN_, 1, CW_, 2>(                 \
                              s, cnt, x, wd, bd, w_hi, w_lo, bp, res, y, q, dry_run, nullptr);  \
  }
  if (q->stride == 1) {
    if (q->ow <= 8) SPX_DWP_CFG(0, 1, 8, 8, 16, 4, 2, 1);
    if (q->c <= 32) SPX_DWP_CFG(4, 1, 8, 16, 32, 4, 1, 2);
    SPX_DWP_CFG(1, 1, 8, 16, 32, 4, 1, 2);
  }
  if (q->ow <= 8) SPX_DWP_CFG(2, 2, 8, 8, 16, 1, 1, 2);
  // Stride 2 with long reductions: 32-channel halo blocks on 64-pixel tiles.
  // A warp's lanes then read two whole 128-byte pixels (the 16-channel
  // blocks put the four pixels a warp reads on the same 16 banks, a 4-way
  // conflict); the smaller tiles cost per-tile work, which only the longer
  // K loops repay (measured: 192 -> 64 at 28x28 69.7 -> 60.8 us, 96 -> 24
  // at 112x112 285.9 -> 312.9 us, b256).
  if (q->c > 160) SPX_DWP_CFG(5, 2, 4, 16, 32, 2, 1, 2);
  SPX_DWP_CFG(3, 2, 8, 16, 16, 2, 1, 2);
#undef SPX_DWP_CFG
}

}  // namespace spx
