// Tensor-core GEMM for sm_100a: TMA -> shared memory -> tcgen05.mma (kind::tf32)
// with the accumulator in TMEM, split "3xTF32" so results keep fp32 accuracy.
//
// Serves the dense contractions whose operands are both K-contiguous:
// pointwise (1x1, stride 1) convolutions over NHWC activations with OHWI
// weights (A = x as [M = n*h*w][K = ic], B = w as [N = oc][K]), and
// fully_connected / linear layers (B = W[out][in]).
//
// Precision: every fp32 operand x is split into hi = rna_tf32(x) and
// lo = rna_tf32(x - hi) (activations on chip, weights either on chip or once
// at load); each k-step issues lo*hi + hi*lo + hi*hi into an fp32 TMEM
// accumulator.  Relative error per product is ~2^-21 (the neglected lo*lo
// term ~2^-22).  The tensor core's accumulate rounds toward zero, so the
// remaining error grows with the K/8 accumulation steps: about 1e-5 of the
// running-sum magnitude at K = 1000 (the kernel tests bound it by K).
//
// Structure: one CTA per SM, persistent over output tiles (n-tile fastest so
// consecutive tiles share the A tile in L2), 18 warps:
//   warp 16     TMA producer: per k-block an A tile 128 x 32 and either a B
//               tile BN x 32 or, with pre-split weights, its hi and lo tiles,
//               into an S-stage ring (128-byte swizzle, mbarrier tx counts).
//   warps 8-15  converters: split A (and B unless pre-split) of a landed
//               stage, hi in place and lo into a second buffer, then
//               fence.proxy.async + arrive.
//   warp 17     TMEM owner and MMA issuer (one thread): 12 UMMAs per k-block
//               (4 k-steps x 3 products); a commit frees the stage; a commit at
//               the end of a tile hands one of two TMEM accumulators
//               (2 x BN columns) to the epilogue.
//   warps 0-7   epilogue, 32 columns at a time (two warps per TMEM lane
//               quarter, alternating chunks): each warp loads its 32 TMEM
//               lanes x 32 columns, transposes them through a private padded
//               smem tile (warp-synchronous, no block barrier) and then
//               applies bias, residual and activation while reading and
//               writing whole 128-byte row segments of C, so stores are
//               coalesced.  Releasing the accumulator lets tile i's epilogue
//               overlap tile i+1's k-loop.
// Every wait is bounded (globaltimer); on timeout the CTA raises an abort flag,
// records a device status, drains its own in-flight copies and MMAs, frees
// TMEM and exits.  The host reads the status at the next sync.
#include <cuda.h>

#include <mutex>

#include "spx_internal.cuh"

namespace spx {

__device__ int g_tc_status = 0;
int g_tc_epi12 = 1;
int g_tc_conv2 = 1;
int g_tc_lo_tmem = 0;
int g_tc_cat = 1;
int g_tc_acc4 = 1;

#ifdef SPX_TC_TRACE
// Development-only pipeline trace of CTA 0 (not compiled into the library).
__device__ unsigned long long g_tc_trace[16][64];
#define TC_TRACE(ev, i)                                                     \
  do {                                                                      \
    if (blockIdx.x == 0 && (i) < 64) g_tc_trace[ev][i] = gtimer();          \
  } while (0)
#else
#define TC_TRACE(ev, i) \
  do {                  \
  } while (0)
#endif

namespace {

constexpr int kBM = 128;         // UMMA M: output rows per tile
constexpr int kBK = 32;          // fp32 elements per k-block (one 128-byte row)
constexpr int kEpiWarps = 8;     // two per TMEM lane quarter (default)
constexpr int kMaxAcc = 4;       // TMEM accumulators (2, or 4 with two epilogue groups)
constexpr int kMaxEpiWarps = 12; // three per quarter: short k-loops with 3+ chunks per quarter
constexpr int kConvWarps = 8;
constexpr int kProducerWarp = kEpiWarps + kConvWarps;
constexpr int kMmaWarp = kProducerWarp + 1;
constexpr int kThreads = (kMmaWarp + 1) * 32;  // 18 warps
constexpr int kMaxStages = 8;
constexpr int kEpiStride = 36;   // floats per row of a warp's transpose tile
// Per-warp epilogue slot (1024-aligned): a 32 x 32 fp32 TMA staging tile in
// 128-byte-swizzled layout (4 KB), or the padded transpose tile of the
// fallback path (32 x kEpiStride floats).
constexpr uint32_t kEpiSlot = 5120;
constexpr uint32_t kATileBytes = kBM * kBK * 4;       // 16 KB
constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait
constexpr unsigned long long kDrainNs = 200000000ull;     // 0.2 s drain on abort

struct TcArgs {
  int M, N, K, BN, n_tiles, m_tiles, k_blocks, stages;
  uint32_t idesc, tmem_cols, stage_bytes, b_bytes;
  int presplit;  // B arrives as hi and lo tiles: converters split A only
  int tma_store; // C (and the residual) move through TMA, 32 x 32 boxes per warp
  const float* bias;
  const float* res;
  float* c;
  int64_t ldc;
  float alpha;
  int act;
  int vec4;
  // Implicit-GEMM convolution (conv != 0): A is gathered per k-block by a
  // 4-D TMA box over the NHWC input; an M tile is a patch of tn images x th
  // rows x tw columns of output pixels (tn * th * tw <= 128 rows).
  int conv;
  int oh, ow, ic_blocks, kw, sh, pt, pl;
  int th, tw, tn, tiles_h, tiles_w;
  uint32_t a_tx;  // bytes one A load delivers
  int groups;     // epilogue groups taking alternate tiles (1, or 2 for N <= 32 with TMA stores)
  int nacc;       // TMEM accumulators: 2 per group
  int conv_groups;  // converter groups splitting alternate stages (1 or 2)
  int last_ksteps;  // 8-wide k-steps of the last k-block that hold columns < K
  int b_resident;   // one k-block and one n-tile: pre-split B loaded once, not per stage
  int lo_tmem;      // activation lo terms in two TMEM slots (A operand from TMEM)
  int lo_col;       // first TMEM column of the two 32-column lo slots
  uint32_t smem_bytes;  // dynamic shared memory of the launch
  int cat;              // raw A x [B hi; B lo] as one N = 2 BN product (+ lo x hi): an
                        // accumulator spans 2 BN columns, the epilogue adds the halves
  uint32_t idesc2;      // instruction descriptor with N = 2 BN
  int bias_n;           // bias entries staged in shared memory (n_tiles * BN), 0 = read from global
  int epi_warps;  // epilogue warps in use (4, 8 or 12): long k-loops trade them for stages,
                  // 1-block k-loops take 12 (warps 8-11 leave the converters)
};

__device__ __forceinline__ uint32_t su32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on the phase with the given parity.  Returns false when the
// CTA is aborting (another role timed out) or this wait itself timed out.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                         unsigned long long limit = kTimeoutNs,
                                         int max_sleep_ns = 128) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  int sleep_ns = 16;
  for (;;) {
    // Back off between polls so waiting warps leave issue slots and the
    // shared-memory pipe to the warps doing work.
    if (max_sleep_ns > 0) {
      __nanosleep(sleep_ns);
      sleep_ns = sleep_ns * 2 < max_sleep_ns ? sleep_ns * 2 : max_sleep_ns;
    }
#pragma unroll 1
    for (int i = 0; i < 4; ++i)
      if (bar_try(b, parity)) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > limit) {
      *abort_flag = 1;
      atomicExch(&g_tc_status, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(su32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Output pixel index (n * oh + oy) * ow + ox of row r of conv M tile mt, or
// -1 for rows outside the patch or the map.
__device__ __forceinline__ int64_t conv_row(const TcArgs& p, int mt, int r) {
  const int per = p.th * p.tw;
  if (r >= p.tn * per) return -1;
  const int ni = r / per, rem = r % per;
  const int tx = mt % p.tiles_w;
  const int t2 = mt / p.tiles_w;
  const int ty = t2 % p.tiles_h;
  const int nb = t2 / p.tiles_h;
  const int img = nb * p.tn + ni;
  const int oy = ty * p.th + rem / p.tw, ox = tx * p.tw + rem % p.tw;
  if (oy >= p.oh || ox >= p.ow) return -1;
  const int64_t pix = ((int64_t)img * p.oh + oy) * p.ow + ox;
  return pix < p.M ? pix : -1;
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes grouped in 8-row (1024-byte) atoms.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused, K fits one row)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // swizzle: 128B
  return d;
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}
// A operand from tensor memory (lane = row, one 32-bit column per k element).
__device__ __forceinline__ void umma_tf32_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}
// This thread's TMEM lane, 16 consecutive columns from taddr.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(su32(src))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  return __uint_as_float(h);
}

// tf32 round-to-nearest, ties away from zero, on the bit pattern: adding half
// a tf32 ulp (bit 12) to the magnitude and clearing the 13 dropped bits rounds
// |x| half-up, which is ties-away for a sign-magnitude format.  Finite inputs
// only (infinities and NaNs are handled by the callers).
__device__ __forceinline__ uint32_t rna13(uint32_t b) { return (b + 0x1000u) & 0xFFFFE000u; }

// hi = rna_tf32(x), lo = rna_tf32(x - hi).  For finite x, x - hi is exact; for
// inf / nan hi keeps the special value (nan made quiet) and lo is zero, so
// the hi*hi product carries it.
__device__ __forceinline__ void split1(float x, float& hi, float& lo) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7F800000u) == 0x7F800000u) {
    hi = __uint_as_float((b & 0x007FFFFFu) ? 0x7FFFFFFFu : b);
    lo = 0.0f;
    return;
  }
  hi = __uint_as_float(rna13(b));
  lo = __uint_as_float(rna13(__float_as_uint(x - hi)));
}
__device__ __forceinline__ float split_lo(float x, float h) {
  const float r = x - h;
  return r == r ? tf32_rna(r) : 0.0f;
}
__device__ __forceinline__ void split4(const float4& v, float4& h, float4& l) {
  split1(v.x, h.x, l.x);
  split1(v.y, h.y, l.y);
  split1(v.z, h.z, l.z);
  split1(v.w, h.w, l.w);
}
// lo-only split for an operand the MMA reads raw: kind::tf32 uses the upper
// 19 bits of each 32-bit element (sign, exponent, 10 mantissa bits) and
// ignores the low 13, so the raw fp32 tile already is hi = trunc_tf32(x) and
// only lo = rna_tf32(x - trunc_tf32(x)) (exact difference, below one tf32
// ulp) is written.  inf / nan: lo = 0 and the raw special value carries the
// product.  The tensor-core GEMM tests at fp32 tolerance check this reading.
__device__ __forceinline__ float lo_of_raw(float x) {
  const uint32_t b = __float_as_uint(x);
  if ((b & 0x7F800000u) == 0x7F800000u) return 0.0f;
  return __uint_as_float(rna13(__float_as_uint(x - __uint_as_float(b & 0xFFFFE000u))));
}
__device__ __forceinline__ void split_lo_buffer(const float4* x, float4* lo, int n16, int tid,
                                                int nthr) {
  int i = tid;
  for (; i + 3 * nthr < n16; i += 4 * nthr) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = x[i + j * nthr];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      lo[i + j * nthr] =
          make_float4(lo_of_raw(v[j].x), lo_of_raw(v[j].y), lo_of_raw(v[j].z), lo_of_raw(v[j].w));
  }
  for (; i < n16; i += nthr) {
    const float4 v = x[i];
    lo[i] = make_float4(lo_of_raw(v.x), lo_of_raw(v.y), lo_of_raw(v.z), lo_of_raw(v.w));
  }
}

// In-place hi / separate lo split of n16 16-byte vectors, all loads of a
// thread's batch of four issued before its stores.
__device__ __forceinline__ void split_buffer(float4* hi, float4* lo, int n16, int tid, int nthr) {
  int i = tid;
  for (; i + 3 * nthr < n16; i += 4 * nthr) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = hi[i + j * nthr];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 h, l;
      split4(v[j], h, l);
      lo[i + j * nthr] = l;
      hi[i + j * nthr] = h;
    }
  }
  for (; i < n16; i += nthr) {
    float4 h, l;
    split4(hi[i], h, l);
    lo[i] = l;
    hi[i] = h;
  }
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// v += the 32 columns at taddr (two 16-column loads, fewer live registers).
__device__ __forceinline__ void add_tmem32(uint32_t taddr, float (&v)[32]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr + (uint32_t)(h * 16)));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[16 * h + i] += __uint_as_float(r[i]);
  }
}

template <int AG>  // activation group (act_group of p.act)
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmBlo,
                   const __grid_constant__ CUtensorMap tmC,
                   const __grid_constant__ CUtensorMap tmR, const TcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = p.stages;
  // Resident weights (one k-block, one n-tile): B hi | lo loaded once.
  uint8_t* bres = smem + (size_t)S * p.stage_bytes;
  uint8_t* epi = bres + (p.b_resident ? 2 * (size_t)p.b_bytes : 0);  // epi_warps slots of kEpiSlot bytes
  uint64_t* full = (uint64_t*)(epi + p.epi_warps * kEpiSlot);
  uint64_t* conv = full + kMaxStages;
  uint64_t* empty = conv + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + kMaxAcc;
  uint64_t* rfull = tempty + kMaxAcc;  // per epilogue warp: residual box landed
  uint64_t* drain = rfull + kMaxEpiWarps;
  uint64_t* bfull = drain + 1;  // resident weights landed
  uint64_t* lo_empty = bfull + 1;  // [2]: MMAs reading a TMEM lo slot are done
  uint32_t* tmem_slot = (uint32_t*)(lo_empty + 2);
  // B's offset within a stage: after the raw A tile and, unless the lo terms
  // live in TMEM, the A lo tile.
  const uint32_t b_off = p.lo_tmem ? kATileBytes : 2 * kATileBytes;
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // Bias of every n tile (zero past N, or without a bias) where shared memory
  // has room: the TMA epilogue then reads it as broadcasts, not global loads.
  float* bias_s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 512);
  for (int i = threadIdx.x; i < p.bias_n; i += kThreads)
    bias_s[i] = (p.bias && i < p.N) ? __ldg(p.bias + i) : 0.f;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Converters: warps conv_lo .. kEpiWarps + kConvWarps - 1.
  const int conv_lo = p.epi_warps > kEpiWarps ? p.epi_warps : kEpiWarps;
  const int conv_threads = (kEpiWarps + kConvWarps - conv_lo) * 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&conv[s], conv_threads / p.conv_groups);
      bar_init(&empty[s], 1);
    }
    for (int a = 0; a < p.nacc; ++a) {
      bar_init(&tfull[a], 1);
      bar_init(&tempty[a], p.epi_warps / p.groups * 32);
    }
    for (int w = 0; w < kMaxEpiWarps; ++w) bar_init(&rfull[w], 1);
    bar_init(drain, 1);
    bar_init(bfull, 1);
    bar_init(&lo_empty[0], 1);
    bar_init(&lo_empty[1], 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = p.m_tiles * p.n_tiles;
  // Set-up above touched only this launch's constants (the bias): from here
  // on the previous kernel's output is read and buffers it may read are written.
  pdl_trigger();
  pdl_wait();

  if (warp == kProducerWarp) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, armed = 0, armed_par = 0;
      const uint32_t tx = p.a_tx + (p.b_resident ? 0u : p.b_bytes * (p.presplit ? 2u : 1u));
      if (p.b_resident) {
        bar_expect_tx(bfull, 2 * p.b_bytes);
        tma_load_2d(bres, &tmB, bfull, 0, 0);
        tma_load_2d(bres + p.b_bytes, &tmBlo, bfull, 0, 0);
      }
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const int mt = t / p.n_tiles, nt = t % p.n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!bar_wait(&empty[s], ph ^ 1, abort_flag, kTimeoutNs, 64)) goto producer_done;
          uint8_t* st = smem + (size_t)s * p.stage_bytes;
          bar_expect_tx(&full[s], tx);
          if (kb == 0) TC_TRACE(0, (t - blockIdx.x) / gridDim.x);
          if (p.conv) {
            // k-block -> (tap, 32-channel block); the box starts at the
            // patch origin shifted by the tap, padding comes from the zero fill.
            const int tap = kb / p.ic_blocks, cb = kb % p.ic_blocks;
            const int ky = tap / p.kw, kx = tap % p.kw;
            const int tx0 = mt % p.tiles_w, t2 = mt / p.tiles_w;
            const int ty0 = t2 % p.tiles_h, nb = t2 / p.tiles_h;
            tma_load_4d(st, &tmA, &full[s], cb * kBK, tx0 * p.tw * p.sh + kx - p.pl,
                        ty0 * p.th * p.sh + ky - p.pt, nb * p.tn);
          } else {
            tma_load_2d(st, &tmA, &full[s], kb * kBK, mt * kBM);
          }
          if (!p.b_resident) {
            tma_load_2d(st + b_off, &tmB, &full[s], kb * kBK, nt * p.BN);
            if (p.presplit)
              tma_load_2d(st + b_off + p.b_bytes, &tmBlo, &full[s], kb * kBK,
                          nt * p.BN);
          }
          armed |= 1u << s;
          armed_par = (armed_par & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_flag) {  // let this CTA's own copies land before it exits
        if (p.b_resident) {
          volatile int never = 0;
          bar_wait(bfull, 0, &never, kDrainNs);
        }
        for (int i = 0; i < S; ++i)
          if (armed & (1u << i)) {
            volatile int never = 0;
            bar_wait(&full[i], (armed_par >> i) & 1, &never, kDrainNs);
          }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool issued = false;
      if (p.b_resident && !bar_wait(bfull, 0, abort_flag, kTimeoutNs, 64)) goto mma_done;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        if (!bar_wait(&tempty[acc], aph ^ 1, abort_flag, kTimeoutNs, 64)) goto mma_done;
        TC_TRACE(2, (t - blockIdx.x) / gridDim.x);
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * p.BN * (1 + p.cat));
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!bar_wait(&conv[s], ph, abort_flag, kTimeoutNs, 64)) goto mma_done;
          if (kb == 0) TC_TRACE(3, (t - blockIdx.x) / gridDim.x);
          tc_fence_after();
          const uint32_t a_hi = su32(smem + (size_t)s * p.stage_bytes);
          const uint32_t a_lo = a_hi + kATileBytes;
          const uint32_t b_hi = p.b_resident ? su32(bres) : a_hi + b_off;
          const uint32_t lo_t = tmem + (uint32_t)p.lo_col + (uint32_t)((s & 1) * kBK);
          const uint32_t b_lo = b_hi + p.b_bytes;
          // The last k-block stops at the last k-step holding real columns.
          const int ksteps = kb == p.k_blocks - 1 ? p.last_ksteps : kBK / 8;
#pragma unroll
          for (int k = 0; k < kBK / 8; ++k) {
            if (k >= ksteps) break;
            const uint32_t off = k * 32;  // 8 tf32 = 32 bytes along K
            const uint64_t dah = sdesc(a_hi + off), dal = sdesc(a_lo + off);
            const uint64_t dbh = sdesc(b_hi + off), dbl = sdesc(b_lo + off);
            if (p.cat) {
              // B hi and lo are adjacent 128-byte rows: one N = 2 BN operand.
              umma_tf32(d, dah, dbh, p.idesc2, (kb | k) ? 1u : 0u);
              umma_tf32(d, dal, dbh, p.idesc, 1u);
              continue;
            }
            if (p.lo_tmem)
              umma_tf32_ta(d, lo_t + (uint32_t)(k * 8), dbh, p.idesc, (kb | k) ? 1u : 0u);
            else
              umma_tf32(d, dal, dbh, p.idesc, (kb | k) ? 1u : 0u);
            umma_tf32(d, dah, dbl, p.idesc, 1u);
            umma_tf32(d, dah, dbh, p.idesc, 1u);
          }
          issued = true;
          umma_commit(&empty[s]);
          if (p.lo_tmem) umma_commit(&lo_empty[s & 1]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        TC_TRACE(4, (t - blockIdx.x) / gridDim.x);
        if (++acc == p.nacc) {
          acc = 0;
          aph ^= 1;
        }
      }
    mma_done:
      if (*abort_flag && issued) {  // wait for this CTA's MMAs before TMEM is freed
        umma_commit(drain);
        volatile int never = 0;
        bar_wait(drain, 0, &never, kDrainNs);
      }
    }
  } else if (warp >= conv_lo) {
    // ---------------- converters (hi/lo split) ----------------
    // With conv_groups = 2 the two halves take the even and the odd stages
    // of an even-sized ring, so two stages are split at once.
    const int gthreads = conv_threads / p.conv_groups;
    const int cg = (threadIdx.x - conv_lo * 32) / gthreads;
    const int ct = (threadIdx.x - conv_lo * 32) % gthreads;
    int s = 0;
    uint32_t ph = 0, lph[2] = {0, 0};
    // TMEM lo: thread = tile row (its warp's TMEM lane quarter), the group's
    // warps of one quarter share the row's 32 columns.
    const int wpq = gthreads / 128;  // warps per lane quarter in a group (1 or 2)
    const int lo_cols = kBK / wpq;
    const int lo_c0 = ((ct >> 5) >> 2) * lo_cols;
    const int lo_row = (warp & 3) * 32 + lane;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (s % p.conv_groups == cg) {
          if (!bar_wait(&full[s], ph, abort_flag, kTimeoutNs, 256)) goto conv_done;
          if (kb == 0 && ct == 0) TC_TRACE(7, (t - blockIdx.x) / gridDim.x);
          uint8_t* st = smem + (size_t)s * p.stage_bytes;
          if (p.lo_tmem) {
            // The slot's previous readers (the MMAs of stage s - 2) are done.
            if (!bar_wait(&lo_empty[s & 1], lph[s & 1] ^ 1, abort_flag, kTimeoutNs, 64))
              goto conv_done;
            lph[s & 1] ^= 1;
            tc_fence_after();
            const uint8_t* rowp = st + lo_row * 128;
            const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) +
                                   (uint32_t)(p.lo_col + (s & 1) * kBK + lo_c0);
            for (int h = 0; h < lo_cols; h += 16) {
              uint32_t r[16];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int c4 = (lo_c0 + h) / 4 + q;  // 16-byte chunk of the 128-byte row
                const float4 v =
                    *reinterpret_cast<const float4*>(rowp + ((c4 ^ (lo_row & 7)) << 4));
                r[4 * q + 0] = __float_as_uint(lo_of_raw(v.x));
                r[4 * q + 1] = __float_as_uint(lo_of_raw(v.y));
                r[4 * q + 2] = __float_as_uint(lo_of_raw(v.z));
                r[4 * q + 3] = __float_as_uint(lo_of_raw(v.w));
              }
              tmem_st16(taddr + (uint32_t)h, r);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            bar_arrive(&conv[s]);
            if (kb == 0 && ct == 0) TC_TRACE(1, (t - blockIdx.x) / gridDim.x);
            goto next_stage;
          }
          split_lo_buffer((const float4*)st, (float4*)(st + kATileBytes), kATileBytes / 16, ct,
                          gthreads);
          if (!p.presplit)
            split_buffer((float4*)(st + b_off), (float4*)(st + b_off + p.b_bytes),
                         p.b_bytes / 16, ct, gthreads);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          bar_arrive(&conv[s]);
          if (kb == 0 && ct == 0) TC_TRACE(1, (t - blockIdx.x) / gridDim.x);
        }
      next_stage:
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  conv_done:;
  } else if (warp >= p.epi_warps) {
    // epilogue warp not in use for this launch
  } else if (p.tma_store) {
    // ---------------- epilogue via TMA (warps 0 .. kEpiWarps-1) ----------------
    // Warp w reads TMEM lane quarter w % 4 (lane = tile row) and takes every
    // (kEpiWarps / 4)-th 32-column chunk starting at chunk w / 4.  Per chunk:
    // lane 0 frees the warp's staging tile (previous store has read it) and
    // TMA-loads the residual box into it; lanes add bias / residual, apply the
    // activation, write their row back 128-byte swizzled; lane 0 TMA-stores
    // the 32 x 32 box.  No block-wide barrier; stores run asynchronously.
    // With two groups (one 32-column chunk per quarter: N <= 32), warps 0-3
    // take the CTA's even tiles and warps 4-7 the odd ones, each group
    // cycling over its own two of the four accumulators.
    const int wpg = p.epi_warps / p.groups;       // warps per group
    const int grp = warp / wpg;
    int acc = grp;
    int issuer = 31;  // lane that issued the last store from this warp's staging
    uint32_t aph = 0, rph = 0;
    uint8_t* stg = epi + warp * kEpiSlot;
    float4* srow = reinterpret_cast<float4*>(stg + lane * 128);
    const int sw = lane & 7;
    bool ok = true;
    for (int t = blockIdx.x + grp * gridDim.x; t < total; t += p.groups * gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      ok = bar_wait(&tfull[acc], aph, abort_flag, kTimeoutNs, 128) && ok;
      if (threadIdx.x == 0) TC_TRACE(5, (t - blockIdx.x) / gridDim.x);
      if (__any_sync(0xffffffffu, !ok)) break;
      tc_fence_after();
      const int quarter = warp & 3;
      const uint32_t tbase =
          tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.BN * (1 + p.cat));
      const int row0 = mt * kBM + quarter * 32;
      for (int c0 = ((warp % wpg) >> 2) * 32; c0 < p.BN; c0 += 32 * (wpg / 4)) {
        const int n0 = nt * p.BN + c0;
        if (n0 >= p.N) break;  // uniform across the warp
        // The lane that issued the previous store waits until it has read the
        // staging tile; the next store is issued by the following lane, so no
        // lane's proxy fence has to wait behind its own in-flight store.
        const bool trc = warp == 0 && lane == 0 && c0 == 0;
        if (trc) TC_TRACE(8, (t - blockIdx.x) / gridDim.x);
        // The accumulator chunk comes out of TMEM first (it does not touch
        // the staging tile), so its latency overlaps the wait for the
        // previous store's read of the staging tile.
        float v[32];
        tmem_ld32(tbase + (uint32_t)c0, v);
        if (p.cat) add_tmem32(tbase + (uint32_t)(p.BN + c0), v);
        if (trc) TC_TRACE(9, (t - blockIdx.x) / gridDim.x);
        if (lane == issuer) bulk_wait_read0();
        const int next = (issuer + 1) & 31;
        if (lane == next) {
          if (p.res) {
            bar_expect_tx(&rfull[warp], 32 * 32 * 4);
            tma_load_2d(stg, &tmR, &rfull[warp], n0, row0);
          }
        }
        __syncwarp();
        if (trc) TC_TRACE(10, (t - blockIdx.x) / gridDim.x);
        if (p.res) {
          ok = bar_wait(&rfull[warp], rph, abort_flag) && ok;
          rph ^= 1;
        }
        with_act_group<AG>(p.act, [&](auto tag) {
          constexpr int A = decltype(tag)::value;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int nq = n0 + 4 * q;
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.bias_n) b4 = reinterpret_cast<const float4*>(bias_s + n0)[q];
            else if (p.bias && nq < p.N) b4 = __ldg(reinterpret_cast<const float4*>(p.bias + nq));
            const float4 r4 = p.res ? srow[q ^ sw] : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 o;
            o.x = act_c<A>(v[4 * q + 0] * p.alpha + b4.x + r4.x);
            o.y = act_c<A>(v[4 * q + 1] * p.alpha + b4.y + r4.y);
            o.z = act_c<A>(v[4 * q + 2] * p.alpha + b4.z + r4.z);
            o.w = act_c<A>(v[4 * q + 3] * p.alpha + b4.w + r4.w);
            srow[q ^ sw] = o;
          }
        });
        if (trc) TC_TRACE(11, (t - blockIdx.x) / gridDim.x);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (trc) TC_TRACE(12, (t - blockIdx.x) / gridDim.x);
        if (lane == next) {
          tma_store_2d(&tmC, stg, n0, row0);
          bulk_commit();
        }
#ifdef SPX_TC_TRACE
        __syncwarp();
        if (trc) TC_TRACE(13, (t - blockIdx.x) / gridDim.x);
#endif
        issuer = next;
      }
      tc_fence_before();
      bar_arrive(&tempty[acc]);
      if (threadIdx.x == 0) TC_TRACE(6, (t - blockIdx.x) / gridDim.x);
      acc += p.groups;
      if (acc >= p.nacc) {
        acc -= p.nacc;
        aph ^= 1;
      }
    }
    bulk_wait_all();  // every lane that issued stores waits for them
  } else {
    // ---------------- epilogue (warps 0 .. kEpiWarps-1) ----------------
    // Warp w reads TMEM lane quarter w % 4 and takes every
    // (kEpiWarps / 4)-th 32-column chunk starting at chunk w / 4.
    int acc = 0;
    uint32_t aph = 0;
    float* tile = reinterpret_cast<float*>(epi + warp * kEpiSlot);  // 32 x kEpiStride tile
    const int sub_r = lane >> 3;                 // 0..3: row within a group of 4
    const int sub_c = (lane & 7) * 4;            // first of 4 columns
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      // Uniform per warp: every lane waits on the same barrier phase.
      const bool ok = bar_wait(&tfull[acc], aph, abort_flag, kTimeoutNs, 128);
      if (threadIdx.x == 0) TC_TRACE(5, (t - blockIdx.x) / gridDim.x);
      if (__any_sync(0xffffffffu, !ok)) break;
      tc_fence_after();
      const int quarter = warp & 3;
      const uint32_t tbase =
          tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.BN * (1 + p.cat));
      const int64_t row0 = (int64_t)mt * kBM + quarter * 32;
      for (int c0 = (warp >> 2) * 32; c0 < p.BN; c0 += 32 * (p.epi_warps / 4)) {
        float v[32];
        tmem_ld32(tbase + (uint32_t)c0, v);  // lane = row, 32 consecutive columns
        if (p.cat) add_tmem32(tbase + (uint32_t)(p.BN + c0), v);
        float4* trow = reinterpret_cast<float4*>(tile + lane * kEpiStride);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          trow[q] = make_float4(v[4 * q] * p.alpha, v[4 * q + 1] * p.alpha,
                                v[4 * q + 2] * p.alpha, v[4 * q + 3] * p.alpha);
        __syncwarp();
        const int n = nt * p.BN + c0 + sub_c;
        float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.bias) {
          float* bp = &b4.x;
          if (p.vec4 && n + 3 < p.N) b4 = __ldg(reinterpret_cast<const float4*>(p.bias + n));
          else
            for (int e = 0; e < 4; ++e) bp[e] = n + e < p.N ? p.bias[n + e] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = i * 4 + sub_r;
          const int64_t m = p.conv ? conv_row(p, mt, quarter * 32 + rr) : row0 + rr;
          if (m < 0 || m >= p.M || n >= p.N) continue;
          float4 o = *reinterpret_cast<const float4*>(tile + rr * kEpiStride + sub_c);
          float* op = &o.x;
          const float* bp = &b4.x;
          float* crow = p.c + m * p.ldc;
          with_act_group<AG>(p.act, [&](auto tag) {
            constexpr int A = decltype(tag)::value;
            if (p.vec4 && n + 3 < p.N) {
              float4 r4 = p.res ? *reinterpret_cast<const float4*>(p.res + m * p.ldc + n)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
              const float* rp = &r4.x;
#pragma unroll
              for (int e = 0; e < 4; ++e) op[e] = act_c<A>(op[e] + bp[e] + rp[e]);
              *reinterpret_cast<float4*>(crow + n) = o;
            } else {
              for (int e = 0; e < 4; ++e)
                if (n + e < p.N) {
                  float x = op[e] + bp[e];
                  if (p.res) x += p.res[m * p.ldc + n + e];
                  crow[n + e] = act_c<A>(x);
                }
            }
          });
        }
        __syncwarp();
      }
      tc_fence_before();
      bar_arrive(&tempty[acc]);
      if (threadIdx.x == 0) TC_TRACE(6, (t - blockIdx.x) / gridDim.x);
      acc ^= 1;
      if (!acc) aph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
}

// ===========================================================================
// Few-row GEMM on tensor cores, operands swapped: C[m][n] for M <= 256 rows
// (decode / small-batch linear layers) computed as D[n][m] = W[n][:] . X[m][:]
// so the 128-row UMMA M dimension runs over the weight rows and the batch is
// the UMMA N dimension (16..256).  Weights stream through the CTA exactly
// once; the k range is split over a thread-block cluster along grid.y and the
// partial tiles are summed through distributed shared memory (fixed order,
// deterministic), each CTA of the cluster reducing and storing its share of
// the batch rows.
//   warps 0-3  converters (split W and X tiles to hi / lo), then epilogue:
//              TMEM lanes = weight rows -> partial tile red[m][128] in smem
//   warp 4     TMA producer (W box 128 x 32, X box Mp x 32)
//   warp 5     TMEM owner, MMA issuer
constexpr int kSkThreads = 192;
constexpr int kSkProducer = 4;
constexpr int kSkMma = 5;

struct SkArgs {
  int M, N, K, Mp, k_blocks, kb_per_split, splits, stages;
  int presplit;  // W arrives as hi and lo tiles (pre-split weights): converters split X only
  uint32_t idesc, tmem_cols, stage_bytes, x_bytes;
  const float* bias;
  const float* res;
  float* c;
  int64_t ldc;
  float alpha;
  int act;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `local`'s twin in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* local, uint32_t rank) {
  uint32_t a;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(su32(local)), "r"(rank));
  return a;
}
// Plain (non-volatile) loads so a thread's loads from the peers overlap;
// ordering against the peers' writes comes from the cluster barrier.
__device__ __forceinline__ float ld_cluster(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__global__ void __launch_bounds__(kSkThreads)
    gemm_tc_skinny_kernel(const __grid_constant__ CUtensorMap tmW,
                          const __grid_constant__ CUtensorMap tmWlo,
                          const __grid_constant__ CUtensorMap tmX, const SkArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = p.stages;
  uint64_t* full = (uint64_t*)(smem + (size_t)S * p.stage_bytes);
  uint64_t* conv = full + kMaxStages;
  uint64_t* empty = conv + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = (uint32_t*)(drain + 1);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem);  // [Mp][128] partial, after the k-loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x;
  const int split = (int)cluster_rank();
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
  const int nkb = kb1 > kb0 ? kb1 - kb0 : 0;
  const uint32_t w_bytes = kATileBytes;  // 128 rows x 32 fp32
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&conv[s], 128);
      bar_init(&empty[s], 1);
    }
    bar_init(tfull, 1);
    bar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kSkMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(tmem_slot)),
                 "r"(p.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool have_acc = false;

  if (warp == kSkProducer) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, armed = 0, armed_par = 0;
      for (int i = 0; i < nkb; ++i) {
        if (!bar_wait(&empty[s], ph ^ 1, abort_flag, kTimeoutNs, 64)) break;
        uint8_t* st = smem + (size_t)s * p.stage_bytes;
        bar_expect_tx(&full[s], (p.presplit ? 2 * w_bytes : w_bytes) + p.x_bytes);
        tma_load_2d(st, &tmW, &full[s], (kb0 + i) * kBK, nt * kBM);
        if (p.presplit) tma_load_2d(st + w_bytes, &tmWlo, &full[s], (kb0 + i) * kBK, nt * kBM);
        tma_load_2d(st + 2 * w_bytes, &tmX, &full[s], (kb0 + i) * kBK, 0);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | (ph << s);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      if (*abort_flag) {
        for (int i = 0; i < S; ++i)
          if (armed & (1u << i)) {
            volatile int never = 0;
            bar_wait(&full[i], (armed_par >> i) & 1, &never, kDrainNs);
          }
      }
    }
  } else if (warp == kSkMma) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool issued = false;
      for (int i = 0; i < nkb; ++i) {
        if (!bar_wait(&conv[s], ph, abort_flag, kTimeoutNs, 64)) break;
        tc_fence_after();
        const uint32_t w_hi = su32(smem + (size_t)s * p.stage_bytes);
        const uint32_t w_lo = w_hi + w_bytes;
        const uint32_t x_hi = w_hi + 2 * w_bytes;
        const uint32_t x_lo = x_hi + p.x_bytes;
#pragma unroll
        for (int k = 0; k < kBK / 8; ++k) {
          const uint32_t off = k * 32;
          const uint64_t dwh = sdesc(w_hi + off), dwl = sdesc(w_lo + off);
          const uint64_t dxh = sdesc(x_hi + off), dxl = sdesc(x_lo + off);
          umma_tf32(tmem, dwl, dxh, p.idesc, (i | k) ? 1u : 0u);
          umma_tf32(tmem, dwh, dxl, p.idesc, 1u);
          umma_tf32(tmem, dwh, dxh, p.idesc, 1u);
        }
        issued = true;
        umma_commit(&empty[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      if (issued) umma_commit(tfull);
      if (*abort_flag && issued) {
        umma_commit(drain);
        volatile int never = 0;
        bar_wait(drain, 0, &never, kDrainNs);
      }
    }
  } else {
    // converters, then the TMEM -> smem partial
    const int ct = threadIdx.x;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      ok = bar_wait(&full[s], ph, abort_flag, kTimeoutNs, 256);
      if (!ok) break;
      uint8_t* st = smem + (size_t)s * p.stage_bytes;
      if (!p.presplit)
        split_buffer((float4*)st, (float4*)(st + w_bytes), w_bytes / 16, ct, 128);
      split_buffer((float4*)(st + 2 * w_bytes), (float4*)(st + 2 * w_bytes + p.x_bytes),
                   p.x_bytes / 16, ct, 128);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bar_arrive(&conv[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
    }
    if (nkb > 0) ok = bar_wait(tfull, 0, abort_flag, kTimeoutNs, 128) && ok;
    have_acc = nkb > 0 && ok;
    // Every lane of the warp takes the same branch only when all agree.
    have_acc = __all_sync(0xffffffffu, have_acc);
    tc_fence_after();
    const int row = warp * 32 + lane;  // weight row within the tile
    for (int c0 = 0; c0 < p.Mp; c0 += 32) {
      float v[32];
      if (have_acc) {
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < p.Mp) red[(c0 + j) * kBM + row] = v[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // every partial of the cluster is in shared memory
  if (threadIdx.x < 128) {
    const int row = threadIdx.x;
    const int n = nt * kBM + row;
    if (n < p.N) {
      const float b = p.bias ? p.bias[n] : 0.0f;
      with_act(p.act, [&](auto tag) {
        constexpr int A = decltype(tag)::value;
        uint32_t base[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          base[q] = q < p.splits ? peer_addr(red + row, (uint32_t)q) : 0u;
        // Unrolled: several rows' peer loads are in flight at once (each
        // row still sums its partials in the fixed order below).
#pragma unroll 4
        for (int m = split; m < p.M; m += p.splits) {
          float part[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            part[q] = q < p.splits ? ld_cluster(base[q] + (uint32_t)(m * kBM * 4)) : 0.0f;
          float acc = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) acc += part[q];  // fixed order: deterministic
          float v = acc * p.alpha + b;
          if (p.res) v += p.res[(int64_t)m * p.ldc + n];
          p.c[(int64_t)m * p.ldc + n] = act_c<A>(v);
        }
      });
    }
  }
  cluster_sync_all();  // peers finished reading this CTA's partial
  if (warp == kSkMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(p.tmem_cols));
  }
}

// Pre-splits weights once at load: hi = rna_tf32(w), lo = rna_tf32(w - hi).
__global__ void weights_split_kernel(const float* __restrict__ w, float* __restrict__ hi,
                                     float* __restrict__ lo, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float x = w[i];
    const float h = tf32_rna(x);
    hi[i] = h;
    lo[i] = split_lo(x, h);
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 2-D fp32 tensor map over rows x cols (cols contiguous, row pitch ld), box
// box_rows x 32 columns, 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
             int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SPX_OK;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = kNumSms;
  }
  return n;
}


// ===========================================================================
// Fused inverted-residual front half on tensor cores: 1x1 expand conv
// (3xTF32 UMMAs, accumulators in TMEM) + bias + activation + 3x3 depthwise +
// bias + activation, the expanded tensor never leaving the chip.
//
// Persistent CTA, one per SM, walking spatial tiles (TH x TW outputs of one
// image).  Per spatial tile the TMA producer loads the block input's halo
// box (IH x IW pixels x 32 channels, zero fill past cin and past the map)
// once; the converters split it into tf32 hi / lo tiles; then for every
// 32-channel chunk of the expanded width the MMA warp computes the expanded
// halo [pixels x 32] into one of two TMEM accumulators (3 M tiles of 128
// pixel rows), and the eight epilogue warps move it through bias,
// activation and the out-of-map zeroing (the depthwise padding applies to
// the expanded tensor) into a shared-memory tile, then run the depthwise
// rows on it and store the output.  The expand weights (all chunks, hi and
// lo) stay resident in shared memory.
//   warp 0      TMA producer        warp 1   TMEM owner, MMA issuer
//   warps 2-5   converters          warps 6-13  epilogue + depthwise
constexpr int kXdwThreads = 14 * 32;
constexpr int kXdwEpi0 = 6;  // first epilogue warp

struct XdwArgs {
  int n, ih, iw, cin, ce, oh, ow, pt, pl;
  int tiles_h, tiles_w, nch, ksteps;
  uint32_t xbytes, row_bytes, idesc;
  const float* be;
  const float* wd;
  const float* bd;
  float* y;
};

__device__ __forceinline__ void epi_bar() {  // the 256 epilogue threads
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

template <int S, int TH, int TW, int R, int ACT>
__global__ void __launch_bounds__(kXdwThreads, 1)
    xdw_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmWh,
                  const __grid_constant__ CUtensorMap tmWl, const XdwArgs p) {
  constexpr int IH = (TH - 1) * S + 3, IW = (TW - 1) * S + 3;
  constexpr int NPIX = IH * IW;
  constexpr int NROW = (NPIX + 7) / 8 * 8;
  constexpr int MT = (NPIX + kBM - 1) / kBM;
  constexpr uint32_t kXB = NROW * 128;
  constexpr int CG = 8;  // 4-channel groups of a 32-channel chunk
  static_assert((TH / R) * TW * CG == 256, "one epilogue thread per (rows, column, group)");
  static_assert(MT * 32 * 2 <= 256, "two accumulators of MT x 32 columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* xraw = smem;
  uint8_t* xhi = xraw + kXB;
  uint8_t* xlo = xhi + kXB;
  uint8_t* wres = xlo + kXB;                              // [nch][hi 4 KB | lo 4 KB]
  float* es = (float*)(wres + (size_t)p.nch * 8192);      // [NPIX][32], 16-byte chunks swizzled
  uint64_t* bars = (uint64_t*)(es + NPIX * 32);
  uint64_t* bfull = bars + 0;
  uint64_t* xraw_full = bars + 1;
  uint64_t* xraw_empty = bars + 2;
  uint64_t* xsplit_full = bars + 3;
  uint64_t* xsplit_empty = bars + 4;
  uint64_t* tfull = bars + 5;   // [2]
  uint64_t* tempty = bars + 7;  // [2]
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = (uint32_t*)(bars + 10);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.n * p.tiles_h * p.tiles_w;
  if (threadIdx.x == 0) {
    bar_init(bfull, 1);
    bar_init(xraw_full, 1);
    bar_init(xraw_empty, 128);
    bar_init(xsplit_full, 128);
    bar_init(xsplit_empty, 1);
    for (int a = 0; a < 2; ++a) {
      bar_init(&tfull[a], 1);
      bar_init(&tempty[a], 256);
    }
    bar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto coords = [&](int st, int& img, int& ty, int& tx) {
    tx = st % p.tiles_w;
    const int r = st / p.tiles_w;
    ty = r % p.tiles_h;
    img = r / p.tiles_h;
  };

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      bool armed = false;
      uint32_t armed_par = 0;
      bar_expect_tx(bfull, (uint32_t)p.nch * 8192);
      for (int c = 0; c < p.nch; ++c) {
        tma_load_2d(wres + (size_t)c * 8192, &tmWh, bfull, 0, c * 32);
        tma_load_2d(wres + (size_t)c * 8192 + 4096, &tmWl, bfull, 0, c * 32);
      }
      uint32_t ph = 0;
      for (int st = blockIdx.x; st < total; st += gridDim.x) {
        if (!bar_wait(xraw_empty, ph ^ 1, abort_flag, kTimeoutNs, 64)) break;
        int img, ty, tx;
        coords(st, img, ty, tx);
        bar_expect_tx(xraw_full, p.xbytes);
        tma_load_4d(xraw, &tmX, xraw_full, 0, tx * TW * S - p.pl, ty * TH * S - p.pt, img);
        armed = true;
        armed_par = ph;
        ph ^= 1;
      }
      if (*abort_flag) {
        volatile int never = 0;
        bar_wait(bfull, 0, &never, kDrainNs);
        if (armed) bar_wait(xraw_full, armed_par, &never, kDrainNs);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool issued = false;
      uint32_t xph = 0;
      int it = 0;  // chunk counter over the whole launch
      if (!bar_wait(bfull, 0, abort_flag, kTimeoutNs, 64)) goto mma_done;
      for (int st = blockIdx.x; st < total; st += gridDim.x) {
        if (!bar_wait(xsplit_full, xph, abort_flag, kTimeoutNs, 64)) goto mma_done;
        xph ^= 1;
        tc_fence_after();
        for (int c = 0; c < p.nch; ++c, ++it) {
          const int a = it & 1;
          const uint32_t aph = (uint32_t)(it >> 1) & 1u;
          if (!bar_wait(&tempty[a], aph ^ 1, abort_flag, kTimeoutNs, 64)) goto mma_done;
          tc_fence_after();
          const uint32_t wh = su32(wres + (size_t)c * 8192), wl = wh + 4096;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint32_t d = tmem + (uint32_t)(a * MT * 32 + m * 32);
            const uint32_t xh = su32(xhi + m * kBM * 128), xl = su32(xlo + m * kBM * 128);
            for (int k = 0; k < p.ksteps; ++k) {
              const uint32_t off = k * 32;
              umma_tf32(d, sdesc(xl + off), sdesc(wh + off), p.idesc, k ? 1u : 0u);
              umma_tf32(d, sdesc(xh + off), sdesc(wl + off), p.idesc, 1u);
              umma_tf32(d, sdesc(xh + off), sdesc(wh + off), p.idesc, 1u);
            }
          }
          issued = true;
          umma_commit(&tfull[a]);
        }
        umma_commit(xsplit_empty);  // the split x tile is free once these MMAs finish
      }
    mma_done:
      if (*abort_flag && issued) {
        umma_commit(drain);
        volatile int never = 0;
        bar_wait(drain, 0, &never, kDrainNs);
      }
    }
  } else if (warp < kXdwEpi0) {
    // ---------------- converters: raw halo -> hi / lo ----------------
    const int ct = threadIdx.x - 64;
    uint32_t rph = 0, sph = 0;
    for (int st = blockIdx.x; st < total; st += gridDim.x) {
      if (!bar_wait(xraw_full, rph, abort_flag, kTimeoutNs, 256)) break;
      rph ^= 1;
      if (!bar_wait(xsplit_empty, sph ^ 1, abort_flag, kTimeoutNs, 256)) break;
      sph ^= 1;
      const float4* src = reinterpret_cast<const float4*>(xraw);
      float4* hi = reinterpret_cast<float4*>(xhi);
      float4* lo = reinterpret_cast<float4*>(xlo);
      const int chunks = 2 * p.ksteps;  // 16-byte chunks of K that the MMAs read
#pragma unroll 4
      for (int i = ct; i < NPIX * 8; i += 128) {
        if (((i & 7) ^ ((i >> 3) & 7)) >= chunks) continue;
        const float4 v = src[i];
        const float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        lo[i] = make_float4(split_lo(v.x, h.x), split_lo(v.y, h.y), split_lo(v.z, h.z),
                            split_lo(v.w, h.w));
        hi[i] = h;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bar_arrive(xraw_empty);
      bar_arrive(xsplit_full);
    }
  } else {
    // ---------------- epilogue + depthwise (256 threads) ----------------
    const int et = threadIdx.x - kXdwEpi0 * 32;
    const int quarter = warp & 3;
    const int group = (warp - kXdwEpi0) >> 2;  // 0 or 1: which M tiles this warp drains
    const int cg = et % CG;
    const int ox_l = (et / CG) % TW;
    const int rb = et / (CG * TW);
    int it = 0;
    for (int st = blockIdx.x; st < total; st += gridDim.x) {
      int img, ty, tx;
      coords(st, img, ty, tx);
      const int y0 = ty * TH * S - p.pt, x0 = tx * TW * S - p.pl;
      for (int c = 0; c < p.nch; ++c, ++it) {
        const int a = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        const bool ok = bar_wait(&tfull[a], aph, abort_flag, kTimeoutNs, 128);
        (void)ok;
        epi_bar();  // previous chunk's depthwise reads of es are done; abort is uniform
        if (*abort_flag) break;
        tc_fence_after();
        // TMEM -> es: this warp drains M tiles group, group + 2, ...
        const int c0 = c * 32;
        for (int m = group; m < MT; m += 2) {
          float v[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * MT * 32 + m * 32), v);
          const int r = m * kBM + quarter * 32 + lane;  // halo pixel
          if (r < NPIX) {
            const int py = y0 + r / IW, px = x0 + r % IW;
            const bool in = py >= 0 && py < p.ih && px >= 0 && px < p.iw;
            float4* row = reinterpret_cast<float4*>(es + r * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const int ch = c0 + 4 * q;
              float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
              if (p.be && ch < p.ce) b4 = __ldg(reinterpret_cast<const float4*>(p.be + ch));
              float4 e;
              e.x = in ? act_c<ACT>(v[4 * q + 0] + b4.x) : 0.0f;
              e.y = in ? act_c<ACT>(v[4 * q + 1] + b4.y) : 0.0f;
              e.z = in ? act_c<ACT>(v[4 * q + 2] + b4.z) : 0.0f;
              e.w = in ? act_c<ACT>(v[4 * q + 3] + b4.w) : 0.0f;
              row[q ^ (r & 7)] = e;  // swizzled: conflict-free across a warp's rows
            }
          }
        }
        tc_fence_before();
        bar_arrive(&tempty[a]);
        epi_bar();  // es complete
        // Depthwise rows (dw_tma_kernel's walk) on the expanded halo.
        const int ch = c0 + cg * 4;
        const bool live = ch < p.ce;
        float4 wr[9];
#pragma unroll
        for (int k = 0; k < 9; ++k)
          wr[k] = live ? __ldg(reinterpret_cast<const float4*>(p.wd + (size_t)k * p.ce + ch))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 bv = (p.bd && live) ? __ldg(reinterpret_cast<const float4*>(p.bd + ch))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = bv;
#pragma unroll
        for (int j = 0; j < (R - 1) * S + 3; ++j) {
          const int iy = rb * R * S + j;
          float4 rowv[3];
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const int pix = iy * IW + ox_l * S + kx;
            rowv[kx] = reinterpret_cast<const float4*>(es + pix * 32)[cg ^ (pix & 7)];
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = j - r * S;
            if (ky < 0 || ky >= 3) continue;
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
              const float4 w4 = wr[ky * 3 + kx];
              acc[r].x = fmaf(rowv[kx].x, w4.x, acc[r].x);
              acc[r].y = fmaf(rowv[kx].y, w4.y, acc[r].y);
              acc[r].z = fmaf(rowv[kx].z, w4.z, acc[r].z);
              acc[r].w = fmaf(rowv[kx].w, w4.w, acc[r].w);
            }
          }
        }
        const int ox = tx * TW + ox_l;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int oy = ty * TH + rb * R + r;
          if (oy < p.oh && ox < p.ow && live) {
            float4 v = acc[r];
            v.x = act_c<ACT>(v.x);
            v.y = act_c<ACT>(v.y);
            v.z = act_c<ACT>(v.z);
            v.w = act_c<ACT>(v.w);
            *reinterpret_cast<float4*>(p.y + (((size_t)img * p.oh + oy) * p.ow + ox) * p.ce + ch) =
                v;
          }
        }
      }
      if (*abort_flag) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}

template <int S, int TH, int TW, int R, int ACT>
int launch_xdw(cudaStream_t s, const float* x, const float* we_hi, const float* we_lo,
               const float* be, const float* wd, const float* bd, float* y,
               const spx_expand_dw_params* q) {
  constexpr int IH = (TH - 1) * S + 3, IW = (TW - 1) * S + 3;
  constexpr int NPIX = IH * IW;
  constexpr int NROW = (NPIX + 7) / 8 * 8;
  XdwArgs p = {};
  p.n = q->n;
  p.ih = q->ih;
  p.iw = q->iw;
  p.cin = q->cin;
  p.ce = q->ce;
  p.oh = q->oh;
  p.ow = q->ow;
  p.pt = q->pad_top;
  p.pl = q->pad_left;
  p.tiles_h = (q->oh + TH - 1) / TH;
  p.tiles_w = (q->ow + TW - 1) / TW;
  p.nch = (q->ce + 31) / 32;
  p.ksteps = (q->cin + 7) / 8;
  p.xbytes = NPIX * 128;
  p.idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(32 >> 3) << 17) |
            ((uint32_t)(kBM >> 4) << 24);
  p.be = be;
  p.wd = wd;
  p.bd = bd;
  p.y = y;
  const size_t smem = 1024 + 3 * (size_t)NROW * 128 + (size_t)p.nch * 8192 +
                      (size_t)NPIX * 32 * 4 + 128;
  if (smem > 227 * 1024) return -1;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap mx, mwh, mwl;
  cuuint64_t dims[4] = {(cuuint64_t)q->cin, (cuuint64_t)q->iw, (cuuint64_t)q->ih,
                        (cuuint64_t)q->n};
  cuuint64_t strides[3] = {(cuuint64_t)q->cin * 4, (cuuint64_t)q->iw * q->cin * 4,
                           (cuuint64_t)q->ih * q->iw * q->cin * 4};
  cuuint32_t box[4] = {(cuuint32_t)kBK, (cuuint32_t)IW, (cuuint32_t)IH, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "expand_dw x map encode failed (%d)", (int)r);
  int rc;
  if ((rc = make_map(&mwh, we_hi, q->ce, q->cin, q->cin, 32))) return rc;
  if ((rc = make_map(&mwl, we_lo, q->ce, q->cin, q->cin, 32))) return rc;
  auto kern = xdw_tc_kernel<S, TH, TW, R, ACT>;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (attr != cudaSuccess) return check_cuda(attr, "expand_dw_tc: smem attribute");
  const int total = p.n * p.tiles_h * p.tiles_w;
  const int grid = total < sm_count() ? total : sm_count();
  kern<<<grid, kXdwThreads, smem, s>>>(mx, mwh, mwl, p);
  return SPX_OK;
}
}  // namespace

bool gemm_tc_eligible(const float* a, int64_t lda, const float* b, int64_t ldb, int M, int N,
                      int K, const float* c, int64_t ldc) {
  auto al16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
  return M > 0 && N > 0 && K > 0 && K % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 && lda >= K &&
         ldb >= K && al16(a) && al16(b) && ldc >= N && c != nullptr;
}

namespace {
// 4-D fp32 tensor map over an NHWC activation (dims C, W, H, N) whose box is
// one conv M tile's worth of one k-block: 32 channels x tw x th x tn pixels,
// traversed with the conv stride in W and H, 128-byte swizzle, zero fill.
int make_conv_map(CUtensorMap* map, const float* x, const spx_conv_params* q, int tw, int th,
                  int tn) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SPX_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)q->ic, (cuuint64_t)q->iw, (cuuint64_t)q->ih,
                        (cuuint64_t)q->n};
  cuuint64_t strides[3] = {(cuuint64_t)q->ic * 4, (cuuint64_t)q->iw * q->ic * 4,
                           (cuuint64_t)q->ih * q->iw * q->ic * 4};
  cuuint32_t box[4] = {(cuuint32_t)kBK, (cuuint32_t)(tw * q->stride_w),
                       (cuuint32_t)(th * q->stride_h), (cuuint32_t)tn};
  cuuint32_t estr[4] = {1, (cuuint32_t)q->stride_w, (cuuint32_t)q->stride_h, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)x, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SPX_ERR_CUDA, "conv tensor map encode failed (%d)", (int)r);
  return SPX_OK;
}
}  // namespace

bool conv_tc_eligible(const float* x, const float* w, const float* y,
                      const spx_conv_params* q) {
  auto al16 = [](const void* v) { return ((uintptr_t)v & 15) == 0; };
  const int dh = q->dilation_h > 0 ? q->dilation_h : 1, dw = q->dilation_w > 0 ? q->dilation_w : 1;
  return q->weight_layout == SPX_WEIGHT_OHWI && dh == 1 && dw == 1 && q->ic % kBK == 0 &&
         q->stride_h == q->stride_w && q->stride_h <= 8 && q->ow * q->stride_w <= 256 &&
         q->oc > 0 && al16(x) && al16(w) && y != nullptr &&
         (int64_t)q->n * q->oh * q->ow < INT32_MAX;
}

int launch_conv_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* w,
                   const float* w_lo, const float* bias, const float* res, float* y,
                   const spx_conv_params* q) {
  // Output patch per 128-row tile: whole rows (tw = ow when it fits), as
  // many rows as fit, and several images when a whole map fits.
  const int tw = q->ow <= kBM ? q->ow : kBM;
  int th = kBM / tw;
  if (th > q->oh) th = q->oh;
  // Fewer, fuller row bands: the smallest th with the same number of bands.
  const int bands = (q->oh + th - 1) / th;
  th = (q->oh + bands - 1) / bands;
  int tn = th == q->oh ? kBM / (th * tw) : 1;
  if (tn > q->n) tn = q->n;
  if (tn < 1) tn = 1;
  if (tw * q->stride_w > 256 || th * q->stride_h > 256)
    return fail(SPX_ERR_UNSUPPORTED, "conv_tc: patch exceeds a TMA box");
  CUtensorMap mx;
  int rc = make_conv_map(&mx, x, q, tw, th, tn);
  if (rc) return rc;
  ConvGeom g = {q->oh, q->ow, q->ic / kBK, q->kw, q->stride_h, q->pad_top, q->pad_left,
                th, tw, tn, (q->oh + th - 1) / th, (q->ow + tw - 1) / tw};
  const int K = q->kh * q->kw * q->ic;
  return launch_gemm_tc(s, cnt, x, K, w, w_lo, K, q->n * q->oh * q->ow, q->oc, K, bias, res, y,
                        q->oc, 1.0f, q->activation, &g, &mx, (q->n + tn - 1) / tn);
}

// Per-shape configuration of gemm_tc_kernel (no device access): tile width,
// ring depth, warp roles, accumulators.  `conv` marks the implicit-GEMM conv
// mode, `m_tiles` is the number of 128-row tiles, `vec4` whether C / residual
// / bias allow 16-byte access.
int plan_gemm_tc(TcArgs& p, int M, int N, int K, bool presplit, bool conv, int m_tiles,
                 bool vec4) {
  p = TcArgs{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.presplit = presplit;
  // N tile: a multiple of 32 (the epilogue's chunk), at most 256 (UMMA N),
  // halved while there are fewer than two tiles per SM.
  const int nt0 = (N + 255) / 256;
  p.BN = ((N + nt0 - 1) / nt0 + 31) / 32 * 32;
  p.m_tiles = m_tiles;
  // More, narrower tiles only pay while the k-loop is short: every n-tile
  // re-splits the same A tiles and narrow UMMAs cost nearly as much to issue
  // as wide ones.
  const int kb_total = (K + kBK - 1) / kBK;
  // With very few tiles (tiny M) narrower tiles win regardless of K.
  while (p.BN > 32 && (int64_t)p.m_tiles * ((N + p.BN - 1) / p.BN) <
                          (kb_total <= 4 ? 2 * sm_count() : sm_count() / 2))
    p.BN = (p.BN / 2 + 31) / 32 * 32;
  // Few waves of tiles (small M, e.g. 7x7 maps): pick the N tile that
  // minimises waves x per-tile cost, so the last wave is not mostly idle.
  // A tile's cost is modelled as its width plus a fixed 64 columns' worth
  // for the A side (load and split, the same for every width).
  {
    const int sms = sm_count();
    const int64_t tiles = (int64_t)p.m_tiles * ((N + p.BN - 1) / p.BN);
    if (tiles < 6 * sms) {
      int best_bn = p.BN;
      int64_t best = ((tiles + sms - 1) / sms) * (p.BN + 64);
      for (int bn = p.BN - 32; bn >= 64; bn -= 32) {
        const int64_t t = (int64_t)p.m_tiles * ((N + bn - 1) / bn);
        const int64_t cost = ((t + sms - 1) / sms) * (bn + 64);
        if (cost < best) {
          best = cost;
          best_bn = bn;
        }
      }
      p.BN = best_bn;
    }
  }
  // At least two pipeline stages must fit next to the epilogue tiles; long
  // k-loops count with four epilogue warps (below), so a 256-wide tile keeps
  // its width (wide tiles read A once per 256 columns: measured 120 -> 169
  // fp32 TFLOP/s at 4096 x 3072 x 768, 141 -> 203 at 50176 x 1024 x 512).
  const int full_budget = 227 * 1024 - 1024 - kEpiWarps * (int)kEpiSlot - 512;
  const int fit_budget = kb_total >= 8 ? 227 * 1024 - 1024 - 4 * (int)kEpiSlot - 512 : full_budget;
  while (p.BN > 32 && fit_budget / (int)(2 * kATileBytes + 2 * (uint32_t)p.BN * kBK * 4) < 2)
    p.BN = (p.BN / 2 + 31) / 32 * 32;
  // Long k-loops keep the tensor pipe busy only with several stages in
  // flight; their epilogue is rare, so when that buys a third stage, or the
  // second one, they give up half the epilogue warps (and their staging
  // tiles).
  p.epi_warps = kEpiWarps;
  {
    const int bn_stage = (int)(2 * kATileBytes + 2 * (uint32_t)p.BN * kBK * 4);
    const int half_budget = 227 * 1024 - 1024 - 4 * (int)kEpiSlot - 512;
    if (kb_total >= 8 && full_budget / bn_stage < 3 &&
        (half_budget / bn_stage >= 3 || full_budget / bn_stage < 2))
      p.epi_warps = 4;
    // One or two k-blocks per tile (K <= 64, the expand layers): the
    // converters are mostly idle and the epilogue's per-chunk latency sets
    // the tile period, so four converter warps become a third epilogue warp
    // per lane quarter when that saves a round of chunks (measured: 64 ->
    // 384 at 14x14, b256, 36.8 -> 34.6 us; no gain from three k-blocks).
    const int chunks = (p.BN + 31) / 32;
    const int wide_budget = 227 * 1024 - 1024 - kMaxEpiWarps * (int)kEpiSlot - 512;
    if (g_tc_epi12 && kb_total <= 2 && (chunks + 2) / 3 < (chunks + 1) / 2 &&
        wide_budget / bn_stage >= 2)
      p.epi_warps = kMaxEpiWarps;
  }
  p.n_tiles = (N + p.BN - 1) / p.BN;
  p.k_blocks = (K + kBK - 1) / kBK;
  p.last_ksteps = conv ? kBK / 8 : (K - (p.k_blocks - 1) * kBK + 7) / 8;
  p.b_bytes = (uint32_t)p.BN * kBK * 4;
  p.b_resident = g_tc_epi12 && p.presplit && !conv && p.k_blocks == 1 && p.n_tiles == 1;
  p.vec4 = vec4;
  p.tma_store = p.vec4 && !conv;
  // One 32-column chunk per lane quarter: the two halves of the epilogue take
  // alternate tiles (four accumulators) so two tiles drain at once.
  p.groups = (g_tc_epi12 && p.tma_store && p.BN == 32 && p.epi_warps == kEpiWarps) ? 2 : 1;
  p.nacc = 2 * p.groups;
  // Several k-blocks with pre-split weights: the activations' lo terms go to
  // two 32-column TMEM slots after the accumulators (registers -> TMEM, the
  // lo*hi MMA reads A from TMEM), so a stage holds only the raw A tile and B.
  p.lo_tmem = g_tc_lo_tmem && p.presplit && p.k_blocks >= 2 && p.epi_warps <= kEpiWarps &&
              p.nacc * p.BN + 2 * kBK <= 512;
  p.cat = g_tc_cat && p.BN <= 128 && !p.lo_tmem;
  // One k-block per tile (the expand layers): the epilogue sets the pace, so
  // three or four accumulators (three separate products, no concatenated
  // N = 2 BN one) let the tensor core run ahead of a slow chunk.
  if (g_tc_acc4 && p.groups == 1 && p.tma_store && p.k_blocks == 1 && 3 * p.BN <= 512) {
    p.nacc = 4 * p.BN <= 512 ? 4 : 3;
    p.cat = 0;
  }
  p.lo_col = p.nacc * p.BN;
  const int budget = 227 * 1024 - 1024 - p.epi_warps * (int)kEpiSlot - 512 -
                     (p.b_resident ? 2 * (int)p.b_bytes : 0);
  p.stage_bytes = (p.lo_tmem ? 1 : 2) * kATileBytes + (p.b_resident ? 0 : 2 * p.b_bytes);
  p.stages = budget / (int)p.stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  if (p.stages < 2) return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc: tile does not fit");
  // The lo-in-TMEM rings are deep enough to give up a stage for an even
  // count (two converter groups, below).
  if (p.lo_tmem && g_tc_conv2 && p.stages % 2 && p.stages > 2) --p.stages;
  // Two converter groups own the even and the odd stages: each group then
  // meets every one of its stages once per pass of the ring, so its mbarrier
  // parities stay in step.  That needs an even stage count.
  p.conv_groups =
      (g_tc_conv2 && p.epi_warps <= kEpiWarps && p.k_blocks > 1 && p.stages % 2 == 0) ? 2 : 1;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.nacc * p.BN * (1 + p.cat) + (p.lo_tmem ? 2 * kBK : 0))) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = (1u << 4)                          // accumulator F32
            | (2u << 7) | (2u << 10)           // A, B: TF32
            | ((uint32_t)(p.BN >> 3) << 17)    // N
            | ((uint32_t)(kBM >> 4) << 24);    // M
  p.idesc2 = (p.idesc & ~(0x3Fu << 17)) | ((uint32_t)((2 * p.BN) >> 3) << 17);
  p.smem_bytes = 1024 + (uint32_t)p.stages * p.stage_bytes +
                 (p.b_resident ? 2 * p.b_bytes : 0u) + (uint32_t)p.epi_warps * kEpiSlot + 512;
  // The bias goes to shared memory only where the plan leaves room for it.
  const int bias_n = p.n_tiles * p.BN;
  if (p.tma_store && bias_n <= 4096 && p.smem_bytes + (uint32_t)bias_n * 4 <= 227u * 1024u) {
    p.bias_n = bias_n;
    p.smem_bytes += (uint32_t)bias_n * 4;
  }
  return SPX_OK;
}

int launch_gemm_tc(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda, const float* b,
                   const float* b_lo, int64_t ldb, int M, int N, int K, const float* bias,
                   const float* res, float* c, int64_t ldc, float alpha, int act,
                   const ConvGeom* conv, const void* conv_map, int conv_img_groups) {
  TcArgs p;
  auto al16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
  const bool vec4 = (ldc % 4 == 0) && al16(c) && (!res || al16(res)) && (!bias || al16(bias));
  const int m_tiles =
      conv ? conv_img_groups * conv->tiles_h * conv->tiles_w : (M + kBM - 1) / kBM;
  int rc0 = plan_gemm_tc(p, M, N, K, b_lo != nullptr, conv != nullptr, m_tiles, vec4);
  if (rc0) return rc0;
  p.bias = bias;
  p.res = res;
  p.c = c;
  p.ldc = ldc;
  p.alpha = alpha;
  p.act = act;
  p.a_tx = kATileBytes;
  CUtensorMap ma, mb, mblo;
  int rc;
  if (conv) {
    p.conv = 1;
    p.oh = conv->oh;
    p.ow = conv->ow;
    p.ic_blocks = conv->ic_blocks;
    p.kw = conv->kw;
    p.sh = conv->sh;
    p.pt = conv->pt;
    p.pl = conv->pl;
    p.th = conv->th;
    p.tw = conv->tw;
    p.tn = conv->tn;
    p.tiles_h = conv->tiles_h;
    p.tiles_w = conv->tiles_w;
    p.a_tx = (uint32_t)(conv->tn * conv->th * conv->tw) * kBK * 4;
    ma = *reinterpret_cast<const CUtensorMap*>(conv_map);
  } else if ((rc = make_map(&ma, a, M, K, lda, kBM))) {
    return rc;
  }
  if ((rc = make_map(&mb, b, N, K, ldb, p.BN))) return rc;
  mblo = mb;
  if (p.presplit && (rc = make_map(&mblo, b_lo, N, K, ldb, p.BN))) return rc;
  CUtensorMap mc = ma, mr = ma;
  if (p.tma_store) {
    if ((rc = make_map(&mc, c, M, N, ldc, 32))) return rc;
    if (res && (rc = make_map(&mr, res, M, N, ldc, 32))) return rc;
  }
  const size_t smem = p.smem_bytes;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(gemm_tc_kernel<0>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(gemm_tc_kernel<1>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "gemm_tc: smem attribute");
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  const cudaError_t le = launch_pdl(act_group(p.act) ? gemm_tc_kernel<1> : gemm_tc_kernel<0>,
                                    dim3(grid), dim3(kThreads), smem, s, ma, mb, mblo, mc, mr, p);
  if (le != cudaSuccess) return check_cuda(le, "gemm_tc launch");
  return after_launch(cnt, "gemm_tc");
}

bool gemm_tc_skinny_eligible(const float* a, int64_t lda, const float* w, int64_t ldw, int M,
                             int N, int K) {
  auto al16 = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
  return M >= 1 && M <= 256 && N > 0 && K > 0 && K % 4 == 0 && lda % 4 == 0 && ldw % 4 == 0 &&
         lda >= K && ldw >= K && al16(a) && al16(w);
}

int launch_gemm_tc_skinny(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda,
                          const float* w, const float* w_lo, int64_t ldw, int M, int N, int K,
                          const float* bias, const float* res, float* c, int64_t ldc,
                          float alpha, int act) {
  if (!gemm_tc_skinny_eligible(a, lda, w, ldw, M, N, K) || ldc < N || !c)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc_skinny: operands not eligible");
  SkArgs p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  p.Mp = (M + 15) / 16 * 16;
  p.presplit = w_lo != nullptr;
  if (w_lo && ((uintptr_t)w_lo & 15)) return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc_skinny: w_lo");
  p.k_blocks = (K + kBK - 1) / kBK;
  const int tiles = (N + kBM - 1) / kBM;
  // Two CTAs per SM; split k over a cluster until the grid fills them.
  int splits = (2 * sm_count()) / tiles;
  if (splits > 8) splits = 8;
  if (splits > p.k_blocks) splits = p.k_blocks;
  if (splits < 1) splits = 1;
  p.kb_per_split = (p.k_blocks + splits - 1) / splits;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.x_bytes = (uint32_t)p.Mp * kBK * 4;
  p.stage_bytes = 2 * kATileBytes + 2 * p.x_bytes;
  p.stages = p.Mp <= 64 ? 2 : (p.Mp <= 128 ? 3 : 2);
  uint32_t cols = 32;
  while (cols < (uint32_t)p.Mp) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(p.Mp >> 3) << 17) |
            ((uint32_t)(kBM >> 4) << 24);
  p.bias = bias;
  p.res = res;
  p.c = c;
  p.ldc = ldc;
  p.alpha = alpha;
  p.act = act;
  CUtensorMap mw, mwlo, mx;
  int rc;
  if ((rc = make_map(&mw, w, N, K, ldw, kBM))) return rc;
  mwlo = mw;
  if (w_lo && (rc = make_map(&mwlo, w_lo, N, K, ldw, kBM))) return rc;
  if ((rc = make_map(&mx, a, M, K, lda, p.Mp))) return rc;
  size_t smem = 1024 + (size_t)p.stages * p.stage_bytes + 256;
  const size_t red_bytes = (size_t)p.Mp * kBM * 4;
  if (red_bytes > (size_t)p.stages * p.stage_bytes)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc_skinny: partial tile does not fit");
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(gemm_tc_skinny_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "gemm_tc_skinny: smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, p.splits, 1);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = p.splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_skinny_kernel, mw, mwlo, mx, p);
  if (e != cudaSuccess) return check_cuda(e, "gemm_tc_skinny launch");
  return after_launch(cnt, "gemm_tc_skinny");
}

int launch_weights_split(cudaStream_t s, int64_t* cnt, const float* w, float* hi, float* lo,
                         int64_t n) {
  if (n <= 0) return n == 0 ? SPX_OK : fail(SPX_ERR_INVALID_ARGUMENT, "weights_split: n < 0");
  weights_split_kernel<<<grid_for(n, 256), 256, 0, s>>>(w, hi, lo, n);
  return after_launch(cnt, "weights_split");
}

#ifdef SPX_TC_TRACE
extern "C" int spx_tc_trace_fetch(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_tc_trace, sizeof(g_tc_trace)) == cudaSuccess ? 0 : 3;
}
#endif

// Host-side view of the tensor-core GEMM's per-shape plan (no device work):
// out[0..15] = BN, n_tiles, k_blocks, last_ksteps, stages, stage_bytes,
// epi_warps, conv_groups, epilogue groups, accumulators, TMEM columns,
// resident weights, dynamic smem bytes, m_tiles, converter threads, grid,
// lo terms in TMEM.
extern "C" int spx_gemm_tc_plan(int32_t M, int32_t N, int32_t K, int32_t presplit, int32_t conv,
                                int32_t vec4, int32_t* out, int32_t n_out) {
  if (!out || n_out < 17 || M <= 0 || N <= 0 || K <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_tc_plan: bad arguments");
  TcArgs p;
  const int m_tiles = (M + kBM - 1) / kBM;
  int rc = plan_gemm_tc(p, M, N, K, presplit != 0, conv != 0, m_tiles, vec4 != 0);
  if (rc) return rc;
  const int conv_lo = p.epi_warps > kEpiWarps ? p.epi_warps : kEpiWarps;
  const int tiles = p.m_tiles * p.n_tiles;
  const int32_t v[17] = {p.BN, p.n_tiles, p.k_blocks, p.last_ksteps, p.stages,
                         (int32_t)p.stage_bytes, p.epi_warps, p.conv_groups, p.groups, p.nacc,
                         (int32_t)p.tmem_cols, p.b_resident, (int32_t)p.smem_bytes, p.m_tiles,
                         (kEpiWarps + kConvWarps - conv_lo) * 32,
                         tiles < sm_count() ? tiles : sm_count(), p.lo_tmem};
  for (int i = 0; i < 17; ++i) out[i] = v[i];
  return SPX_OK;
}

int launch_expand_dw_tc(cudaStream_t s, int64_t* cnt, const float* x, const float* we_hi,
                        const float* we_lo, const float* be, const float* wd, const float* bd,
                        float* y, const spx_expand_dw_params* q) {
  auto al16 = [](const void* v) { return ((uintptr_t)v & 15) == 0; };
  if (!x || !we_hi || !we_lo || !wd || !y || !q) return -1;
  if ((q->cin != 16 && q->cin != 24 && q->cin != 32) || q->ce % 4 || q->ce > 256 ||
      (q->stride != 1 && q->stride != 2) || q->act_expand != q->act_dw ||
      (q->act_expand != SPX_ACT_RELU6 && q->act_expand != SPX_ACT_NONE))
    return -1;
  if (q->oh != (q->ih + q->stride - 1) / q->stride || q->ow != (q->iw + q->stride - 1) / q->stride)
    return -1;
  if (!al16(x) || !al16(we_hi) || !al16(we_lo) || !al16(wd) || !al16(y) || (be && !al16(be)) ||
      (bd && !al16(bd)))
    return -1;
  if ((int64_t)q->n * q->oh * q->ow * q->ce >= INT32_MAX) return -1;
  const bool r6 = q->act_expand == SPX_ACT_RELU6;
  int rc;
  if (q->stride == 1)
    rc = r6 ? launch_xdw<1, 14, 16, 7, SPX_ACT_RELU6>(s, x, we_hi, we_lo, be, wd, bd, y, q)
            : launch_xdw<1, 14, 16, 7, SPX_ACT_NONE>(s, x, we_hi, we_lo, be, wd, bd, y, q);
  else
    rc = r6 ? launch_xdw<2, 4, 16, 2, SPX_ACT_RELU6>(s, x, we_hi, we_lo, be, wd, bd, y, q)
            : launch_xdw<2, 4, 16, 2, SPX_ACT_NONE>(s, x, we_hi, we_lo, be, wd, bd, y, q);
  if (rc != SPX_OK) return rc;
  return after_launch(cnt, "expand_dw_tc");
}

int tc_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
  }
  return v;
}

}  // namespace spx
