// Kernels of the TinyLlama decode path (the `llama_step` graph of
// source/xla_hlo/tools/export_llama.py:269-365 run with a KV cache instead of
// the reference's full re-computation over the padded 64-token window,
// run_llama_spirv.py:190-260):
//
//  * gemm_rows: C[m][n] = act(alpha * A[m] . W[n] + bias[n] + R[m][n]) for a
//    few activation rows (m < 8).  Decode GEMMs are weight-streaming: one warp
//    owns one output column, reads that weight row once with 16-byte loads
//    (eight in flight per lane) and keeps the m row accumulators in
//    registers.  A is read through L1, where every warp of the SM shares it.
//    Paired mode computes the gate column n and the up column n + pair_off
//    together and writes silu(gate) * up: the SwiGLU MLP's first GEMM and its
//    activation in one pass.
//  * rope_kv_append: rotate-half RoPE from the reference's cos / sin tables
//    (run_llama_spirv.py:87-97) on the q and k slices of the fused QKV
//    projection, q to the attention input, k and v appended to the KV cache
//    at position pos[0] + t.
//  * attention_kv: grouped-query attention of the new tokens over the cache
//    (causal: key j is visible to the query at position p when j <= p), one
//    CTA per (sequence, kv head, query chunk) sharing the cache tiles among
//    its query heads, online softmax over 64-key tiles.
//  * token_commit / argmax_partial / argmax_merge: greedy-decode bookkeeping
//    on the device (history, position counter) and the vocab-parallel argmax
//    of the tensor-parallel lm_head.
#include "spx_internal.cuh"

namespace spx {
namespace {

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

constexpr int kRowsWarps = 8;
constexpr int kRowsUnroll = 8;

template <int MR, bool PAIR, int A>
__global__ void __launch_bounds__(kRowsWarps * 32) gemm_rows_kernel(
    const float* __restrict__ a, int64_t lda, const float* __restrict__ w, int64_t ldw, int M,
    int N, int K, const float* __restrict__ bias, const float* __restrict__ res, float* c,
    int64_t ldc, float alpha, int64_t pair_off, float rms_eps,
    unsigned long long* __restrict__ amax) {
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * kRowsWarps + (threadIdx.x >> 5);
  if (n >= N) return;
  const int k4 = K >> 2;
  const float4* wr = reinterpret_cast<const float4*>(w + (int64_t)n * ldw);
  const float4* wu = reinterpret_cast<const float4*>(w + ((int64_t)n + pair_off) * ldw);
  const bool rms = rms_eps >= 0.0f;
  float acc[MR], accu[PAIR ? MR : 1], ss[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    acc[m] = 0.0f;
    ss[m] = 0.0f;
    if constexpr (PAIR) accu[m] = 0.0f;
  }
  for (int i0 = lane; i0 < k4; i0 += 32 * kRowsUnroll) {
    float4 wv[kRowsUnroll], uv[PAIR ? kRowsUnroll : 1];
#pragma unroll
    for (int j = 0; j < kRowsUnroll; ++j) {
      const int i = i0 + 32 * j;
      wv[j] = i < k4 ? __ldcs(wr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (PAIR) uv[j] = i < k4 ? __ldcs(wu + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kRowsUnroll; ++j) {
      const int i = i0 + 32 * j;
      if (i < k4) {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m < M) {
            const float4 av = __ldg(reinterpret_cast<const float4*>(a + m * lda) + i);
            acc[m] = dot4(av, wv[j], acc[m]);
            if constexpr (PAIR) accu[m] = dot4(av, uv[j], accu[m]);
            if (rms) ss[m] = dot4(av, av, ss[m]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    acc[m] = warp_sum32(acc[m]);
    if constexpr (PAIR) accu[m] = warp_sum32(accu[m]);
    if (rms) {
      // RMSNorm of the A row folded in: (x / rms(x)) . w = (x . w) / rms(x)
      // (the norm's gain is folded into the weights by the caller).
      const float inv = 1.0f / sqrtf(warp_sum32(ss[m]) / (float)K + rms_eps);
      acc[m] *= inv;
      if constexpr (PAIR) accu[m] *= inv;
    }
  }
  // Lane m writes row m.
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (lane == m && m < M) {
      float v;
      if constexpr (PAIR) {
        const float g = alpha * acc[m], u = alpha * accu[m];
        v = (g / (1.0f + expf(-g))) * u;
      } else {
        v = alpha * acc[m];
        if (bias) v += bias[n];
        if (res) v += res[(int64_t)m * ldc + n];
        v = act_c<A>(v);
      }
      c[(int64_t)m * ldc + n] = v;
      if (amax) {
        // Greedy argmax fused into the lm_head: one 64-bit key per row,
        // (order-preserving bits of v, ~n), so atomicMax keeps the largest
        // value and, among equal values, the smallest column.
        const uint32_t u = __float_as_uint(v);
        const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        atomicMax(amax + m, ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)n));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE + KV append.  qkv row r = b * T + t holds [q heads | k heads | v heads]
// of head_dim each.  cos / sin tables are [max_seq][head_dim].
__global__ void rope_kv_append_kernel(const float* __restrict__ qkv, int64_t ld_qkv,
                                      const float* __restrict__ cos_t,
                                      const float* __restrict__ sin_t,
                                      const int32_t* __restrict__ pos_p, float* __restrict__ q_out,
                                      float* __restrict__ kc, float* __restrict__ vc, int B,
                                      int T, int Hq, int Hkv, int D, int max_seq) {
  const int half = D >> 1;
  const int slots = Hq + 2 * Hkv;
  const int64_t total = (int64_t)B * T * slots * half;
  const int pos0 = *pos_p;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    int64_t r = idx / half;
    const int slot = (int)(r % slots);
    r /= slots;
    const int t = (int)(r % T);
    const int b = (int)(r / T);
    const int p = pos0 + t;
    if (p >= max_seq) continue;
    const float* src = qkv + ((int64_t)b * T + t) * ld_qkv + (int64_t)slot * D;
    const float x1 = src[i], x2 = src[i + half];
    if (slot < Hq + Hkv) {
      const float* cr = cos_t + (int64_t)p * D;
      const float* sr = sin_t + (int64_t)p * D;
      // x * cos + rotate_half(x) * sin, rotate_half(x) = [-x2, x1]
      // (export_llama.py:288-296), each product rounded as written.
      const float o1 = __fadd_rn(__fmul_rn(x1, cr[i]), __fmul_rn(-x2, sr[i]));
      const float o2 = __fadd_rn(__fmul_rn(x2, cr[i + half]), __fmul_rn(x1, sr[i + half]));
      float* dst;
      if (slot < Hq) {
        dst = q_out + (((int64_t)b * T + t) * Hq + slot) * D;
      } else {
        dst = kc + (((int64_t)b * Hkv + (slot - Hq)) * max_seq + p) * D;
      }
      dst[i] = o1;
      dst[i + half] = o2;
    } else {
      float* dst = vc + (((int64_t)b * Hkv + (slot - Hq - Hkv)) * max_seq + p) * D;
      dst[i] = x1;
      dst[i + half] = x2;
    }
  }
}

// ---------------------------------------------------------------------------
// Attention over the KV cache, head_dim 64.  Block = 8 warps; the CTA serves
// the G query heads of one kv head for TQ consecutive new tokens of one
// sequence: pairs (g, t) are dealt to warps round-robin, PP pairs per warp.
constexpr int kAttD = 64;
constexpr int kAttKeys = 64;
constexpr int kAttWarps = 8;

template <int PP>
__global__ void __launch_bounds__(kAttWarps * 32) attention_kv_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ out, const int32_t* __restrict__ pos_p, int T, int Hq, int Hkv,
    int max_seq, int TQ, float scale) {
  __shared__ float ks[kAttKeys][kAttD + 1];
  __shared__ float vs[kAttKeys][kAttD];
  __shared__ float qs[kAttWarps * PP][kAttD];
  const int G = Hq / Hkv;
  const int kvh = blockIdx.x;
  const int b = blockIdx.y;
  const int t0 = blockIdx.z * TQ;
  const int nt = min(TQ, T - t0);
  const int npairs = G * nt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos0 = *pos_p;
  // Stage the queries (pairs in order p = t_local * G + g).
  for (int e = threadIdx.x; e < npairs * kAttD; e += blockDim.x) {
    const int pr = e / kAttD, d = e % kAttD;
    const int tl = pr / G, g = pr % G;
    qs[pr][d] = q[(((int64_t)b * T + t0 + tl) * Hq + kvh * G + g) * kAttD + d];
  }
  float m_run[PP], l_run[PP], o0[PP], o1[PP];
#pragma unroll
  for (int j = 0; j < PP; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.0f;
    o0[j] = 0.0f;
    o1[j] = 0.0f;
  }
  const int last_pos = min(pos0 + t0 + nt - 1, max_seq - 1);
  const float* kb = kc + ((int64_t)b * Hkv + kvh) * max_seq * kAttD;
  const float* vb = vc + ((int64_t)b * Hkv + kvh) * max_seq * kAttD;
  for (int k0 = 0; k0 <= last_pos; k0 += kAttKeys) {
    __syncthreads();
    const int nk = min(kAttKeys, last_pos + 1 - k0);
    for (int e = threadIdx.x; e < nk * (kAttD / 4); e += blockDim.x) {
      const int j = e / (kAttD / 4), d4 = e % (kAttD / 4);
      const float4 kv4 = *reinterpret_cast<const float4*>(kb + (int64_t)(k0 + j) * kAttD + d4 * 4);
      const float4 vv4 = *reinterpret_cast<const float4*>(vb + (int64_t)(k0 + j) * kAttD + d4 * 4);
      ks[j][d4 * 4 + 0] = kv4.x;
      ks[j][d4 * 4 + 1] = kv4.y;
      ks[j][d4 * 4 + 2] = kv4.z;
      ks[j][d4 * 4 + 3] = kv4.w;
      *reinterpret_cast<float4*>(&vs[j][d4 * 4]) = vv4;
    }
    __syncthreads();
#pragma unroll
    for (int jj = 0; jj < PP; ++jj) {
      const int pr = warp + jj * kAttWarps;
      if (pr >= npairs) continue;
      const int qpos = pos0 + t0 + pr / G;
      // Scores of keys k0 + lane and k0 + lane + 32.
      float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 16
      for (int d = 0; d < kAttD; ++d) {
        const float qd = qs[pr][d];
        s0 = fmaf(qd, ks[lane][d], s0);
        s1 = fmaf(qd, ks[lane + 32][d], s1);
      }
      const bool ok0 = lane < nk && k0 + lane <= qpos;
      const bool ok1 = lane + 32 < nk && k0 + lane + 32 <= qpos;
      s0 = ok0 ? s0 * scale : -INFINITY;
      s1 = ok1 ? s1 * scale : -INFINITY;
      float mt = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      if (mt == -INFINITY) continue;  // no visible key in this tile
      const float m_new = fmaxf(m_run[jj], mt);
      const float corr = expf(m_run[jj] - m_new);
      const float p0 = ok0 ? expf(s0 - m_new) : 0.0f;
      const float p1 = ok1 ? expf(s1 - m_new) : 0.0f;
      l_run[jj] = l_run[jj] * corr + warp_sum32(p0 + p1);
      float a0 = o0[jj] * corr, a1 = o1[jj] * corr;
      for (int j = 0; j < nk; ++j) {
        const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
        a0 = fmaf(pj, vs[j][lane], a0);
        a1 = fmaf(pj, vs[j][lane + 32], a1);
      }
      o0[jj] = a0;
      o1[jj] = a1;
      m_run[jj] = m_new;
    }
  }
#pragma unroll
  for (int jj = 0; jj < PP; ++jj) {
    const int pr = warp + jj * kAttWarps;
    if (pr >= npairs) continue;
    const int tl = pr / G, g = pr % G;
    float* op = out + (((int64_t)b * T + t0 + tl) * Hq + kvh * G + g) * kAttD;
    const float inv = 1.0f / l_run[jj];
    op[lane] = o0[jj] * inv;
    op[lane + 32] = o1[jj] * inv;
  }
}

// ---------------------------------------------------------------------------
// state[0] = position (tokens in the cache), state[1] = generated count.
// With `keys` (fused lm_head argmax), ids[b] is decoded from keys[b] first
// and the key is reset for the next step.
__global__ void token_commit_kernel(int32_t* __restrict__ ids, int32_t* __restrict__ hist,
                                    int32_t* state, int B, int advance, int hist_cap,
                                    unsigned long long* __restrict__ keys) {
  const int step = state[1];
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    if (keys) {
      ids[b] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[b] & 0xFFFFFFFFull));
      keys[b] = 0ull;
    }
    if (step < hist_cap) hist[(int64_t)step * B + b] = ids[b];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    state[0] += advance;
    state[1] = step + 1;
  }
}

// Packed (value, global index) argmax of each row, first maximum wins.
__global__ void argmax_partial_kernel(const float* __restrict__ x, int64_t ldx, int rows,
                                      int cols, int col_offset, float2* __restrict__ packed) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* xr = x + (int64_t)r * ldx;
  float best = -3.4028234663852886e+38f;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < cols; j += blockDim.x) {
    const float v = xr[j];
    if (v > best || (v == best && j < bi)) { best = v; bi = j; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -3.4028234663852886e+38f;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) packed[r] = make_float2(best, __int_as_float(bi + col_offset));
  }
}

// packed: [parts][rows] (value, index bits); larger value wins, ties go to
// the smaller index.
__global__ void argmax_merge_kernel(const float2* __restrict__ packed, int parts, int rows,
                                    int32_t* __restrict__ ids) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    float best = -3.4028234663852886e+38f;
    int bi = 0x7fffffff;
    for (int p = 0; p < parts; ++p) {
      const float2 e = packed[(int64_t)p * rows + r];
      const int i = __float_as_int(e.y);
      if (e.x > best || (e.x == best && i < bi)) { best = e.x; bi = i; }
    }
    ids[r] = bi;
  }
}

// y[r][j] = silu(gu[r][j]) * gu[r][j + f] over rows of the fused gate|up
// projection (row stride ld).
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, int64_t ld, float* __restrict__ y,
                                   int64_t ldy, int rows, int f) {
  const int64_t total = (int64_t)rows * f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / f), j = (int)(i % f);
    const float g = gu[(int64_t)r * ld + j], u = gu[(int64_t)r * ld + f + j];
    y[(int64_t)r * ldy + j] = (g / (1.0f + expf(-g))) * u;
  }
}

template <int MR, bool PAIR>
void rows_launch(cudaStream_t s, int act, const float* a, int64_t lda, const float* w,
                 int64_t ldw, int M, int N, int K, const float* bias, const float* res, float* c,
                 int64_t ldc, float alpha, int64_t pair_off, float rms_eps,
                 unsigned long long* amax) {
  const int grid = (N + kRowsWarps - 1) / kRowsWarps;
  if constexpr (PAIR) {
    gemm_rows_kernel<MR, true, SPX_ACT_NONE><<<grid, kRowsWarps * 32, 0, s>>>(
        a, lda, w, ldw, M, N, K, bias, res, c, ldc, alpha, pair_off, rms_eps, nullptr);
  } else {
    host_with_act(act, [&](auto tag) {
      constexpr int A = decltype(tag)::value;
      gemm_rows_kernel<MR, false, A><<<grid, kRowsWarps * 32, 0, s>>>(
          a, lda, w, ldw, M, N, K, bias, res, c, ldc, alpha, pair_off, rms_eps, amax);
    });
  }
}

bool al16p(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

bool gemm_rows_eligible(const float* a, int64_t lda, const float* w, int64_t ldw, int M, int K) {
  return M >= 1 && M <= 8 && K > 0 && K % 4 == 0 && lda % 4 == 0 && ldw % 4 == 0 && al16p(a) &&
         al16p(w);
}

int launch_gemm_rows(cudaStream_t s, int64_t* cnt, const float* a, int64_t lda, const float* w,
                     int64_t ldw, int M, int N, int K, const float* bias, const float* res,
                     float* c, int64_t ldc, float alpha, int act, int64_t pair_off,
                     float rms_eps, unsigned long long* amax) {
  if (!gemm_rows_eligible(a, lda, w, ldw, M, K) || N <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "gemm_rows: operands not eligible");
  const bool pair = pair_off > 0;
  // Row counts are rounded up to 1, 2, 4 or 8 accumulators.
  const int mr = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
#define SPX_ROWS(MRV)                                                                          \
  (pair ? rows_launch<MRV, true>(s, act, a, lda, w, ldw, M, N, K, bias, res, c, ldc, alpha,    \
                                 pair_off, rms_eps, nullptr)                                   \
        : rows_launch<MRV, false>(s, act, a, lda, w, ldw, M, N, K, bias, res, c, ldc, alpha,   \
                                  pair_off, rms_eps, amax))
  switch (mr) {
    case 1: SPX_ROWS(1); break;
    case 2: SPX_ROWS(2); break;
    case 4: SPX_ROWS(4); break;
    default: SPX_ROWS(8); break;
  }
#undef SPX_ROWS
  return after_launch(cnt, "gemm_rows");
}

int launch_rope_kv_append(cudaStream_t s, int64_t* cnt, const float* qkv, int64_t ld_qkv,
                          const float* cos_t, const float* sin_t, const int32_t* pos,
                          float* q_out, float* kc, float* vc, int B, int T, int Hq, int Hkv,
                          int D, int max_seq) {
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2 || max_seq <= 0 ||
      ld_qkv < (int64_t)(Hq + 2 * Hkv) * D)
    return fail(SPX_ERR_INVALID_ARGUMENT, "rope_kv_append: bad shape");
  const int64_t total = (int64_t)B * T * (Hq + 2 * Hkv) * (D / 2);
  rope_kv_append_kernel<<<grid_for(total, 256), 256, 0, s>>>(qkv, ld_qkv, cos_t, sin_t, pos, q_out,
                                                             kc, vc, B, T, Hq, Hkv, D, max_seq);
  return after_launch(cnt, "rope_kv_append");
}

int launch_attention_kv(cudaStream_t s, int64_t* cnt, const float* q, const float* kc,
                        const float* vc, float* out, const int32_t* pos, int B, int T, int Hq,
                        int Hkv, int D, int max_seq, float scale) {
  if (D != kAttD) return fail(SPX_ERR_UNSUPPORTED, "attention_kv: head_dim must be 64");
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || max_seq <= 0)
    return fail(SPX_ERR_INVALID_ARGUMENT, "attention_kv: bad shape");
  const int G = Hq / Hkv;
  if (G > 4 * kAttWarps) return fail(SPX_ERR_UNSUPPORTED, "attention_kv: group above 32 heads");
  // Tokens per CTA: as many as keep every warp at <= 4 (g, t) pairs.
  int TQ = (4 * kAttWarps) / G;
  if (TQ > T) TQ = T;
  const int pairs = G * TQ;
  const int pp = (pairs + kAttWarps - 1) / kAttWarps;
  dim3 grid(Hkv, B, (T + TQ - 1) / TQ);
  if (grid.y > 65535 || grid.z > 65535)
    return fail(SPX_ERR_UNSUPPORTED, "attention_kv: grid too large");
  switch (pp) {
    case 1:
      attention_kv_kernel<1><<<grid, kAttWarps * 32, 0, s>>>(q, kc, vc, out, pos, T, Hq, Hkv,
                                                             max_seq, TQ, scale);
      break;
    case 2:
      attention_kv_kernel<2><<<grid, kAttWarps * 32, 0, s>>>(q, kc, vc, out, pos, T, Hq, Hkv,
                                                             max_seq, TQ, scale);
      break;
    default:
      attention_kv_kernel<4><<<grid, kAttWarps * 32, 0, s>>>(q, kc, vc, out, pos, T, Hq, Hkv,
                                                             max_seq, TQ, scale);
      break;
  }
  return after_launch(cnt, "attention_kv");
}

int launch_token_commit(cudaStream_t s, int64_t* cnt, int32_t* ids, int32_t* hist,
                        int32_t* state, int B, int advance, int hist_cap,
                        unsigned long long* keys) {
  if (B <= 0 || hist_cap <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "token_commit: bad shape");
  token_commit_kernel<<<1, 256, 0, s>>>(ids, hist, state, B, advance, hist_cap, keys);
  return after_launch(cnt, "token_commit");
}

int launch_argmax_partial(cudaStream_t s, int64_t* cnt, const float* x, int64_t ldx, int rows,
                          int cols, int col_offset, float* packed) {
  if (rows <= 0 || cols <= 0 || ldx < cols)
    return fail(SPX_ERR_INVALID_ARGUMENT, "argmax_partial: bad shape");
  argmax_partial_kernel<<<rows, 512, 0, s>>>(x, ldx, rows, cols, col_offset,
                                             reinterpret_cast<float2*>(packed));
  return after_launch(cnt, "argmax_partial");
}

int launch_swiglu_rows(cudaStream_t s, int64_t* cnt, const float* gu, int64_t ld, float* y,
                       int64_t ldy, int rows, int f) {
  if (rows <= 0 || f <= 0 || ld < 2 * (int64_t)f || ldy < f)
    return fail(SPX_ERR_INVALID_ARGUMENT, "swiglu_rows: bad shape");
  swiglu_rows_kernel<<<grid_for((int64_t)rows * f, 256), 256, 0, s>>>(gu, ld, y, ldy, rows, f);
  return after_launch(cnt, "swiglu_rows");
}

int launch_argmax_merge(cudaStream_t s, int64_t* cnt, const float* packed, int parts, int rows,
                        int32_t* ids) {
  if (rows <= 0 || parts <= 0) return fail(SPX_ERR_INVALID_ARGUMENT, "argmax_merge: bad shape");
  argmax_merge_kernel<<<grid_for(rows, 128), 128, 0, s>>>(
      reinterpret_cast<const float2*>(packed), parts, rows, ids);
  return after_launch(cnt, "argmax_merge");
}

}  // namespace spx
