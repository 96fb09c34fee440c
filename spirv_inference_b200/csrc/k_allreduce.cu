// One-shot all-reduce over peer memory (NVLink / NVSwitch), for the small
// messages of tensor-parallel decode (a few KB to ~1 MB per step, where a
// library all-reduce is launch- and protocol-bound).
//
// Every rank owns a communicator buffer: two data slots of max_bytes and a
// flag array, exported with cudaIpcGetMemHandle and opened by every peer.
// A producer (the row-parallel GEMM) writes its partial sum straight into
// slot s of its own buffer; spx_op_allreduce then, per CTA:
//   1. takes the next epoch from a device-side counter (so a captured CUDA
//      graph replays with fresh epochs),
//   2. publishes it to flags[cta][my rank] of every peer (release, system
//      scope, after a system fence that orders the partial sums),
//   3. waits until every peer's epoch for this CTA has reached its own
//      (acquire loads; bounded by a %globaltimer limit, 2 s unless the
//      "ar_wait_limit_us" option says otherwise, after which it records an
//      error status and returns without touching the output),
//   4. sums its slice of slot s over all ranks with plain loads from the
//      peers' memory into the local output.
// Consecutive all-reduces must alternate the two slots: a rank rewrites slot
// s only after it has passed the barrier of the next all-reduce, which every
// peer enters only after finishing its reads of slot s.  No multicast and no
// TMA are used on peer memory.
#include <cuda_runtime.h>

#include <vector>

#include "spx_internal.cuh"

struct spx_ar {
  int device = 0, rank = 0, world = 0;
  size_t max_bytes = 0;
  uint8_t* base = nullptr;             // [slot 0 | slot 1 | flags | epochs]
  std::vector<uint8_t*> peers;         // peers' bases (own base at index rank)
  float** d_peers = nullptr;           // device array of world slot-0 pointers
  unsigned long long** d_flags = nullptr;
  bool opened = false;
};

namespace spx {

__device__ int g_ar_status = 0;

namespace {

constexpr int kArMaxCtas = 32;
constexpr int kArMaxRanks = 8;
constexpr size_t kFlagBytes = (size_t)kArMaxCtas * kArMaxRanks * 8;
constexpr size_t kEpochBytes = (size_t)kArMaxCtas * 8;

__device__ __forceinline__ unsigned long long ar_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// peers[r]: rank r's slot-0 base; flags[r]: rank r's flag array.
__global__ void __launch_bounds__(512) allreduce_kernel(
    float* const* __restrict__ peers, unsigned long long* const* __restrict__ flags,
    unsigned long long* __restrict__ epochs, int rank, int world, int64_t slot_off, float* out,
    int64_t n4, unsigned long long limit_ns) {
  __shared__ int s_ok;
  const int cta = blockIdx.x;
  if (threadIdx.x == 0) {
    __threadfence_system();  // this rank's partial sums before the signal
    const unsigned long long e = epochs[cta] + 1;
    epochs[cta] = e;
    for (int r = 0; r < world; ++r) st_release_sys(flags[r] + cta * kArMaxRanks + rank, e);
    int ok = 1;
    const unsigned long long t0 = ar_now();
    for (int r = 0; r < world && ok; ++r) {
      const unsigned long long* f = flags[rank] + cta * kArMaxRanks + r;
      while (ld_acquire_sys(f) < e) {
        if (ar_now() - t0 > limit_ns) {
          atomicExch(&g_ar_status, 1);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  // This CTA's slice of the float4 range.
  const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
  const int64_t lo = (int64_t)cta * per, hi = min(n4, lo + per);
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {  // fixed rank order: identical sums on every rank
      const float4 v =
          __ldcv(reinterpret_cast<const float4*>(peers[r] + slot_off) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

}  // namespace

int ar_take_status() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ar_status, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (v) {
    int zero = 0;
    cudaMemcpyToSymbol(g_ar_status, &zero, sizeof(int));
  }
  return v;
}

}  // namespace spx

using namespace spx;

extern "C" {

int spx_ar_create(int32_t device, int32_t rank, int32_t world, size_t max_bytes, spx_ar** out) {
  if (!out) return fail(SPX_ERR_INVALID_ARGUMENT, "ar_create: null");
  *out = nullptr;
  if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world)
    return fail(SPX_ERR_INVALID_ARGUMENT, "ar_create: rank %d of %d (at most %d ranks)", rank,
                world, kArMaxRanks);
  if (max_bytes == 0 || max_bytes % 16)
    return fail(SPX_ERR_INVALID_ARGUMENT, "ar_create: max_bytes must be a positive multiple of 16");
  int rc = check_cuda(cudaSetDevice(device), "ar_create: cudaSetDevice");
  if (rc) return rc;
  spx_ar* a = new spx_ar();
  a->device = device;
  a->rank = rank;
  a->world = world;
  a->max_bytes = max_bytes;
  const size_t total = 2 * max_bytes + kFlagBytes + kEpochBytes;
  rc = check_cuda(cudaMalloc((void**)&a->base, total), "ar_create: cudaMalloc");
  if (!rc) rc = check_cuda(cudaMemset(a->base, 0, total), "ar_create: cudaMemset");
  if (!rc) rc = check_cuda(cudaMalloc((void**)&a->d_peers, world * sizeof(float*)), "ar_create");
  if (!rc)
    rc = check_cuda(cudaMalloc((void**)&a->d_flags, world * sizeof(unsigned long long*)),
                    "ar_create");
  if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "ar_create: sync");
  if (rc) {
    if (a->base) cudaFree(a->base);
    if (a->d_peers) cudaFree(a->d_peers);
    if (a->d_flags) cudaFree(a->d_flags);
    delete a;
    return rc;
  }
  *out = a;
  return SPX_OK;
}

int spx_ar_handle(spx_ar* a, void* handle, size_t handle_bytes) {
  if (!a || !handle) return fail(SPX_ERR_INVALID_ARGUMENT, "ar_handle: null");
  if (handle_bytes < sizeof(cudaIpcMemHandle_t))
    return fail(SPX_ERR_INVALID_ARGUMENT, "ar_handle: buffer below %zu bytes",
                sizeof(cudaIpcMemHandle_t));
  cudaIpcMemHandle_t h;
  int rc = check_cuda(cudaSetDevice(a->device), "ar_handle: cudaSetDevice");
  if (!rc) rc = check_cuda(cudaIpcGetMemHandle(&h, a->base), "cudaIpcGetMemHandle");
  if (!rc) memcpy(handle, &h, sizeof(h));
  return rc;
}

size_t spx_ar_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int spx_ar_open(spx_ar* a, const void* handles) {
  if (!a || !handles) return fail(SPX_ERR_INVALID_ARGUMENT, "ar_open: null");
  if (a->opened) return fail(SPX_ERR_INVALID_ARGUMENT, "ar_open: already open");
  int rc = check_cuda(cudaSetDevice(a->device), "ar_open: cudaSetDevice");
  if (rc) return rc;
  a->peers.assign(a->world, nullptr);
  for (int r = 0; r < a->world; ++r) {
    if (r == a->rank) {
      a->peers[r] = a->base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, (const uint8_t*)handles + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    rc = check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                    "cudaIpcOpenMemHandle");
    if (rc) return rc;
    a->peers[r] = (uint8_t*)p;
  }
  std::vector<float*> slots(a->world);
  std::vector<unsigned long long*> flags(a->world);
  for (int r = 0; r < a->world; ++r) {
    slots[r] = (float*)a->peers[r];
    flags[r] = (unsigned long long*)(a->peers[r] + 2 * a->max_bytes);
  }
  rc = check_cuda(cudaMemcpy(a->d_peers, slots.data(), a->world * sizeof(float*),
                             cudaMemcpyHostToDevice),
                  "ar_open: peers");
  if (!rc)
    rc = check_cuda(cudaMemcpy(a->d_flags, flags.data(),
                               a->world * sizeof(unsigned long long*), cudaMemcpyHostToDevice),
                    "ar_open: flags");
  if (!rc) a->opened = true;
  return rc;
}

float* spx_ar_slot(spx_ar* a, int32_t slot) {
  if (!a || slot < 0 || slot > 1) return nullptr;
  return (float*)(a->base + (size_t)slot * a->max_bytes);
}

int spx_op_allreduce(spx_graph* g, spx_ar* a, int32_t slot, float* out, int64_t n) {
  if (!g || !a || !out) return fail(SPX_ERR_INVALID_ARGUMENT, "allreduce: null");
  if (!a->opened) return fail(SPX_ERR_INVALID_ARGUMENT, "allreduce: peers not opened");
  if (slot < 0 || slot > 1) return fail(SPX_ERR_INVALID_ARGUMENT, "allreduce: slot 0 or 1");
  if (n <= 0 || n % 4 || (size_t)n * 4 > a->max_bytes || ((uintptr_t)out & 15))
    return fail(SPX_ERR_INVALID_ARGUMENT,
                "allreduce: n must be a positive multiple of 4 floats within max_bytes, out "
                "16-byte aligned");
  const int64_t n4 = n / 4;
  int ctas = (int)((n4 + 2047) / 2048);  // ~32 KB per CTA
  if (ctas > kArMaxCtas) ctas = kArMaxCtas;
  if (ctas < 1) ctas = 1;
  unsigned long long* epochs =
      (unsigned long long*)(a->base + 2 * a->max_bytes + kFlagBytes);
  allreduce_kernel<<<ctas, 512, 0, g->stream>>>(a->d_peers, a->d_flags, epochs, a->rank,
                                                 a->world, (int64_t)slot * (int64_t)(a->max_bytes / 4),
                                                 out, n4,
                                                 (unsigned long long)g_ar_wait_limit_us * 1000ull);
  return after_launch(&g->launches, "allreduce");
}

int spx_ar_reset(spx_ar* a) {
  if (!a) return fail(SPX_ERR_INVALID_ARGUMENT, "ar_reset: null");
  int rc = check_cuda(cudaSetDevice(a->device), "ar_reset: cudaSetDevice");
  if (!rc)
    rc = check_cuda(cudaMemset(a->base + 2 * a->max_bytes, 0, kFlagBytes + kEpochBytes),
                    "ar_reset: cudaMemset");
  if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "ar_reset: sync");
  return rc;
}

int spx_ar_destroy(spx_ar* a) {
  if (!a) return SPX_OK;
  cudaSetDevice(a->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < (int)a->peers.size(); ++r)
    if (r != a->rank && a->peers[r]) cudaIpcCloseMemHandle(a->peers[r]);
  if (a->base) cudaFree(a->base);
  if (a->d_peers) cudaFree(a->d_peers);
  if (a->d_flags) cudaFree(a->d_flags);
  delete a;
  return SPX_OK;
}

}  // extern "C"
