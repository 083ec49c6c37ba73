// All-reduce of row-parallel partial products over NVLink peer memory, for
// the tensor-parallel split of a decoder layer (O and down projections: each
// rank holds a block-aligned slice of K, its product is a partial sum of the
// full output, and every rank needs the total).
//
// Each rank owns one "peer region" (cudaMalloc, shared with the other ranks
// of the node through CUDA IPC; no multicast object):
//   [0, 256)      ready flags, one u32 per rank
//   [256, 512)    done flags, one u32 per rank
//   [512, 516)    this rank's call counter (epoch)
//   [1024, ...)   the partial product (floats), written by the caller
// One call, on every rank in the same order:
//   1. epoch = ++counter (device side, so the call replays correctly from a
//      CUDA graph);
//   2. make the partial visible system-wide and set ready[rank] = epoch in
//      every peer's region (release stores over NVLink);
//   3. wait until every peer has set this rank's ready[peer] >= epoch
//      (acquire loads, bounded by a time limit);
//   4. out[i] = sum over ranks 0..world-1 of partial[i], in rank order, so
//      every rank computes bit-identical totals;
//   5. set done[rank] = epoch in every peer and wait for all done flags, so
//      no rank overwrites its partial while a peer still reads it.
// A wait that runs out (after hyq_set_peer_timeout_ms, 5 s by default) sets
// HYQ_DEV_TIMEOUT_PEER in the status word and the call returns without
// writing `out`.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "../../include/hyq.h"
#include "hyq_common.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace {

constexpr int kMaxPeers = 8;
constexpr int kPeerDataOffset = HYQ_PEER_DATA_OFFSET;
// How long a call waits for the other ranks' flags (hyq_set_peer_timeout_ms;
// 5 s by default), read when the call is issued.
std::atomic<uint64_t> g_peer_wait_ns{5000000000ull};

struct PeerArgs {
  uint64_t region[kMaxPeers];
  int rank, world;
  int64_t n;
  float* out;
  unsigned* status;
  uint64_t wait_ns;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_volatile_f4(const float4* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ float ld_volatile_f(const float* p) {
  float v;
  asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// Wait (one thread) until flags[q] >= epoch for every peer q != rank.
__device__ bool wait_flags(const unsigned* flags, int rank, int world, unsigned epoch, uint64_t wait_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    for (uint32_t it = 0;; ++it) {
      if ((int)(ld_acquire_sys(flags + q) - epoch) >= 0) break;
      if ((it & 255u) == 255u && globaltimer_ns() - t0 > wait_ns) return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(512) peer_allreduce_kernel(const __grid_constant__ PeerArgs a) {
  __shared__ unsigned epoch_s;
  __shared__ int ok_s;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.region[a.rank]);
  if (threadIdx.x == 0) {
    unsigned* ctr = reinterpret_cast<unsigned*>(mine + 512);
    const unsigned e = *ctr + 1;
    *ctr = e;
    epoch_s = e;
    __threadfence_system();  // the partial written before this kernel, system-wide
    for (int q = 0; q < a.world; ++q)
      if (q != a.rank) st_release_sys(reinterpret_cast<unsigned*>(a.region[q]) + a.rank, e);
    ok_s = wait_flags(reinterpret_cast<const unsigned*>(mine), a.rank, a.world, e, a.wait_ns) ? 1 : 0;
    if (!ok_s) atomicOr(a.status, DEV_TIMEOUT_PEER);
  }
  __syncthreads();
  if (!ok_s) return;
  const int64_t n4 = ((a.n & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0) ? a.n / 4 : 0;
  for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < a.world; ++q) {
      const float4 v = ld_volatile_f4(reinterpret_cast<const float4*>(a.region[q] + kPeerDataOffset) + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    reinterpret_cast<float4*>(a.out)[i] = s;
  }
  for (int64_t i = 4 * n4 + threadIdx.x; i < a.n; i += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < a.world; ++q)
      s += ld_volatile_f(reinterpret_cast<const float*>(a.region[q] + kPeerDataOffset) + i);
    a.out[i] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned e = epoch_s;
    for (int q = 0; q < a.world; ++q)
      if (q != a.rank) st_release_sys(reinterpret_cast<unsigned*>(a.region[q] + 256) + a.rank, e);
    if (!wait_flags(reinterpret_cast<const unsigned*>(mine + 256), a.rank, a.world, e, a.wait_ns))
      atomicOr(a.status, DEV_TIMEOUT_PEER);
  }
}

}  // namespace
}  // namespace hyq

extern "C" {

int hyq_set_peer_timeout_ms(int ms) {
  if (ms < 1 || ms > 600000) return hyq::api_fail(HYQ_E_INVALID, "set_peer_timeout_ms: %d ms (1 .. 600000)", ms);
  hyq::g_peer_wait_ns.store((uint64_t)ms * 1000000ull, std::memory_order_relaxed);
  return HYQ_OK;
}

int hyq_peer_alloc(size_t data_bytes, void** region, void* ipc_handle) {
  if (!region || !ipc_handle) return hyq::api_fail(HYQ_E_INVALID, "peer_alloc: null output");
  *region = nullptr;
  void* p = nullptr;
  const size_t bytes = HYQ_PEER_DATA_OFFSET + (data_bytes + 15) / 16 * 16;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_NOMEM, "peer_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return hyq::api_fail(HYQ_E_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof h);
  *region = p;
  return HYQ_OK;
}

int hyq_peer_open(const void* ipc_handle, void** region) {
  if (!ipc_handle || !region) return hyq::api_fail(HYQ_E_INVALID, "peer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(region, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "peer_open: %s", cudaGetErrorString(e));
  return HYQ_OK;
}

int hyq_peer_close(void* region) {
  const cudaError_t e = cudaIpcCloseMemHandle(region);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "peer_close: %s", cudaGetErrorString(e));
  return HYQ_OK;
}

int hyq_peer_free(void* region) {
  const cudaError_t e = cudaFree(region);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "peer_free: %s", cudaGetErrorString(e));
  return HYQ_OK;
}

int hyq_peer_allreduce(const uint64_t* regions, int rank, int world, int64_t n, float* out, void* stream) {
  if (!regions || !out) return hyq::api_fail(HYQ_E_INVALID, "peer_allreduce: null argument");
  if (world < 1 || world > hyq::kMaxPeers || rank < 0 || rank >= world)
    return hyq::api_fail(HYQ_E_INVALID, "peer_allreduce: rank %d of %d (at most %d ranks)", rank, world,
                         hyq::kMaxPeers);
  if (n < 0) return hyq::api_fail(HYQ_E_SHAPE, "peer_allreduce: negative length");
  hyq::PeerArgs a{};
  for (int q = 0; q < world; ++q) {
    if (!regions[q] || (regions[q] & 255)) return hyq::api_fail(HYQ_E_ALIGN, "peer_allreduce: region %d", q);
    a.region[q] = regions[q];
  }
  a.rank = rank;
  a.world = world;
  a.n = n;
  a.out = out;
  a.wait_ns = hyq::g_peer_wait_ns.load(std::memory_order_relaxed);
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  hyq::peer_allreduce_kernel<<<1, 512, 0, (cudaStream_t)stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "peer_allreduce: %s", cudaGetErrorString(e));
  return HYQ_OK;
}

}  // extern "C"
