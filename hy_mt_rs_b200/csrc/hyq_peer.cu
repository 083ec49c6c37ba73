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

// ---------------------------------------------------------------------------
// Expert-parallel exchange over the same kind of region: rank r's block for
// rank q (rows of `row_floats` floats) is pushed into q's region at data
// slot r, so that each rank finds every source's block for it in its own
// region.  Header words used: ready[src] at [0, 256), started[src] at
// [256, 512), the call counter (epoch) at 512, a CTA counter at 516 and an
// abort word at 520.  One call is two launches, on every rank in the same
// order:
//   open (one thread): epoch e = counter + 1; started[rank] = e in every
//     peer; wait until every peer has started e as well (then each peer's
//     stream has finished with the data of exchange e - 1 in its region);
//   push (grid (row CTAs, destinations)): copy rows [0, valid[q]) of block q
//     (and, with `last_row`, the block's last row) into q's slot; every CTA
//     fences system-wide and counts itself; the last one sets ready[rank] = e
//     in every peer, waits for every peer's ready flag of e and stores e in
//     the counter.
// The next kernel in the stream reads the blocks from this rank's region.
// A wait that runs out sets HYQ_DEV_TIMEOUT_PEER (the open step also raises
// the abort word so that nothing is pushed).
struct XchgArgs {
  uint64_t region[kMaxPeers];
  int rank, world;
  const float* send;     // [world][rows][row_floats]
  const int32_t* valid;  // rows of each block to send (null: all)
  int rows, row_floats, last_row;
  int64_t slot;          // floats between slots of a region's data area
  unsigned* status;
  uint64_t wait_ns;
};

__global__ void peer_xchg_open_kernel(const __grid_constant__ XchgArgs a) {
  if (threadIdx.x != 0) return;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.region[a.rank]);
  const unsigned e = *reinterpret_cast<volatile unsigned*>(mine + 512) + 1;
  __threadfence_system();  // this rank's reads of exchange e - 1's data are ordered before the flag
  for (int q = 0; q < a.world; ++q)
    if (q != a.rank) st_release_sys(reinterpret_cast<unsigned*>(a.region[q] + 256) + a.rank, e);
  const bool ok = wait_flags(reinterpret_cast<const unsigned*>(mine + 256), a.rank, a.world, e, a.wait_ns);
  *reinterpret_cast<volatile int*>(mine + 520) = ok ? 0 : 1;
  if (!ok) atomicOr(a.status, DEV_TIMEOUT_PEER);
}

__global__ void __launch_bounds__(512) peer_xchg_push_kernel(const __grid_constant__ XchgArgs a) {
  __shared__ int last_s;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.region[a.rank]);
  const bool aborted = *reinterpret_cast<volatile int*>(mine + 520) != 0;
  const unsigned e = *reinterpret_cast<volatile unsigned*>(mine + 512) + 1;
  const int q = (int)blockIdx.y;
  if (!aborted) {
    int n = a.valid ? a.valid[q] : a.rows;
    n = n < 0 ? 0 : (n > a.rows ? a.rows : n);
    const float* src = a.send + (size_t)q * a.rows * a.row_floats;
    float* dst = reinterpret_cast<float*>(a.region[q] + kPeerDataOffset) + (size_t)a.rank * a.slot;
    const bool v4 = (a.row_floats & 3) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                                                 (uintptr_t)(a.slot * 4)) & 15) == 0;
    for (int r = (int)blockIdx.x; r < n + (a.last_row && n < a.rows ? 1 : 0); r += (int)gridDim.x) {
      const int row = r < n ? r : a.rows - 1;  // the block's last row, after the valid ones
      const float* s = src + (size_t)row * a.row_floats;
      float* d = dst + (size_t)row * a.row_floats;
      if (v4) {
        for (int i = threadIdx.x; i < a.row_floats / 4; i += blockDim.x)
          reinterpret_cast<float4*>(d)[i] = reinterpret_cast<const float4*>(s)[i];
      } else {
        for (int i = threadIdx.x; i < a.row_floats; i += blockDim.x) d[i] = s[i];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* cnt = reinterpret_cast<unsigned*>(mine + 516);
    last_s = atomicAdd(cnt, 1u) == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (!last_s || threadIdx.x != 0) return;
  *reinterpret_cast<volatile unsigned*>(mine + 516) = 0;
  if (!aborted) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank) st_release_sys(reinterpret_cast<unsigned*>(a.region[p]) + a.rank, e);
    if (!wait_flags(reinterpret_cast<const unsigned*>(mine), a.rank, a.world, e, a.wait_ns))
      atomicOr(a.status, DEV_TIMEOUT_PEER);
  }
  *reinterpret_cast<volatile unsigned*>(mine + 512) = e;
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

int hyq_peer_exchange(const uint64_t* regions, int rank, int world, size_t region_data_bytes, const float* send,
                      int rows, int row_floats, const int32_t* valid, int last_row, int64_t slot_floats,
                      void* stream) {
  if (!regions || !send) return hyq::api_fail(HYQ_E_INVALID, "peer_exchange: null argument");
  if (world < 1 || world > hyq::kMaxPeers || rank < 0 || rank >= world)
    return hyq::api_fail(HYQ_E_INVALID, "peer_exchange: rank %d of %d (at most %d ranks)", rank, world,
                         hyq::kMaxPeers);
  if (rows < 1 || row_floats < 1 || slot_floats < (int64_t)rows * row_floats)
    return hyq::api_fail(HYQ_E_SHAPE, "peer_exchange: %d rows of %d floats do not fit a slot of %lld floats", rows,
                         row_floats, (long long)slot_floats);
  if ((size_t)world * (size_t)slot_floats * sizeof(float) > region_data_bytes)
    return hyq::api_fail(HYQ_E_SHAPE, "peer_exchange: %d slots of %lld floats exceed the regions' %zu data bytes",
                         world, (long long)slot_floats, region_data_bytes);
  hyq::XchgArgs a{};
  for (int q = 0; q < world; ++q) {
    if (!regions[q] || (regions[q] & 255)) return hyq::api_fail(HYQ_E_ALIGN, "peer_exchange: region %d", q);
    a.region[q] = regions[q];
  }
  a.rank = rank;
  a.world = world;
  a.send = send;
  a.valid = valid;
  a.rows = rows;
  a.row_floats = row_floats;
  a.last_row = last_row ? 1 : 0;
  a.slot = slot_floats;
  a.wait_ns = hyq::g_peer_wait_ns.load(std::memory_order_relaxed);
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  hyq::peer_xchg_open_kernel<<<1, 32, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    const unsigned gx = (unsigned)(rows < 64 ? rows : 64);
    hyq::peer_xchg_push_kernel<<<dim3(gx, (unsigned)world), 512, 0, st>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "peer_exchange: %s", cudaGetErrorString(e));
  return HYQ_OK;
}

}  // extern "C"
