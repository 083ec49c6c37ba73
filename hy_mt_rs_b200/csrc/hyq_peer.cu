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
  // Row sources other than a packed send buffer (mode):
  //   0: block q row i = send[(q rows + i)];
  //   1 (expert dispatch): block q holds this rank's grouped rows for q's
  //     experts, off[q El] .. off[(q + 1) El], row i = send[row_token[off[q
  //     El] + i]] (send = the layer's token rows, `src_rows` of them), and
  //     its last row starts with the int32 bit patterns of q's experts' row
  //     counts;
  //   2 (expert return): block q row i = send[gather[q (rows) + i]] for i <
  //     valid[q] (send = the expert outputs, `src_rows` of them).
  int mode;
  const int32_t* off;
  const int32_t* gather;  // mode 1: row_token; mode 2: inverse permutation
  int el;                 // experts per rank (mode 1)
  int src_rows;
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
    float* dst = reinterpret_cast<float*>(a.region[q] + kPeerDataOffset) + (size_t)a.rank * a.slot;
    int n, g0 = 0;
    if (a.mode == 1) {
      // grouped rows of q's experts, then (first CTA) the count row
      g0 = a.off[q * a.el];
      n = a.off[(q + 1) * a.el] - g0;
      if (blockIdx.x == 0)
        for (int e = threadIdx.x; e < a.el; e += blockDim.x)
          reinterpret_cast<int32_t*>(dst + (size_t)(a.rows - 1) * a.row_floats)[e] =
              a.off[q * a.el + e + 1] - a.off[q * a.el + e];
    } else {
      n = a.valid ? a.valid[q] : a.rows;
    }
    const int cap_rows = a.mode == 1 ? a.rows - 1 : a.rows;
    n = n < 0 ? 0 : (n > cap_rows ? cap_rows : n);
    const float* src = a.send + (a.mode == 0 ? (size_t)q * a.rows * a.row_floats : 0);
    const bool v4 = (a.row_floats & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.send) | reinterpret_cast<uintptr_t>(dst) |
                                                 (uintptr_t)(a.slot * 4)) & 15) == 0;
    const bool extra = a.mode == 0 && a.last_row && n < a.rows;
    for (int r = (int)blockIdx.x; r < n + (extra ? 1 : 0); r += (int)gridDim.x) {
      const int row = r < n ? r : a.rows - 1;  // the block's last row, after the valid ones
      int sr = row;  // source row
      if (a.mode != 0) {
        sr = a.mode == 1 ? a.gather[g0 + row] : a.gather[(size_t)q * a.rows + row];
        sr = sr < 0 ? 0 : (sr >= a.src_rows ? a.src_rows - 1 : sr);
      }
      const float* s = src + (size_t)sr * a.row_floats;
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

// Receive side of the expert exchange, one CTA: from the count rows the
// sources left in this rank's region (source s's block at row s * stride,
// its count row at row cap), the expert-major gather index of the expert
// products, the local experts' row offsets, the inverse (expert-major row of
// each received row, for the return) and the rows received from each source.
constexpr int kPlanMax = 1024;  // world x experts per rank
struct PlanArgs {
  const float* data;  // this rank's region data
  int world, el, cap, hidden;
  int64_t slot;
  int32_t* perm;      // [world cap]
  int32_t* off;       // [el + 1]
  int32_t* inv;       // [world cap]
  int32_t* back;      // [world]
};

__global__ void __launch_bounds__(1024) moe_ep_plan_kernel(const __grid_constant__ PlanArgs a) {
  __shared__ int cnt[kPlanMax];   // [s][e]
  __shared__ int src0[kPlanMax];  // first row of (s, e) in source s's block
  __shared__ int base[kPlanMax];  // first expert-major row of (e, s), in (e, s) order
  __shared__ int total_s;
  const int W = a.world, El = a.el, n = W * El;
  const int64_t stride = a.slot / a.hidden;
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    const int s = k / El, e = k - s * El;
    const int32_t* row = reinterpret_cast<const int32_t*>(a.data + (size_t)s * a.slot + (size_t)a.cap * a.hidden);
    const int c = row[e];
    cnt[k] = c < 0 ? 0 : (c > a.cap ? a.cap : c);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < W; ++s) {
      int acc = 0;
      for (int e = 0; e < El; ++e) {
        // a source never sends more than cap rows in all
        const int c = acc + cnt[s * El + e] > a.cap ? a.cap - acc : cnt[s * El + e];
        cnt[s * El + e] = c;
        src0[s * El + e] = acc;
        acc += c;
      }
      a.back[s] = acc;
    }
    int t = 0;
    for (int e = 0; e < El; ++e) {
      a.off[e] = t;
      for (int s = 0; s < W; ++s) {
        base[e * W + s] = t;
        t += cnt[s * El + e];
      }
    }
    a.off[El] = t;
    total_s = t;
  }
  __syncthreads();
  const int total = total_s, R = W * a.cap;
  for (int t = threadIdx.x; t < R; t += blockDim.x) {
    if (t >= total) {
      a.perm[t] = 0;
      continue;
    }
    int lo = 0, hi = n - 1;  // last (e, s) whose base <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (base[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    while (lo + 1 < n && base[lo + 1] <= t) ++lo;  // skip empty runs that share a base
    const int e = lo / W, s = lo - e * W;
    const int i = src0[s * El + e] + (t - base[lo]);
    a.perm[t] = (int32_t)(s * stride + i);
    a.inv[s * a.cap + i] = t;
  }
}

// The returned rows home: the rows this rank sent to rank q come back into
// its region at slot q, row i = grouped row off[q El] + i of `out`.
struct HomeArgs {
  const float* data;
  const int32_t* off;
  int world, el, cap, hidden;
  int64_t slot;
  float* out;
};

__global__ void __launch_bounds__(512) moe_ep_home_kernel(const __grid_constant__ HomeArgs a) {
  const int q = (int)blockIdx.y;
  const int g0 = a.off[q * a.el];
  int n = a.off[(q + 1) * a.el] - g0;
  n = n < 0 ? 0 : (n > a.cap ? a.cap : n);
  const bool v4 = (a.hidden & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.data) | reinterpret_cast<uintptr_t>(a.out) |
                                           (uintptr_t)(a.slot * 4)) & 15) == 0;
  for (int r = (int)blockIdx.x; r < n; r += (int)gridDim.x) {
    const float* s = a.data + (size_t)q * a.slot + (size_t)r * a.hidden;
    float* d = a.out + (size_t)(g0 + r) * a.hidden;
    if (v4) {
      for (int i = threadIdx.x; i < a.hidden / 4; i += blockDim.x)
        reinterpret_cast<float4*>(d)[i] = reinterpret_cast<const float4*>(s)[i];
    } else {
      for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) d[i] = s[i];
    }
  }
}

// Regions, rank and sizes shared by the exchange entry points.
int xchg_setup(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
               int64_t need_floats, const char* what, XchgArgs& a) {
  if (!regions) return api_fail(HYQ_E_INVALID, "%s: null regions", what);
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return api_fail(HYQ_E_INVALID, "%s: rank %d of %d (at most %d ranks)", what, rank, world, kMaxPeers);
  if (need_floats < 1 || slot_floats < need_floats)
    return api_fail(HYQ_E_SHAPE, "%s: a block of %lld floats does not fit a slot of %lld floats", what,
                    (long long)need_floats, (long long)slot_floats);
  if ((size_t)world * (size_t)slot_floats * sizeof(float) > region_data_bytes)
    return api_fail(HYQ_E_SHAPE, "%s: %d slots of %lld floats exceed the regions' %zu data bytes", what, world,
                    (long long)slot_floats, region_data_bytes);
  a = XchgArgs{};
  for (int q = 0; q < world; ++q) {
    if (!regions[q] || (regions[q] & 255)) return api_fail(HYQ_E_ALIGN, "%s: region %d", what, q);
    a.region[q] = regions[q];
  }
  a.rank = rank;
  a.world = world;
  a.slot = slot_floats;
  a.wait_ns = g_peer_wait_ns.load(std::memory_order_relaxed);
  return api_status_word(&a.status);
}

int xchg_launch(const XchgArgs& a, void* stream, const char* what) {
  cudaStream_t st = (cudaStream_t)stream;
  peer_xchg_open_kernel<<<1, 32, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    const unsigned gx = (unsigned)(a.rows < 64 ? a.rows : 64);
    peer_xchg_push_kernel<<<dim3(gx, (unsigned)a.world), 512, 0, st>>>(a);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return api_fail(HYQ_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return HYQ_OK;
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
  if (!send) return hyq::api_fail(HYQ_E_INVALID, "peer_exchange: null send");
  if (rows < 1 || row_floats < 1) return hyq::api_fail(HYQ_E_SHAPE, "peer_exchange: %d rows of %d floats", rows, row_floats);
  hyq::XchgArgs a;
  int rc = hyq::xchg_setup(regions, rank, world, region_data_bytes, slot_floats, (int64_t)rows * row_floats,
                           "peer_exchange", a);
  if (rc) return rc;
  a.send = send;
  a.valid = valid;
  a.rows = rows;
  a.row_floats = row_floats;
  a.last_row = last_row ? 1 : 0;
  return hyq::xchg_launch(a, stream, "peer_exchange");
}

int hyq_moe_ep_dispatch(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                        const float* x, int tokens, int hidden, const int32_t* off, const int32_t* row_token,
                        int experts_per_rank, int cap, void* stream) {
  if (!x || !off || !row_token) return hyq::api_fail(HYQ_E_INVALID, "moe_ep_dispatch: null argument");
  if (tokens < 1 || hidden < 1 || cap < 1 || experts_per_rank < 1 || experts_per_rank > hidden)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_ep_dispatch: %d tokens, hidden %d, cap %d, %d experts per rank", tokens,
                         hidden, cap, experts_per_rank);
  hyq::XchgArgs a;
  int rc = hyq::xchg_setup(regions, rank, world, region_data_bytes, slot_floats, (int64_t)(cap + 1) * hidden,
                           "moe_ep_dispatch", a);
  if (rc) return rc;
  a.mode = 1;
  a.send = x;
  a.src_rows = tokens;
  a.off = off;
  a.gather = row_token;
  a.el = experts_per_rank;
  a.rows = cap + 1;
  a.row_floats = hidden;
  return hyq::xchg_launch(a, stream, "moe_ep_dispatch");
}

int hyq_moe_ep_plan(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                    int hidden, int cap, int experts_per_rank, int32_t* perm, int32_t* expert_off, int32_t* inv,
                    int32_t* back_rows, void* stream) {
  if (!perm || !expert_off || !inv || !back_rows) return hyq::api_fail(HYQ_E_INVALID, "moe_ep_plan: null output");
  if (hidden < 1 || cap < 1 || experts_per_rank < 1 || experts_per_rank > hidden ||
      (int64_t)world * experts_per_rank > hyq::kPlanMax || slot_floats % hidden)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_ep_plan: hidden %d, cap %d, %d experts per rank (at most %d with the ranks)",
                         hidden, cap, experts_per_rank, hyq::kPlanMax);
  hyq::XchgArgs x;
  int rc = hyq::xchg_setup(regions, rank, world, region_data_bytes, slot_floats, (int64_t)(cap + 1) * hidden,
                           "moe_ep_plan", x);
  if (rc) return rc;
  hyq::PlanArgs a{};
  a.data = reinterpret_cast<const float*>(regions[rank] + HYQ_PEER_DATA_OFFSET);
  a.world = world;
  a.el = experts_per_rank;
  a.cap = cap;
  a.hidden = hidden;
  a.slot = slot_floats;
  a.perm = perm;
  a.off = expert_off;
  a.inv = inv;
  a.back = back_rows;
  hyq::moe_ep_plan_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_ep_plan: %s", cudaGetErrorString(e));
}

int hyq_moe_ep_return(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                      const float* y, int hidden, const int32_t* inv, const int32_t* back_rows, int cap,
                      void* stream) {
  if (!y || !inv || !back_rows) return hyq::api_fail(HYQ_E_INVALID, "moe_ep_return: null argument");
  if (hidden < 1 || cap < 1) return hyq::api_fail(HYQ_E_SHAPE, "moe_ep_return: hidden %d, cap %d", hidden, cap);
  hyq::XchgArgs a;
  int rc = hyq::xchg_setup(regions, rank, world, region_data_bytes, slot_floats, (int64_t)cap * hidden,
                           "moe_ep_return", a);
  if (rc) return rc;
  a.mode = 2;
  a.send = y;
  a.src_rows = world * cap;
  a.gather = inv;
  a.valid = back_rows;
  a.rows = cap;
  a.row_floats = hidden;
  return hyq::xchg_launch(a, stream, "moe_ep_return");
}

int hyq_moe_ep_home(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                    int hidden, const int32_t* off, int experts_per_rank, int cap, float* out, void* stream) {
  if (!off || !out) return hyq::api_fail(HYQ_E_INVALID, "moe_ep_home: null argument");
  if (hidden < 1 || cap < 1 || experts_per_rank < 1)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_ep_home: hidden %d, cap %d, %d experts per rank", hidden, cap,
                         experts_per_rank);
  hyq::XchgArgs x;
  int rc = hyq::xchg_setup(regions, rank, world, region_data_bytes, slot_floats, (int64_t)cap * hidden,
                           "moe_ep_home", x);
  if (rc) return rc;
  hyq::HomeArgs a{};
  a.data = reinterpret_cast<const float*>(regions[rank] + HYQ_PEER_DATA_OFFSET);
  a.off = off;
  a.world = world;
  a.el = experts_per_rank;
  a.cap = cap;
  a.hidden = hidden;
  a.slot = slot_floats;
  a.out = out;
  hyq::moe_ep_home_kernel<<<dim3((unsigned)(cap < 64 ? cap : 64), (unsigned)world), 512, 0, (cudaStream_t)stream>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_ep_home: %s", cudaGetErrorString(e));
}

}  // extern "C"
