// Shared device helpers for the hyq kernels (sm_100a).
//
// Block geometry follows hy-mt-rs src/quant.rs:17-63 (DType, block_len,
// block_bytes).  Synchronisation uses mbarriers and bulk-async copies
// (cp.async.bulk, the TMA 1-D engine); every wait is bounded in time so that a
// lost completion turns into a status word the host can read instead of a hung
// GPU.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace hyq {

// DType order of quant.rs:19-27; the C ABI uses the same values.
enum DType : int { F32 = 0, F16 = 1, Q4_K = 2, Q6_K = 3, Q8_0 = 4, Q2_0C = 5, STQ1_0 = 6 };

__host__ __device__ constexpr int block_len(int t) {
  return (t == F32 || t == F16) ? 1 : (t == Q8_0 ? 32 : (t == Q2_0C ? 512 : 256));
}

__host__ __device__ constexpr int block_bytes(int t) {
  return t == F32 ? 4
       : t == F16 ? 2
       : t == Q4_K ? 144
       : t == Q6_K ? 210
       : t == Q8_0 ? 34
       : t == Q2_0C ? 130
       : t == STQ1_0 ? 42 : 0;
}

// Device status bits (OR-ed into a status word owned by the library).
enum : unsigned {
  DEV_TIMEOUT_FULL = 1u,   // consumer gave up waiting for a stage to land
  DEV_TIMEOUT_EMPTY = 2u,  // producer gave up waiting for a stage to drain
  DEV_TIMEOUT_DRAIN = 4u,  // exit path gave up waiting for copies in flight
  DEV_BAD_ARGS = 8u,       // kernel saw arguments the host should have rejected
  DEV_TIMEOUT_PEER = 16u,  // a peer all-reduce gave up waiting for another rank's flag
  DEV_TIMEOUT_GRID = 32u,  // a persistent kernel gave up waiting at a grid-wide barrier
};

// Bound on any single wait (nanoseconds of %globaltimer).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Suspend-time hint of a try_wait (ns): a waiting warp sleeps until the
// phase completes or this much time passes, instead of spinning and taking
// issue slots from the warps that do the work.  Bounded waits re-check their
// abort flag and time limit every 64 tries.
constexpr uint32_t kTryWaitSuspendNs = 1000000;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kTryWaitSuspendNs)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of an mbarrier, giving up after kWaitLimitNs or as
// soon as another thread of the CTA raised `*abort` (abort may be null: then
// only the time bound applies).  Returns false on give-up (the caller then
// records a status bit and leaves its loop).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

// Make prior generic-proxy accesses of shared memory ordered before later
// async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk-async copy global -> shared (16-byte aligned addresses, size a multiple
// of 16), completing `bytes` of transaction count on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// L2 policy for data read once per call (streamed weights): such lines go
// first when L2 needs room, so the weights do not push kernel code,
// parameters and activations out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// Exact IEEE binary16 -> f32 of the `half` crate (finite values are exact,
// NaNs are quieted with their payload).  Used where decode output bits matter.
__device__ __forceinline__ float half_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  if ((h & 0x7fffu) == 0) return __uint_as_float(sign);
  if (e == 0x1f) return __uint_as_float(m ? (sign | 0x7fc00000u | (m << 13)) : (sign | 0x7f800000u));
  if (e == 0) {
    const int lz = __clz(m) - 21;  // shifts that bring bit 10 up
    m = (m << lz) & 0x3ffu;
    return __uint_as_float(sign | ((uint32_t)(113 - lz) << 23) | (m << 13));
  }
  return __uint_as_float(sign | ((e + 112u) << 23) | (m << 13));
}

// Fast f16 -> f32 for scales inside dot products (hardware conversion; exact
// for every finite value).
__device__ __forceinline__ float half_to_f32(uint32_t h) {
  float f;
  asm("{ .reg .b16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
  return f;
}

// Little-endian loads of 16/32 bits from shared memory at a 2-byte aligned
// address.
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 2u) * 8u;
  return __funnelshift_r(w[0], w[1], sh);
}

// N consecutive 32-bit words starting at a 2-byte aligned shared address.
template <int N>
__device__ __forceinline__ void lds_words_a2(const uint8_t* p, uint32_t (&out)[N]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (uint32_t)(a & 2u) * 8u;
  uint32_t t[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) t[i] = w[i];
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(t[i], t[i + 1], sh);
}

__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  return __dp4a(a, b, (unsigned)c);
}

// unsigned bytes of a times signed bytes of b
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  return __dp4a((int)a, (int)b, c);
}

// All-reduce of a flag over the threads of named barrier `id` (`count`
// threads, a multiple of 32): true only if every participant passed true.
__device__ __forceinline__ bool bar_red_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Programmatic dependent launch.  `grid_dependency_wait` returns once every
// grid this one depends on has completed and its memory is visible (at once
// when the launch carried no programmatic dependency);
// `allow_dependents_launch` lets the next grid in the stream be scheduled
// before this one completes.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void bar_sync_named(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// dot_avx2's reduction of its two 8-lane accumulators (quant.rs:2562-2596)
// when n % 16 == 0: lane l of the 16-lane group [b, b + 16) holds
// accumulator lane l; every lane of the group returns the dot.
__device__ __forceinline__ float x86_lane_sum(float acc, unsigned mask) {
  const int lane = threadIdx.x & 31, l = lane & 15, base = lane & 16;
  const float sum = __fadd_rn(acc, __shfl_sync(mask, acc, base + ((l + 8) & 15)));
  float h = -0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) h = __fadd_rn(h, __shfl_sync(mask, sum, base + k));
  return __fadd_rn(h, -0.0f);
}

// dot_avx2 order (quant.rs:2562-2596: two 8-lane FMA accumulators per 16
// floats, their lane sums, a scalar tail) over n floats, by the 16 lanes
// [b, b + 16) of a warp (b = lane & 16), one per AVX2 accumulator lane.  Every lane of the group returns
// the result.  `mask` covers the calling lanes.
__device__ __forceinline__ float dot_x86(const float* a, const float* b, int n, unsigned mask) {
  const int lane = threadIdx.x & 31;
  const int l = lane & 15, base = lane & 16;
  const int chunks = n / 16;
  float acc = 0.f;
#pragma unroll 8
  for (int c = 0; c < chunks; ++c) acc = fmaf(a[16 * c + l], b[16 * c + l], acc);
  // sum[l] = s0[l] + s1[l] for l < 8
  float sum = __fadd_rn(acc, __shfl_sync(mask, acc, base + ((l + 8) & 15)));
  const int simd_end = chunks * 16, vec_end = n / 8 * 8;
  if (vec_end > simd_end && l < 8) sum = fmaf(a[simd_end + l], b[simd_end + l], sum);
  float h = -0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) h = __fadd_rn(h, __shfl_sync(mask, sum, base + k));
  float t = -0.0f;
  for (int i = vec_end; i < n; ++i) t = __fadd_rn(t, __fmul_rn(a[i], b[i]));
  return __fadd_rn(h, t);
}

// Asynchronous 16- and 4-byte copies global -> shared (cp.async), their
// commit groups and waits (this thread's copies).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The same dot_avx2 order (quant.rs:2562-2596) computed by one thread: the
// sixteen accumulator lanes are registers, followed by the same pairwise lane
// sums, horizontal sum and scalar tail as dot_x86.  a and b are 16-byte
// aligned when n % 4 == 0 (float4 loads).
__device__ __forceinline__ float dot_x86_thread(const float* a, const float* b, int n) {
  float acc[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) acc[l] = 0.f;
  const int chunks = n / 16;
  if ((n & 3) == 0) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll 2
    for (int c = 0; c < chunks; ++c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 x = a4[4 * c + j], y = b4[4 * c + j];
        acc[4 * j] = fmaf(x.x, y.x, acc[4 * j]);
        acc[4 * j + 1] = fmaf(x.y, y.y, acc[4 * j + 1]);
        acc[4 * j + 2] = fmaf(x.z, y.z, acc[4 * j + 2]);
        acc[4 * j + 3] = fmaf(x.w, y.w, acc[4 * j + 3]);
      }
    }
  } else {
    for (int c = 0; c < chunks; ++c) {
#pragma unroll
      for (int l = 0; l < 16; ++l) acc[l] = fmaf(a[16 * c + l], b[16 * c + l], acc[l]);
    }
  }
  float sum[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) sum[l] = __fadd_rn(acc[l], acc[l + 8]);
  const int simd_end = chunks * 16, vec_end = n / 8 * 8;
  if (vec_end > simd_end) {
#pragma unroll
    for (int l = 0; l < 8; ++l) sum[l] = fmaf(a[simd_end + l], b[simd_end + l], sum[l]);
  }
  float h = -0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) h = __fadd_rn(h, sum[k]);
  float t = -0.0f;
  for (int i = vec_end; i < n; ++i) t = __fadd_rn(t, __fmul_rn(a[i], b[i]));
  return __fadd_rn(h, t);
}

}  // namespace hyq
