// Bit-exact block decoders, the f32 dot, and int8 activation quantization.
//
// decode: hy-mt-rs src/quant.rs:1066-1079 (decode) and :2405-2486
// (decode_unchecked).  Every product/difference is rounded separately with
// __fmul_rn/__fsub_rn: the Rust code never fuses them, and the golden vectors
// pin the exact f32 bits.
//
// Q8 quantization: quant.rs:904-922 (Q8::quantize_into), :869-892
// (max_abs_neon), :967-991 (quantize_group_neon), :945-963 (deinterleave_q2c).
#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {

// One thread per output value: coalesced stores, block headers served by L1.
template <int T>
__global__ void __launch_bounds__(256) decode_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                                     int64_t n_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_out) return;
  constexpr int BL = block_len(T), BB = block_bytes(T);
  const int64_t b = i / BL;
  dst[i] = decode_elem<T>(src + b * BB, (int)(i - b * BL));
}

cudaError_t launch_decode(int dtype, const void* src, float* dst, int64_t n_out, cudaStream_t st) {
  if (n_out == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n_out + 255) / 256);
  const uint8_t* s = static_cast<const uint8_t*>(src);
  switch (dtype) {
    case F32: decode_kernel<F32><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case F16: decode_kernel<F16><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case Q4_K: decode_kernel<Q4_K><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case Q6_K: decode_kernel<Q6_K><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case Q8_0: decode_kernel<Q8_0><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case Q2_0C: decode_kernel<Q2_0C><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    case STQ1_0: decode_kernel<STQ1_0><<<grid, 256, 0, st>>>(s, dst, n_out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// f32 dot product (quant.rs:2500).  One CTA; deterministic tree order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) dot_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                   int64_t n, float* __restrict__ out) {
  __shared__ float part[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(a[i], b[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v;
  }
}

cudaError_t launch_dot(const float* a, const float* b, int64_t n, float* out, cudaStream_t st) {
  dot_kernel<<<1, 1024, 0, st>>>(a, b, n, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Q8 activation quantization, one CTA (256 threads) per 256-element group.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) q8_quantize_kernel(const float* __restrict__ x, int64_t len,
                                                          int8_t* __restrict__ values, float* __restrict__ scales,
                                                          int8_t* __restrict__ values_q2c) {
  __shared__ float red_max[8];
  __shared__ int red_nan[8];
  __shared__ float tail_max[8];
  __shared__ int8_t qv[256];
  const int64_t g0 = (int64_t)blockIdx.x * 256;
  const int n = (int)(len - g0 < 256 ? len - g0 : 256);
  const int t = threadIdx.x;
  const int simd_n = n / 16 * 16;  // vector part of quantize_group_neon / max_abs_neon
  const float v = t < n ? x[g0 + t] : 0.f;
  const float av = fabsf(v);
  // Vector part: NEON fmax propagates NaN.  Tail: Rust f32::max ignores it.
  float vm = (t < simd_n && !isnan(av)) ? av : 0.f;
  int vn = (t < simd_n && isnan(av)) ? 1 : 0;
  float tm = (t >= simd_n && t < n && !isnan(av)) ? av : -1.f;  // -1: "no value"
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, o));
    vn |= __shfl_xor_sync(0xffffffffu, vn, o);
    tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
  }
  if ((t & 31) == 0) {
    red_max[t >> 5] = vm;
    red_nan[t >> 5] = vn;
    tail_max[t >> 5] = tm;
  }
  __syncthreads();
  float m = 0.f, tmax = -1.f;
  int anynan = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    m = fmaxf(m, red_max[w]);
    anynan |= red_nan[w];
    tmax = fmaxf(tmax, tail_max[w]);
  }
  if (anynan) m = __int_as_float(0x7fc00000);
  if (tmax >= 0.f) m = isnan(m) ? tmax : fmaxf(m, tmax);  // tail folds over the vector result
  float scale = 0.f, inverse = 0.f;
  if (m > 0.f) {
    scale = __fdiv_rn(m, 127.f);
    inverse = __fdiv_rn(127.f, m);
  }
  if (t == 0) scales[blockIdx.x] = scale;
  if (t < n) {
    const float s = __fmul_rn(v, inverse);
    int q;
    if (t < simd_n) {
      // vcvtnq_s32_f32 then two saturating narrows: round-to-nearest-even,
      // NaN -> 0, clamp to [-128, 127].
      q = isnan(s) ? 0 : max(-128, min(127, __float2int_rn(s)));
    } else {
      float r = roundf(s);
      q = isnan(r) ? 0 : (int)fminf(127.f, fmaxf(-127.f, r));
    }
    values[g0 + t] = (int8_t)q;
    qv[t] = (int8_t)q;
  }
  __syncthreads();
  if (values_q2c && t < n) {
    // De-interleave within each full 64-element chunk: t[k*16+j] = s[4j+k].
    const int64_t gi = g0 + t;
    const int64_t chunk0 = gi / 64 * 64;
    int8_t out;
    if (chunk0 + 64 <= len) {
      const int r = (int)(gi - chunk0), k = r >> 4, j = r & 15;
      out = qv[(int)(chunk0 - g0) + 4 * j + k];
    } else {
      out = qv[t];
    }
    values_q2c[gi] = out;
  }
}

cudaError_t launch_q8_quantize(const float* x, int64_t len, int8_t* values, float* scales, int8_t* values_q2c,
                               cudaStream_t st) {
  if (len == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((len + 255) / 256);
  q8_quantize_kernel<<<grid, 256, 0, st>>>(x, len, values, scales, values_q2c);
  return cudaGetLastError();
}

}  // namespace hyq
