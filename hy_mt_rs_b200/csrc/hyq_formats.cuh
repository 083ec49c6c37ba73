// Per-element decoders shared by the decode kernel and the fallback GEMV.
//
// Each returns weight `o` (0 <= o < block_len) of the block at `x`, with the
// operation order of hy-mt-rs src/quant.rs:2405-2486 (decode_unchecked):
// separate f32 roundings, no fused multiply-add.
#pragma once

#include "hyq_common.cuh"

namespace hyq {

// Tencent STQ1_0 codebook, a format table (quant.rs:1081-1084).  Internal
// linkage: every translation unit that includes this header gets its copy.
static __constant__ uint8_t kStqCodebook[32] = {
    0xa9, 0x89, 0x29, 0x09, 0xa6, 0x86, 0x26, 0x06, 0x9a, 0x92, 0x1a, 0x12, 0x6a, 0x62, 0x4a, 0x42,
    0x01, 0x21, 0x81, 0xa1, 0x04, 0x24, 0x84, 0xa4, 0x10, 0x18, 0x90, 0x98, 0x40, 0x48, 0x60, 0x68,
};

__device__ __forceinline__ uint32_t ld_u16_le(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

template <int T>
__device__ __forceinline__ float decode_elem(const uint8_t* __restrict__ x, int o) {
  if (T == F32) {
    return __uint_as_float(ld_u16_le(x) | (ld_u16_le(x + 2) << 16));
  } else if (T == F16) {
    return half_bits_to_f32(ld_u16_le(x));
  } else if (T == Q8_0) {
    return __fmul_rn(half_bits_to_f32(ld_u16_le(x)), (float)(int8_t)x[2 + o]);
  } else if (T == Q2_0C) {
    const int c = (x[2 + o / 4] >> (2 * (o % 4))) & 3;
    return __fmul_rn((float)(2 * c - 3), half_bits_to_f32(ld_u16_le(x)));
  } else if (T == STQ1_0) {
    const int chunk = o >> 6, r = o & 63, p = r >> 4, j = r & 15;
    const int g = chunk * 16 + j;
    const int code = (x[g >> 1] >> (4 * (g & 1))) & 15;
    const int sign = (x[32 + (g >> 3)] >> (g & 7)) & 1;
    const int cb = kStqCodebook[(sign << 4) | code];
    return __fmul_rn((float)(((cb >> (2 * p)) & 3) - 1), half_bits_to_f32(ld_u16_le(x + 40)));
  } else if (T == Q4_K) {
    const float d = half_bits_to_f32(ld_u16_le(x)), dmin = half_bits_to_f32(ld_u16_le(x + 2));
    const uint8_t* sc = x + 4;
    const int group = o >> 6, r = o & 63, h = r >> 5, l = r & 31;
    const int j = group * 2 + h;
    int s, m;
    if (j < 4) {
      s = sc[j] & 63;
      m = sc[j + 4] & 63;
    } else {
      s = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
      m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const int q = x[16 + group * 32 + l];
    const int nib = h ? (q >> 4) : (q & 15);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)nib), __fmul_rn(dmin, (float)m));
  } else {  // Q6_K
    const float d = half_bits_to_f32(ld_u16_le(x + 208));
    const int chunk = o >> 7, r = o & 127, p = r >> 5, half = (r >> 4) & 1, ii = r & 15;
    const int qv = x[chunk * 64 + half * 16 + (p & 1) * 32 + ii];
    const int hv = x[128 + chunk * 32 + half * 16 + ii];
    const int q = ((qv >> ((p >> 1) * 4)) & 15) | (((hv >> (2 * p)) & 3) << 4);
    const float s = __fmul_rn(d, (float)(int8_t)x[192 + chunk * 8 + 2 * p + half]);
    return __fmul_rn(s, (float)(q - 32));
  }
}

// STQ1_0 codebook (quant.rs:1081-1123) looked up for four groups at once:
// `hw` holds their four 4-bit nibble codes, `s4` their four sign bits; byte
// b of the result is the 4-digit pattern (2 bits per lane p, digit - 1 =
// weight / d) of group b.  The sign-1 half of the table is the digit-wise
// negation of the sign-0 half (entry 16 + n = 0xaa - entry n), so PRMT reads
// the 16 sign-0 entries from four register tables, a byte mask picks the half
// by nibble bit 3, and the sign swaps each digit d for 2 - d.
__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t stq_patterns4(uint32_t hw, uint32_t s4) {
  const uint32_t T0 = 0x092989a9u, T1 = 0x062686a6u, T2 = 0x121a929au, T3 = 0x424a626au;
  const uint32_t sel = hw & 0x7777u;
  const uint32_t p0 = prmt_b32(T0, T1, sel), p1 = prmt_b32(T2, T3, sel);
  const uint32_t m3 = prmt_b32(hw << 4, hw, 0xD9C8u);           // 0xff where nibble bit 3 is set
  const uint32_t sm = prmt_b32(s4 * 0x10204080u, 0u, 0xBA98u);  // 0xff where the sign bit is set
  const uint32_t cb = (p0 & ~m3) | (p1 & m3);
  return cb ^ (sm & (cb ^ (0xaaaaaaaau - cb)));
}

}  // namespace hyq
