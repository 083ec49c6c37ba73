/*
 * hyq_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the block-quantized CPU kernels of hy-mt-rs
 * (src/quant.rs), used as the parity checker for the CUDA library and as the
 * timed CPU baseline.  Nothing in the product links or calls this file: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg
 * load it.  The reference itself is Rust and cannot be compiled here (no
 * cargo/rustc), so this restatement stands in for it; it is pinned against
 * the reference's own golden decoder vectors (tests/fixtures/quant.json of the
 * reference, copied to tests/golden/quant.json).
 *
 * Two accumulation orders are restated exactly:
 *   - the x86_64 path (f32 activations; AVX2 `dot` with two 8-lane FMA
 *     accumulators, quant.rs:2562-2596), which is what the reference runs on
 *     the B200 host; and
 *   - the aarch64 SDOT path (int8 activations; per-lane int32 sums and
 *     lane-wise f32 FMA, quant.rs:1493-1561, 1877-1959, 2241-2335).
 * Build with -ffp-contract=off: Rust never contracts a*b+c, and every fused
 * operation of the reference (FMA intrinsics) is written here as fmaf().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* DType order of quant.rs:19-27. */
enum { T_F32 = 0, T_F16 = 1, T_Q4_K = 2, T_Q6_K = 3, T_Q8_0 = 4, T_Q2_0C = 5, T_STQ1_0 = 6 };

/* quant.rs:43-50 */
int hyo_block_len(int t) {
  switch (t) {
    case T_F32: case T_F16: return 1;
    case T_Q8_0: return 32;
    case T_Q2_0C: return 512;
    case T_Q4_K: case T_Q6_K: case T_STQ1_0: return 256;
    default: return 0;
  }
}

/* quant.rs:52-62 */
int hyo_block_bytes(int t) {
  switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    case T_Q8_0: return 34;
    case T_Q2_0C: return 130;
    case T_STQ1_0: return 42;
    default: return 0;
  }
}

/* DType::from_id (quant.rs:30-41). profile: 1 standard, 2 tencent-q2-0c,
 * 3 tencent-stq1.  Returns -1 for an unsupported id/profile pair. */
int hyo_dtype_from_id(uint32_t id, int profile) {
  switch (id) {
    case 0: return T_F32;
    case 1: return T_F16;
    case 8: return T_Q8_0;
    case 12: return T_Q4_K;
    case 14: return T_Q6_K;
    case 40: return profile == 2 ? T_Q2_0C : -1;
    case 42: return profile == 3 ? T_STQ1_0 : -1;
    default: return -1;
  }
}

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary16 -> f32 as the `half` crate 2.x does it (exact for every
 * finite value; NaNs are quieted with their payload kept).  quant.rs:845-847. */
float hyo_half(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ffu;
  if ((h & 0x7fffu) == 0) return bits_f32(sign);
  if (exp == 0x1f) {
    if (man == 0) return bits_f32(sign | 0x7f800000u);
    return bits_f32(sign | 0x7fc00000u | (man << 13));
  }
  if (exp == 0) {
    /* subnormal: renormalise */
    int e = 0;
    while (!(man & 0x400u)) { man <<= 1; ++e; }
    man &= 0x3ffu;
    return bits_f32(sign | ((uint32_t)(127 - 15 - e + 1) << 23) | (man << 13));
  }
  return bits_f32(sign | ((exp + 127 - 15) << 23) | (man << 13));
}

static inline float half_at(const uint8_t* p) { return hyo_half((uint16_t)(p[0] | (p[1] << 8))); }

/* Format table of the Tencent STQ1_0 codebook (quant.rs:1081-1084). */
static const uint8_t STQ_CODEBOOK[32] = {
  0xa9, 0x89, 0x29, 0x09, 0xa6, 0x86, 0x26, 0x06, 0x9a, 0x92, 0x1a, 0x12, 0x6a, 0x62, 0x4a, 0x42,
  0x01, 0x21, 0x81, 0xa1, 0x04, 0x24, 0x84, 0xa4, 0x10, 0x18, 0x90, 0x98, 0x40, 0x48, 0x60, 0x68,
};

/* stq_digits_scalar (quant.rs:1103-1123): group g lane p -> output
 * (g/16)*64 + g%16 + 16p, value ((cb >> 2p) & 3) - 1, times `scale`. */
static void stq_digits(const uint8_t* b, float scale, float* out) {
  for (int g = 0; g < 64; ++g) {
    uint8_t code = (b[g >> 1] >> (4 * (g & 1))) & 15;
    uint8_t sign = (b[32 + (g >> 3)] >> (g & 7)) & 1;
    uint8_t cb = STQ_CODEBOOK[(sign << 4) | code];
    for (int p = 0; p < 4; ++p)
      out[(g / 16) * 64 + (g % 16) + 16 * p] = (float)((int)((cb >> (2 * p)) & 3) - 1) * scale;
  }
}

/* decode_unchecked (quant.rs:2405-2486), x86 branches.  Every product is a
 * separate f32 rounding (no FMA), as in Rust. */
static void decode_block(int t, const uint8_t* x, float* y) {
  switch (t) {
    case T_F32: { uint32_t u; memcpy(&u, x, 4); y[0] = bits_f32(u); break; }
    case T_F16: y[0] = half_at(x); break;
    case T_Q8_0: {
      float d = half_at(x);
      for (int i = 0; i < 32; ++i) y[i] = d * (float)(int8_t)x[2 + i];
      break;
    }
    case T_Q2_0C: {
      float d = half_at(x);
      for (int i = 0; i < 512; ++i)
        y[i] = (float)(2 * (int)((x[2 + i / 4] >> (2 * (i % 4))) & 3) - 3) * d;
      break;
    }
    case T_STQ1_0: stq_digits(x, half_at(x + 40), y); break;
    case T_Q4_K: {
      float d = half_at(x), dmin = half_at(x + 2);
      const uint8_t* sc = x + 4;
      for (int group = 0; group < 4; ++group) {
        float dm[2][2];
        for (int h = 0; h < 2; ++h) {
          int j = group * 2 + h;
          uint8_t s, m;
          if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
          else {
            s = (uint8_t)((sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4));
            m = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
          }
          dm[h][0] = d * (float)s;
          dm[h][1] = dmin * (float)m;
        }
        for (int l = 0; l < 32; ++l) {
          uint8_t q = x[16 + group * 32 + l];
          y[group * 64 + l] = dm[0][0] * (float)(q & 15) - dm[0][1];
          y[group * 64 + 32 + l] = dm[1][0] * (float)(q >> 4) - dm[1][1];
        }
      }
      break;
    }
    case T_Q6_K: {
      float d = half_at(x + 208);
      for (int chunk = 0; chunk < 2; ++chunk) {
        const uint8_t* ql = x + chunk * 64;
        const uint8_t* qh = x + 128 + chunk * 32;
        const uint8_t* sc = x + 192 + chunk * 8;
        for (int p = 0; p < 4; ++p) {
          int nib = (p >> 1) * 4, bits = 2 * p;
          for (int half = 0; half < 2; ++half) {
            float s = d * (float)(int8_t)sc[2 * p + half];
            for (int i = 0; i < 16; ++i) {
              uint8_t qv = ql[half * 16 + (p & 1) * 32 + i], hv = qh[half * 16 + i];
              int q = ((qv >> nib) & 15) | (((hv >> bits) & 3) << 4);
              y[chunk * 128 + p * 32 + half * 16 + i] = s * (float)(q - 32);
            }
          }
        }
      }
      break;
    }
  }
}

/* decode (quant.rs:1066-1079): 0 on success, -1 on a partial block or a
 * byte count that does not match. */
int hyo_decode(int t, const uint8_t* bytes, size_t nbytes, float* out, size_t nout) {
  int bl = hyo_block_len(t), bb = hyo_block_bytes(t);
  if (!bl) return -1;
  if (nout % (size_t)bl) return -1;
  if (nbytes != nout / bl * bb) return -1;
  size_t blocks = nout / bl;
  for (size_t i = 0; i < blocks; ++i) decode_block(t, bytes + i * bb, out + i * bl);
  return 0;
}

/* dot_scalar (quant.rs:2518-2520): sequential sum of a*b from -0.0. */
float hyo_dot_scalar(const float* a, const float* b, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* dot_avx2 (quant.rs:2562-2596): two 8-lane FMA accumulators over 16-wide
 * chunks, an 8-wide tail into their sum, a sequential lane sum, then the
 * scalar tail. */
float hyo_dot(const float* a, const float* b, size_t n) {
  float s0[8] = {0}, s1[8] = {0}, sum[8];
  size_t chunks = n / 16;
  for (size_t c = 0; c < chunks; ++c) {
    const float* pa = a + c * 16; const float* pb = b + c * 16;
    for (int l = 0; l < 8; ++l) {
      s0[l] = fmaf(pa[l], pb[l], s0[l]);
      s1[l] = fmaf(pa[8 + l], pb[8 + l], s1[l]);
    }
  }
  for (int l = 0; l < 8; ++l) sum[l] = s0[l] + s1[l];
  size_t simd_end = chunks * 16, vec_end = n / 8 * 8;
  for (size_t i = simd_end; i < vec_end; i += 8)
    for (int l = 0; l < 8; ++l) sum[l] = fmaf(a[i + l], b[i + l], sum[l]);
  float lanes = -0.0f;
  for (int l = 0; l < 8; ++l) lanes += sum[l];
  return lanes + hyo_dot_scalar(a + vec_end, b + vec_end, n - vec_end);
}

static inline size_t row_bytes_of(int t, int64_t K) {
  return (size_t)(K / hyo_block_len(t)) * (size_t)hyo_block_bytes(t);
}

/* One packed row against f32 activations, x86 batch-1 path of
 * Weight::matmul (quant.rs:179-268):
 *   STQ1_0: stq_row_dot  (quant.rs:1264-1280; stq_dot :1248-1262)
 *   Q6_K:   q6_row_dot   (quant.rs:1728-1743; q6_dot :1712-1726)
 *   Q2_0C:  q2c_row_dot  (quant.rs:2169-2188, scalar)
 *   F32/F16: whole-row decode + dot (quant.rs:225-238)
 *   Q4_K/Q8_0: per-block decode + dot, summed (quant.rs:239-266). */
float hyo_row_dot_f32(int t, const uint8_t* row, const float* x, int64_t K) {
  int bl = hyo_block_len(t), bb = hyo_block_bytes(t);
  int64_t nb = K / bl;
  switch (t) {
    case T_STQ1_0: {
      float sum = 0.0f, digits[256];
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 42;
        float d = half_at(blk + 40);
        stq_digits(blk, 1.0f, digits);
        sum += d * hyo_dot(digits, x + b * 256, 256);
      }
      return sum;
    }
    case T_Q6_K: {
      float sum = 0.0f, dec[256];
      for (int64_t b = 0; b < nb; ++b) {
        decode_block(T_Q6_K, row + b * 210, dec);
        sum += hyo_dot(dec, x + b * 256, 256);
      }
      return sum;
    }
    case T_Q2_0C: {
      float sum = 0.0f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * 130;
        float d = half_at(blk);
        const float* xs = x + b * 512;
        for (int i = 0; i < 512; ++i) {
          float w = (float)(2 * (int)((blk[2 + i / 4] >> (2 * (i % 4))) & 3) - 3);
          sum += d * w * xs[i];
        }
      }
      return sum;
    }
    case T_F32: case T_F16: {
      float* v = (float*)malloc(sizeof(float) * (size_t)K);
      for (int64_t i = 0; i < K; ++i) decode_block(t, row + i * bb, v + i);
      float r = hyo_dot(v, x, (size_t)K);
      free(v);
      return r;
    }
    default: {
      float sum = 0.0f, scratch[512];
      for (int64_t b = 0; b < nb; ++b) {
        decode_block(t, row + b * bb, scratch);
        sum += hyo_dot(scratch, x + b * bl, (size_t)bl);
      }
      return sum;
    }
  }
}

/* Weight::matmul (quant.rs:159-344), x86 order, output [batch, rows].
 *   batch == 1: hyo_row_dot_f32 per row.
 *   2 <= batch < 8: whole-row decode, then dot per batch item (quant.rs:312-336).
 *   batch >= 8: the reference decodes 64-row tiles and multiplies them with
 *     Candle's CPU GEMM (gemm 0.19.0, not in the reference tree).  That GEMM's
 *     summation order is not restated: this oracle accumulates each output in
 *     f64 and rounds once (parity for this branch is tolerance-based).
 * threads <= 0 uses the OpenMP default. */
void hyo_matmul(int t, const uint8_t* w, int64_t K, int64_t N, const float* x, int64_t batch,
                float* y, int threads) {
  size_t rb = row_bytes_of(t, K);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  if (batch == 1) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r) y[r] = hyo_row_dot_f32(t, w + r * rb, x, K);
    return;
  }
  if (batch < 8) {
#pragma omp parallel
    {
      float* v = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
      for (int64_t r = 0; r < N; ++r) {
        hyo_decode(t, w + r * rb, rb, v, (size_t)K);
        for (int64_t b = 0; b < batch; ++b) y[b * N + r] = hyo_dot(v, x + b * K, (size_t)K);
      }
      free(v);
    }
    return;
  }
#pragma omp parallel
  {
    float* v = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < N; ++r) {
      hyo_decode(t, w + r * rb, rb, v, (size_t)K);
      for (int64_t b = 0; b < batch; ++b) {
        const float* xb = x + b * K;
        double acc = 0.0;
        for (int64_t i = 0; i < K; ++i) acc += (double)v[i] * (double)xb[i];
        y[b * N + r] = (float)acc;
      }
    }
    free(v);
  }
}

/* The decode half of the batch >= 8 branch of Weight::matmul
 * (quant.rs:280-296): rows decoded to f32 (decode_unchecked per row) in
 * parallel, out[r * K ..] = row r.  The benchmark's CPU arm multiplies the
 * result with a BLAS f32 GEMM in place of Candle's. */
void hyo_decode_rows(int t, const uint8_t* w, int64_t K, int64_t N, float* out, int threads) {
  size_t rb = row_bytes_of(t, K);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r) hyo_decode(t, w + r * rb, rb, out + r * K, (size_t)K);
}

/* SiLU gate as written at quant.rs:573-574 (and every other arm). */
static inline float silu_mul(float g, float u) {
  float silu = g / (1.0f + expf(-g));
  return silu * u;
}

/* matmul_gate_up_silu (quant.rs:724-841), x86 order. */
void hyo_gate_up_silu(int t, const uint8_t* gate, const uint8_t* up, int64_t K, int64_t N,
                      const float* x, float* y, int threads) {
  size_t rb = row_bytes_of(t, K);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r) {
    float g = hyo_row_dot_f32(t, gate + r * rb, x, K);
    float u = hyo_row_dot_f32(t, up + r * rb, x, K);
    y[r] = silu_mul(g, u);
  }
}

/* ---------------------------------------------------------------------- */
/* int8 activations (aarch64 reference path)                               */
/* ---------------------------------------------------------------------- */

static inline float rust_max(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a > b ? a : b;
}

/* NEON fmax semantics: NaN in either operand gives NaN. */
static inline float neon_max(float a, float b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}

static inline int8_t sat_i8_from_rne(float v) {
  /* vcvtnq_s32_f32 (round to nearest even, NaN -> 0, saturating), then
   * vqmovn_s32 and vqmovn_s16: net saturation to [-128, 127]. */
  if (isnan(v)) return 0;
  float r = nearbyintf(v); /* default rounding mode: nearest even */
  if (r > 127.0f) return 127;
  if (r < -128.0f) return -128;
  return (int8_t)r;
}

/* Q8::quantize_into (quant.rs:904-922) with max_abs_neon (:869-892),
 * quantize_group_neon (:967-991) and deinterleave_q2c (:945-963).
 * values/values_q2c: len int8; scales: ceil(len/256) f32. */
void hyo_q8_quantize(const float* input, int64_t len, int8_t* values, float* scales,
                     int8_t* values_q2c) {
  for (int64_t g0 = 0, gi = 0; g0 < len; g0 += 256, ++gi) {
    int64_t n = len - g0 < 256 ? len - g0 : 256;
    const float* src = input + g0;
    int64_t chunks = n / 16;
    float m = 0.0f;
    for (int64_t i = 0; i < chunks * 16; ++i) m = neon_max(m, fabsf(src[i]));
    for (int64_t i = chunks * 16; i < n; ++i) m = rust_max(m, fabsf(src[i]));
    float scale = 0.0f, inverse = 0.0f;
    if (m > 0.0f) { scale = m / 127.0f; inverse = 127.0f / m; }
    scales[gi] = scale;
    int64_t i = 0;
    for (; i + 16 <= n; ++i) values[g0 + i] = sat_i8_from_rne(src[i] * inverse);
    for (; i < n; ++i) {
      float v = roundf(src[i] * inverse);
      if (isnan(v)) { values[g0 + i] = 0; continue; }
      if (v > 127.0f) v = 127.0f;
      if (v < -127.0f) v = -127.0f;
      values[g0 + i] = (int8_t)v;
    }
  }
  if (values_q2c) {
    int64_t i = 0;
    for (; i + 64 <= len; i += 64)
      for (int k = 0; k < 4; ++k)
        for (int j = 0; j < 16; ++j) values_q2c[i + 16 * k + j] = values[i + 4 * j + k];
    for (; i < len; ++i) values_q2c[i] = values[i];
  }
}

/* sdot lane i += sum_{b<4} a[4i+b] * d[4i+b] over one 16-byte vector. */
static inline void sdot16(int32_t acc[4], const int8_t* a, const int8_t* d) {
  for (int i = 0; i < 4; ++i)
    for (int b = 0; b < 4; ++b) acc[i] += (int32_t)a[4 * i + b] * (int32_t)d[4 * i + b];
}

/* vaddvq_f32: pairwise (a0+a1)+(a2+a3). */
static inline float addv4(const float v[4]) { return (v[0] + v[1]) + (v[2] + v[3]); }

/* stq_row_dot_sdot (quant.rs:1493-1561). */
static float stq_row_dot_q8(const uint8_t* row, int64_t K, const int8_t* xq, const float* xs) {
  float row_acc[4] = {0, 0, 0, 0};
  int64_t nb = K / 256;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * 42;
    float block_scale = half_at(blk + 40) * xs[b];
    int32_t acc[4] = {0, 0, 0, 0};
    const int8_t* xp = xq + b * 256;
    for (int c = 0; c < 4; ++c) {
      int8_t planes[4][16];
      for (int j = 0; j < 16; ++j) {
        int g = c * 16 + j;
        uint8_t code = (blk[g >> 1] >> (4 * (g & 1))) & 15;
        uint8_t sign = (blk[32 + (g >> 3)] >> (g & 7)) & 1;
        uint8_t cb = STQ_CODEBOOK[(sign << 4) | code];
        for (int p = 0; p < 4; ++p) planes[p][j] = (int8_t)(((cb >> (2 * p)) & 3) - 1);
      }
      for (int p = 0; p < 4; ++p) sdot16(acc, xp + c * 64 + 16 * p, planes[p]);
    }
    for (int i = 0; i < 4; ++i) row_acc[i] = fmaf((float)acc[i], block_scale, row_acc[i]);
  }
  return addv4(row_acc);
}

/* q6_row_dot_sdot (quant.rs:2241-2335). */
static float q6_row_dot_q8(const uint8_t* row, int64_t K, const int8_t* xq, const float* xs) {
  float r0[4] = {0, 0, 0, 0}, r1[4] = {0, 0, 0, 0};
  int64_t nb = K / 256;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * 210;
    float d = half_at(blk + 208) * xs[b];
    const int8_t* xp = xq + b * 256;
    for (int c = 0; c < 2; ++c) {
      const uint8_t* ql = blk + c * 64;
      const uint8_t* qh = blk + 128 + c * 32;
      const uint8_t* sc = blk + 192 + c * 8;
      for (int p = 0; p < 4; ++p) {
        for (int h = 0; h < 2; ++h) {
          int8_t dig[16];
          for (int i = 0; i < 16; ++i) {
            uint8_t qv = ql[(p & 1) * 32 + h * 16 + i], hv = qh[h * 16 + i];
            int q = ((qv >> ((p >> 1) * 4)) & 15) | (((hv >> (2 * p)) & 3) << 4);
            dig[i] = (int8_t)(q - 32);
          }
          int32_t acc[4] = {0, 0, 0, 0};
          sdot16(acc, xp + c * 128 + p * 32 + h * 16, dig);
          float plane = d * (float)(int8_t)sc[2 * p + h];
          float* ra = h ? r1 : r0;
          for (int i = 0; i < 4; ++i) ra[i] = fmaf((float)acc[i], plane, ra[i]);
        }
      }
    }
  }
  float s[4];
  for (int i = 0; i < 4; ++i) s[i] = r0[i] + r1[i];
  return addv4(s);
}

/* q2c_row_dot_sdot (quant.rs:1877-1959) on de-interleaved activations; the
 * dual-row kernel (:1961-2118) gives each row the same result. */
static float q2c_row_dot_q8(const uint8_t* row, int64_t K, const int8_t* xq2c, const float* xs) {
  float row_acc[4] = {0, 0, 0, 0};
  int64_t nb = K / 512;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = row + b * 130;
    float d = half_at(blk);
    const uint8_t* payload = blk + 2;
    const int8_t* xp = xq2c + b * 512;
    for (int h = 0; h < 2; ++h) {
      float scale = d * xs[2 * b + h];
      int32_t acc[4] = {0, 0, 0, 0};
      for (int c = 0; c < 4; ++c) {
        const uint8_t* raw = payload + 64 * h + 16 * c;
        for (int k = 0; k < 4; ++k) {
          int8_t v[16];
          for (int j = 0; j < 16; ++j) v[j] = (int8_t)(2 * ((raw[j] >> (2 * k)) & 3) - 3);
          sdot16(acc, xp + 256 * h + 64 * c + 16 * k, v);
        }
      }
      for (int i = 0; i < 4; ++i) row_acc[i] = fmaf((float)acc[i], scale, row_acc[i]);
    }
  }
  return addv4(row_acc);
}

/* One packed row against Q8 activations.  STQ1_0 / Q6_K / Q2_0C follow the
 * reference's SDOT kernels (row_dot_q8_raw, quant.rs:2219-2233).  Q4_K, Q8_0,
 * F16 and F32 have no int8 kernel in the reference: for them this returns
 * sum_i decode(w)_i * (q_i * s_g) accumulated in f64 and rounded once. */
float hyo_row_dot_q8(int t, const uint8_t* row, int64_t K, const int8_t* values,
                     const float* scales, const int8_t* values_q2c) {
  switch (t) {
    case T_STQ1_0: return stq_row_dot_q8(row, K, values, scales);
    case T_Q6_K: return q6_row_dot_q8(row, K, values, scales);
    case T_Q2_0C: return q2c_row_dot_q8(row, K, values_q2c, scales);
    default: {
      float* v = (float*)malloc(sizeof(float) * (size_t)K);
      hyo_decode(t, row, row_bytes_of(t, K), v, (size_t)K);
      double acc = 0.0;
      for (int64_t i = 0; i < K; ++i)
        acc += (double)v[i] * ((double)values[i] * (double)scales[i / 256]);
      free(v);
      return (float)acc;
    }
  }
}

/* gemv_q8_fast (quant.rs:353-380) over all rows. */
void hyo_gemv_q8(int t, const uint8_t* w, int64_t K, int64_t N, const int8_t* values,
                 const float* scales, const int8_t* values_q2c, float* y, int threads) {
  size_t rb = row_bytes_of(t, K);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r) y[r] = hyo_row_dot_q8(t, w + r * rb, K, values, scales, values_q2c);
}

/* matmul_gate_up_silu_fast (quant.rs:540-651). */
void hyo_gate_up_silu_q8(int t, const uint8_t* gate, const uint8_t* up, int64_t K, int64_t N,
                         const int8_t* values, const float* scales, const int8_t* values_q2c,
                         float* y, int threads) {
  size_t rb = row_bytes_of(t, K);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < N; ++r) {
    float g = hyo_row_dot_q8(t, gate + r * rb, K, values, scales, values_q2c);
    float u = hyo_row_dot_q8(t, up + r * rb, K, values, scales, values_q2c);
    y[r] = silu_mul(g, u);
  }
}

int hyo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------------------
 * Dense decoder step primitives (x86 branches of src/model.rs), for the
 * full-model decode parity test.  No golden vectors exist for these (the
 * reference's logits fixtures need its real GGUF files): parity unpinned.
 * ------------------------------------------------------------------------ */

/* rms_norm_into (model.rs:785-830, x86 loop :827-829):
 * variance = dot(x, x) / n; scale = recip(sqrt(variance + eps));
 * out = (x * scale) * w. */
void hyo_rms_norm(const float* x, const float* w, int64_t n, float eps, float* out) {
  const float variance = hyo_dot(x, x, (size_t)n) / (float)n;
  const float scale = 1.0f / sqrtf(variance + eps);
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* rms_norm over rows of width `dim` in place (model.rs:832-872): the
 * per-head q/k norm of the Dense architecture (model.rs:443-446). */
void hyo_rms_norm_rows(float* v, int64_t rows, const float* w, int64_t dim, float eps) {
  for (int64_t r = 0; r < rows; ++r) hyo_rms_norm(v + r * dim, w, dim, eps, v + r * dim);
}

/* Rotary table for one position (model.rs:378-391): (pos * freq).sin_cos()
 * with freq_j = rope_base.powf(-2 j / head_dim) (model.rs:266-272). */
void hyo_rope_table(int64_t pos, int head_dim, float rope_base, float* cos_out, float* sin_out) {
  for (int j = 0; j < head_dim / 2; ++j) {
    const float freq = powf(rope_base, -2.0f * (float)j / (float)head_dim);
    const float a = (float)pos * freq;
    sin_out[j] = sinf(a);
    cos_out[j] = cosf(a);
  }
}

/* rope_with_cache (model.rs:874-913, x86 loop :907-912), per head of `dim`. */
void hyo_rope(float* v, int64_t heads, int64_t dim, const float* cos_s, const float* sin_s) {
  const int64_t half = dim / 2;
  for (int64_t h = 0; h < heads; ++h) {
    float* head = v + h * dim;
    for (int64_t j = 0; j < half; ++j) {
      const float a = head[j], b = head[j + half];
      head[j] = a * cos_s[j] - b * sin_s[j];
      head[j + half] = a * sin_s[j] + b * cos_s[j];
    }
  }
}

/* attention_into for one query token (model.rs:949-1021, x86 branch):
 * keys/values hold `past + 1` positions of kv_heads * dim floats. */
void hyo_attention(const float* q, const float* keys, const float* values, int heads, int kv_heads, int dim,
                   int64_t past, float* out) {
  const int64_t kv_width = (int64_t)kv_heads * dim;
  const int repeats = heads / kv_heads;
  const float scale = 1.0f / sqrtf((float)dim);
  const int64_t visible = past + 1;
  float* scores = (float*)malloc(sizeof(float) * (size_t)visible);
  for (int h = 0; h < heads; ++h) {
    const int kvh = h / repeats;
    const float* query = q + (int64_t)h * dim;
    float* o = out + (int64_t)h * dim;
    for (int d = 0; d < dim; ++d) o[d] = 0.0f;
    for (int64_t pos = 0; pos < visible; ++pos)
      scores[pos] = hyo_dot(query, keys + pos * kv_width + (int64_t)kvh * dim, (size_t)dim) * scale;
    float max = -INFINITY;
    for (int64_t pos = 0; pos < visible; ++pos) max = fmaxf(max, scores[pos]);
    float sum = 0.0f;
    for (int64_t pos = 0; pos < visible; ++pos) {
      scores[pos] = expf(scores[pos] - max);
      sum += scores[pos];
    }
    const float inv_sum = 1.0f / sum;
    for (int64_t pos = 0; pos < visible; ++pos) {
      const float p = scores[pos] * inv_sum;
      const float* val = values + pos * kv_width + (int64_t)kvh * dim;
      for (int d = 0; d < dim; ++d) o[d] += p * val[d];
    }
  }
  free(scores);
}

/* route (model.rs:728-767) for one token: sigmoid with the reference's two
 * branches; indices ordered by sigmoid + bias descending under
 * f32::total_cmp (ties: lower index first); the first `used` kept; weights
 * sigmoid / max(sum of the kept sigmoids in that order, f16 MIN_POSITIVE) *
 * scale when normalize, else sigmoid / 1 * scale. */
static int32_t hyo_total_key(float v) {
  int32_t b;
  memcpy(&b, &v, 4);
  return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

void hyo_moe_route(const float* logits, int experts, const float* bias, int used, int normalize, float scale,
                   int32_t* idx_out, float* w_out) {
  float* sig = (float*)malloc(sizeof(float) * (size_t)experts);
  int32_t* key = (int32_t*)malloc(sizeof(int32_t) * (size_t)experts);
  char* taken = (char*)calloc((size_t)experts, 1);
  for (int e = 0; e < experts; ++e) {
    const float x = logits[e];
    float s;
    if (x >= 0.0f) {
      s = 1.0f / (1.0f + expf(-x));
    } else {
      const float ev = expf(x);
      s = ev / (1.0f + ev);
    }
    sig[e] = s;
    key[e] = hyo_total_key(s + bias[e]);
  }
  float sum = 0.0f;
  for (int k = 0; k < used; ++k) {
    int best = -1;
    for (int e = 0; e < experts; ++e)
      if (!taken[e] && (best < 0 || key[e] > key[best])) best = e;  /* ties keep the lower index */
    taken[best] = 1;
    idx_out[k] = best;
    sum += sig[best];
  }
  const float min_pos = 6.103515625e-05f; /* half::f16::MIN_POSITIVE */
  if (!normalize) sum = 1.0f;
  else if (!(sum >= min_pos)) sum = min_pos; /* f32::max: a NaN sum gives the bound */
  for (int k = 0; k < used; ++k) w_out[k] = sig[idx_out[k]] / sum * scale;
  free(sig);
  free(key);
  free(taken);
}
