// Batch-1 matrix-vector products over packed GGUF rows (sm_100a): kernels.
// Included by one translation unit per packed format (hyq_gemv_<fmt>.cu).
//
// Reference behaviour (hy-mt-rs src/quant.rs):
//   Weight::matmul batch 1          :159-270   (f32 activations)
//   gemv_q8 (quantize + SDOT rows)  :346-380   (int8 activations)
//   gemv_q8_fast / compute_chunk_q8 :353-439
//   gemv_qkv(_fast)                 :441-538, :653-721
//   matmul_gate_up_silu(_fast)      :540-651, :723-841
//
// Engine.  Rows are streamed, never re-read: a persistent CTA per SM owns a
// ring of shared-memory stages; one producer thread fills each stage with a
// tile of consecutive packed rows using cp.async.bulk (one contiguous copy of
// the packed bytes, unchanged) and an mbarrier transaction count; 12 consumer
// warps decode the codes out of shared memory and reduce them against the
// activations.  The activations are prepared once per CTA into shared memory
// in the order the codes come out of each format's decoder, then every lane
// keeps the 64-column "units" it owns in registers for the CTA's lifetime.  A
// row is split over KS warps when K is too wide for one warp's registers or
// when splitting gives the grid enough row tiles.
//
// Arithmetic.  Codes are multiplied in the integer domain with dp4a:
//   XQ8 / XQ8F (NP=1): the reference's Q8 activations, given (gemv_q8_fast)
//     or computed in the CTA prologue from f32 input exactly as
//     Q8::quantize_into does (gemv_q8); per 256-column group the exact
//     integer sum is scaled by (weight scale * activation scale), as the SDOT
//     kernels do (quant.rs:1511-1557, 1891-1955, 2257-2332).
//   XF32 (NP=3): each f32 activation is written as a 24-bit integer X times
//     a power-of-two group scale 2^(e-22) (e = exponent of the 256-column
//     group's max |x|) and split exactly into three signed bytes.  Products
//     and sums are exact integers; the only roundings are |dX| <= 1/2 per
//     activation (2^(e-23) absolute) and the final f32 accumulation: f32-level
//     accuracy.
#pragma once

#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace gemv {

constexpr int kCW = 12;                    // consumer warps (13 warps: <= 128 registers)
constexpr int kThreads = (kCW + 1) * 32;   // + one producer warp
constexpr int kMaxStages = 32;
constexpr int kRedOffset = 528;            // partial sums: 2 copies x 12 warps x 4 rows x (gate, up)
constexpr int kHeaderBytes = 2048;         // barriers [0,512), abort flag, partial sums [528,1296), x barrier
constexpr int kXBarOffset = 1296;          // mbarrier of the activation copy
constexpr int kNormScaleOffset = 1312;     // the RMSNorm scale of the fused-norm form
constexpr int kNormMaxPerThread = 16;      // fused norm: K <= kNormMaxPerThread * kCW * 32
constexpr int kXStageMax = 32768;          // f32 activations up to this many bytes arrive by one bulk copy
constexpr int kConsumerBarrier = 15;       // named barrier of the 12 consumer warps

// Activation modes.
enum XMode : int { XF32 = 0, XQ8 = 1, XQ8F = 2 };

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t ld_s32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t ld_s16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ uint4 ld_s128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

// N consecutive 32-bit words at a 2-byte aligned shared address (reads one
// word past the span when the address is 4-byte aligned).
template <int N>
__device__ __forceinline__ void ld_s_words(uint32_t a, uint32_t (&out)[N]) {
  const uint32_t base = a & ~3u;
  const uint32_t sh = (a & 2u) * 8u;
  uint32_t t[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) t[i] = ld_s32(base + 4 * i);
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(t[i], t[i + 1], sh);
}

struct MatDev {
  const uint8_t* w;
  float* y;
  int64_t rows;
  int64_t batch_begin;
};

struct Params {
  MatDev mat[3];
  const uint8_t* up;
  int n_mat;
  int64_t total_batches;
  int K, U, row_bytes;
  int ks, rg, slice;   // K-split, row groups (rg*ks == kCW), units per slice
  int stages;
  int half_bytes;      // bytes of one row-tile buffer
  int stage_bytes;
  int x_off;           // shared-memory offset of the prepared activations
  int x_raw_off;       // shared-memory offset of the f32 activation copy (0: read x from global memory)
  int x_pad_off;       // shared-memory offset of its padded copy (65 floats per 64-column unit; 0: none)
  int stage_off;       // shared-memory offset of stage 0
  int xmode;
  const float* x;      // XF32 / XQ8F
  const int8_t* xq;    // XQ8
  const float* xs;     // XQ8
  // Fused forms (f32 activations staged in shared memory only): with norm_w
  // set, the staged x is replaced by RMSNorm(x) * norm_w before use
  // (rms_norm_into, model.rs:785-830); with residual set, every output adds
  // into y instead of replacing it (add, model.rs:1043-1071).
  const float* norm_w;
  float eps;
  int residual;
  unsigned* status;
};

// ---------------------------------------------------------------------------
// Unit geometry.  A unit is 64 columns that one lane owns; its columns are
// listed in "unit order" (two runs of 32), and code word j byte b of the
// decoded unit multiplies column rel(j, b) of that list.
// ---------------------------------------------------------------------------
template <int FMT>
__device__ __forceinline__ void unit_runs(int u, int& c0, int& c1) {
  if (FMT == Q6_K) {
    const int B = u >> 2, c = (u >> 1) & 1, pp = u & 1;
    c0 = B * 256 + c * 128 + pp * 32;  // plane pp of chunk c, then plane pp+2
    c1 = c0 + 64;
  } else {
    c0 = u * 64;
    c1 = c0 + 32;
  }
}

template <int FMT>
__host__ __device__ constexpr int rel(int j, int b) {
  return FMT == Q2_0C ? 16 * (j >> 2) + 4 * b + (j & 3)
       : FMT == STQ1_0 ? 16 * (j & 3) + 4 * (j >> 2) + b
       : 4 * j + b;
}

template <int FMT>
__device__ __forceinline__ int unit_col(int u, int r) {
  int c0, c1;
  unit_runs<FMT>(u, c0, c1);
  return r < 32 ? c0 + r : c1 + (r - 32);
}

template <int FMT>
__host__ __device__ constexpr int nseg() {
  return FMT == Q6_K ? 4 : ((FMT == Q4_K || FMT == Q8_0) ? 2 : 1);
}

template <int NP>
struct XUnit {
  uint32_t w[NP][16];
  int xsum[4];
  float sg;
};

struct WUnit {
  uint32_t c[16];
  float s[4];
  float m[2];
  int si[4];  // the same sub-block scales as integers (Q4_K: scale / min codes, Q6_K: int8 scales)
};

// ---------------------------------------------------------------------------
// Activation prologue: all consumer threads write the activations of every
// unit into shared memory as words[piece][j][u] (u fastest), plus one scale
// per 256-column group; each lane then loads its own units into registers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync %0, %1;" ::"r"(kConsumerBarrier), "r"(kCW * 32) : "memory");
}

template <int FMT, int NP>
__device__ void prepare_x(const Params& p, uint8_t* smem) {
  uint32_t* words = reinterpret_cast<uint32_t*>(smem + p.x_off);
  const int U = p.U, G = U >> 2;
  float* sg = reinterpret_cast<float*>(words + NP * 16 * U);
  float* gaux = sg + G;  // XF32: 2^(22-e); XQ8F: 127/max
  const int ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  // f32 activations come into shared memory with one bulk copy (after the
  // preceding grid has completed); the maxima and the words read them there.
  const float* xsrc = p.x;
  if (p.x_raw_off) {
    const uint32_t xbar = smem_addr(smem + kXBarOffset);
    float* raw = reinterpret_cast<float*>(smem + p.x_raw_off);
    const uint32_t bytes = (uint32_t)p.K * 4u;
    if (ctid == 0) {
      mbar_arrive_expect_tx(xbar, bytes);
      bulk_g2s(smem_addr(raw), p.x, bytes, xbar);
    }
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages);
    if (!mbar_wait(xbar, 0, abort_flag)) {
      if (ctid == 0) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
        *abort_flag = 1;
        // no copy may land after the CTA is gone
        if (!mbar_wait(xbar, 0, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
      }
    }
    xsrc = raw;
    if (p.norm_w) {
      // RMSNorm of the staged row, as the separate norm kernel computes it:
      // dot(x, x) in the x86 order (lane l of 16 accumulates columns l,
      // l + 16, ... in sequence; K % 16 == 0), scale = 1 / sqrt(d / K + eps),
      // x = (x * scale) * w.  The norm weights of this thread's columns load
      // while lanes 0-15 sum.
      float* scale_s = reinterpret_cast<float*>(smem + kNormScaleOffset);
      const int nt = kCW * 32, K = p.K;
      float wv[kNormMaxPerThread];
#pragma unroll
      for (int j = 0; j < kNormMaxPerThread; ++j) wv[j] = (ctid + j * nt < K) ? p.norm_w[ctid + j * nt] : 0.f;
      if (ctid < 16) {
        float acc = 0.f;
        for (int c0 = 0; c0 < K / 16; c0 += 16) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = raw[16 * (c0 + j) + ctid];
#pragma unroll
          for (int j = 0; j < 16; ++j) acc = fmaf(v[j], v[j], acc);
        }
        const float d = x86_lane_sum(acc, 0xffffu);
        if (ctid == 0) *scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)K), p.eps)));
      }
      consumers_sync();
      const float scale = *scale_s;
#pragma unroll
      for (int j = 0; j < kNormMaxPerThread; ++j) {
        const int i = ctid + j * nt;
        if (i < K) raw[i] = __fmul_rn(__fmul_rn(raw[i], scale), wv[j]);
      }
      consumers_sync();
    }
  }
  // The activation words read the four columns of a unit's code word, for
  // the units of consecutive lanes: in the staged copy those sit 64 floats
  // apart, one shared-memory bank.  The group-maxima pass therefore also
  // writes a copy with one float of padding per 64-column unit, where they
  // fall in consecutive banks.
  float* xpad = (p.x_pad_off && p.xmode != XQ8) ? reinterpret_cast<float*>(smem + p.x_pad_off) : nullptr;
  if (p.xmode == XQ8) {
    for (int g = ctid; g < G; g += kCW * 32) sg[g] = p.xs[g];
  } else {
    // Group maxima: one warp per 256-column group.
    for (int g = warp; g < G; g += kCW) {
      const float4* src = reinterpret_cast<const float4*>(xsrc + 256 * g);
      const float4 a = src[lane], b = src[32 + lane];
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      if (xpad) {
        const int c0 = 256 * g + 4 * lane, c1 = c0 + 128;  // column c -> c + c / 64
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xpad[c0 + (c0 >> 6) + e] = v[e];
          xpad[c1 + (c1 >> 6) + e] = v[4 + e];
        }
      }
      float m = 0.f;
      int bad = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float av = fabsf(v[i]);
        bad |= isnan(av) ? 1 : 0;
        bad |= (NP == 3 && isinf(av)) ? 1 : 0;
        m = fmaxf(m, av);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
      }
      if (lane == 0) {
        if (NP == 3) {
          // |x| <= m < 2^e: x * 2^(22-e) is an exact scaling below 2^22.
          int e = 0;
          frexpf(m, &e);
          if (bad) {
            sg[g] = __int_as_float(0x7fc00000);
            gaux[g] = 0.f;
          } else if (22 - e <= 127 && e - 22 >= -126) {
            sg[g] = __int_as_float((127 + e - 22) << 23);
            gaux[g] = __int_as_float((127 + 22 - e) << 23);
          } else {
            sg[g] = ldexpf(1.f, e - 22);
            gaux[g] = ldexpf(1.f, 22 - e);
          }
        } else {
          // Q8::quantize_into (quant.rs:904-922): a NaN in the group makes the
          // max NaN (NEON fmax), and then scale = inverse = 0.
          const float mm = bad ? __int_as_float(0x7fc00000) : m;
          float scale = 0.f, inverse = 0.f;
          if (mm > 0.f) {
            scale = __fdiv_rn(mm, 127.f);
            inverse = __fdiv_rn(127.f, mm);
          }
          sg[g] = scale;
          gaux[g] = inverse;
        }
      }
    }
    consumers_sync();
  }
  // Item (j, u) is word j of unit u, items u-fastest over the consumer
  // threads; (j, u) advance by increments (no division per item).  A signed
  // 24-bit X = p0 + 2^8 p1 + 2^16 p2 (signed bytes) has p0 = X mod 2^8 as a
  // byte, p1 = ((X + 2^7) >> 8) mod 2^8 and p2 = ((X + 2^7 + 2^15) >> 16).
  const float* xw = xpad ? xpad : xsrc;
  const int padsh = xpad ? 6 : 31;  // column c reads xw[c + (c >> padsh)]
  const int du = (kCW * 32) % U, dj = (kCW * 32) / U;
  for (int u = ctid % U, j = ctid / U; j < 16;) {
    if (p.xmode == XQ8) {
      uint32_t w0 = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) w0 |= ((uint32_t)(uint8_t)p.xq[unit_col<FMT>(u, rel<FMT>(j, b))]) << (8 * b);
      words[j * U + u] = w0;
    } else {
      const float sc = gaux[u >> 2];
      int X[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int col = unit_col<FMT>(u, rel<FMT>(j, b));
        const float xc = xw[col + (col >> padsh)];
        if (p.xmode == XQ8F) {
          // vcvtnq_s32_f32 + saturating narrows: nearest-even, NaN -> 0.
          const float q = __fmul_rn(xc, sc);
          X[b] = isnan(q) ? 0 : max(-128, min(127, __float2int_rn(q)));
        } else {
          X[b] = sc == 0.f ? 0 : __float2int_rn(xc * sc);
        }
      }
      words[j * U + u] = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
      if (NP == 3) {
#pragma unroll
        for (int b = 0; b < 4; ++b) X[b] = (X[b] + 128) >> 8;
        words[(16 + j) * U + u] =
            __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
        for (int b = 0; b < 4; ++b) X[b] = (X[b] + 128) >> 8;
        words[(32 + j) * U + u] =
            __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
      }
    }
    u += du;
    j += dj;
    if (u >= U) {
      u -= U;
      ++j;
    }
  }
  consumers_sync();
}

// One output row: stored, or (residual form) added to the row's value y_old.
__device__ __forceinline__ void emit_row(const Params& p, int m, int64_t row, float out, float y_old) {
  p.mat[m].y[row] = p.residual ? __fadd_rn(y_old, out) : out;
}

template <int FMT, int NP>
__device__ __forceinline__ void load_x(const Params& p, const uint8_t* smem, int u, bool valid, XUnit<NP>& xu) {
  const uint32_t* words = reinterpret_cast<const uint32_t*>(smem + p.x_off);
  const float* sg = reinterpret_cast<const float*>(words + NP * 16 * p.U);
  constexpr int NS = nseg<FMT>(), WPS = 16 / NS;
#pragma unroll
  for (int pc = 0; pc < NP; ++pc)
#pragma unroll
    for (int j = 0; j < 16; ++j) xu.w[pc][j] = valid ? words[(pc * 16 + j) * p.U + u] : 0u;
  xu.sg = valid ? sg[u >> 2] : 0.f;
#pragma unroll
  for (int s = 0; s < 4; ++s) xu.xsum[s] = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
    for (int j = s * WPS; j < (s + 1) * WPS; ++j) {
      a0 = __dp4a((int)xu.w[0][j], 0x01010101, a0);
      if (NP == 3) {
        a1 = __dp4a((int)xu.w[NP > 1 ? 1 : 0][j], 0x01010101, a1);
        a2 = __dp4a((int)xu.w[NP > 2 ? 2 : 0][j], 0x01010101, a2);
      }
    }
    xu.xsum[s] = NP == 3 ? a0 + (a1 << 8) + (a2 << 16) : a0;
  }
  // constants of combine() for the 2-bit and ternary formats
  if (FMT == Q2_0C || FMT == STQ1_0) {
    if (NP == 1) xu.xsum[0] *= FMT == Q2_0C ? 96 : 64;
    xu.sg *= FMT == Q2_0C ? (1.0f / 32.0f) : (1.0f / 64.0f);
  }
}

// ---------------------------------------------------------------------------
// Weight unit decode from shared memory.  `row` is the shared address of the
// row (2-byte aligned; Q4_K rows are 16-byte aligned).
// ---------------------------------------------------------------------------
template <int FMT>
__device__ __forceinline__ void decode_unit(uint32_t row, int u, WUnit& wu) {
  if (FMT == Q2_0C) {
    // quant.rs:2419-2432: 2-bit code c -> (2c - 3) * d, four codes per byte.
    const uint32_t blk = row + (u >> 3) * 130;
    wu.s[0] = half_to_f32(ld_s16(blk));
    uint32_t q[4];
    ld_s_words<4>(blk + 2 + 16 * (u & 7), q);
    // Plane k keeps its codes in place (c << 2k): seg_dot divides by 4^k.
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) wu.c[4 * i + k] = q[i] & (0x03030303u << (2 * k));
  } else if (FMT == STQ1_0) {
    // quant.rs:1103-1123: group g of chunk c: codebook[(sign << 4) | nibble],
    // lane p -> column 16p + (g % 16).  Four groups at a time: PRMT looks the
    // codebook up in registers, byte masks pick the half by nibble bit 3 and
    // by the sign bit.
    const uint32_t blk = row + (u >> 2) * 42;
    const int c = u & 3;
    wu.s[0] = half_to_f32(ld_s16(blk + 40));
    uint32_t nb[2];
    ld_s_words<2>(blk + 8 * c, nb);
    const uint32_t sbits = ld_s16(blk + 32 + 2 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t hw = (i & 1) ? (nb[i >> 1] >> 16) : (nb[i >> 1] & 0xffffu);
      const uint32_t cb = stq_patterns4(hw, (sbits >> (4 * i)) & 15u);
#pragma unroll
      for (int pl = 0; pl < 4; ++pl) wu.c[4 * i + pl] = cb & (0x03030303u << (2 * pl));
    }
  } else if (FMT == Q4_K) {
    // quant.rs:2437-2461.
    const uint32_t blk = row + (u >> 2) * 144;
    const int g = u & 3;
    const uint4 h = ld_s128(blk);
    const float d = half_to_f32(h.x & 0xffffu), dmin = half_to_f32(h.x >> 16);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = 2 * g + hh;
      uint32_t s, m;
      if (j < 4) {
        s = (h.y >> (8 * j)) & 63u;
        m = (h.z >> (8 * j)) & 63u;
      } else {
        const int k = j - 4;
        const uint32_t hi = (h.w >> (8 * k)) & 0xffu;
        s = (hi & 15u) | ((((h.y >> (8 * k)) & 0xffu) >> 6) << 4);
        m = (hi >> 4) | ((((h.z >> (8 * k)) & 0xffu) >> 6) << 4);
      }
      wu.s[hh] = d * (float)s;
      wu.m[hh] = dmin * (float)m;
      wu.si[hh] = (int)s;
      wu.si[2 + hh] = (int)m;
    }
    wu.s[2] = d;     // the f32 path applies d and dmin once per unit (combine)
    wu.s[3] = dmin;
    const uint4 q0 = ld_s128(blk + 16 + 32 * g);
    const uint4 q1 = ld_s128(blk + 32 + 32 * g);
    const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wu.c[i] = q[i] & 0x0f0f0f0fu;
      wu.c[8 + i] = (q[i] >> 4) & 0x0f0f0f0fu;
    }
  } else if (FMT == Q6_K) {
    // quant.rs:2462-2483; this unit holds planes pp and pp+2 of chunk c.
    const uint32_t blk = row + (u >> 2) * 210;
    const int c = (u >> 1) & 1, pp = u & 1;
    uint32_t ql[8], qh[8];
    ld_s_words<8>(blk + 64 * c + 32 * pp, ql);
    ld_s_words<8>(blk + 128 + 32 * c, qh);
    const uint32_t s01 = ld_s16(blk + 192 + 8 * c + 2 * pp);
    const uint32_t s45 = ld_s16(blk + 196 + 8 * c + 2 * pp);
    wu.m[0] = half_to_f32(ld_s16(blk + 208));
    wu.si[0] = (int)(int8_t)(s01 & 0xffu);
    wu.si[1] = (int)(int8_t)(s01 >> 8);
    wu.si[2] = (int)(int8_t)(s45 & 0xffu);
    wu.si[3] = (int)(int8_t)(s45 >> 8);
#pragma unroll
    for (int k = 0; k < 4; ++k) wu.s[k] = (float)wu.si[k];
    // code = low nibble | (2 high bits << 4): the high bits of plane pp sit
    // at bits 2pp..2pp+1 of each qh byte, those of plane pp+2 four bits up.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t h0 = pp ? (qh[i] << 2) : (qh[i] << 4);
      const uint32_t h1 = pp ? (qh[i] >> 2) : qh[i];
      wu.c[i] = (ql[i] & 0x0f0f0f0fu) | (h0 & 0x30303030u);
      wu.c[8 + i] = ((ql[i] >> 4) & 0x0f0f0f0fu) | (h1 & 0x30303030u);
    }
  } else {  // Q8_0, quant.rs:2413-2418
    const uint32_t blk = row + u * 68;
    wu.s[0] = half_to_f32(ld_s16(blk));
    wu.s[1] = half_to_f32(ld_s16(blk + 34));
    uint32_t q0[8], q1[8];
    ld_s_words<8>(blk + 2, q0);
    ld_s_words<8>(blk + 36, q1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wu.c[i] = q0[i];
      wu.c[8 + i] = q1[i];
    }
  }
}

template <int FMT>
__device__ __forceinline__ int dp4(uint32_t code, uint32_t x, int acc) {
  return FMT == Q8_0 ? dp4a_ss(code, x, acc) : dp4a_us(code, x, acc);
}

// Integer sum of codes x activations over words [j0, j1) of a unit: exact
// in 32 bits for one activation byte plane; the three planes of the f32 path
// are combined in 64 bits.
// Q2_0C and STQ1_0 words: word j holds plane k = j & 3 of its codes in
// place, i.e. code << 2k, so plane k sums carry a factor 4^k; one accumulator
// per plane keeps the four dp4a chains independent.  Returns
// 64 a0 + 16 a1 + 4 a2 + a3 = 64 x the exact code-activation sum.
template <int FMT>
__device__ __forceinline__ int plane_dot64(const WUnit& wu, const uint32_t (&x)[16]) {
  int a[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) a[j & 3] = dp4<FMT>(wu.c[j], x[j], a[j & 3]);
  return a[3] + 4 * (a[2] + 4 * (a[1] + 4 * a[0]));
}

// 64 x sum(code * activation) over a unit, one plane (NP=1) or the three
// exact planes of the f32 path (NP=3, 64-bit).
template <int FMT, int NP>
__device__ __forceinline__ long long plane_dot64_np(const WUnit& wu, const XUnit<NP>& xu) {
  const int a0 = plane_dot64<FMT>(wu, xu.w[0]);
  if (NP == 1) return a0;
  const int a1 = plane_dot64<FMT>(wu, xu.w[NP > 1 ? 1 : 0]);
  const int a2 = plane_dot64<FMT>(wu, xu.w[NP > 2 ? 2 : 0]);
  return (long long)a0 + ((long long)a1 << 8) + ((long long)a2 << 16);
}

template <int FMT, int NP>
__device__ __forceinline__ long long seg_dot(const WUnit& wu, const XUnit<NP>& xu, int j0, int j1) {
  if (NP == 1) {
    int a = 0;
#pragma unroll
    for (int j = j0; j < j1; ++j) a = dp4<FMT>(wu.c[j], xu.w[0][j], a);
    return a;
  } else {
    int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
    for (int j = j0; j < j1; ++j) {
      a0 = dp4<FMT>(wu.c[j], xu.w[0][j], a0);
      a1 = dp4<FMT>(wu.c[j], xu.w[NP > 1 ? 1 : 0][j], a1);
      a2 = dp4<FMT>(wu.c[j], xu.w[NP > 2 ? 2 : 0][j], a2);
    }
    return (long long)a0 + ((long long)a1 << 8) + ((long long)a2 << 16);
  }
}

// int -> float for the NP=1 (32-bit) and NP=3 (64-bit) sums.
template <int NP>
__device__ __forceinline__ float to_f(long long v) {
  return NP == 1 ? (float)(int)v : __ll2float_rn(v);
}

template <int FMT, int NP>
__device__ __forceinline__ float combine(const WUnit& wu, const XUnit<NP>& xu, float acc) {
  if (FMT == Q2_0C || FMT == STQ1_0) {
    // Q2_0C: sum (2c - 3) x = 2 sum c x - 3 sum x; STQ1_0: digit = code - 1.
    // With V = 64 sum c x - C sum x (C = 96 / 64) the sum is V / D (D = 32
    // / 64); load_x pre-multiplies xsum by C (NP=1) and pre-divides the
    // activation scale by D, an exact power of two, so the product equals
    // sum * (weight scale * activation scale) rounded once, as before.
    constexpr int C = FMT == Q2_0C ? 96 : 64;
    if (NP == 1) return fmaf((float)((int)plane_dot64_np<FMT, NP>(wu, xu) - xu.xsum[0]), wu.s[0] * xu.sg, acc);
    const long long v = plane_dot64_np<FMT, NP>(wu, xu) - (long long)C * xu.xsum[0];
    return fmaf(__ll2float_rn(v), wu.s[0] * xu.sg, acc);
  } else if (FMT == Q4_K && NP == 3) {
    // f32 path: sum (d s_h q - dmin m_h) X over the unit's two 32-column
    // sub-blocks = d sum_h s_h (sum q X)_h - dmin sum_h m_h (sum X)_h, with
    // s_h, m_h the 6-bit scale and min codes: two exact integers, one
    // conversion and one scale each.
    int A[3] = {0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int j = 8 * h; j < 8 * h + 8; ++j) {
        a0 = dp4<FMT>(wu.c[j], xu.w[0][j], a0);
        a1 = dp4<FMT>(wu.c[j], xu.w[NP > 1 ? 1 : 0][j], a1);
        a2 = dp4<FMT>(wu.c[j], xu.w[NP > 2 ? 2 : 0][j], a2);
      }
      A[0] += wu.si[h] * a0;
      A[1] += wu.si[h] * a1;
      A[2] += wu.si[h] * a2;
    }
    const long long qx = (long long)A[0] + ((long long)A[1] << 8) + ((long long)A[2] << 16);
    const long long mx = (long long)wu.si[2] * xu.xsum[0] + (long long)wu.si[3] * xu.xsum[1];
    const float t = __fsub_rn(__fmul_rn(wu.s[2], __ll2float_rn(qx)), __fmul_rn(wu.s[3], __ll2float_rn(mx)));
    return fmaf(t, xu.sg, acc);
  } else if (FMT == Q4_K) {
    // sum (d1 q - m1) x = d1 sum q x - m1 sum x, per 32-column sub-block
    const float a0 = to_f<NP>(seg_dot<FMT, NP>(wu, xu, 0, 8));
    const float a1 = to_f<NP>(seg_dot<FMT, NP>(wu, xu, 8, 16));
    float t = wu.s[0] * a0 - wu.m[0] * (float)xu.xsum[0];
    t += wu.s[1] * a1 - wu.m[1] * (float)xu.xsum[1];
    return fmaf(t, xu.sg, acc);
  } else if (FMT == Q6_K && NP == 3) {
    // f32 path: the four 16-weight planes' scales are int8, so the unit's
    // sum_s sc_s sum_i (q_i - 32) X_i is one exact integer (per activation
    // byte plane |sum| < 2^25), converted once and scaled by d * s_x.
    int A[3] = {0, 0, 0};
    long long xs = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
      for (int j = 4 * s; j < 4 * s + 4; ++j) {
        a0 = dp4<FMT>(wu.c[j], xu.w[0][j], a0);
        a1 = dp4<FMT>(wu.c[j], xu.w[NP > 1 ? 1 : 0][j], a1);
        a2 = dp4<FMT>(wu.c[j], xu.w[NP > 2 ? 2 : 0][j], a2);
      }
      A[0] += wu.si[s] * a0;
      A[1] += wu.si[s] * a1;
      A[2] += wu.si[s] * a2;
      xs += (long long)wu.si[s] * xu.xsum[s];
    }
    const long long t = (long long)A[0] + ((long long)A[1] << 8) + ((long long)A[2] << 16) - 32ll * xs;
    return fmaf(__ll2float_rn(t), wu.m[0] * xu.sg, acc);
  } else if (FMT == Q6_K) {
    // per 16-weight plane: (q - 32) x, scaled by (d * s_x) * sc
    const float ds = wu.m[0] * xu.sg;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const long long a = seg_dot<FMT, NP>(wu, xu, 4 * s, 4 * s + 4) - 32ll * xu.xsum[s];
      acc = fmaf(to_f<NP>(a), ds * wu.s[s], acc);
    }
    return acc;
  } else {  // Q8_0
    acc = fmaf(to_f<NP>(seg_dot<FMT, NP>(wu, xu, 0, 8)), wu.s[0] * xu.sg, acc);
    return fmaf(to_f<NP>(seg_dot<FMT, NP>(wu, xu, 8, 16)), wu.s[1] * xu.sg, acc);
  }
}

__device__ __forceinline__ void batch_of(const Params& p, int64_t bt, int R, int& m, int64_t& row0, int& nrows) {
  m = 0;
  if (p.n_mat > 1 && bt >= p.mat[1].batch_begin) m = 1;
  if (p.n_mat > 2 && bt >= p.mat[2].batch_begin) m = 2;
  row0 = (bt - p.mat[m].batch_begin) * R;
  const int64_t left = p.mat[m].rows - row0;
  nrows = (int)(left < R ? left : R);
}

// Row tiles land in shared memory as the 16-byte aligned window around them:
// [floor16(src), floor16(src + bytes)) by one bulk copy, and the last
// (src + bytes) % 16 bytes by plain loads, so row data starts at
// dst + (src & 15).  stage_tail must run before the arrive that releases the
// stage; stage_bulk after it.
__device__ __forceinline__ uint32_t stage_tail(uint8_t* dst, const uint8_t* src, int64_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src);
  const uintptr_t a0 = a & ~uintptr_t(15);
  const uintptr_t a1 = a + (uintptr_t)bytes;
  const uintptr_t b1 = (a1 & ~uintptr_t(15)) > a0 ? (a1 & ~uintptr_t(15)) : a0;
  const uint8_t* t = reinterpret_cast<const uint8_t*>(b1);
  uint8_t* d = dst + (b1 - a0);
  for (uintptr_t k = 0; k < a1 - b1; ++k) d[k] = t[k];
  return (uint32_t)(b1 - a0);
}

__device__ __forceinline__ void stage_bulk(uint8_t* dst, const uint8_t* src, uint32_t bulk, uint32_t bar,
                                           uint64_t policy) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
  if (bulk) bulk_g2s_hint(smem_addr(dst), reinterpret_cast<const void*>(a0), bulk, bar, policy);
}

// Reduce V = 2^k per-lane values over the warp with a transposed butterfly:
// each level keeps half of the values and exchanges the other half, so V rows
// cost (V-1) + (5-k) shuffles instead of 5V.  Afterwards lane l holds the
// total of value index reduce_index<V>(l) in v[0].
template <int V>
__device__ __forceinline__ void warp_reduce_multi(float (&v)[V], int lane) {
  int n = V;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < V / 2; ++j) {
        if (j < n / 2) {
          const float send = upper ? v[j] : v[j + n / 2];
          const float keep = upper ? v[j + n / 2] : v[j];
          v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n /= 2;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
}

template <int V>
__device__ __forceinline__ int reduce_index(int lane) {
  int idx = 0, n = V;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      if (lane & o) idx += n / 2;
      n /= 2;
    }
  }
  return idx;
}

// The lowest lane of each group that holds one reduced index.
template <int V>
__device__ __forceinline__ bool reduce_writer(int lane) {
  constexpr int k = V == 1 ? 0 : (V == 2 ? 1 : (V == 4 ? 2 : 3));
  return (lane & ((32 >> k) - 1)) == 0;
}

// The RW rows x UPL units of one warp in one tile, as straight-line code so
// that their loads and dp4a chains interleave.  CHECK (the last tile of a
// matrix, or lanes without a unit): rows past the tile's end re-read row 0
// and are never written; a lane without a unit decodes unit 0 and keeps its
// sums unchanged.
template <int FMT, int NP, int UPL, int RW, bool PAIR, bool CHECK>
__device__ __forceinline__ void tile_rows(uint32_t base, uint32_t baseu, int row_bytes, int rg, int rgi, int nrows,
                                          const int (&ui)[UPL], const bool (&uv)[UPL], const XUnit<NP> (&xu)[UPL],
                                          float (&g)[RW], float (&u)[RW]) {
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
      const int r = rgi + rg * rr;
      const uint32_t off = (uint32_t)(((CHECK && r >= nrows) ? 0 : r) * row_bytes);
      WUnit wu;
      decode_unit<FMT>(base + off, ui[i], wu);
      const float gv = combine<FMT, NP>(wu, xu[i], g[rr]);
      g[rr] = (!CHECK || uv[i]) ? gv : g[rr];
      if (PAIR) {
        WUnit wv;
        decode_unit<FMT>(baseu + off, ui[i], wv);
        const float uvv = combine<FMT, NP>(wv, xu[i], u[rr]);
        u[rr] = (!CHECK || uv[i]) ? uvv : u[rr];
      }
    }
  }
}

// Variants that also come in a two-CTAs-per-SM build (DUAL: <= 72 registers,
// 26 warps per SM): the int8 path of the 2-bit and ternary formats with one
// unit per lane, whose dp4a and shared-load chains need more warps to hide
// their latency.  The others take the whole SM.
__host__ __device__ constexpr bool dual_variant(int fmt, int np, int upl, bool pair) {
  return (fmt == Q2_0C || fmt == STQ1_0) && np == 1 && upl == 1 && !pair;
}

template <int FMT, int NP, int UPL, int RW, bool PAIR, bool DUAL>
__global__ void __launch_bounds__(kThreads, DUAL ? 2 : 1) gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages);
  float* red = reinterpret_cast<float*>(smem + kRedOffset);
  uint8_t* stages = smem + p.stage_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const int R = p.rg * RW;  // rows per tile: RW per row group

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), kCW);
    }
    mbar_init(smem_addr(smem + kXBarOffset), 1);
    *abort_flag = 0;
    mbar_fence_init();
    // With an overlapped launch the next product may start streaming its
    // weights now; everything it reads from this grid waits for completion.
    allow_dependents_launch();
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------ producer ------------------------------
    // The packed weights are read-only for the whole call sequence, so the
    // first ring of tiles is fetched before the preceding grid completes
    // (overlapped launches only); the bounded waits start after it has.
    if (lane == 0) {
      // Each packed weight byte is used once per call.
      const uint64_t policy = l2_evict_first_policy();
      int64_t issued = 0;
      int s = 0;
      uint32_t par = 1;  // phase of the empty barrier being waited for, from the second lap
      for (int64_t bt = blockIdx.x; bt < p.total_batches; bt += gridDim.x, ++issued) {
        if (issued == S) grid_dependency_wait();
        if (issued >= S) {
          if (!mbar_wait(smem_addr(&empty[s]), par, abort_flag)) {
            atomicOr(p.status, DEV_TIMEOUT_EMPTY);
            *abort_flag = 1;
            break;
          }
        }
        fence_proxy_async_smem();
        int m, nrows;
        int64_t row0;
        batch_of(p, bt, R, m, row0, nrows);
        uint8_t* dst = stages + (size_t)s * p.stage_bytes;
        const int64_t bytes = (int64_t)nrows * p.row_bytes;
        const uint8_t* src = p.mat[m].w + row0 * p.row_bytes;
        const uint32_t bar = smem_addr(&full[s]);
        const uint8_t* srcu = PAIR ? p.up + row0 * p.row_bytes : nullptr;
        const uint32_t b0 = stage_tail(dst, src, bytes);
        const uint32_t b1 = PAIR ? stage_tail(dst + p.half_bytes, srcu, bytes) : 0u;
        mbar_arrive_expect_tx(bar, b0 + b1);
        stage_bulk(dst, src, b0, bar, policy);
        if (PAIR) stage_bulk(dst + p.half_bytes, srcu, b1, bar, policy);
        if (++s == S) {
          s = 0;
          par ^= 1u;
        }
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      const int64_t last = issued;
      for (int64_t k = (last > S ? last - S : 0); k < last; ++k) {
        const int s = (int)(k % S);
        const uint32_t par = (uint32_t)((k / S) & 1);
        if (!mbar_wait(smem_addr(&full[s]), par, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
      }
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  grid_dependency_wait();  // x is the preceding grid's output; y may be its input
  prepare_x<FMT, NP>(p, smem);
  const int ksi = warp % p.ks, rgi = warp / p.ks;
  XUnit<NP> xu[UPL];
  int uu[UPL];
  bool uv[UPL];
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    const int local = lane + 32 * i;
    uu[i] = ksi * p.slice + local;
    uv[i] = local < p.slice && uu[i] < p.U;
    load_x<FMT, NP>(p, smem, uu[i], uv[i], xu[i]);
  }
  const int ridx = reduce_index<RW>(lane);
  const bool writer = reduce_writer<RW>(lane);
  const uint32_t stages_s = smem_addr(stages);
  int ui[UPL];
  bool lanes_ok = true;
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    ui[i] = uv[i] ? uu[i] : 0;
    lanes_ok = lanes_ok && uv[i];
  }
  const bool all_units = __all_sync(0xffffffffu, lanes_ok);
  const int row_bytes = p.row_bytes, rg = p.rg;

  // Ring slot and phase advance by increments (no division per tile).
  int s = 0;
  uint32_t par = 0;
  int64_t it = 0;
  for (int64_t bt = blockIdx.x; bt < p.total_batches; bt += gridDim.x, ++it) {
    int m, nrows;
    int64_t row0;
    batch_of(p, bt, R, m, row0, nrows);
    const int r = rgi + p.rg * ridx;  // the row this lane holds after the reduction
    const bool emits = writer && r < nrows && (p.ks == 1 || ksi == 0);
    // residual form: the row's current value, loaded while the tile computes
    const float y_old = (p.residual && emits) ? __ldcg(p.mat[m].y + row0 + r) : 0.f;
    bool ok = mbar_wait(smem_addr(&full[s]), par, abort_flag);
    // The warps that share a row leave together, or the named barrier below
    // would wait for a warp that is gone.
    if (p.ks > 1) ok = bar_red_and(1 + rgi, p.ks * 32, ok);
    if (!ok) {
      if (lane == 0) atomicOr(p.status, DEV_TIMEOUT_FULL);
      *abort_flag = 1;
      break;
    }
    const uint32_t tile = stages_s + (uint32_t)s * (uint32_t)p.stage_bytes;
    const uint32_t base = tile + (uint32_t)(reinterpret_cast<uintptr_t>(p.mat[m].w + row0 * row_bytes) & 15);
    const uint32_t baseu =
        tile + (uint32_t)p.half_bytes +
        (PAIR ? (uint32_t)(reinterpret_cast<uintptr_t>(p.up + row0 * row_bytes) & 15) : 0u);
    float g[RW], u[RW];
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) g[rr] = u[rr] = 0.f;
    // (UPL 4 keeps one copy: two do not fit in 128 registers.)
    if (UPL <= 3 && all_units && nrows == R)
      tile_rows<FMT, NP, UPL, RW, PAIR, (UPL > 3)>(base, baseu, row_bytes, rg, rgi, nrows, ui, uv, xu, g, u);
    else
      tile_rows<FMT, NP, UPL, RW, PAIR, true>(base, baseu, row_bytes, rg, rgi, nrows, ui, uv, xu, g, u);
    warp_reduce_multi<RW>(g, lane);
    if (PAIR) warp_reduce_multi<RW>(u, lane);
    if (p.ks == 1) {
      if (emits) {
        float out = g[0];
        if (PAIR) out = (g[0] / (1.0f + expf(-g[0]))) * u[0];  // quant.rs:573-574
        emit_row(p, m, row0 + r, out, y_old);
      }
    } else {
      // Partial sums of the ks warps of each row, double-buffered by tile
      // parity: a writer two tiles ahead has passed this group's barrier of
      // the next tile, which the reader reaches only after reading.
      float* rb = red + (it & 1) * (2 * kCW * 4);
      if (writer) {
        rb[((rgi * RW + ridx) * p.ks + ksi) * 2] = g[0];
        rb[((rgi * RW + ridx) * p.ks + ksi) * 2 + 1] = PAIR ? u[0] : 0.f;
      }
      bar_sync_named(1 + rgi, p.ks * 32);
      if (emits) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < p.ks; ++k) {
          gs += rb[((rgi * RW + ridx) * p.ks + k) * 2];
          us += rb[((rgi * RW + ridx) * p.ks + k) * 2 + 1];
        }
        float out = gs;
        if (PAIR) out = (gs / (1.0f + expf(-gs))) * us;
        emit_row(p, m, row0 + r, out, y_old);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[s]));
    if (++s == S) {
      s = 0;
      par ^= 1u;
    }
  }
}

// Launch geometry chosen by the host (hyq_gemv.cu, make_plan).
struct Plan {
  bool streaming = false;
  int ks = 1, slice = 0, upl = 1, rw = 1, stages = 0, half_bytes = 0, stage_bytes = 0;
  int x_bytes = 0;
  int x_raw_bytes = 0, x_raw_off = 0;  // staged f32 activations (0: none)
  int x_pad_off = 0;                    // their padded copy (with the staged copy)
  int64_t total_batches = 0;
  int64_t batch_begin[3] = {};
  size_t smem = 0;
  int smem_cap = 0;
  int grid = 0;
  int ctas_per_sm = 1;
  // Launch as a programmatic dependent of the preceding grid in the stream
  // (the caller guarantees no kernel still in flight writes the weights).
  bool overlap = false;
};

template <int FMT, int NP, int UPL, int RW, bool PAIR, bool DUAL>
cudaError_t run_stream(const Params& p, const Plan& pl, cudaStream_t st) {
  auto k = gemv_kernel<FMT, NP, UPL, RW, PAIR, DUAL>;
  // Raise the dynamic shared-memory limit once per device and instantiation.
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem_cap);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  if (pl.overlap) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, p);
  }
  k<<<pl.grid, kThreads, pl.smem, st>>>(p);
  return cudaGetLastError();
}

template <int FMT, int NP, int UPL, bool PAIR>
cudaError_t dispatch_rw(const Params& p, const Plan& pl, cudaStream_t st) {
  if constexpr (dual_variant(FMT, NP, UPL, PAIR)) {
    if (pl.ctas_per_sm == 2) {
      switch (pl.rw) {
        case 1: return run_stream<FMT, NP, UPL, 1, PAIR, true>(p, pl, st);
        case 2: return run_stream<FMT, NP, UPL, 2, PAIR, true>(p, pl, st);
        default: return run_stream<FMT, NP, UPL, 4, PAIR, true>(p, pl, st);
      }
    }
  }
  switch (pl.rw) {
    case 1: return run_stream<FMT, NP, UPL, 1, PAIR, false>(p, pl, st);
    case 2: return run_stream<FMT, NP, UPL, 2, PAIR, false>(p, pl, st);
    default: return run_stream<FMT, NP, UPL, 4, PAIR, false>(p, pl, st);
  }
}

template <int FMT, int NP, bool PAIR>
cudaError_t dispatch_upl(const Params& p, const Plan& pl, cudaStream_t st) {
  if constexpr (NP == 3) {
    return dispatch_rw<FMT, NP, 1, PAIR>(p, pl, st);
  } else {
    switch (pl.upl) {
      case 1: return dispatch_rw<FMT, NP, 1, PAIR>(p, pl, st);
      case 2: return dispatch_rw<FMT, NP, 2, PAIR>(p, pl, st);
      case 3: return dispatch_rw<FMT, NP, 3, PAIR>(p, pl, st);
      default: return dispatch_rw<FMT, NP, 4, PAIR>(p, pl, st);
    }
  }
}

// Entry of one format's translation unit.
template <int FMT>
cudaError_t dispatch_fmt(const Params& p, const Plan& pl, bool pair, cudaStream_t st) {
  if (p.xmode == XF32)
    return pair ? dispatch_upl<FMT, 3, true>(p, pl, st) : dispatch_upl<FMT, 3, false>(p, pl, st);
  return pair ? dispatch_upl<FMT, 1, true>(p, pl, st) : dispatch_upl<FMT, 1, false>(p, pl, st);
}

}  // namespace gemv
}  // namespace hyq
