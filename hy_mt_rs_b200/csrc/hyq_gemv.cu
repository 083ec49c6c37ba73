// Batch-1 matrix-vector products over packed GGUF rows (sm_100a).
//
// Reference behaviour (hy-mt-rs src/quant.rs):
//   Weight::matmul batch 1          :159-270   (f32 activations)
//   gemv_q8_fast / compute_chunk_q8 :353-439   (int8 activations, SDOT rows)
//   gemv_qkv(_fast)                 :441-538, :653-721
//   matmul_gate_up_silu(_fast)      :540-651, :723-841
//
// Engine.  Rows are streamed, never re-read: a persistent CTA per SM owns a
// ring of shared-memory stages; one producer thread fills each stage with a
// tile of consecutive packed rows using cp.async.bulk (one contiguous copy,
// packed bytes unchanged) and an mbarrier transaction count; 12 consumer warps
// decode the codes out of shared memory and reduce them against the
// activations, which every lane keeps in registers for the CTA's lifetime
// (each lane owns fixed 64-column "units" of the row).  A row is split over KS
// warps when K is too wide for one warp's registers or when splitting gives
// the grid enough row tiles.
//
// Arithmetic.  Codes are multiplied in the integer domain with dp4a:
//   int8 path (NP=1): the reference's Q8 activations; per 256-column group
//     the exact integer sum is scaled by (weight scale * activation scale),
//     as the SDOT kernels do (quant.rs:1511-1557, 1891-1955, 2257-2332).
//   f32 path (NP=3): each f32 activation is written as a 24-bit integer X
//     times a power-of-two group scale (2^(e-22), e = exponent of the group's
//     max |x|), split exactly into three signed bytes.  Products and sums are
//     exact integers; the only rounding is |dx| <= 2^(e-23) per activation and
//     the final f32 accumulation, i.e. f32-level accuracy.
#include <cstdio>

#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {

namespace {

constexpr int kCW = 12;                    // consumer warps (13 warps: <= 128 registers)
constexpr int kThreads = (kCW + 1) * 32;   // + one producer warp
constexpr int kMaxStages = 32;
constexpr int kHeaderBytes = 2048;         // barriers, abort flag, partial sums
constexpr int kRedOffset = 1024;           // partial sums: 2 copies x 16 warps x (gate, up)

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
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
  int ks, rg, slice;  // K-split, row groups (rg*ks == kCW), units per slice
  int stages;
  int half_bytes;     // bytes of one row-tile buffer
  int stage_bytes;
  const float* x;
  const int8_t* xq;
  const float* xs;
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
};

// ---------------------------------------------------------------------------
// Activation setup (once per CTA).
// ---------------------------------------------------------------------------
template <int FMT>
__device__ __forceinline__ void setup_x_i8(const Params& p, int u, bool valid, XUnit<1>& xu) {
  uint32_t n[16];
  if (valid) {
    int c0, c1;
    unit_runs<FMT>(u, c0, c1);
    const uint4* r0 = reinterpret_cast<const uint4*>(p.xq + c0);
    const uint4* r1 = reinterpret_cast<const uint4*>(p.xq + c1);
    const uint4 a = r0[0], b = r0[1], c = r1[0], d = r1[1];
    n[0] = a.x; n[1] = a.y; n[2] = a.z; n[3] = a.w;
    n[4] = b.x; n[5] = b.y; n[6] = b.z; n[7] = b.w;
    n[8] = c.x; n[9] = c.y; n[10] = c.z; n[11] = c.w;
    n[12] = d.x; n[13] = d.y; n[14] = d.z; n[15] = d.w;
    xu.sg = p.xs[u >> 2];
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) n[i] = 0;
    xu.sg = 0.f;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t w = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int r = rel<FMT>(j, b);
      w |= ((n[r >> 2] >> (8 * (r & 3))) & 0xffu) << (8 * b);
    }
    xu.w[0][j] = w;
  }
  constexpr int NS = nseg<FMT>(), WPS = 16 / NS;
#pragma unroll
  for (int s = 0; s < 4; ++s) xu.xsum[s] = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    int acc = 0;
#pragma unroll
    for (int k = s * WPS; k < (s + 1) * WPS; ++k) acc = __dp4a((int)n[k], 0x01010101, acc);
    xu.xsum[s] = acc;
  }
}

template <int FMT>
__device__ __forceinline__ void setup_x_f32(const Params& p, int u, bool valid, XUnit<3>& xu) {
  float xv[64];
  float m = 0.f;
  bool bad = false;
  if (valid) {
    int c0, c1;
    unit_runs<FMT>(u, c0, c1);
    const float4* r0 = reinterpret_cast<const float4*>(p.x + c0);
    const float4* r1 = reinterpret_cast<const float4*>(p.x + c1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = r0[i], b = r1[i];
      xv[4 * i] = a.x; xv[4 * i + 1] = a.y; xv[4 * i + 2] = a.z; xv[4 * i + 3] = a.w;
      xv[32 + 4 * i] = b.x; xv[33 + 4 * i] = b.y; xv[34 + 4 * i] = b.z; xv[35 + 4 * i] = b.w;
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float a = fabsf(xv[i]);
      bad |= !(a <= 3.0e38f);  // inf or NaN
      m = fmaxf(m, a);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) xv[i] = 0.f;
  }
  // The four units of a 256-column group sit on four consecutive lanes.
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  int badi = bad ? 1 : 0;
  badi |= __shfl_xor_sync(0xffffffffu, badi, 1);
  badi |= __shfl_xor_sync(0xffffffffu, badi, 2);
  int ex = 0;
  frexpf(m, &ex);
  int X[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) X[i] = badi ? 0 : __float2int_rn(ldexpf(xv[i], 22 - ex));
  xu.sg = badi ? __int_as_float(0x7fc00000) : ldexpf(1.f, ex - 22);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int v = X[rel<FMT>(j, b)];
      const int p0 = (int)(int8_t)(v & 0xff);
      const int t = (v - p0) >> 8;
      const int p1 = (int)(int8_t)(t & 0xff);
      const int p2 = (t - p1) >> 8;
      w0 |= ((uint32_t)p0 & 0xffu) << (8 * b);
      w1 |= ((uint32_t)p1 & 0xffu) << (8 * b);
      w2 |= ((uint32_t)p2 & 0xffu) << (8 * b);
    }
    xu.w[0][j] = w0;
    xu.w[1][j] = w1;
    xu.w[2][j] = w2;
  }
  constexpr int NS = nseg<FMT>(), CPS = 64 / NS;
#pragma unroll
  for (int s = 0; s < 4; ++s) xu.xsum[s] = 0;
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    int acc = 0;
#pragma unroll
    for (int k = s * CPS; k < (s + 1) * CPS; ++k) acc += X[k];
    xu.xsum[s] = acc;
  }
}

// ---------------------------------------------------------------------------
// Weight unit decode from shared memory (row pointer 2-byte aligned; Q4_K
// rows are 16-byte aligned).
// ---------------------------------------------------------------------------
template <int FMT>
__device__ __forceinline__ void decode_unit(const uint8_t* row, int u, WUnit& wu) {
  if (FMT == Q2_0C) {
    // quant.rs:2419-2432: 2-bit code c -> (2c - 3) * d, four codes per byte.
    const uint8_t* blk = row + (u >> 3) * 130;
    wu.s[0] = half_to_f32(lds_u16(blk));
    uint32_t q[4];
    lds_words_a2<4>(blk + 2 + 16 * (u & 7), q);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) wu.c[4 * i + k] = (q[i] >> (2 * k)) & 0x03030303u;
  } else if (FMT == STQ1_0) {
    // quant.rs:1103-1123: group g of chunk c: codebook[(sign << 4) | nibble],
    // lane p -> column 16p + (g % 16).  Four groups at a time: PRMT looks the
    // codebook up in registers, byte masks pick the half by nibble bit 3 and
    // by the sign bit.
    const uint8_t* blk = row + (u >> 2) * 42;
    const int c = u & 3;
    wu.s[0] = half_to_f32(lds_u16(blk + 40));
    uint32_t nb[2];
    lds_words_a2<2>(blk + 8 * c, nb);
    const uint32_t sbits = lds_u16(blk + 32 + 2 * c);
    const uint32_t T0 = 0x092989a9u, T1 = 0x062686a6u, T2 = 0x121a929au, T3 = 0x424a626au;
    const uint32_t T4 = 0xa1812101u, T5 = 0xa4842404u, T6 = 0x98901810u, T7 = 0x68604840u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t hw = (i & 1) ? (nb[i >> 1] >> 16) : (nb[i >> 1] & 0xffffu);
      const uint32_t sel = hw & 0x7777u;
      const uint32_t p0 = prmt(T0, T1, sel), p1 = prmt(T2, T3, sel);
      const uint32_t p2 = prmt(T4, T5, sel), p3 = prmt(T6, T7, sel);
      const uint32_t m3 = prmt(hw << 4, hw, 0xD9C8u);
      const uint32_t s4 = (sbits >> (4 * i)) & 15u;
      const uint32_t sm = prmt(s4 * 0x10204080u, 0u, 0xBA98u);
      const uint32_t lo = (p0 & ~m3) | (p1 & m3);
      const uint32_t hi = (p2 & ~m3) | (p3 & m3);
      const uint32_t cb = (lo & ~sm) | (hi & sm);
#pragma unroll
      for (int pl = 0; pl < 4; ++pl) wu.c[4 * i + pl] = (cb >> (2 * pl)) & 0x03030303u;
    }
  } else if (FMT == Q4_K) {
    // quant.rs:2437-2461.
    const uint8_t* blk = row + (u >> 2) * 144;
    const int g = u & 3;
    const uint4 h = *reinterpret_cast<const uint4*>(blk);
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
    }
    const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
    const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
    const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wu.c[i] = q[i] & 0x0f0f0f0fu;
      wu.c[8 + i] = (q[i] >> 4) & 0x0f0f0f0fu;
    }
  } else if (FMT == Q6_K) {
    // quant.rs:2462-2483; this unit holds planes pp and pp+2 of chunk c.
    const uint8_t* blk = row + (u >> 2) * 210;
    const int c = (u >> 1) & 1, pp = u & 1;
    uint32_t ql[8], qh[8];
    lds_words_a2<8>(blk + 64 * c + 32 * pp, ql);
    lds_words_a2<8>(blk + 128 + 32 * c, qh);
    const uint32_t s01 = lds_u16(blk + 192 + 8 * c + 2 * pp);
    const uint32_t s45 = lds_u16(blk + 196 + 8 * c + 2 * pp);
    wu.m[0] = half_to_f32(lds_u16(blk + 208));
    wu.s[0] = (float)(int8_t)(s01 & 0xffu);
    wu.s[1] = (float)(int8_t)(s01 >> 8);
    wu.s[2] = (float)(int8_t)(s45 & 0xffu);
    wu.s[3] = (float)(int8_t)(s45 >> 8);
    const int sh = 2 * pp;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wu.c[i] = (ql[i] & 0x0f0f0f0fu) | (((qh[i] >> sh) & 0x03030303u) << 4);
      wu.c[8 + i] = ((ql[i] >> 4) & 0x0f0f0f0fu) | (((qh[i] >> (sh + 4)) & 0x03030303u) << 4);
    }
  } else {  // Q8_0, quant.rs:2413-2418
    const uint8_t* blk = row + u * 68;
    wu.s[0] = half_to_f32(lds_u16(blk));
    wu.s[1] = half_to_f32(lds_u16(blk + 34));
    uint32_t q0[8], q1[8];
    lds_words_a2<8>(blk + 2, q0);
    lds_words_a2<8>(blk + 36, q1);
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

// Integer sum of codes x activations over words [j0, j1) of a unit.
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

template <int FMT, int NP>
__device__ __forceinline__ float combine(const WUnit& wu, const XUnit<NP>& xu, float acc) {
  if (FMT == Q2_0C) {
    const long long a = 2 * seg_dot<FMT, NP>(wu, xu, 0, 16) - 3ll * xu.xsum[0];
    return fmaf(__ll2float_rn(a), wu.s[0] * xu.sg, acc);
  } else if (FMT == STQ1_0) {
    const long long a = seg_dot<FMT, NP>(wu, xu, 0, 16) - (long long)xu.xsum[0];
    return fmaf(__ll2float_rn(a), wu.s[0] * xu.sg, acc);
  } else if (FMT == Q4_K) {
    const float a0 = __ll2float_rn(seg_dot<FMT, NP>(wu, xu, 0, 8));
    const float a1 = __ll2float_rn(seg_dot<FMT, NP>(wu, xu, 8, 16));
    float t = wu.s[0] * a0 - wu.m[0] * (float)xu.xsum[0];
    t += wu.s[1] * a1 - wu.m[1] * (float)xu.xsum[1];
    return fmaf(t, xu.sg, acc);
  } else if (FMT == Q6_K) {
    const float ds = wu.m[0] * xu.sg;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const long long a = seg_dot<FMT, NP>(wu, xu, 4 * s, 4 * s + 4) - 32ll * xu.xsum[s];
      acc = fmaf(__ll2float_rn(a), ds * wu.s[s], acc);
    }
    return acc;
  } else {  // Q8_0
    acc = fmaf(__ll2float_rn(seg_dot<FMT, NP>(wu, xu, 0, 8)), wu.s[0] * xu.sg, acc);
    return fmaf(__ll2float_rn(seg_dot<FMT, NP>(wu, xu, 8, 16)), wu.s[1] * xu.sg, acc);
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

__device__ __forceinline__ void stage_bulk(uint8_t* dst, const uint8_t* src, uint32_t bulk, uint32_t bar) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
  if (bulk) bulk_g2s(smem_addr(dst), reinterpret_cast<const void*>(a0), bulk, bar);
}

template <int FMT, int NP, int UPL, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * kMaxStages);
  float* red = reinterpret_cast<float*>(smem + kRedOffset);
  uint8_t* stages = smem + kHeaderBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const int R = p.rg;  // rows per tile: one per row group

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), kCW);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      int64_t issued = 0;
      for (int64_t bt = blockIdx.x; bt < p.total_batches; bt += gridDim.x, ++issued) {
        const int s = (int)(issued % S);
        if (issued >= S) {
          const uint32_t par = (uint32_t)(((issued / S) - 1) & 1);
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
        stage_bulk(dst, src, b0, bar);
        if (PAIR) stage_bulk(dst + p.half_bytes, srcu, b1, bar);
      }
      // Do not leave while copies into this CTA's shared memory are in flight.
      const int64_t last = issued;
      for (int64_t k = (last > S ? last - S : 0); k < last; ++k) {
        const int s = (int)(k % S);
        const uint32_t par = (uint32_t)((k / S) & 1);
        if (!mbar_wait(smem_addr(&full[s]), par, nullptr)) {
          atomicOr(p.status, DEV_TIMEOUT_DRAIN);
        }
      }
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int ksi = warp % p.ks, rgi = warp / p.ks;
  XUnit<NP> xu[UPL];
  int uu[UPL];
  bool uv[UPL];
#pragma unroll
  for (int i = 0; i < UPL; ++i) {
    const int local = lane + 32 * i;
    uu[i] = ksi * p.slice + local;
    uv[i] = local < p.slice && uu[i] < p.U;
    if (NP == 1) setup_x_i8<FMT>(p, uu[i], uv[i], reinterpret_cast<XUnit<1>&>(xu[i]));
    else setup_x_f32<FMT>(p, uu[i], uv[i], reinterpret_cast<XUnit<3>&>(xu[i]));
  }

  int64_t it = 0;
  for (int64_t bt = blockIdx.x; bt < p.total_batches; bt += gridDim.x, ++it) {
    const int s = (int)(it % S);
    const uint32_t par = (uint32_t)((it / S) & 1);
    bool ok = mbar_wait(smem_addr(&full[s]), par, abort_flag);
    // The warps that share a row leave together, or the named barrier below
    // would wait for a warp that is gone.
    if (p.ks > 1) ok = bar_red_and(1 + rgi, p.ks * 32, ok);
    if (!ok) {
      if (lane == 0) atomicOr(p.status, DEV_TIMEOUT_FULL);
      *abort_flag = 1;
      break;
    }
    int m, nrows;
    int64_t row0;
    batch_of(p, bt, R, m, row0, nrows);
    const uint8_t* tile = stages + (size_t)s * p.stage_bytes;
    const int skew = (int)(reinterpret_cast<uintptr_t>(p.mat[m].w + row0 * p.row_bytes) & 15);
    const int r = rgi;
    float g = 0.f, uacc = 0.f;
    if (r < nrows) {
      const uint8_t* rowp = tile + skew + r * p.row_bytes;
      const uint8_t* rowu = tile + p.half_bytes + (PAIR ? (int)(reinterpret_cast<uintptr_t>(p.up + row0 * p.row_bytes) & 15) : 0) + r * p.row_bytes;
#pragma unroll
      for (int i = 0; i < UPL; ++i) {
        if (uv[i]) {
          WUnit wu;
          decode_unit<FMT>(rowp, uu[i], wu);
          g = combine<FMT, NP>(wu, xu[i], g);
          if (PAIR) {
            WUnit wv;
            decode_unit<FMT>(rowu, uu[i], wv);
            uacc = combine<FMT, NP>(wv, xu[i], uacc);
          }
        }
      }
      g = warp_sum(g);
      if (PAIR) uacc = warp_sum(uacc);
    }
    if (p.ks == 1) {
      if (r < nrows && lane == 0) {
        float out = g;
        if (PAIR) out = (g / (1.0f + expf(-g))) * uacc;  // quant.rs:573-574
        p.mat[m].y[row0 + r] = out;
      }
    } else {
      // Partial sums of the ks warps of this row, double-buffered by tile
      // parity: a writer two tiles ahead has passed this group's barrier of
      // the next tile, which the reader reaches only after reading.
      float* rb = red + (it & 1) * (2 * kCW);
      if (lane == 0) {
        rb[(r * p.ks + ksi) * 2] = g;
        rb[(r * p.ks + ksi) * 2 + 1] = uacc;
      }
      bar_sync_named(1 + rgi, p.ks * 32);
      if (ksi == 0 && lane == 0 && r < nrows) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < p.ks; ++k) {
          gs += rb[(r * p.ks + k) * 2];
          us += rb[(r * p.ks + k) * 2 + 1];
        }
        float out = gs;
        if (PAIR) out = (gs / (1.0f + expf(-gs))) * us;
        p.mat[m].y[row0 + r] = out;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[s]));
  }
}

// ---------------------------------------------------------------------------
// Fallback: one warp per row, per-element decode straight from global memory.
// Used for F32/F16 weights and for shapes or pointers the streaming engine
// does not take (K not a multiple of 256, unaligned buffers).
// ---------------------------------------------------------------------------
template <int T, bool PAIR>
__global__ void __launch_bounds__(256) gemv_fallback_kernel(const __grid_constant__ Params p) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr int BL = block_len(T), BB = block_bytes(T);
  int64_t total = 0;
  for (int m = 0; m < p.n_mat; ++m) total += p.mat[m].rows;
  for (int64_t gr = gw; gr < total; gr += nw) {
    int m = 0;
    int64_t r = gr;
    while (m + 1 < p.n_mat && r >= p.mat[m].rows) r -= p.mat[m++].rows;
    const uint8_t* row = p.mat[m].w + r * p.row_bytes;
    const uint8_t* rowu = PAIR ? p.up + r * p.row_bytes : nullptr;
    float g = 0.f, u = 0.f;
    for (int k = lane; k < p.K; k += 32) {
      const float xv = p.x ? p.x[k] : (float)p.xq[k] * p.xs[k >> 8];
      const int b = k / BL, o = k - b * BL;
      g = fmaf(decode_elem<T>(row + b * BB, o), xv, g);
      if (PAIR) u = fmaf(decode_elem<T>(rowu + b * BB, o), xv, u);
    }
    g = warp_sum(g);
    if (PAIR) u = warp_sum(u);
    if (lane == 0) p.mat[m].y[r] = PAIR ? (g / (1.0f + expf(-g))) * u : g;
  }
}

int g_num_sms = 0;
int g_smem_optin = 0;

void device_limits() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached_dev = -1;
  if (cached_dev != dev) {
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cached_dev = dev;
  }
}

struct Plan {
  bool streaming = false;
  int ks = 1, slice = 0, upl = 1, stages = 0, half_bytes = 0, stage_bytes = 0;
  int64_t total_batches = 0;
  int64_t batch_begin[3] = {};
  size_t smem = 0;
  int grid = 0;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

Plan make_plan(const GemvJob& j) {
  Plan pl;
  device_limits();
  const int t = j.dtype;
  const bool pair = j.up != nullptr;
  if (t == F32 || t == F16) return pl;
  if (j.K % 256 != 0) return pl;
  for (int m = 0; m < j.n_mat; ++m)
    if (!aligned16(j.w[m])) return pl;
  if (pair && !aligned16(j.up)) return pl;
  if (j.x ? !aligned16(j.x) : !aligned16(j.xq)) return pl;
  const int U = (int)(j.K / 64);
  const int np = j.x ? 3 : 1;
  const int upl_max = np == 1 ? 4 : 1;
  const int64_t row_bytes = j.K / block_len(t) * block_bytes(t);
  int64_t total_rows = 0;
  for (int m = 0; m < j.n_mat; ++m) total_rows += j.rows[m];
  const int smem_cap = g_smem_optin > 0 ? g_smem_optin : 227 * 1024;
  int chosen = 0;
  static const int kSplits[] = {1, 2, 3, 4, 6, 12};
  for (int ks : kSplits) {
    // Units per K-split slice, rounded to whole 256-column groups.
    const int slice = ((U + ks - 1) / ks + 3) / 4 * 4;
    const int upl = (slice + 31) / 32;
    if (upl > upl_max) continue;
    const int rg = kCW / ks;
    const int64_t half = ((int64_t)rg * row_bytes + 32 + 15) / 16 * 16;
    const int64_t stage = half * (pair ? 2 : 1);
    if (kHeaderBytes + 2 * stage > smem_cap) continue;
    int64_t batches = 0;
    for (int m = 0; m < j.n_mat; ++m) batches += (j.rows[m] + rg - 1) / rg;
    chosen = ks;
    pl.ks = ks;
    pl.slice = slice;
    pl.upl = upl;
    pl.half_bytes = (int)half;
    pl.stage_bytes = (int)stage;
    // Prefer the first split that gives every SM two row tiles.
    if (batches >= 2LL * g_num_sms) break;
  }
  if (!chosen) return pl;
  const int rg = kCW / pl.ks;
  pl.total_batches = 0;
  for (int m = 0; m < j.n_mat; ++m) {
    pl.batch_begin[m] = pl.total_batches;
    pl.total_batches += (j.rows[m] + rg - 1) / rg;
  }
  int stages = (int)((smem_cap - kHeaderBytes) / pl.stage_bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return pl;
  pl.stages = stages;
  pl.smem = (size_t)kHeaderBytes + (size_t)stages * pl.stage_bytes;
  pl.grid = (int)(pl.total_batches < g_num_sms ? pl.total_batches : g_num_sms);
  pl.streaming = pl.grid > 0;
  (void)total_rows;
  return pl;
}

template <int FMT, int NP, int UPL, bool PAIR>
cudaError_t run_stream(const Params& p, const Plan& pl, cudaStream_t st) {
  auto k = gemv_kernel<FMT, NP, UPL, PAIR>;
  // Raise the dynamic shared-memory limit once per device and instantiation.
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         g_smem_optin > 0 ? g_smem_optin : (int)pl.smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  k<<<pl.grid, kThreads, pl.smem, st>>>(p);
  return cudaGetLastError();
}

template <int FMT, int NP, bool PAIR>
cudaError_t dispatch_upl(const Params& p, const Plan& pl, cudaStream_t st) {
  if constexpr (NP == 3) {
    return run_stream<FMT, NP, 1, PAIR>(p, pl, st);
  } else {
    switch (pl.upl) {
      case 1: return run_stream<FMT, NP, 1, PAIR>(p, pl, st);
      case 2: return run_stream<FMT, NP, 2, PAIR>(p, pl, st);
      case 3: return run_stream<FMT, NP, 3, PAIR>(p, pl, st);
      default: return run_stream<FMT, NP, 4, PAIR>(p, pl, st);
    }
  }
}

template <int FMT>
cudaError_t dispatch_np(const Params& p, const Plan& pl, bool pair, cudaStream_t st) {
  if (p.x) return pair ? dispatch_upl<FMT, 3, true>(p, pl, st) : dispatch_upl<FMT, 3, false>(p, pl, st);
  return pair ? dispatch_upl<FMT, 1, true>(p, pl, st) : dispatch_upl<FMT, 1, false>(p, pl, st);
}

template <int T>
cudaError_t run_fallback(const Params& p, bool pair, int64_t total_rows, cudaStream_t st) {
  device_limits();
  int64_t blocks = (total_rows + 7) / 8;
  const int64_t cap = (int64_t)(g_num_sms > 0 ? g_num_sms : 148) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (pair) gemv_fallback_kernel<T, true><<<(unsigned)blocks, 256, 0, st>>>(p);
  else gemv_fallback_kernel<T, false><<<(unsigned)blocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

int gemv_engine(const GemvJob& job) { return make_plan(job).streaming ? 0 : 1; }

cudaError_t launch_gemv(const GemvJob& j, cudaStream_t st) {
  Params p{};
  p.n_mat = j.n_mat;
  int64_t total_rows = 0;
  for (int m = 0; m < j.n_mat; ++m) {
    p.mat[m].w = j.w[m];
    p.mat[m].y = j.y[m];
    p.mat[m].rows = j.rows[m];
    total_rows += j.rows[m];
  }
  if (total_rows == 0) return cudaSuccess;
  p.up = j.up;
  p.K = (int)j.K;
  p.U = (int)(j.K / 64);
  p.row_bytes = (int)(j.K / block_len(j.dtype) * block_bytes(j.dtype));
  p.x = j.x;
  p.xq = j.xq;
  p.xs = j.xs;
  p.status = j.status;
  const bool pair = j.up != nullptr;
  const Plan pl = make_plan(j);
  if (!pl.streaming) {
    switch (j.dtype) {
      case F32: return run_fallback<F32>(p, pair, total_rows, st);
      case F16: return run_fallback<F16>(p, pair, total_rows, st);
      case Q4_K: return run_fallback<Q4_K>(p, pair, total_rows, st);
      case Q6_K: return run_fallback<Q6_K>(p, pair, total_rows, st);
      case Q8_0: return run_fallback<Q8_0>(p, pair, total_rows, st);
      case Q2_0C: return run_fallback<Q2_0C>(p, pair, total_rows, st);
      case STQ1_0: return run_fallback<STQ1_0>(p, pair, total_rows, st);
      default: return cudaErrorInvalidValue;
    }
  }
  for (int m = 0; m < j.n_mat; ++m) p.mat[m].batch_begin = pl.batch_begin[m];
  p.total_batches = pl.total_batches;
  p.ks = pl.ks;
  p.rg = kCW / pl.ks;
  p.slice = pl.slice;
  p.stages = pl.stages;
  p.half_bytes = pl.half_bytes;
  p.stage_bytes = pl.stage_bytes;
  switch (j.dtype) {
    case Q4_K: return dispatch_np<Q4_K>(p, pl, pair, st);
    case Q6_K: return dispatch_np<Q6_K>(p, pl, pair, st);
    case Q8_0: return dispatch_np<Q8_0>(p, pl, pair, st);
    case Q2_0C: return dispatch_np<Q2_0C>(p, pl, pair, st);
    case STQ1_0: return dispatch_np<STQ1_0>(p, pl, pair, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace hyq
