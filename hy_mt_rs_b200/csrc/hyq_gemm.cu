// Batched products over packed GGUF rows on the 5th-generation tensor cores
// (tcgen05 / TMEM), sm_100a.
//
// Reference behaviour: Weight::matmul with batch >= 2 (hy-mt-rs
// src/quant.rs:272-343): Y[batch, N] = X[batch, K] . W^T, where the reference
// decodes 64-row tiles to f32 and multiplies them with Candle's CPU GEMM.
//
// Tile: 128 weight rows (the MMA's M) x BN tokens (the MMA's N: 64, 128 or 256)
// x K, with D = W_tile . X_tile^T accumulated in f32 in tensor memory.
// The decoded weights (operand A) never touch shared memory: each dequant
// thread owns one weight row = one TMEM lane and stores its fp16 pairs with
// tcgen05.st, and the MMA reads A from tensor memory.  Shared memory carries
// only the activation tiles (TMA in, MMA out) and the packed weight bytes,
// which keeps it below its bandwidth at full tensor-core rate.
// Within every 64-column K step the activations are stored in the order the
// dequantizer produces weight pairs (see k_perm), so both operands agree on
// the K order without shuffles.  Roles:
//   warp 0  : TMA producer -- packed weight block columns (2-D tensor map over
//             the raw GGUF bytes: 128 rows x one block column, taken as the
//             16-byte aligned window around it) and fp16 activation tiles
//             (SWIZZLE_128B);
//   warp 1  : allocates TMEM and issues tcgen05.mma (one elected thread),
//             releasing each stage with tcgen05.commit;
//   warps 2-17: four groups of 4 warps taking K steps in turn; warp w serves
//             TMEM lanes 32*(w%4).. (its rows), decodes the packed block
//             column into the fp16 A stage in tensor memory, waits for the
//             stores and signals the stage (four steps' stores in flight
//             hide their latency); all of them then run the epilogue
//             (tcgen05.ld -> f32 stores of Y), a quarter of the columns per
//             group.
// (The 2-SM variant below keeps two groups: warps 2-9.)
// Tensor memory (512 columns): accumulator in columns [0, BN), A stage s in
// columns [BN + 32 s, BN + 32 s + 32) (128 lanes x 64 fp16).
// Operands are fp16 (both), accumulation f32.  Weights are decoded with fp16
// arithmetic from exact integer codes: 1024 + q is built in the fp16 bit
// pattern, 1024 (and the Q6_K offset 32) is subtracted exactly, and one fused
// multiply-add with the fp16 sub-block scale and min rounds the result.  The
// product stays inside the 1e-3 relative-L2 bound.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>

#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace gemm {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BK = 64;           // K per stage: one 128-byte swizzle row of fp16
constexpr int WS = 2;            // packed weight block-column stages
constexpr int kDequantWarps = 8;   // 2-SM kernel: two groups of 4 warps; each group takes every other K step
constexpr int kGroupWarps = 4;     // one thread per weight row, 64 weights per step
constexpr int kThreads = (2 + kDequantWarps) * 32;
constexpr int kGroups = 4;         // 1-SM kernel: dequant groups taking K steps in turn
constexpr int kThreads1 = (2 + kGroups * kGroupWarps) * 32;
constexpr int kTmemCols = 512;

// Activation / decoded-weight stages for a BN-token tile (shared memory
// holds S activation tiles and two packed block columns).  The split-operand
// form (below) holds two activation tiles and two A stages per step and
// keeps two accumulators: 4 stages at 128 tokens, 6 at 64.
__host__ __device__ constexpr int stages_for(int bn, bool split = false) {
  return split ? (bn == 128 ? 4 : 6) : (bn == 256 ? 5 : 8);
}

// Split-operand form (hyq_set_gemm_precision(HYQ_GEMM_F32)): every weight w
// (decoded exactly in f32, as decode_unchecked) and every activation x is
// written as hi + lo / 2^11 with hi = fp16(w) and lo = fp16((w - hi) * 2^11)
// (w - hi is exact, and the scale keeps lo a normal fp16 number), so each
// operand carries 22 significant bits.  Per 16-column K chunk three MMAs run:
// hi.hi into the main accumulator, hi.lo and lo.hi into a correction
// accumulator; the epilogue returns main + correction / 2^11.  Only the
// lo.lo term (2^-22 relative) is left out, so products reach f32 accuracy
// at three times the tensor-core instructions (Ootomo and Yokota, "Recovering
// single precision accuracy from Tensor Cores while surpassing the FP32
// theoretical peak performance", 2022, with the scaled low part).
constexpr float kSplitScale = 2048.0f;
constexpr float kSplitInv = 1.0f / 2048.0f;

// Token tile (the MMA's N) for products of m activation rows (per expert in
// expert mode): a 64-token tile for at most 64 rows, so that small batches
// do not spend tensor-core time on zero-filled rows.
inline int token_tile(int64_t m) { return m >= 256 ? 256 : m > 64 ? 128 : 64; }

// K columns of one packed block column (the unit of a weight TMA load) and
// its packed bytes per row.
__host__ __device__ constexpr int wcol_for(int fmt) {
  return fmt == Q8_0 ? 128 : fmt == Q2_0C ? 512 : 256;
}
__host__ __device__ constexpr int wbytes_for(int fmt) {
  return fmt == Q4_K ? 144 : fmt == Q6_K ? 210 : fmt == Q8_0 ? 136 : fmt == Q2_0C ? 130 : 42;
}

// Bytes per row of the packed block-column tile (TMA box inner size).
// (the 16-byte aligned window around one block column: packed bytes + skew)
__host__ __device__ constexpr int wbox_for(int fmt) {
  return fmt == Q4_K ? 144 : fmt == Q6_K ? 224 : fmt == Q8_0 ? 160 : fmt == Q2_0C ? 144 : 64;
}

struct Params {
  int K, N, M;
  int steps_per_split;  // K steps of one split-K slice (a whole number of block columns)
  int row_bytes;
  int wcol;             // K columns per packed block-column tile
  int wbox;             // bytes per row of that tile (TMA box inner size)
  int wbytes;           // packed bytes of one row per block column
  int g;                // rows per 16-byte-aligned pitch of the weight tensor map (1, 2, 4 or 8)
  float* y;             // split-K partials [splits, M, N] (N = all matrices' columns), or unused
  unsigned* status;
  // Matrices sharing the activations (QKV): row tile t belongs to matrix m
  // for seg_tile0[m] <= t < seg_tile0[m + 1]; its output is ys[m] [M,
  // seg_rows[m]], or columns seg_col0[m].. of the split-K partials.
  int n_seg;
  int seg_tile0[4];
  int seg_rows[3];
  int seg_col0[3];
  float* ys[3];
  // Gate/up pair (matmul_gate_up_silu): a 128-row tile holds 64 gate and the
  // same 64 up rows, interleaved by 16 in each 32-lane TMEM quarter; the
  // output is silu(gate x) * (up x) in ys[0] [M, seg_rows[0]] (split-K:
  // gate partials in columns 0.., up partials in columns seg_rows[0]..).
  int gate_up;
  // Expert mode: CTA x serves expert x / expert_tiles, whose weight rows
  // start at e * expert_rows and whose activation rows are expert_off[e] ..
  // expert_off[e + 1]; a CTA whose token tile holds none of them returns.
  const int32_t* expert_off;
  int expert_tiles;
  int expert_rows;
  // Tail split (tail_z > 1; 1-SM kernel, 1-D grid): CTAs [0, tail_begin)
  // take whole tiles t = CTA index (row tile t % tiles_x, token tile t /
  // tiles_x); the last tiles t >= tail_begin, which would run as a thin last
  // wave, are cut into tail_z K-slices of tail_steps steps, one CTA each.  A
  // slice writes its partial tile to tail_part [tail tile][slice][BN tokens]
  // [BM tile rows] for tail_reduce_kernel.
  int tail_z;
  int tail_begin;
  int tail_steps;
  int tiles_x;
  float* tail_part;
};

template <int FMT, int BN, bool SPLIT = false>
struct Smem {
  static constexpr int S = stages_for(BN, SPLIT);
  static constexpr int x_half = BN * 128;                   // one fp16 activation tile
  static constexpr int x_tile = x_half * (SPLIT ? 2 : 1);   // hi tile, then the lo tile
  // offsets from the 1024-aligned base
  static constexpr int x = 0;
  static constexpr int w = x + S * x_tile;
  static constexpr int w_stage = (BM * wbox_for(FMT) + 1023) / 1024 * 1024;
  static constexpr int bars = w + WS * w_stage;
  // barriers: xfull[S], afull[S], empty[S], wfull[WS], wempty[WS], accfull
  static constexpr int n_bars = 3 * S + 2 * WS + 1;
  static constexpr int misc = bars + 8 * n_bars;  // tmem address, abort flag
  static constexpr int total = misc + 16;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major, SWIZZLE_128B: 8-row groups 1024 bytes apart (SBO), LBO unused
  // (1), descriptor version 1, layout type 2.
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (TMEM) += A (TMEM, 128 lanes x 16 fp16) . B (shared memory descriptor)^T
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane <- o[0..31].
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&o)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3]), "r"(o[4]), "r"(o[5]), "r"(o[6]), "r"(o[7]), "r"(o[8]), "r"(o[9]),
      "r"(o[10]), "r"(o[11]), "r"(o[12]), "r"(o[13]), "r"(o[14]), "r"(o[15]), "r"(o[16]), "r"(o[17]), "r"(o[18]),
      "r"(o[19]), "r"(o[20]), "r"(o[21]), "r"(o[22]), "r"(o[23]), "r"(o[24]), "r"(o[25]), "r"(o[26]), "r"(o[27]),
      "r"(o[28]), "r"(o[29]), "r"(o[30]), "r"(o[31])
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void st_s128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
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

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// K order inside one 64-column step.  Slot pair P = 16h + 4t + j (h: which
// thread of the row, t: 32-bit word, j: pair inside the word) holds columns
// c + T[j][0], c + T[j][1] with c = 16h + 4t; T is the order in which pairs of
// codes fall out of a 32-bit word with (w >> 4k) & 0x000F000F.
//
// Q8_0 keeps the natural order.  Q2_0C: word t of the step's 16 code bytes,
// code k of its bytes (0, 2) or (1, 3) (ab = 0 / 1): pair P = 8t + 2k + ab
// holds columns 16t + 4ab + k and + 8.  STQ1_0: lane p of the patterns of
// groups 4i + (0, 2) or (1, 3): pair P = 8i + 2p + ab holds columns
// 4i + ab + 16p and + 2.
__host__ __device__ constexpr int k_perm(int fmt, int slot) {
  const int P = slot >> 1, e = slot & 1;
  if (fmt == Q8_0) return slot;
  if (fmt == Q2_0C) return 16 * (P >> 3) + 4 * (P & 1) + ((P >> 1) & 3) + 8 * e;
  if (fmt == STQ1_0) return 4 * (P >> 3) + (P & 1) + 2 * e + 16 * ((P >> 1) & 3);
  const int h = P >> 4, t = (P >> 2) & 3, j = P & 3;
  const int c = 16 * h + 4 * t;
  // Q4_K, j = 0..3: (0,2) (32,34) (1,3) (33,35)  [low / high nibbles]
  // Q6_K, j = 0..3: (0,2) (1,3) (32,34) (33,35)  [plane p0 / plane p0+1]
  const int off = fmt == Q4_K ? (j & 1) * 32 + (j >> 1) : (j >> 1) * 32 + (j & 1);
  return c + off + 2 * e;
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t h2_splat(float f) {
  __half h = __float2half_rn(f);
  const uint32_t u = *reinterpret_cast<unsigned short*>(&h);
  return u | (u << 16);
}

__device__ __forceinline__ uint2 ld_s64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

// Decode one row's 64 weights of K step `j4` of the block column (the row's
// bytes start at `row`) into 32 fp16x2 words in k_perm order: word P holds
// slot pair P, i.e. TMEM column P of the row's A stage.
template <int FMT>
__device__ __forceinline__ void decode64(uint32_t row, int j4, uint32_t (&o)[32]) {
  constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
  if constexpr (FMT == Q8_0) {
    // Step j4 of a 4-block column: blocks 2 j4, 2 j4 + 1 (quant.rs:2413-2418,
    // d * q).  Flipping the sign bit gives q + 128 in 0..255; PRMT places two
    // such bytes under fp16 1024's exponent; subtracting 1152 leaves q.
    const uint32_t k1152 = 0x64806480u;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const uint32_t blk = row + (2 * j4 + b) * 34;
      const uint32_t d = ld_s16(blk);
      const uint32_t d2 = d | (d << 16);
      uint32_t w[8];
      ld_s_words<8>(blk + 2, w);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t u = w[t] ^ 0x80808080u;
        o[16 * b + 2 * t] = hmul2_u(hsub2_u(prmt_b32(u, 0x64646464u, 0x4140u), k1152), d2);
        o[16 * b + 2 * t + 1] = hmul2_u(hsub2_u(prmt_b32(u, 0x64646464u, 0x4342u), k1152), d2);
      }
    }
  } else if constexpr (FMT == Q2_0C) {
    // One 512-weight block per block column (quant.rs:2419-2432: (2c - 3) d,
    // four codes per byte); step j4 = code bytes 16 j4 .. + 15.
    const uint32_t d = ld_s16(row);
    const uint32_t d2 = d | (d << 16);
    uint32_t w[4];
    ld_s_words<4>(row + 2 + 16 * j4, w);
    const uint32_t k2 = 0x40004000u, km3 = 0xC200C200u;  // fp16 2, -3
#pragma unroll
    for (int t = 0; t < 4; ++t) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int ab = 0; ab < 2; ++ab) {
          const uint32_t v = ((w[t] >> (2 * k + 8 * ab)) & 0x00030003u) | kMagic;  // 1024 + c
          const uint32_t c = hsub2_u(v, kMagic);
          o[8 * t + 2 * k + ab] = hmul2_u(hfma2_u(c, k2, km3), d2);  // (2c - 3) d, rounded once
        }
      }
    }
  } else if constexpr (FMT == STQ1_0) {
    // One 256-weight block per block column; step j4 = chunk j4 (16 groups,
    // columns 64 j4 + g % 16 + 16 p): (digit - 1) d (quant.rs:1103-1123).
    const uint32_t d = ld_s16(row + 40);
    const uint32_t d2 = d | (d << 16);
    uint32_t nb[2];
    ld_s_words<2>(row + 8 * j4, nb);
    const uint32_t sbits = ld_s16(row + 32 + 2 * j4);
    const uint32_t k1025 = 0x64016401u;  // fp16 1025
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t hw = (i & 1) ? (nb[i >> 1] >> 16) : (nb[i >> 1] & 0xffffu);
      const uint32_t cb = stq_patterns4(hw, (sbits >> (4 * i)) & 15u);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int ab = 0; ab < 2; ++ab) {
          const uint32_t v = ((cb >> (2 * p + 8 * ab)) & 0x00030003u) | kMagic;  // 1024 + digit
          o[8 * i + 2 * p + ab] = hmul2_u(hsub2_u(v, k1025), d2);
        }
      }
    }
  } else if constexpr (FMT == Q4_K) {
    const int g = j4;  // 64-column group of the 256-column block
    const uint4 hd = ld_s128(row);
    const float d = half_to_f32(hd.x & 0xffffu), dmin = half_to_f32(hd.x >> 16);
    uint32_t sm[2], mm[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = 2 * g + hh;
      uint32_t sc, mn;
      if (j < 4) {
        sc = (hd.y >> (8 * j)) & 63u;
        mn = (hd.z >> (8 * j)) & 63u;
      } else {
        const int k = j - 4;
        const uint32_t hi = (hd.w >> (8 * k)) & 0xffu;
        sc = (hi & 15u) | ((((hd.y >> (8 * k)) & 0xffu) >> 6) << 4);
        mn = (hi >> 4) | ((((hd.z >> (8 * k)) & 0xffu) >> 6) << 4);
      }
      sm[hh] = h2_splat(d * (float)sc);
      mm[hh] = h2_splat(-(dmin * (float)mn));
    }
    // 32 quant bytes: low nibbles -> columns 0..31, high nibbles -> 32..63
    const uint4 q0 = ld_s128(row + 16 + 32 * g), q1 = ld_s128(row + 32 + 32 * g);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t v = ((w[c] >> (4 * j)) & 0x000f000fu) | kMagic;  // 1024 + q, exact
        const int hi = j & 1;                                          // high nibble: sub-block 2g+1
        o[4 * c + j] = hfma2_u(hsub2_u(v, kMagic), sm[hi], mm[hi]);
      }
    }
  } else {  // Q6_K
    static_assert(FMT == Q6_K, "format without a GEMM decoder");
    const int chunk = j4 >> 1, p0 = 2 * (j4 & 1);
    const int nsh = (p0 >> 1) * 4;
    uint32_t A[8], B[8], H[8];
    ld_s_words<8>(row + chunk * 64, A);       // plane p0 (low or high nibbles)
    ld_s_words<8>(row + chunk * 64 + 32, B);  // plane p0+1
    ld_s_words<8>(row + 128 + chunk * 32, H);
    const float d = half_to_f32(ld_s16(row + 208));
    const uint32_t sc0 = ld_s16(row + 192 + chunk * 8 + 2 * p0);      // plane p0, halves 0/1
    const uint32_t sc1 = ld_s16(row + 192 + chunk * 8 + 2 * p0 + 2);  // plane p0+1
    uint32_t sv[2][2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      sv[0][hh] = h2_splat(d * (float)(int8_t)((sc0 >> (8 * hh)) & 0xffu));
      sv[1][hh] = h2_splat(d * (float)(int8_t)((sc1 >> (8 * hh)) & 0xffu));
    }
    const uint32_t k1056 = 0x64206420u;  // fp16 1056 = 1024 + 32
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int hh = c >> 2;  // columns 0..15 use half 0, 16..31 half 1
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t src = j < 2 ? A[c] : B[c];
        const int bsh = 8 * (j & 1);          // bytes (0,2) or (1,3)
        const int hsh = 2 * (p0 + (j >> 1));  // qh bits of this plane
        const uint32_t lo = ((src >> (nsh + bsh)) & 0x000f000fu) | kMagic;
        const uint32_t hb = (H[c] >> (hsh + bsh)) & 0x00030003u;
        const uint32_t v = lo | (hb << 4);  // 1024 + q6, exact
        o[4 * c + j] = hmul2_u(hsub2_u(v, k1056), sv[j >> 1][hh]);
      }
    }
  }
}

// Split-operand decode: the row's 64 weights of K step j4 as decode64
// orders them, each as hi (word P of `hi`) plus lo / 2^11 (word P of `lo`),
// where hi + lo / 2^11 equals the reference's f32 weight (decode_unchecked)
// to 22 significant bits.
//   Q8_0, Q2_0C: the weight is an integer code k (|k| <= 128) times the fp16
//     block scale d; hi = fp16(k d) and the residual k d - hi is a multiple of
//     ulp(d) with at most 8 significant bits, so fma.rn.f16x2(k, d, -hi) is
//     exact and lo = 2^11 times it: hi + lo / 2^11 = k d exactly.
//   STQ1_0: k is -1, 0 or 1, so hi = k d exactly and lo = 0 (no lo MMA).
//   Q4_K, Q6_K: the reference rounds in f32 (d sc q - dmin m, d sc (q - 32)),
//     so the weight is computed in f32 with those roundings and split.
__device__ __forceinline__ void split2(float a, float b, uint32_t& h, uint32_t& l) {
  const __half2 hh = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(hh);
  h = *reinterpret_cast<const uint32_t*>(&hh);
  l = pack_h2(__fmul_rn(__fsub_rn(a, hf.x), kSplitScale), __fmul_rn(__fsub_rn(b, hf.y), kSplitScale));
}

// exact f32 of the 16-bit integers in the two halves of v (each < 2^16), less `off`
__device__ __forceinline__ float2 u16x2_to_f32(uint32_t v, float off) {
  return make_float2(__fsub_rn(__uint_as_float((v & 0xffffu) | 0x4B000000u), 8388608.0f + off),
                     __fsub_rn(__uint_as_float((v >> 16) | 0x4B000000u), 8388608.0f + off));
}

template <int FMT>
__device__ __forceinline__ void decode64_split(uint32_t row, int j4, uint32_t (&hi)[32], uint32_t (&lo)[32]) {
  constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024 in both halves
  constexpr uint32_t kNeg = 0x80008000u;
  constexpr uint32_t k2048 = 0x68006800u;   // fp16 2^11 in both halves
  if constexpr (FMT == Q8_0) {
    const uint32_t k1152 = 0x64806480u;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const uint32_t blk = row + (2 * j4 + b) * 34;
      const uint32_t d = ld_s16(blk);
      const uint32_t d2 = d | (d << 16);
      uint32_t w[8];
      ld_s_words<8>(blk + 2, w);
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t u = w[t] ^ 0x80808080u;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t q = hsub2_u(prmt_b32(u, 0x64646464u, h ? 0x4342u : 0x4140u), k1152);
          const uint32_t x = hmul2_u(q, d2);
          hi[16 * b + 2 * t + h] = x;
          lo[16 * b + 2 * t + h] = hmul2_u(hfma2_u(q, d2, x ^ kNeg), k2048);
        }
      }
    }
  } else if constexpr (FMT == Q2_0C) {
    const uint32_t d = ld_s16(row);
    const uint32_t d2 = d | (d << 16);
    uint32_t w[4];
    ld_s_words<4>(row + 2 + 16 * j4, w);
    const uint32_t k2 = 0x40004000u, km3 = 0xC200C200u;  // fp16 2, -3
#pragma unroll
    for (int t = 0; t < 4; ++t) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
#pragma unroll
        for (int ab = 0; ab < 2; ++ab) {
          const uint32_t v = ((w[t] >> (2 * k + 8 * ab)) & 0x00030003u) | kMagic;
          const uint32_t c = hfma2_u(hsub2_u(v, kMagic), k2, km3);  // 2c - 3, exact
          const uint32_t x = hmul2_u(c, d2);
          hi[8 * t + 2 * k + ab] = x;
          lo[8 * t + 2 * k + ab] = hmul2_u(hfma2_u(c, d2, x ^ kNeg), k2048);
        }
      }
    }
  } else if constexpr (FMT == STQ1_0) {
    decode64<STQ1_0>(row, j4, hi);  // (digit - 1) d is exact in fp16
#pragma unroll
    for (int P = 0; P < 32; ++P) lo[P] = 0u;
  } else if constexpr (FMT == Q4_K) {
    const int g = j4;
    const uint4 hd = ld_s128(row);
    const float d = half_to_f32(hd.x & 0xffffu), dmin = half_to_f32(hd.x >> 16);
    float sm[2], mm[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int j = 2 * g + hh;
      uint32_t sc, mn;
      if (j < 4) {
        sc = (hd.y >> (8 * j)) & 63u;
        mn = (hd.z >> (8 * j)) & 63u;
      } else {
        const int k = j - 4;
        const uint32_t hi8 = (hd.w >> (8 * k)) & 0xffu;
        sc = (hi8 & 15u) | ((((hd.y >> (8 * k)) & 0xffu) >> 6) << 4);
        mn = (hi8 >> 4) | ((((hd.z >> (8 * k)) & 0xffu) >> 6) << 4);
      }
      sm[hh] = __fmul_rn(d, (float)sc);     // exact
      mm[hh] = __fmul_rn(dmin, (float)mn);  // exact
    }
    const uint4 q0 = ld_s128(row + 16 + 32 * g), q1 = ld_s128(row + 32 + 32 * g);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int h = j & 1;
        const float2 q = u16x2_to_f32((w[c] >> (4 * j)) & 0x000f000fu, 0.0f);
        split2(__fsub_rn(__fmul_rn(sm[h], q.x), mm[h]), __fsub_rn(__fmul_rn(sm[h], q.y), mm[h]), hi[4 * c + j],
               lo[4 * c + j]);
      }
    }
  } else {  // Q6_K
    static_assert(FMT == Q6_K, "format without a split decoder");
    const int chunk = j4 >> 1, p0 = 2 * (j4 & 1);
    const int nsh = (p0 >> 1) * 4;
    uint32_t A[8], B[8], H[8];
    ld_s_words<8>(row + chunk * 64, A);
    ld_s_words<8>(row + chunk * 64 + 32, B);
    ld_s_words<8>(row + 128 + chunk * 32, H);
    const float d = half_to_f32(ld_s16(row + 208));
    const uint32_t sc0 = ld_s16(row + 192 + chunk * 8 + 2 * p0);
    const uint32_t sc1 = ld_s16(row + 192 + chunk * 8 + 2 * p0 + 2);
    float sv[2][2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      sv[0][hh] = __fmul_rn(d, (float)(int8_t)((sc0 >> (8 * hh)) & 0xffu));  // exact
      sv[1][hh] = __fmul_rn(d, (float)(int8_t)((sc1 >> (8 * hh)) & 0xffu));
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int hh = c >> 2;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t src = j < 2 ? A[c] : B[c];
        const int bsh = 8 * (j & 1);
        const int hsh = 2 * (p0 + (j >> 1));
        const uint32_t q6 = ((src >> (nsh + bsh)) & 0x000f000fu) | (((H[c] >> (hsh + bsh)) & 0x00030003u) << 4);
        const float2 q = u16x2_to_f32(q6, 32.0f);  // q - 32
        const float s = sv[j >> 1][hh];
        split2(__fmul_rn(s, q.x), __fmul_rn(s, q.y), hi[4 * c + j], lo[4 * c + j]);
      }
    }
  }
}

template <int FMT, int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads1, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w0, const __grid_constant__ CUtensorMap tmap_w1,
                const __grid_constant__ CUtensorMap tmap_w2, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_xlo, const __grid_constant__ Params p) {
  using L = Smem<FMT, BN, SPLIT>;
  constexpr int S = L::S;
  // Tensor memory: the accumulator(s) in columns [0, kAcc), A stage s (hi,
  // and for SPLIT the scaled lo after it) at kAcc + kAStage * s.
  constexpr int kAcc = SPLIT ? 2 * BN : BN;
  constexpr int kAStage = SPLIT ? 64 : 32;
  // With an even number of stages the MMA thread releases them in pairs:
  // one tcgen05.commit costs about as much issue time as two MMAs, so one
  // commit per two K steps (on the pair's first barrier) saves it half the
  // time.  Waiters of stage s wait on barrier rel(s).
  constexpr bool kPairRelease = S % 2 == 0;
  auto rel = [](int s) { return kPairRelease ? (s & ~1) : s; };
  static_assert(kAcc + kAStage * S <= kTmemCols, "accumulators and A stages exceed tensor memory");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  const uint32_t raw_s = smem_addr(smem_raw);
  const uint32_t base = (raw_s + 1023u) & ~1023u;
  uint8_t* base_g = smem_raw + (base - raw_s);
  const uint32_t bars = base + L::bars;
  auto xfull = [&](int s) { return bars + 8 * s; };
  auto afull = [&](int s) { return bars + 8 * (S + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * S + s); };
  auto wfull = [&](int s) { return bars + 8 * (3 * S + s); };
  auto wempty = [&](int s) { return bars + 8 * (3 * S + WS + s); };
  const uint32_t accfull = bars + 8 * (3 * S + 2 * WS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_g + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_g + L::misc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 32) {
    // the descriptors are kernel parameters: fetch them during the set-up
    prefetch_tmap(&tmap_x);
    if (SPLIT) prefetch_tmap(&tmap_xlo);
    prefetch_tmap(&tmap_w0);
    if (p.n_seg > 1 || p.gate_up) prefetch_tmap(&tmap_w1);
    if (p.n_seg > 2) prefetch_tmap(&tmap_w2);
  }
  if (p.expert_off) grid_dependency_wait();  // the expert offsets come from the previous grid
  // this CTA's row tile, token tile and K-slice
  int bx = (int)blockIdx.x, by = (int)blockIdx.y, bz = (int)blockIdx.z;
  int tail = -1;  // tail split: index of this CTA's tail tile
  if (p.tail_z > 1) {
    int t = bx;
    if (t >= p.tail_begin) {
      const int j = t - p.tail_begin;
      tail = j / p.tail_z;
      bz = j - tail * p.tail_z;
      t = p.tail_begin + tail;
    }
    by = t / p.tiles_x;
    bx = t - by * p.tiles_x;
  }
  int tok0 = by * BN;
  int tok_end = p.M;  // activation rows of this tile end here
  // row tile -> matrix and its first row (a gate/up tile covers 64 rows of each)
  int seg = 0;
  while (seg + 1 < p.n_seg && bx >= p.seg_tile0[seg + 1]) ++seg;
  const int tile_rows = p.gate_up ? BM / 2 : BM;
  int row0 = (bx - p.seg_tile0[seg]) * tile_rows;
  int wrow0 = row0;  // first row in the weight tensor map
  if (p.expert_off) {
    const int e = bx / p.expert_tiles;
    const int t_end = p.expert_off[e + 1];
    tok0 = p.expert_off[e] + by * BN;
    if (tok0 >= t_end) return;  // nothing allocated or armed yet
    tok_end = t_end;
    row0 = (bx % p.expert_tiles) * tile_rows;
    wrow0 = e * p.expert_rows + row0;
  }
  constexpr int steps_per_w = wcol_for(FMT) / BK;  // p.wcol
  // split-K slice of this CTA: K steps [kbeg, kbeg + nk)
  const int slice_steps = tail >= 0 ? p.tail_steps : p.steps_per_split;
  const int kbeg = bz * slice_steps;
  const int nk_all = p.K / BK;
  const int nk = min(slice_steps, nk_all - kbeg);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(xfull(s), 1);
      mbar_init(afull(s), kGroupWarps);
      mbar_init(empty(s), 1);
    }
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull(s), 1);
      // every group with a K step in the block column releases it
      mbar_init(wempty(s), min(kGroups, p.wcol / BK) * kGroupWarps);
    }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    // TMEM: accumulator (BN columns) and the A stages.  One CTA per SM (the
    // shared-memory footprint allows no second one), so all 512 columns.
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // set-up above overlaps the previous grid's tail (launch_ex); data after
  grid_dependency_wait();
  allow_dependents_launch();

  if (warp == 0) {
    // ------------------------------ TMA producer ----------------------------
    if (lane == 0) {
      int issued_x = 0, issued_w = 0;
      bool ok = true;
      for (int ks = 0; ks < nk && ok; ++ks) {
        if (ks % steps_per_w == 0) {
          const int wb = ks / steps_per_w, ws = wb % WS;
          if (wb >= WS && !mbar_wait(wempty(ws), ((wb / WS) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          // The tensor map sees g rows as one pitch (a multiple of 16 bytes):
          // one load per row class j fetches rows row0 + j, + j + g, ...;
          // a gate/up tile loads 64 rows of each matrix.
          const int64_t kb = (kbeg + ks) / steps_per_w;
          mbar_arrive_expect_tx(wfull(ws), (uint32_t)(BM * p.wbox));
          for (int mt = 0; mt < (p.gate_up ? 2 : 1); ++mt) {
            const int mi = p.gate_up ? mt : seg;
            const CUtensorMap* map = mi == 0 ? &tmap_w0 : (mi == 1 ? &tmap_w1 : &tmap_w2);
            for (int j = 0; j < p.g; ++j) {
              const int x0 = (int)(((int64_t)j * p.row_bytes + kb * p.wbytes) & ~int64_t(15));
              tma_load_2d(base + L::w + ws * L::w_stage + (mt * tile_rows + j * (tile_rows / p.g)) * p.wbox, map,
                          x0, wrow0 / p.g, wfull(ws));
            }
          }
          ++issued_w;
        }
        const int s = ks % S;
        if (ks >= S && !mbar_wait(empty(rel(s)), ((ks / S) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(xfull(s), (uint32_t)L::x_tile);
        tma_load_2d(base + L::x + s * L::x_tile, &tmap_x, (kbeg + ks) * BK, tok0, xfull(s));
        if (SPLIT) tma_load_2d(base + L::x + s * L::x_tile + L::x_half, &tmap_xlo, (kbeg + ks) * BK, tok0, xfull(s));
        ++issued_x;
      }
      if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_EMPTY);
        *abort_flag = 1;
      }
      // Drain: no copy may land after this CTA is gone.
      for (int k = (issued_x > S ? issued_x - S : 0); k < issued_x; ++k)
        if (!mbar_wait(xfull(k % S), (k / S) & 1, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
      for (int k = (issued_w > WS ? issued_w - WS : 0); k < issued_w; ++k)
        if (!mbar_wait(wfull(k % WS), (k / WS) & 1, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    // idesc: f32 accumulate, fp16 A and B, both K-major, N = BN, M = BM.
    const uint32_t idesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    int ks = 0;
    for (; ks < nk; ++ks) {
      const int s = ks % S;
      const uint32_t par = (ks / S) & 1;
      if (!mbar_wait(afull(s), par, abort_flag) || !mbar_wait(xfull(s), par, abort_flag)) {
        if (lane == 0) atomicOr(p.status, DEV_TIMEOUT_FULL);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a0 = tmem + (uint32_t)(kAcc + kAStage * s);
        const uint32_t b0 = base + L::x + s * L::x_tile;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint32_t acc = (ks > 0 || k > 0) ? 1u : 0u;
          umma_f16_ts(tmem, a0 + 8 * k, sw128_desc(b0 + 32 * k), idesc, acc);
          if constexpr (SPLIT) {
            // correction accumulator: hi.lo + lo.hi (STQ1_0 weights have no lo part)
            umma_f16_ts(tmem + BN, a0 + 8 * k, sw128_desc(b0 + L::x_half + 32 * k), idesc, acc);
            if constexpr (FMT != STQ1_0) umma_f16_ts(tmem + BN, a0 + 32 + 8 * k, sw128_desc(b0 + 32 * k), idesc, 1u);
          }
        }
        if (!kPairRelease || (ks & 1) || ks == nk - 1) umma_commit(empty(rel(s)));
      }
      __syncwarp();
    }
    // All issued MMAs have completed once accfull flips.
    if (lane == 0) umma_commit(accfull);
    __syncwarp();
  } else {
    // --------------------------- dequant + epilogue ---------------------------
    const int grp = (warp - 2) / kGroupWarps;  // K steps grp, grp + kGroups, ...
    // A warp reaches only TMEM lanes 32*(warp%4)..+31: those are its rows.
    const int r = (warp & 3) * 32 + lane;  // weight row of the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    // TMEM lane r holds row rl of matrix mt (gate/up: lanes 16..31 of each
    // quarter are the up rows); that row is row rl / g of row class rl % g
    // in shared memory, its bytes `skew` into the class's aligned window.
    constexpr int kSpw = steps_per_w;  // K steps per block column
    const int gsh = p.g == 1 ? 0 : p.g == 2 ? 1 : p.g == 4 ? 2 : 3;  // g = 1, 2, 4 or 8
    const int mt = p.gate_up ? ((r & 31) >> 4) : 0;
    const int rl = p.gate_up ? 16 * (r >> 5) + (r & 15) : r;
    const int jc = rl & (p.g - 1);
    const uint32_t row_off = (uint32_t)((mt * tile_rows + jc * (tile_rows >> gsh) + (rl >> gsh)) * p.wbox);
    const int64_t skew0 = (int64_t)jc * p.row_bytes;
    const int64_t kb0 = kbeg / kSpw;  // split slices are whole block columns
    for (int ks = grp; ks < nk; ks += kGroups) {
      const int wb = ks / kSpw, ws = wb % WS;
      bool ok = true;
      // first step of this block column that this group handles
      if (ks % kSpw < kGroups) ok = mbar_wait(wfull(ws), (wb / WS) & 1, abort_flag);
      const int s = ks % S;
      if (ok && ks >= S) ok = mbar_wait(empty(rel(s)), ((ks / S) - 1) & 1, abort_flag);
      if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();  // the MMAs that read this A stage are complete
      const int skew = (int)((skew0 + (kb0 + wb) * wbytes_for(FMT)) & 15);
      const uint32_t rowp = base + L::w + ws * L::w_stage + row_off + skew;
      if constexpr (SPLIT) {
        uint32_t hi[32], lo[32];
        decode64_split<FMT>(rowp, ks % kSpw, hi, lo);
        tmem_st32(tmem + lane_base + (uint32_t)(kAcc + kAStage * s), hi);
        if constexpr (FMT != STQ1_0) tmem_st32(tmem + lane_base + (uint32_t)(kAcc + kAStage * s + 32), lo);
      } else {
        uint32_t o[32];
        decode64<FMT>(rowp, ks % kSpw, o);
        tmem_st32(tmem + lane_base + (uint32_t)(kAcc + kAStage * s), o);
      }
      // Every writer waits for its tensor-memory stores and orders them
      // before the barrier; the warp then signals the stage once.
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(afull(s));
        // last step of this block column that this group handles
        if (ks % kSpw >= kSpw - kGroups || ks + kGroups >= nk) mbar_arrive(wempty(ws));
      }
    }
    // Epilogue: all dequant warps; warp w reads TMEM lanes 32*(w%4) .. +31,
    // group g (warps 2 + 4g ..) the columns [g BN / kGroups, (g + 1) BN /
    // kGroups), 32 at a time (two loads, one wait); columns past the tile's
    // tokens are skipped.
    {
      const bool ok = mbar_wait(accfull, 0, nullptr);
      tc_fence_after();
      if (ok && !*abort_flag) {
        const int q = warp & 3;
        constexpr int kCols = BN / kGroups;
        static_assert(kCols % 32 == 0 || kCols == 16, "16- or 32-column epilogue batches");
        // SPLIT: 16 columns of each accumulator per wait
        constexpr int kBatch = (kCols < 32 || SPLIT) ? 16 : 32;
        const int cbeg = grp * kCols;
        const int cend = min(cbeg + kCols, tok_end - tok0);
        const bool split = p.y != nullptr;
        const int rows_m = p.seg_rows[seg];
        float* yz = split ? p.y + (size_t)bz * p.M * p.N : nullptr;
        // tail slice: this CTA's partial tile, [BN tokens][BM tile rows]
        float* tp = tail >= 0 ? p.tail_part + ((size_t)tail * p.tail_z + bz) * BN * BM : nullptr;
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += kBatch) {
          uint32_t v[32];
          const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                "=r"(v[15])
              : "r"(ta));
          if constexpr (kBatch == 32 || SPLIT) {
            // the next 16 columns, or (SPLIT) the same 16 of the correction accumulator
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                "%13, %14, %15}, [%16];"
                : "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
                  "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
                  "=r"(v[30]), "=r"(v[31])
                : "r"(ta + (SPLIT ? (uint32_t)BN : 16u)));
          }
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if constexpr (SPLIT) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              v[i] = __float_as_uint(__fadd_rn(__uint_as_float(v[i]), __fmul_rn(__uint_as_float(v[16 + i]), kSplitInv)));
          }
          if (tp) {
            // TMEM lane 32 q + lane is tile row 32 q + lane (gate/up: lanes
            // 16..31 of each quarter are up rows, kept at tile rows 64..)
            const int lr = p.gate_up ? 64 * (lane >> 4) + 16 * q + (lane & 15) : 32 * q + lane;
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
              if (tok0 + c0 + i < tok_end) tp[(size_t)(c0 + i) * BM + lr] = __uint_as_float(v[i]);
          } else if (!p.gate_up) {
            const int row = row0 + 32 * q + lane;
            if (row < rows_m) {
#pragma unroll
              for (int i = 0; i < kBatch; ++i) {
                const int tok = tok0 + c0 + i;
                if (tok >= tok_end) continue;
                if (split) yz[(size_t)tok * p.N + p.seg_col0[seg] + row] = __uint_as_float(v[i]);
                else p.ys[seg][(size_t)tok * rows_m + row] = __uint_as_float(v[i]);
              }
            }
          } else {
            // lanes 0..15: gate rows, lanes 16..31: the same up rows
            const int hi = lane >> 4;
            const int row = row0 + 16 * q + (lane & 15);
            float u[kBatch];
#pragma unroll
            for (int i = 0; i < kBatch; ++i) u[i] = __shfl_down_sync(0xffffffffu, __uint_as_float(v[i]), 16);
            if (row < rows_m) {
#pragma unroll
              for (int i = 0; i < kBatch; ++i) {
                const int tok = tok0 + c0 + i;
                if (tok >= tok_end) continue;
                if (split) {
                  yz[(size_t)tok * p.N + hi * rows_m + row] = __uint_as_float(v[i]);
                } else if (!hi) {
                  // silu(g) * u = g / (1 + e^-g) * u (quant.rs:573-574), with
                  // the fast exponential and division when the operands are
                  // fp16; SPLIT as the batch-1 products compute it
                  const float g = __uint_as_float(v[i]);
                  p.ys[0][(size_t)tok * rows_m + row] =
                      SPLIT ? (g / (1.0f + expf(-g))) * u[i] : __fdividef(g, 1.0f + __expf(-g)) * u[i];
                }
              }
            }
          }
        }
      } else if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes a 256-row x 256-token tile
// with tcgen05.mma.cta_group::2 (M = 256, N = 256).  CTA rank r holds weight
// rows [128 r, 128 r + 128) -- its own packed block columns, dequant warps
// and TMEM lanes (A operand and accumulator) -- and tokens [128 r, 128 r +
// 128) of the activation tile in its shared memory (half of the MMA's B).
// Each SM therefore streams half the activation bytes of the 1-SM tile per
// flop.  Rank 0 issues the MMAs; its barriers collect both CTAs' readiness:
//   xfull[s]: armed by rank 0 for both halves; each CTA's TMA load completes
//             its bytes on rank 0's barrier (cta_group::2 form, no multicast);
//   afull[s]: 4 dequant warps of each CTA arrive (rank 1 remotely);
//   empty[s], accfull: tcgen05.commit with a CTA mask arrives in both CTAs.
// ---------------------------------------------------------------------------
constexpr int kPairStages = 8;
constexpr int kPairHalf = 128;  // tokens per CTA (half of the MMA's N)

template <int FMT>
struct Smem2 {
  static constexpr int S = kPairStages;
  static constexpr int x_tile = kPairHalf * 128;  // 128 tokens x 64 fp16
  static constexpr int x = 0;
  static constexpr int w = x + S * x_tile;
  static constexpr int w_stage = (BM * wbox_for(FMT) + 1023) / 1024 * 1024;
  static constexpr int bars = w + WS * w_stage;
  static constexpr int n_bars = 3 * S + 2 * WS + 1;
  static constexpr int misc = bars + 8 * n_bars;
  static constexpr int total = misc + 16;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on the barrier at the same offset in CTA `rank` of the cluster.
// The data it publishes (tensor-memory stores) is ordered by tcgen05.wait::st
// and the tcgen05 thread-sync fences, so the arrive keeps the default
// CTA-scope release and needs no cluster-wide fence.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t local_bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(map_to_rank(local_bar, rank)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
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

// mbar_wait for barriers that receive arrivals from the other CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, const volatile int* abort) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

// TMA load into this CTA's shared memory whose bytes complete on the barrier
// of rank 0 (cluster address `bar0`).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar0) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar0)
      : "memory");
}

__device__ __forceinline__ void umma_f16_ts_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs once the issued MMAs end.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((unsigned short)3)
      : "memory");
}

template <int FMT>
__global__ void __launch_bounds__(kThreads1, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ Params p) {
  using L = Smem2<FMT>;
  constexpr int S = L::S;
  constexpr int NACC = 2 * kPairHalf;  // accumulator columns (the pair's tokens)
  // stages released in pairs (one commit per two K steps), as gemm_kernel
  static_assert(S % 2 == 0, "paired stage release");
  auto rel = [](int s) { return s & ~1; };
  static_assert(NACC + 32 * S <= kTmemCols, "accumulator and A stages exceed tensor memory");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_s = smem_addr(smem_raw);
  const uint32_t base = (raw_s + 1023u) & ~1023u;
  uint8_t* base_g = smem_raw + (base - raw_s);
  const uint32_t bars = base + L::bars;
  auto xfull = [&](int s) { return bars + 8 * s; };
  auto afull = [&](int s) { return bars + 8 * (S + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * S + s); };
  auto wfull = [&](int s) { return bars + 8 * (3 * S + s); };
  auto wempty = [&](int s) { return bars + 8 * (3 * S + WS + s); };
  const uint32_t accfull = bars + 8 * (3 * S + 2 * WS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_g + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_g + L::misc + 4);

  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * BM;  // this CTA's 128 rows (the pair covers 2 x 128)
  const int tokp = blockIdx.y * NACC;  // the pair's first token
  constexpr int steps_per_w = wcol_for(FMT) / BK;  // p.wcol
  const int kbeg = blockIdx.z * p.steps_per_split;
  const int nk = min(p.steps_per_split, p.K / BK - kbeg);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(xfull(s), 1);
      mbar_init(afull(s), 2 * kGroupWarps);
      mbar_init(empty(s), 1);
    }
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull(s), 1);
      // every group with a K step in the block column releases it
      mbar_init(wempty(s), min(kGroups, steps_per_w) * kGroupWarps);
    }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    // Both CTAs allocate, from the same warp, the same 512 columns.
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  // barriers of both CTAs exist before any cross-CTA arrive or copy
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ----------------------------
    if (lane == 0) {
      int issued_x = 0, issued_w = 0;
      bool ok = true;
      for (int ks = 0; ks < nk && ok; ++ks) {
        if (ks % steps_per_w == 0) {
          const int wb = ks / steps_per_w, ws = wb % WS;
          if (wb >= WS && !mbar_wait(wempty(ws), ((wb / WS) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          const int64_t kb = (kbeg + ks) / steps_per_w;
          mbar_arrive_expect_tx(wfull(ws), (uint32_t)(BM * p.wbox));
          for (int j = 0; j < p.g; ++j) {
            const int x0 = (int)(((int64_t)j * p.row_bytes + kb * p.wbytes) & ~int64_t(15));
            tma_load_2d(base + L::w + ws * L::w_stage + j * (BM / p.g) * p.wbox, &tmap_w, x0, row0 / p.g,
                        wfull(ws));
          }
          ++issued_w;
        }
        const int s = ks % S;
        if (ks >= S && !mbar_wait(empty(rel(s)), ((ks / S) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        // rank 0 expects both halves; each CTA's copy completes there
        if (leader) mbar_arrive_expect_tx(xfull(s), (uint32_t)(2 * L::x_tile));
        tma_load_2d_pair(base + L::x + s * L::x_tile, &tmap_x, (kbeg + ks) * BK, tokp + kPairHalf * (int)crank,
                         map_to_rank(xfull(s), 0));
        ++issued_x;
      }
      if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_EMPTY);
        *abort_flag = 1;
      }
      // Drain.  Both CTAs' activation copies complete on rank 0's barriers,
      // so rank 0 waits for them (the final cluster barrier keeps rank 1
      // resident until then); each CTA waits for its own weight copies.
      if (leader)
        for (int k = (issued_x > S ? issued_x - S : 0); k < issued_x; ++k)
          if (!mbar_wait_cluster(xfull(k % S), (k / S) & 1, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
      for (int k = (issued_w > WS ? issued_w - WS : 0); k < issued_w; ++k)
        if (!mbar_wait(wfull(k % WS), (k / WS) & 1, nullptr)) atomicOr(p.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (rank 0) ---------------------
    if (leader) {
      // idesc: f32 accumulate, fp16 A and B, K-major, N = 256, M = 256.
      const uint32_t idesc = (1u << 4) | ((uint32_t)(NACC >> 3) << 17) | ((uint32_t)((2 * BM) >> 4) << 24);
      for (int ks = 0; ks < nk; ++ks) {
        const int s = ks % S;
        const uint32_t par = (ks / S) & 1;
        if (!mbar_wait_cluster(afull(s), par, abort_flag) || !mbar_wait_cluster(xfull(s), par, abort_flag)) {
          if (lane == 0) atomicOr(p.status, DEV_TIMEOUT_FULL);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = tmem + (uint32_t)(NACC + 32 * s);
          const uint32_t b0 = base + L::x + s * L::x_tile;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_ts_pair(tmem, a0 + 8 * k, sw128_desc(b0 + 32 * k), idesc, (ks > 0 || k > 0) ? 1u : 0u);
          if ((ks & 1) || ks == nk - 1) umma_commit_pair(empty(rel(s)));
        }
        __syncwarp();
      }
      if (lane == 0) umma_commit_pair(accfull);
      __syncwarp();
    }
  } else {
    // --------------------------- dequant + epilogue ---------------------------
    const int grp = (warp - 2) / kGroupWarps;  // K steps grp, grp + kGroups, ...
    const int r = (warp & 3) * 32 + lane;  // weight row of this CTA's half = TMEM lane
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int gsh = p.g == 1 ? 0 : p.g == 2 ? 1 : p.g == 4 ? 2 : 3;  // g = 1, 2, 4 or 8
    const int jc = r & (p.g - 1);
    const uint32_t row_off = (uint32_t)((jc * (BM >> gsh) + (r >> gsh)) * p.wbox);
    const int64_t skew0 = (int64_t)jc * p.row_bytes;
    const int64_t kb0 = kbeg / steps_per_w;
    for (int ks = grp; ks < nk; ks += kGroups) {
      const int wb = ks / steps_per_w, ws = wb % WS;
      bool ok = true;
      if (ks % steps_per_w < kGroups) ok = mbar_wait(wfull(ws), (wb / WS) & 1, abort_flag);
      const int s = ks % S;
      if (ok && ks >= S) ok = mbar_wait(empty(rel(s)), ((ks / S) - 1) & 1, abort_flag);
      if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int skew = (int)((skew0 + (kb0 + wb) * wbytes_for(FMT)) & 15);
      const uint32_t rowp = base + L::w + ws * L::w_stage + row_off + skew;
      uint32_t o[32];
      decode64<FMT>(rowp, ks % steps_per_w, o);
      tmem_st32(tmem + lane_base + (uint32_t)(NACC + 32 * s), o);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_cluster(afull(s), 0);
        if (ks % steps_per_w >= steps_per_w - kGroups || ks + kGroups >= nk) mbar_arrive(wempty(ws));
      }
    }
    {
      // all dequant warps: group g reads the pair's token columns [g NACC /
      // kGroups, (g + 1) NACC / kGroups), 32 at a time (two loads, one wait)
      const bool ok = mbar_wait(accfull, 0, nullptr);
      tc_fence_after();
      if (ok && !*abort_flag) {
        const int q = warp & 3;
        const int row = row0 + 32 * q + lane;
        float* yz = p.y + (size_t)blockIdx.z * p.M * p.N;
        constexpr int kCols = NACC / kGroups;
        static_assert(kCols % 32 == 0, "32-column epilogue batches");
        const int cbeg = grp * kCols, cend = min(cbeg + kCols, p.M - tokp);
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += 32) {
          uint32_t v[32];
          const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                "=r"(v[15])
              : "r"(ta));
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
                "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
                "=r"(v[30]), "=r"(v[31])
              : "r"(ta + 16u));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (row < p.N) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int tok = tokp + c0 + i;
              if (tok < p.M) yz[(size_t)tok * p.N + row] = __uint_as_float(v[i]);
            }
          }
        }
      } else if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // Neither CTA leaves (or frees tensor memory) while the pair's MMAs may
  // still read its shared memory or tensor memory.
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// fp16 copy of the activations for the TMA-fed operand, with every 64-column
// step stored in k_perm order.  One thread per 2 output slots.
template <int FMT>
__global__ void __launch_bounds__(256) to_half_kernel(const float* __restrict__ x, __half2* __restrict__ h,
                                                       int64_t K, int64_t total_pairs,
                                                       const int32_t* __restrict__ rows) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total_pairs) return;
  const int64_t e = 2 * i;  // element index of the first slot
  const int64_t tok = e / K;
  const int64_t kk = e - tok * K;
  const int64_t step0 = kk & ~int64_t(63);
  const int slot = (int)(kk & 63);
  const float* row = x + (rows ? (int64_t)rows[tok] : tok) * K + step0;  // expert mode: gathered rows
  h[i] = __floats2half2_rn(row[k_perm(FMT, slot)], row[k_perm(FMT, slot + 1)]);
}

// Split-operand form: the hi copy at h[0 .. total_pairs) and the scaled lo
// copy (fp16((x - hi) * 2^11)) at h[total_pairs ..), both in k_perm order.
template <int FMT>
__global__ void __launch_bounds__(256) to_half_split_kernel(const float* __restrict__ x, __half2* __restrict__ h,
                                                             int64_t K, int64_t total_pairs,
                                                             const int32_t* __restrict__ rows) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total_pairs) return;
  const int64_t e = 2 * i;
  const int64_t tok = e / K;
  const int64_t kk = e - tok * K;
  const int64_t step0 = kk & ~int64_t(63);
  const int slot = (int)(kk & 63);
  const float* row = x + (rows ? (int64_t)rows[tok] : tok) * K + step0;
  const float a = row[k_perm(FMT, slot)], b = row[k_perm(FMT, slot + 1)];
  const __half2 hi = __floats2half2_rn(a, b);
  const float ah = __low2float(hi), bh = __high2float(hi);
  h[i] = hi;
  h[total_pairs + i] =
      __floats2half2_rn(__fmul_rn(__fsub_rn(a, ah), kSplitScale), __fmul_rn(__fsub_rn(b, bh), kSplitScale));
}

// Conversion with the decoder's residual-stream steps in front (the batched
// forward, model.rs:569-616): one CTA per activation row stages the row
// (hidden, plus delta when given: add, model.rs:1043-1071, written back to
// hidden) and the norm weights in shared memory, computes the RMSNorm scale
// with the x86-order sum of squares (rms_norm_into, model.rs:785-830; the
// arithmetic of the separate add + norm kernel) and converts (x * scale) * w
// as to_half(_split)_kernel converts x.  Shared memory: 2 K floats.
constexpr int kNormConvertMaxK = 16384;

template <int FMT, bool SPLIT>
__global__ void __launch_bounds__(256) to_half_norm_kernel(float* __restrict__ hidden, const float* __restrict__ delta,
                                                            const float* __restrict__ w, float eps,
                                                            __half2* __restrict__ h, int64_t K, int64_t total_pairs) {
  grid_dependency_wait();
  allow_dependents_launch();
  extern __shared__ float norm_smem[];  // [K] row, [K] weights
  __shared__ float scale_s;
  float* xs = norm_smem;
  float* ws = norm_smem + K;
  const int64_t tok = blockIdx.x;
  float* row = hidden + tok * K;
  const float* drow = delta ? delta + tok * K : nullptr;
#pragma unroll 8
  for (int64_t i = threadIdx.x; i < K; i += blockDim.x) {
    const float v = row[i];
    xs[i] = drow ? __fadd_rn(v, drow[i]) : v;
    ws[i] = w[i];
  }
  __syncthreads();
  if (drow)
    for (int64_t i = threadIdx.x; i < K; i += blockDim.x) row[i] = xs[i];
  if (threadIdx.x < 16) {
    const float d = dot_x86(xs, xs, (int)K, 0xffffu);
    if (threadIdx.x == 0) scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)K), eps)));
  }
  __syncthreads();
  const float scale = scale_s;
  const int64_t half_k = K / 2;
  for (int64_t p = threadIdx.x; p < half_k; p += blockDim.x) {
    const int64_t e = 2 * p;
    const int64_t step0 = e & ~int64_t(63);
    const int slot = (int)(e & 63);
    const int64_t ia = step0 + k_perm(FMT, slot), ib = step0 + k_perm(FMT, slot + 1);
    const float a = __fmul_rn(__fmul_rn(xs[ia], scale), ws[ia]);
    const float b = __fmul_rn(__fmul_rn(xs[ib], scale), ws[ib]);
    const __half2 hi = __floats2half2_rn(a, b);
    const int64_t i = tok * half_k + p;
    h[i] = hi;
    if (SPLIT) {
      const float ah = __low2float(hi), bh = __high2float(hi);
      h[total_pairs + i] =
          __floats2half2_rn(__fmul_rn(__fsub_rn(a, ah), kSplitScale), __fmul_rn(__fsub_rn(b, bh), kSplitScale));
    }
  }
}

template <int FMT, bool SPLIT>
cudaError_t launch_norm_convert(const GemmJob& j, __half2* xh2, int64_t pairs, cudaStream_t st) {
  auto k = to_half_norm_kernel<FMT, SPLIT>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         2 * kNormConvertMaxK * (int)sizeof(float));
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  return launch_ex(k, dim3((unsigned)j.M), dim3(256), 2 * (size_t)j.K * sizeof(float), st, j.norm_x, j.norm_delta,
                   j.norm_w, j.norm_eps, xh2, j.K, pairs);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct Geometry {
  int wcol, wbytes, wbox;
  int rows;  // rows per 16-byte-aligned pitch: 16 / gcd(row_bytes, 16)
};

// The weight tensor map needs a pitch that is a multiple of 16 bytes, so it
// treats `rows` consecutive rows as one pitch (Q6_K rows of 28 blocks are
// 5880 bytes: two rows per pitch).  N must be a multiple of it.
bool geometry(int dtype, int64_t K, int64_t N, int64_t row_bytes, Geometry& g) {
  if (K % BK != 0 || (row_bytes & 1)) return false;
  const int r = (int)(row_bytes & 15);
  g.rows = r == 0 ? 1 : (r % 8 == 0 ? 2 : (r % 4 == 0 ? 4 : 8));
  if (N % g.rows != 0) return false;
  switch (dtype) {
#define HYQ_GEOM(F) \
  case F: g.wcol = wcol_for(F); g.wbytes = wbytes_for(F); g.wbox = wbox_for(F); break;
    HYQ_GEOM(Q4_K)
    HYQ_GEOM(Q6_K)
    HYQ_GEOM(Q8_0)  // 4 blocks
    HYQ_GEOM(Q2_0C)
    HYQ_GEOM(STQ1_0)
#undef HYQ_GEOM
    default: return false;
  }
  return K % g.wcol == 0;
}

template <int FMT>
cudaError_t run_pair(const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, int splits, cudaStream_t st) {
  auto k = gemm2_kernel<FMT>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = Smem2<FMT>::total + 1024;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.N / BM), (unsigned)((p.M + 2 * kPairHalf - 1) / (2 * kPairHalf)), (unsigned)splits);
  cfg.blockDim = dim3(kThreads1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, tw, tx, p);
}

// The 2-SM kernel serves single-matrix Q4_K / Q6_K products of at least 256
// tokens whose rows pair up.  With four dequant groups the 7B layer measured
// 777 vs 753 TFLOP/s (2048 tokens) and 575 vs 560 (512 tokens) against the
// 1-SM kernel; per SM its K step takes the same time (the tensor pipe is
// throughput-bound at N = 256).  HYQ_GEMM_PAIR=0 turns it off.
bool use_pair(int64_t N, int64_t M) {
  static const int enabled = [] {
    const char* e = getenv("HYQ_GEMM_PAIR");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return enabled && M >= 256 && N % (2 * BM) == 0;
}

template <int FMT, int BN, bool SPLIT>
cudaError_t run(const CUtensorMap* tw, const CUtensorMap& tx, const CUtensorMap& txlo, const Params& p, int tiles,
                int splits, int64_t max_rows, cudaStream_t st, int ctas_1d = 0) {
  auto k = gemm_kernel<FMT, BN, SPLIT>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = Smem<FMT, BN, SPLIT>::total + 1024;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  // token tiles: of all M rows, or (expert mode) of the most rows one expert can have
  dim3 grid((unsigned)tiles, (unsigned)((max_rows + BN - 1) / BN), (unsigned)splits);
  if (ctas_1d > 0) grid = dim3((unsigned)ctas_1d);  // tail split: tiles and tail slices in one dimension
  return launch_ex(k, grid, dim3(kThreads1), (size_t)smem, st, tw[0], tw[1], tw[2], tx, txlo, p);
}

// Sum of the split-K partials in slice order, written to the matrices'
// outputs (gate/up: silu(sum gate) * sum up).
struct ReduceArgs {
  const float* part;
  int64_t M;
  int N;  // partial columns
  int splits;
  int gate_up;
  int n_seg;
  int seg_col0[3];
  int seg_rows[3];
  float* ys[3];
  int vec4;     // four columns per thread (every column boundary and output 16-byte aligned)
  int precise;  // gate/up SiLU with expf and IEEE division (split-operand products)
};

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float silu_mul(float g, float u, int precise) {
  return precise ? (g / (1.0f + expf(-g))) * u : __fdividef(g, 1.0f + __expf(-g)) * u;
}

__global__ void __launch_bounds__(256) reduce_splits_kernel(const __grid_constant__ ReduceArgs a) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int cols = a.gate_up ? a.seg_rows[0] : a.N;
  if (a.vec4) {
    // the same sums, four columns at a time (16-byte loads in flight)
    const int c4 = cols >> 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.M * c4) return;
    const int64_t tok = i / c4;
    const int c = 4 * (int)(i - tok * c4);
    const int64_t n = a.M * a.N;
    const float* src = a.part + tok * a.N + c;
    float4 s = *reinterpret_cast<const float4*>(src);
    for (int z = 1; z < a.splits; ++z) s = add4(s, *reinterpret_cast<const float4*>(src + (int64_t)z * n));
    if (a.gate_up) {
      const float* su = src + a.seg_rows[0];
      float4 u = *reinterpret_cast<const float4*>(su);
      for (int z = 1; z < a.splits; ++z) u = add4(u, *reinterpret_cast<const float4*>(su + (int64_t)z * n));
      *reinterpret_cast<float4*>(a.ys[0] + tok * a.seg_rows[0] + c) =
          make_float4(silu_mul(s.x, u.x, a.precise), silu_mul(s.y, u.y, a.precise), silu_mul(s.z, u.z, a.precise),
                      silu_mul(s.w, u.w, a.precise));
      return;
    }
    int m = 0;
    while (m + 1 < a.n_seg && c >= a.seg_col0[m + 1]) ++m;
    *reinterpret_cast<float4*>(a.ys[m] + tok * a.seg_rows[m] + (c - a.seg_col0[m])) = s;
    return;
  }
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.M * cols) return;
  const int64_t tok = i / cols;
  const int c = (int)(i - tok * cols);
  const int64_t n = a.M * a.N;
  const float* src = a.part + tok * a.N + c;
  float s = src[0];
  for (int z = 1; z < a.splits; ++z) s += src[(int64_t)z * n];
  if (a.gate_up) {
    const float* su = src + a.seg_rows[0];
    float u = su[0];
    for (int z = 1; z < a.splits; ++z) u += su[(int64_t)z * n];
    a.ys[0][tok * a.seg_rows[0] + c] = silu_mul(s, u, a.precise);  // as in the GEMM epilogue
    return;
  }
  int m = 0;
  while (m + 1 < a.n_seg && c >= a.seg_col0[m + 1]) ++m;
  a.ys[m][tok * a.seg_rows[m] + (c - a.seg_col0[m])] = s;
}

// Tail split: each tail tile's K-slice partials summed in slice order and
// written as the GEMM epilogue writes a whole tile (gate/up: silu(gate) *
// up).  Block (x, t): tail tile t, 256 (token, tile column) pairs.
struct TailArgs {
  const float* part;  // [tail tiles][z][bn tokens][BM tile rows]
  int z, bn, begin, tiles_x, M;
  int gate_up, n_seg, precise;
  int seg_tile0[4];
  int seg_rows[3];
  float* ys[3];
};

__global__ void __launch_bounds__(256) tail_reduce_kernel(const __grid_constant__ TailArgs a) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int tt = (int)blockIdx.y;
  const int t = a.begin + tt;
  const int by = t / a.tiles_x, bx = t - by * a.tiles_x;
  int seg = 0;
  while (seg + 1 < a.n_seg && bx >= a.seg_tile0[seg + 1]) ++seg;
  const int cols = a.gate_up ? BM / 2 : BM;  // output rows of the tile
  const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= a.bn * cols) return;
  const int tl = i / cols, c = i - tl * cols;
  const int tok = by * a.bn + tl;
  const int rows_m = a.seg_rows[seg];
  const int row = (bx - a.seg_tile0[seg]) * cols + c;
  if (tok >= a.M || row >= rows_m) return;
  const size_t stride = (size_t)a.bn * BM;
  const float* src = a.part + (size_t)tt * a.z * stride + (size_t)tl * BM + c;
  float s = src[0];
  for (int z = 1; z < a.z; ++z) s += src[(size_t)z * stride];
  if (a.gate_up) {
    float u = src[BM / 2];
    for (int z = 1; z < a.z; ++z) u += src[(size_t)z * stride + BM / 2];
    a.ys[0][(size_t)tok * rows_m + row] = silu_mul(s, u, a.precise);
    return;
  }
  a.ys[seg][(size_t)tok * rows_m + row] = s;
}

int device_sms() {
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev] > 0 ? sms[dev] : 148;
}

// Split-K slices (in block columns) so that small grids still fill the GPU,
// within one wave of CTAs (one per SM): a second, partial wave costs a whole
// slice's time for a fraction of the SMs.
int choose_splits(int64_t K, int64_t row_tiles, int64_t M, int wcol, int64_t bn) {
  const int64_t tiles = row_tiles * ((M + bn - 1) / bn);
  const int64_t nwb = K / wcol;
  const int64_t sms = device_sms();
  if (tiles >= sms) return 1;
  int64_t z = sms / tiles;
  if (z > nwb) z = nwb;
  if (z > 16) z = 16;
  return (int)(z < 1 ? 1 : z);
}

// Tail split of a grid of at least one wave (fp16 operands, 1-SM kernel):
// when the tiles past the last full wave fill at most half the SMs, they
// are cut into K-slices of whole block columns (up to 16) that run side by
// side in that last wave instead of one tile per SM for a whole tile's
// time.
struct TailPlan {
  int z = 1;      // slices per tail tile (1: no tail split)
  int begin = 0;  // first tail tile
  int tiles = 0;  // tail tiles
  int wb = 0;     // block columns per slice
};

TailPlan tail_plan(int64_t K, int64_t row_tiles, int64_t M, int wcol, int64_t bn) {
  TailPlan t;
  const int64_t tiles = row_tiles * ((M + bn - 1) / bn);
  const int64_t nwb = K / wcol;
  const int64_t sms = device_sms();
  if (tiles < sms || nwb < 2) return t;
  const int64_t rem = tiles % sms;
  if (rem == 0 || 2 * rem > sms) return t;
  int64_t z = sms / rem;
  if (z > nwb) z = nwb;
  if (z > 16) z = 16;
  const int64_t per = (nwb + z - 1) / z;
  z = (nwb + per - 1) / per;
  if (z < 2) return t;
  t.z = (int)z;
  t.begin = (int)(tiles - rem);
  t.tiles = (int)rem;
  t.wb = (int)per;
  return t;
}

// Row tiles of a job and the columns of its split-K partials.
struct Layout {
  int tiles = 0;
  int tile0[4] = {};
  int col0[3] = {};
  int ncols = 0;
};

Layout layout_of(const GemmJob& j) {
  Layout L;
  if (j.experts > 0) {
    // expert e owns row tiles [e * per, (e + 1) * per)
    const int per = (int)((j.rows[0] + (j.gate_up ? BM / 2 : BM) - 1) / (j.gate_up ? BM / 2 : BM));
    L.tiles = j.experts * per;
    L.tile0[1] = L.tiles;
    L.ncols = (int)(j.gate_up ? 2 * j.rows[0] : j.rows[0]);
    return L;
  }
  if (j.gate_up) {
    L.tiles = (int)((j.rows[0] + BM / 2 - 1) / (BM / 2));
    L.tile0[1] = L.tiles;
    L.ncols = (int)(2 * j.rows[0]);
    return L;
  }
  for (int m = 0; m < j.n_mat; ++m) {
    L.tile0[m] = L.tiles;
    L.col0[m] = L.ncols;
    L.tiles += (int)((j.rows[m] + BM - 1) / BM);
    L.ncols += (int)j.rows[m];
  }
  L.tile0[j.n_mat] = L.tiles;
  return L;
}

// The shared tile geometry of a job's matrices, or false when the tensor-core
// path does not take it.
bool job_geometry(const GemmJob& j, Geometry& g) {
  if (j.gate_up ? j.n_mat != 2 : (j.n_mat < 1 || j.n_mat > 3)) return false;
  if (j.experts > 0) {
    if (!j.expert_off || j.n_mat != (j.gate_up ? 2 : 1) || j.expert_max_rows <= 0) return false;
    if ((int64_t)j.experts * j.rows[0] > INT32_MAX / 4) return false;
  }
  if (j.gate_up && j.rows[0] != j.rows[1]) return false;
  const int64_t row_bytes = j.K / block_len(j.dtype) * block_bytes(j.dtype);
  for (int m = 0; m < j.n_mat; ++m) {
    if (!geometry(j.dtype, j.K, j.rows[m], row_bytes, g)) return false;
    if (j.rows[m] > INT32_MAX / 4) return false;
  }
  return j.M <= INT32_MAX / 2;
}

// fp16 activation copy (split-operand form: hi and lo copies)
size_t x_bytes(int64_t K, int64_t M, bool split) {
  return ((size_t)(K * M) * sizeof(__half) * (split ? 2 : 1) + 255) / 256 * 256;
}

// Token tile of a job: by batch size (expert mode: the typical rows per
// expert), at most 128 in the split-operand form (its two accumulators and
// doubled A stages do not fit tensor memory at 256).
int job_token_tile(const GemmJob& j) {
  const int bn = token_tile(j.experts > 0 ? j.M / j.experts : j.M);
  return j.split && bn > 128 ? 128 : bn;
}

}  // namespace gemm

bool gemm_job_supported(const GemmJob& j) {
  gemm::Geometry g;
  if (!gemm::job_geometry(j, g)) return false;
  if (j.norm_w && (j.experts > 0 || j.x_rows || !j.norm_x || j.K > gemm::kNormConvertMaxK)) return false;
  for (int m = 0; m < j.n_mat; ++m)
    if (!j.w[m] || (reinterpret_cast<uintptr_t>(j.w[m]) & 15) != 0) return false;
  return gemm::encode_fn() != nullptr;
}

size_t gemm_job_workspace_bytes(const GemmJob& j) {
  gemm::Geometry g;
  if (!gemm::job_geometry(j, g)) return 0;
  const gemm::Layout L = gemm::layout_of(j);
  const int bn = gemm::job_token_tile(j);
  const int z = j.experts > 0 ? 1 : gemm::choose_splits(j.K, L.tiles, j.M, g.wcol, bn);
  size_t part = z > 1 ? (size_t)z * j.M * L.ncols * sizeof(float) : 0;
  if (j.experts == 0 && !j.split && z == 1) {
    const gemm::TailPlan t = gemm::tail_plan(j.K, L.tiles, j.M, g.wcol, bn);
    if (t.z > 1) part = (size_t)t.tiles * t.z * bn * gemm::BM * sizeof(float);
  }
  return gemm::x_bytes(j.K, j.M, j.split) + part + 16;
}

cudaError_t launch_gemm_job(const GemmJob& j, void* workspace, cudaStream_t st) {
  using namespace gemm;
  Geometry g;
  if (!job_geometry(j, g)) return cudaErrorNotSupported;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const int64_t K = j.K, M = j.M;
  const int64_t row_bytes = K / block_len(j.dtype) * block_bytes(j.dtype);
  const Layout lay = layout_of(j);
  const bool pair = !j.split && j.experts == 0 && !j.gate_up && j.n_mat == 1 &&
                    (j.dtype == Q4_K || j.dtype == Q6_K) && use_pair(j.rows[0], M);
  __half* xh = static_cast<__half*>(workspace);
  {
    const int64_t pairs = K * M / 2;
    const unsigned blocks = (unsigned)((pairs + 255) / 256);
    __half2* xh2 = reinterpret_cast<__half2*>(xh);
    cudaError_t e;
    if (j.norm_w) {
      switch (j.dtype) {
#define HYQ_NORM_X(F)                                                                                  \
  case F:                                                                                              \
    e = j.split ? launch_norm_convert<F, true>(j, xh2, pairs, st) : launch_norm_convert<F, false>(j, xh2, pairs, st); \
    break;
        HYQ_NORM_X(Q4_K)
        HYQ_NORM_X(Q6_K)
        HYQ_NORM_X(Q8_0)
        HYQ_NORM_X(Q2_0C)
        HYQ_NORM_X(STQ1_0)
#undef HYQ_NORM_X
        default: return cudaErrorNotSupported;
      }
      if (e != cudaSuccess) return e;
    } else if (j.split) {
      switch (j.dtype) {
#define HYQ_SPLIT_X(F) \
  case F: e = launch_ex(to_half_split_kernel<F>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
        HYQ_SPLIT_X(Q4_K)
        HYQ_SPLIT_X(Q6_K)
        HYQ_SPLIT_X(Q8_0)
        HYQ_SPLIT_X(Q2_0C)
        HYQ_SPLIT_X(STQ1_0)
#undef HYQ_SPLIT_X
        default: return cudaErrorNotSupported;
      }
      if (e != cudaSuccess) return e;
    } else
    switch (j.dtype) {
      case Q4_K: e = launch_ex(to_half_kernel<Q4_K>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
      case Q6_K: e = launch_ex(to_half_kernel<Q6_K>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
      case Q8_0: e = launch_ex(to_half_kernel<Q8_0>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
      case Q2_0C: e = launch_ex(to_half_kernel<Q2_0C>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
      default: e = launch_ex(to_half_kernel<STQ1_0>, dim3(blocks), dim3(256), 0, st, j.x, xh2, K, pairs, j.x_rows); break;
    }
    if (e != cudaSuccess) return e;
  }
  // expert mode: the typical rows per expert pick the token tile
  const int bn = job_token_tile(j);
  const int tile_rows = j.gate_up ? BM / 2 : BM;
  const int64_t map_mats = j.experts > 0 ? j.experts : 1;  // expert mode: the maps cover every expert
  CUtensorMap tw[3], tx, txlo;
  for (int m = 0; m < 3; ++m) {
    const int mm = m < j.n_mat ? m : 0;  // unused maps repeat the first
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes * g.rows), (cuuint64_t)(map_mats * j.rows[mm] / g.rows)};
    const cuuint64_t strides[1] = {(cuuint64_t)(row_bytes * g.rows)};
    const cuuint32_t box[2] = {(cuuint32_t)g.wbox, (cuuint32_t)(tile_rows / g.rows)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tw[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(j.w[mm]), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)(pair ? kPairHalf : bn)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    // the split-operand lo copy follows the hi copy (K * M halves further)
    txlo = tx;
    if (j.split && enc(&txlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh + K * M, dims, strides, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const int nwb = (int)(K / g.wcol);
  const int z = j.experts > 0 ? 1 : choose_splits(K, lay.tiles, M, g.wcol, bn);
  const int wb_per_split = (nwb + z - 1) / z;
  // slices actually launched (rounding to whole block columns can drop some)
  const int splits = (nwb + wb_per_split - 1) / wb_per_split;
  float* partials =
      splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + x_bytes(K, M, j.split)) : nullptr;
  // whole tiles, then the thin last wave cut into K-slices (fp16 operands)
  const TailPlan tail = (j.experts == 0 && !j.split && !pair && splits == 1)
                            ? tail_plan(K, lay.tiles, M, g.wcol, bn) : TailPlan{};
  Params p{};
  p.K = (int)K;
  p.N = lay.ncols;
  p.M = (int)M;
  p.steps_per_split = wb_per_split * (g.wcol / BK);
  p.row_bytes = (int)row_bytes;
  p.wcol = g.wcol;
  p.wbox = g.wbox;
  p.wbytes = g.wbytes;
  p.g = g.rows;
  p.y = partials;
  p.status = j.status;
  p.n_seg = j.gate_up ? 1 : j.n_mat;
  for (int m = 0; m < 4; ++m) p.seg_tile0[m] = lay.tile0[m];
  for (int m = 0; m < 3; ++m) {
    p.seg_rows[m] = m < j.n_mat ? (int)j.rows[m] : 0;
    p.seg_col0[m] = lay.col0[m];
    p.ys[m] = m < j.n_mat ? j.y[m] : nullptr;
  }
  p.gate_up = j.gate_up ? 1 : 0;
  if (tail.z > 1) {
    p.tail_z = tail.z;
    p.tail_begin = tail.begin;
    p.tail_steps = tail.wb * (g.wcol / BK);
    p.tiles_x = lay.tiles;
    p.tail_part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + x_bytes(K, M, j.split));
  }
  if (j.experts > 0) {
    p.expert_off = j.expert_off;
    p.expert_tiles = lay.tiles / j.experts;
    p.expert_rows = (int)j.rows[0];
  }
  const int64_t max_rows = j.experts > 0 ? (j.expert_max_rows < M ? j.expert_max_rows : M) : M;
  cudaError_t e;
  const int ctas = tail.z > 1 ? tail.begin + tail.tiles * tail.z : 0;
  if (pair) {
    p.N = (int)j.rows[0];
    p.y = splits > 1 ? partials : j.y[0];
    e = j.dtype == Q4_K ? run_pair<Q4_K>(tw[0], tx, p, splits, st) : run_pair<Q6_K>(tw[0], tx, p, splits, st);
  } else {
    switch (j.dtype) {
#define HYQ_RUN(F)                                                                                  \
  case F:                                                                                           \
    if (j.split)                                                                                    \
      e = bn == 128 ? run<F, 128, true>(tw, tx, txlo, p, lay.tiles, splits, max_rows, st)           \
                    : run<F, 64, true>(tw, tx, txlo, p, lay.tiles, splits, max_rows, st);           \
    else                                                                                            \
      e = bn == 256   ? run<F, 256, false>(tw, tx, txlo, p, lay.tiles, splits, max_rows, st, ctas)  \
          : bn == 128 ? run<F, 128, false>(tw, tx, txlo, p, lay.tiles, splits, max_rows, st, ctas)  \
                      : run<F, 64, false>(tw, tx, txlo, p, lay.tiles, splits, max_rows, st, ctas);  \
    break;
      HYQ_RUN(Q4_K)
      HYQ_RUN(Q6_K)
      HYQ_RUN(Q8_0)
      HYQ_RUN(Q2_0C)
      HYQ_RUN(STQ1_0)
#undef HYQ_RUN
      default: return cudaErrorNotSupported;
    }
  }
  if (e != cudaSuccess) return e;
  if (tail.z > 1) {
    TailArgs t{};
    t.part = p.tail_part;
    t.z = tail.z;
    t.bn = bn;
    t.begin = tail.begin;
    t.tiles_x = lay.tiles;
    t.M = (int)M;
    t.gate_up = p.gate_up;
    t.n_seg = p.n_seg;
    t.precise = 0;  // fp16 operands: the epilogue's fast SiLU
    for (int m = 0; m < 4; ++m) t.seg_tile0[m] = p.seg_tile0[m];
    for (int m = 0; m < 3; ++m) {
      t.seg_rows[m] = p.seg_rows[m];
      t.ys[m] = p.ys[m];
    }
    const int per_tile = bn * (j.gate_up ? BM / 2 : BM);
    return launch_ex(tail_reduce_kernel, dim3((unsigned)((per_tile + 255) / 256), (unsigned)tail.tiles), dim3(256), 0,
                     st, t);
  }
  if (splits == 1) return e;
  ReduceArgs r{};
  r.part = partials;
  r.M = M;
  r.N = lay.ncols;
  r.splits = splits;
  r.gate_up = p.gate_up;
  r.precise = j.split ? 1 : 0;
  r.n_seg = p.n_seg;
  for (int m = 0; m < 3; ++m) {
    r.seg_col0[m] = p.seg_col0[m];
    r.seg_rows[m] = p.seg_rows[m];
    r.ys[m] = p.ys[m];
  }
  // four columns per thread when no float4 crosses a matrix boundary and
  // every output row starts 16-byte aligned
  bool v4 = lay.ncols % 4 == 0;
  for (int m = 0; m < r.n_seg; ++m)
    v4 = v4 && r.seg_col0[m] % 4 == 0 && r.seg_rows[m] % 4 == 0 && (reinterpret_cast<uintptr_t>(r.ys[m]) & 15) == 0;
  r.vec4 = v4 ? 1 : 0;
  const int64_t n = M * (j.gate_up ? j.rows[0] : lay.ncols) / (v4 ? 4 : 1);
  return launch_ex(reduce_splits_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, r);
}

// Single-matrix forms used by hyq_matmul and hyq_matmul_noalloc.
static GemmJob single_job(int dtype, const uint8_t* w, int64_t K, int64_t N, const float* x, int64_t M, float* y,
                          unsigned* status, bool split) {
  GemmJob j;
  j.split = split;
  j.dtype = dtype;
  j.n_mat = 1;
  j.w[0] = w;
  j.rows[0] = N;
  j.y[0] = y;
  j.K = K;
  j.M = M;
  j.x = x;
  j.status = status;
  return j;
}

bool gemm_supported(int dtype, int64_t K, int64_t N, int64_t M, const void* w) {
  return gemm_job_supported(
      single_job(dtype, static_cast<const uint8_t*>(w), K, N, nullptr, M, nullptr, nullptr, false));
}

size_t gemm_workspace_bytes(int dtype, int64_t K, int64_t N, int64_t M, bool split) {
  return gemm_job_workspace_bytes(single_job(dtype, nullptr, K, N, nullptr, M, nullptr, nullptr, split));
}

cudaError_t launch_gemm(int dtype, const uint8_t* w, int64_t K, int64_t N, const float* x, int64_t M, float* y,
                        void* workspace, unsigned* status, cudaStream_t st, bool split) {
  return launch_gemm_job(single_job(dtype, w, K, N, x, M, y, status, split), workspace, st);
}

}  // namespace hyq
