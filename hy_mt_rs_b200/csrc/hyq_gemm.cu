// Batched products over packed GGUF rows on the 5th-generation tensor cores
// (tcgen05 / TMEM), sm_100a.
//
// Reference behaviour: Weight::matmul with batch >= 2 (hy-mt-rs
// src/quant.rs:272-343): Y[batch, N] = X[batch, K] . W^T, where the reference
// decodes 64-row tiles to f32 and multiplies them with Candle's CPU GEMM.
//
// Tile: 128 weight rows (the MMA's M) x 128 tokens (the MMA's N) x K, with
// D = W_tile . X_tile^T accumulated in f32 in tensor memory.  Roles:
//   warp 0  : TMA producer -- packed weight block columns (2-D tensor map over
//             the raw GGUF bytes: 128 rows x one block column, taken as the
//             16-byte aligned window around it) and fp16 activation tiles
//             (SWIZZLE_128B);
//   warp 1  : allocates TMEM and issues tcgen05.mma (one elected thread),
//             releasing each stage with tcgen05.commit;
//   warps 2-9: dequantize the packed block column into the fp16 K-major
//             SWIZZLE_128B tile the MMA reads (weights decoded in f32 with
//             the reference's operation order, then rounded to fp16), then
//             fence the writes into the async proxy; warps 2-5 also run the
//             epilogue (tcgen05.ld -> coalesced f32 stores of Y).
// Operands are fp16 (both), accumulation f32: relative error ~4e-4 of the
// f32 reference, inside the 1e-3 relative-L2 bound.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>

#include "hyq_common.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace gemm {

constexpr int BM = 128;          // weight rows per tile (MMA M)
constexpr int BN = 128;          // tokens per tile (MMA N)
constexpr int BK = 64;           // K per stage: one 128-byte swizzle row of fp16
constexpr int S = 4;             // activation / decoded-weight stages
constexpr int WS = 2;            // packed weight block-column stages
constexpr int kDequantWarps = 8;
constexpr int kThreads = (2 + kDequantWarps) * 32;
constexpr int kDequantThreads = kDequantWarps * 32;
constexpr int kTileBytes = 128 * 128;  // one 128-row x 64-fp16 tile

struct Params {
  int K, N, M;
  int row_bytes;
  int wcol;             // K columns per packed block-column tile
  int wbox;             // bytes per row of that tile (TMA box inner size)
  int wbytes;           // packed bytes of one row per block column
  float* y;             // [M, N]
  unsigned* status;
};

struct Smem {
  // offsets from the 1024-aligned base
  static constexpr int x = 0;
  static constexpr int a = x + S * kTileBytes;
  static constexpr int w = a + S * kTileBytes;
  static constexpr int w_stage = 128 * 256;  // max box bytes per row (256) x 128 rows
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

// Decode 32 consecutive weights of one row (K offset `kc` inside the
// block-column tile, a multiple of 32) into 16 fp16x2 words, using the
// reference's f32 operation order (quant.rs:2437-2483) before rounding.
template <int FMT>
__device__ __forceinline__ void decode32(uint32_t row, int kc, uint32_t (&o)[16]) {
  if (FMT == Q4_K) {
    const int g = kc >> 6, hh = (kc >> 5) & 1;  // group of 64, low/high nibbles
    const uint4 h = ld_s128(row);
    const float d = half_to_f32(h.x & 0xffffu), dmin = half_to_f32(h.x >> 16);
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
    const float d1 = d * (float)s, m1 = dmin * (float)m;
    const uint4 q0 = ld_s128(row + 16 + 32 * g), q1 = ld_s128(row + 32 + 32 * g);
    const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t nib = hh ? (q[i] >> 4) & 0x0f0f0f0fu : q[i] & 0x0f0f0f0fu;
      float v[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) v[b] = __fsub_rn(__fmul_rn(d1, (float)((nib >> (8 * b)) & 0xffu)), m1);
      o[2 * i] = pack_h2(v[0], v[1]);
      o[2 * i + 1] = pack_h2(v[2], v[3]);
    }
  } else {  // Q6_K
    const int chunk = kc >> 7, p = (kc >> 5) & 3;
    uint32_t ql[8], qh[8];
    ld_s_words<8>(row + chunk * 64 + (p & 1) * 32, ql);
    ld_s_words<8>(row + 128 + chunk * 32, qh);
    const uint32_t sc = ld_s16(row + 192 + chunk * 8 + 2 * p);
    const float d = half_to_f32(ld_s16(row + 208));
    const float s0 = __fmul_rn(d, (float)(int8_t)(sc & 0xffu));
    const float s1 = __fmul_rn(d, (float)(int8_t)(sc >> 8));
    const int nsh = (p >> 1) * 4, hsh = 2 * p;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = i < 4 ? s0 : s1;  // columns 0..15 use half 0, 16..31 half 1
      float v[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int q = (int)(((ql[i] >> (8 * b + nsh)) & 15u) | (((qh[i] >> (8 * b + hsh)) & 3u) << 4));
        v[b] = __fmul_rn(s, (float)(q - 32));
      }
      o[2 * i] = pack_h2(v[0], v[1]);
      o[2 * i + 1] = pack_h2(v[2], v[3]);
    }
  }
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  const uint32_t raw_s = smem_addr(smem_raw);
  const uint32_t base = (raw_s + 1023u) & ~1023u;
  uint8_t* base_g = smem_raw + (base - raw_s);
  const uint32_t bars = base + Smem::bars;
  auto xfull = [&](int s) { return bars + 8 * s; };
  auto afull = [&](int s) { return bars + 8 * (S + s); };
  auto empty = [&](int s) { return bars + 8 * (2 * S + s); };
  auto wfull = [&](int s) { return bars + 8 * (3 * S + s); };
  auto wempty = [&](int s) { return bars + 8 * (3 * S + WS + s); };
  const uint32_t accfull = bars + 8 * (3 * S + 2 * WS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_g + Smem::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_g + Smem::misc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * BM, tok0 = blockIdx.y * BN;
  const int nk = p.K / BK;
  const int steps_per_w = p.wcol / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(xfull(s), 1);
      mbar_init(afull(s), kDequantThreads);
      mbar_init(empty(s), 1);
    }
    for (int s = 0; s < WS; ++s) {
      mbar_init(wfull(s), 1);
      mbar_init(wempty(s), kDequantThreads);
    }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    // TMEM accumulator: 128 lanes x BN f32 columns.
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
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
          const int x0 = (wb * p.wbytes) & ~15;
          mbar_arrive_expect_tx(wfull(ws), (uint32_t)(BM * p.wbox));
          tma_load_2d(base + Smem::w + ws * Smem::w_stage, &tmap_w, x0, row0, wfull(ws));
          ++issued_w;
        }
        const int s = ks % S;
        if (ks >= S && !mbar_wait(empty(s), ((ks / S) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(xfull(s), (uint32_t)kTileBytes);
        tma_load_2d(base + Smem::x + s * kTileBytes, &tmap_x, ks * BK, tok0, xfull(s));
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
        const uint32_t a0 = base + Smem::a + s * kTileBytes;
        const uint32_t b0 = base + Smem::x + s * kTileBytes;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_f16(tmem, sw128_desc(a0 + 32 * k), sw128_desc(b0 + 32 * k), idesc, (ks > 0 || k > 0) ? 1u : 0u);
        umma_commit(empty(s));
      }
      __syncwarp();
    }
    // All issued MMAs have completed once accfull flips.
    if (lane == 0) umma_commit(accfull);
    __syncwarp();
  } else {
    // --------------------------- dequant + epilogue ---------------------------
    const int dt = threadIdx.x - 64;
    const int r = dt >> 1, h = dt & 1;
    const uint32_t swz = (uint32_t)(r & 7);
    for (int ks = 0; ks < nk; ++ks) {
      const int wb = ks / steps_per_w, ws = wb % WS;
      bool ok = true;
      if (ks % steps_per_w == 0) ok = mbar_wait(wfull(ws), (wb / WS) & 1, abort_flag);
      const int s = ks % S;
      if (ok && ks >= S) ok = mbar_wait(empty(s), ((ks / S) - 1) & 1, abort_flag);
      if (!ok) {
        atomicOr(p.status, DEV_TIMEOUT_FULL);
        *abort_flag = 1;
        break;
      }
      const int skew = (wb * p.wbytes) & 15;
      const uint32_t rowp = base + Smem::w + ws * Smem::w_stage + r * p.wbox + skew;
      const int kc = (ks % steps_per_w) * BK + 32 * h;
      uint32_t o[16];
      decode32<FMT>(rowp, kc, o);
      const uint32_t dst = base + Smem::a + s * kTileBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_s128(dst + ((((uint32_t)(4 * h + c)) ^ swz) << 4), make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]));
      fence_proxy_async_smem();
      mbar_arrive(afull(s));
      if (ks % steps_per_w == steps_per_w - 1) mbar_arrive(wempty(ws));
    }
    // Epilogue: warps 2..5 own TMEM lanes 32*(warp%4) .. +31.
    if (warp < 6) {
      const bool ok = mbar_wait(accfull, 0, nullptr);
      tc_fence_after();
      if (ok && !*abort_flag) {
        const int q = warp & 3;
        const int row = row0 + 32 * q + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t v[16];
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
              "%14, %15}, [%16];"
              : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                "=r"(v[15])
              : "r"(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          if (row < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int tok = tok0 + c0 + i;
              if (tok < p.M) p.y[(size_t)tok * p.N + row] = __uint_as_float(v[i]);
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

// fp16 copy of the activations for the TMA-fed operand.
__global__ void __launch_bounds__(256) to_half_kernel(const float* __restrict__ x, __half* __restrict__ h,
                                                       int64_t n) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    *reinterpret_cast<__half2*>(h + i) = a;
    *reinterpret_cast<__half2*>(h + i + 2) = b;
  } else {
    for (int64_t k = i; k < n; ++k) h[k] = __float2half_rn(x[k]);
  }
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
};

bool geometry(int dtype, int64_t K, int64_t row_bytes, Geometry& g) {
  if (K % BK != 0 || row_bytes % 16 != 0) return false;
  switch (dtype) {
    case Q4_K: g.wcol = 256; g.wbytes = 144; g.wbox = 144; break;
    case Q6_K: g.wcol = 256; g.wbytes = 210; g.wbox = 224; break;
    default: return false;
  }
  return K % g.wcol == 0;
}

template <int FMT>
cudaError_t run(const CUtensorMap& tw, const CUtensorMap& tx, const Params& p, cudaStream_t st) {
  auto k = gemm_kernel<FMT>;
  static int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = Smem::total + 1024;
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  dim3 grid((unsigned)((p.N + BM - 1) / BM), (unsigned)((p.M + BN - 1) / BN));
  k<<<grid, kThreads, smem, st>>>(tw, tx, p);
  return cudaGetLastError();
}

}  // namespace gemm

bool gemm_supported(int dtype, int64_t K, int64_t N, int64_t M, const void* w) {
  gemm::Geometry g;
  const int64_t row_bytes = K / block_len(dtype) * block_bytes(dtype);
  if (!gemm::geometry(dtype, K, row_bytes, g)) return false;
  if ((reinterpret_cast<uintptr_t>(w) & 15) != 0) return false;
  if (N > INT32_MAX / 2 || M > INT32_MAX / 2) return false;
  return gemm::encode_fn() != nullptr;
}

size_t gemm_workspace_bytes(int64_t K, int64_t M) { return (size_t)(K * M) * sizeof(__half) + 16; }

cudaError_t launch_gemm(int dtype, const uint8_t* w, int64_t K, int64_t N, const float* x, int64_t M, float* y,
                        void* workspace, unsigned* status, cudaStream_t st) {
  using namespace gemm;
  Geometry g;
  const int64_t row_bytes = K / block_len(dtype) * block_bytes(dtype);
  if (!geometry(dtype, K, row_bytes, g)) return cudaErrorNotSupported;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  __half* xh = static_cast<__half*>(workspace);
  {
    const int64_t n = K * M;
    const int64_t threads = (n + 3) / 4;
    to_half_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(x, xh, n);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  CUtensorMap tw, tx;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)g.wbox, (cuuint32_t)BM};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  Params p;
  p.K = (int)K;
  p.N = (int)N;
  p.M = (int)M;
  p.row_bytes = (int)row_bytes;
  p.wcol = g.wcol;
  p.wbox = g.wbox;
  p.wbytes = g.wbytes;
  p.y = y;
  p.status = status;
  switch (dtype) {
    case Q4_K: return run<Q4_K>(tw, tx, p, st);
    case Q6_K: return run<Q6_K>(tw, tx, p, st);
    default: return cudaErrorNotSupported;
  }
}

}  // namespace hyq
