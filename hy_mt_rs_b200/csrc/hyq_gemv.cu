// Batch-1 matrix-vector products over packed GGUF rows (sm_100a): host side.
//
// Reference behaviour (hy-mt-rs src/quant.rs):
//   Weight::matmul batch 1          :159-270   (f32 activations)
//   gemv_q8_fast / compute_chunk_q8 :353-439   (int8 activations, SDOT rows)
//   gemv_qkv(_fast)                 :441-538, :653-721
//   matmul_gate_up_silu(_fast)      :540-651, :723-841
//
// make_plan chooses the streaming kernel's geometry (hyq_gemv_impl.cuh) or
// the per-element fallback for shapes and pointers the streaming kernel does
// not take.
#include <cstdlib>

#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace gemv {

extern template cudaError_t dispatch_fmt<Q2_0C>(const Params&, const Plan&, bool, cudaStream_t);
extern template cudaError_t dispatch_fmt<STQ1_0>(const Params&, const Plan&, bool, cudaStream_t);
extern template cudaError_t dispatch_fmt<Q4_K>(const Params&, const Plan&, bool, cudaStream_t);
extern template cudaError_t dispatch_fmt<Q6_K>(const Params&, const Plan&, bool, cudaStream_t);
extern template cudaError_t dispatch_fmt<Q8_0>(const Params&, const Plan&, bool, cudaStream_t);

namespace {

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
    if (p.xmode == XQ8F) {
      // Q8 of each 256-column group (K % 256 == 0: no scalar tail), then the
      // dequantized activation q * scale.
      for (int g0 = 0; g0 < p.K; g0 += 256) {
        float m = 0.f;
        int bad = 0;
        for (int k = lane; k < 256; k += 32) {
          const float a = fabsf(p.x[g0 + k]);
          bad |= isnan(a) ? 1 : 0;
          m = fmaxf(m, a);
        }
        for (int o = 16; o > 0; o >>= 1) {
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          bad |= __shfl_xor_sync(0xffffffffu, bad, o);
        }
        float scale = 0.f, inverse = 0.f;
        if (!bad && m > 0.f) {
          scale = __fdiv_rn(m, 127.f);
          inverse = __fdiv_rn(127.f, m);
        }
        for (int k = g0 + lane; k < g0 + 256; k += 32) {
          const float sv = __fmul_rn(p.x[k], inverse);
          const int q = isnan(sv) ? 0 : max(-128, min(127, __float2int_rn(sv)));
          const float xv = (float)q * scale;
          const int b = k / BL, o = k - b * BL;
          g = fmaf(decode_elem<T>(row + b * BB, o), xv, g);
          if (PAIR) u = fmaf(decode_elem<T>(rowu + b * BB, o), xv, u);
        }
      }
    } else {
      for (int k = lane; k < p.K; k += 32) {
        const float xv = p.xmode == XF32 ? p.x[k] : (float)p.xq[k] * p.xs[k >> 8];
        const int b = k / BL, o = k - b * BL;
        g = fmaf(decode_elem<T>(row + b * BB, o), xv, g);
        if (PAIR) u = fmaf(decode_elem<T>(rowu + b * BB, o), xv, u);
      }
    }
    g = warp_sum(g);
    if (PAIR) u = warp_sum(u);
    if (lane == 0) p.mat[m].y[r] = PAIR ? (g / (1.0f + expf(-g))) * u : g;
  }
}

int g_num_sms = 0;
int g_smem_optin = 0;
int g_smem_dual = 0;  // dynamic shared memory per CTA with two CTAs per SM

void device_limits() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached_dev = -1;
  if (cached_dev != dev) {
    int per_sm = 0, reserved = 0;
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    g_smem_dual = (per_sm / 2 - reserved) / 1024 * 1024;
    if (g_smem_dual > g_smem_optin) g_smem_dual = g_smem_optin;
    cached_dev = dev;
  }
}

// HYQ_GEMV_DUAL=0 keeps one CTA per SM for every variant (for comparisons).
bool dual_enabled() {
  static const int on = [] {
    const char* e = getenv("HYQ_GEMV_DUAL");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

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
  const int np = (j.x && !j.quantize_q8) ? 3 : 1;
  // prepared activations: np byte planes of 16 words per unit, 2 floats per group
  pl.x_bytes = (np * 16 * U + 2 * (U / 4)) * 4;
  // f32 activations staged by one bulk copy when they are small
  pl.x_raw_bytes = (j.x && j.K * 4 <= kXStageMax) ? (int)(j.K * 4) : 0;
  pl.x_raw_off = pl.x_raw_bytes ? (kHeaderBytes + pl.x_bytes + 15) / 16 * 16 : 0;
  // padded copy of the staged activations: 65 floats per 64-column unit
  const int x_pad_bytes = pl.x_raw_bytes ? (int)(j.K / 64 * 65 * 4) : 0;
  pl.x_pad_off = pl.x_raw_bytes ? pl.x_raw_off + pl.x_raw_bytes : 0;
  const int stage_off =
      (kHeaderBytes + pl.x_bytes + (pl.x_raw_bytes ? 16 + pl.x_raw_bytes + x_pad_bytes : 0) + 127) / 128 * 128;
  const int upl_max = np == 1 ? 4 : 1;
  const int64_t row_bytes = j.K / block_len(t) * block_bytes(t);
  int64_t total_rows = 0;
  for (int m = 0; m < j.n_mat; ++m) total_rows += j.rows[m];
  const int smem_cap = g_smem_optin > 0 ? g_smem_optin : 227 * 1024;
  // Pick the K split (ks warps per row) and rows per warp per tile (rw) with
  // the fewest tile waves, weighting each wave by its per-warp work
  // (rw * units per lane) plus a fixed per-tile cost; ties go to fewer splits.
  static const int kSplits[] = {1, 2, 3, 4, 6, 12};
  static const int kRows[] = {4, 2, 1};
  int64_t best = -1;
  for (int ks : kSplits) {
    const int slice = ((U + ks - 1) / ks + 3) / 4 * 4;  // whole 256-column groups
    const int upl = (slice + 31) / 32;
    if (upl > upl_max) continue;
    const int rg = kCW / ks;
    // Two CTAs share an SM for the variants built for it (dual_variant) when
    // every CTA still gets at least two tiles; small products keep one CTA
    // per SM.
    int per_sm = 1;
    if (dual_enabled() && dual_variant(t, np, upl, pair)) {
      int64_t tiles = 0;
      for (int m = 0; m < j.n_mat; ++m) tiles += (j.rows[m] + rg - 1) / rg;  // at rw = 1
      per_sm = tiles >= (int64_t)4 * 4 * g_num_sms ? 2 : 1;  // >= 2 tiles per CTA at rw = 4
    }
    const int cap = per_sm == 2 ? g_smem_dual : smem_cap;
    for (int rw : kRows) {
      const int R = rg * rw;
      const int64_t half = ((int64_t)R * row_bytes + 32 + 15) / 16 * 16;
      const int64_t stage = half * (pair ? 2 : 1);
      if (stage_off + 2 * stage > cap) continue;
      int64_t batches = 0;
      for (int m = 0; m < j.n_mat; ++m) batches += (j.rows[m] + R - 1) / R;
      const int64_t ctas = (int64_t)g_num_sms * per_sm;
      const int64_t waves = (batches + ctas - 1) / ctas;
      const int64_t cost = waves * (rw * upl * (pair ? 2 : 1) + 1);
      if (best < 0 || cost < best) {
        best = cost;
        pl.ks = ks;
        pl.slice = slice;
        pl.upl = upl;
        pl.rw = rw;
        pl.half_bytes = (int)half;
        pl.stage_bytes = (int)stage;
        pl.ctas_per_sm = per_sm;
      }
    }
  }
  if (best < 0) return pl;
  const int R = (kCW / pl.ks) * pl.rw;
  pl.total_batches = 0;
  for (int m = 0; m < j.n_mat; ++m) {
    pl.batch_begin[m] = pl.total_batches;
    pl.total_batches += (j.rows[m] + R - 1) / R;
  }
  const int cap = pl.ctas_per_sm == 2 ? g_smem_dual : smem_cap;
  const int64_t max_grid = (int64_t)g_num_sms * pl.ctas_per_sm;
  int stages = (int)((cap - stage_off) / pl.stage_bytes);
  if (stages > kMaxStages) stages = kMaxStages;
  // No more stages than a CTA has tiles (plus one): small products then
  // initialise fewer barriers and claim less shared memory.
  {
    const int64_t grid = pl.total_batches < max_grid ? pl.total_batches : max_grid;
    const int64_t per_cta = grid > 0 ? (pl.total_batches + grid - 1) / grid : 1;
    if (per_cta + 1 < stages) stages = (int)(per_cta + 1 > 2 ? per_cta + 1 : 2);
  }
  if (stages < 2) return pl;
  pl.stages = stages;
  pl.smem = (size_t)stage_off + (size_t)stages * pl.stage_bytes;
  pl.smem_cap = cap;
  pl.grid = (int)(pl.total_batches < max_grid ? pl.total_batches : max_grid);
  pl.streaming = pl.grid > 0;
  (void)total_rows;
  return pl;
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
}  // namespace gemv

using gemv::make_plan;

int gemv_engine(const GemvJob& job) { return make_plan(job).streaming ? 0 : 1; }

bool gemv_fusable(const GemvJob& job) {
  if (!job.x || job.K > gemv::kNormMaxPerThread * gemv::kCW * 32) return false;
  const gemv::Plan pl = make_plan(job);
  return pl.streaming && pl.x_raw_bytes > 0;
}

cudaError_t launch_gemv(const GemvJob& j, cudaStream_t st) {
  using namespace gemv;
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
  p.xmode = j.x ? (j.quantize_q8 ? XQ8F : XF32) : XQ8;
  p.norm_w = j.norm_w;
  p.eps = j.eps;
  p.residual = j.residual ? 1 : 0;
  p.status = j.status;
  if ((j.norm_w || j.residual) && !gemv_fusable(j)) return cudaErrorNotSupported;
  const bool pair = j.up != nullptr;
  Plan pl = make_plan(j);
  pl.overlap = j.overlap;
  if (!pl.streaming) {
    if (p.xmode == XQ8F && j.K % 256 != 0) return cudaErrorNotSupported;
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
  p.x_off = kHeaderBytes;
  p.x_raw_off = pl.x_raw_off;
  p.x_pad_off = pl.x_pad_off;
  p.stage_off = (int)(pl.smem - (size_t)pl.stages * pl.stage_bytes);
  switch (j.dtype) {
    case Q4_K: return dispatch_fmt<Q4_K>(p, pl, pair, st);
    case Q6_K: return dispatch_fmt<Q6_K>(p, pl, pair, st);
    case Q8_0: return dispatch_fmt<Q8_0>(p, pl, pair, st);
    case Q2_0C: return dispatch_fmt<Q2_0C>(p, pl, pair, st);
    case STQ1_0: return dispatch_fmt<STQ1_0>(p, pl, pair, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace hyq
