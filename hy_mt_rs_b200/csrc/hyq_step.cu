// One Dense decoder token step (hy-mt-rs src/model.rs:374-547) as a single
// persistent kernel: one CTA per SM runs every phase of the step, with a
// grid-wide barrier between dependent phases instead of a kernel boundary.
//
//   embed | per layer: QKV | RoPE + q/k norm + KV append + attention |
//   O (+ residual) | gate/up-SiLU | down (+ residual) | lm_head | argmax
//
// The products are the streaming GEMV engine of hyq_gemv_impl.cuh (the same
// decode, exact three-plane f32 arithmetic and reductions), with two changes
// that only a persistent kernel allows: the producer warp streams the weight
// tiles of all phases back to back (weights are static, so the tiles of the
// next phase are already in shared memory when its barrier opens), and the
// RMSNorm before QKV, gate/up and lm_head runs in every CTA's activation
// prologue (the x86-order sum of the normalised vector, model.rs:785-830),
// the residual add in the product's epilogue (model.rs:1043-1071) and RoPE,
// the q/k norm and the KV append in the attention phase.
//
// Cross-CTA data (activations written in an earlier phase of this launch) is
// read with ld.global.cg (L2), never through a possibly stale L1 line.  Every
// wait is bounded: a barrier or tile wait that runs past kWaitLimitNs raises
// a launch-wide abort word, sets a device status bit, and every CTA leaves at
// its next wait.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <new>
#include <vector>

#include "../../include/hyq.h"
#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace step {

using gemv::XUnit;

enum PhaseKind : int { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2, PH_ARGMAX = 3, PH_FINISH = 4 };

// One phase of the step (host-built table in device memory).
struct Phase {
  int kind;
  // products
  int fmt, rw, pair, n_mat, ks, rg, slice, K, row_bytes, half_bytes;
  int64_t total_batches;
  int64_t batch_begin[3];
  int64_t rows[3];
  const uint8_t* w[3];
  const uint8_t* up;
  float* y[3];
  const float* x;       // activations, or null: the hidden state normalised by norm_w
  const float* norm_w;
  int residual;         // y[0] is the hidden state: hidden[r] += product
  // attention
  float* k_cache;
  float* v_cache;
  const float* q_norm;
  const float* k_norm;
};

struct StepArgs {
  const Phase* phases;
  int n_phases;
  int H, heads, kv_heads, hd, positions, vocab;
  float eps;
  const uint8_t* embed;
  int64_t embed_row_bytes;
  const float* cos_tab;
  const float* sin_tab;
  float* hidden;
  float* q;
  float* k;
  float* v;
  float* attended;
  float* logits;
  int32_t* token;
  int32_t* pos;
  float* attn_ws;            // [heads][splits][2 + hd]
  unsigned* attn_counters;   // [heads], zero between launches
  unsigned* sync;            // [0] barrier arrivals, [1] abort, [2..3] argmax key: zero at launch
  unsigned* status;
  int stages, stage_bytes, stage_off, x_off, x_raw_off, x_pad_off;
};

constexpr int kAttnChunk = 32;
constexpr int kAttnMaxDim = 256;
constexpr int kAttnThreads = 128;   // consumer warps 0-3
constexpr int kAttnBarrier = 13;    // named barrier of those warps

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the consumer warps of every CTA.  Arrivals count up
// from zero through the whole launch (the host zeroes the word before each
// launch), so barrier number `epoch` is complete at epoch * gridDim.x.
__device__ bool grid_barrier(const StepArgs& a, unsigned& epoch, volatile int* cta_abort) {
  __shared__ int ok_s;
  gemv::consumers_sync();
  ++epoch;
  if (threadIdx.x == 0) {
    const unsigned target = epoch * gridDim.x;
    bool ok = *cta_abort == 0;
    // the CTA's writes (ordered before this thread by the barrier above)
    // become visible at gpu scope with the arrival
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    atomicAdd(&a.sync[0], 1u);
    const uint64_t t0 = globaltimer_ns();
    for (unsigned spins = 1; ok && ld_acquire(&a.sync[0]) < target; ++spins) {
      if ((spins & 31u) == 0) {
        if (ld_acquire(&a.sync[1])) ok = false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicExch(&a.sync[1], 1u);
          atomicOr(a.status, DEV_TIMEOUT_GRID);
          ok = false;
        }
      }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (!ok) *cta_abort = 1;
    ok_s = ok;
  }
  gemv::consumers_sync();
  return ok_s != 0;
}

// ---------------------------------------------------------------------------
// Products
// ---------------------------------------------------------------------------
__device__ __forceinline__ void phase_batch(const Phase& P, int64_t bt, int R, int& m, int64_t& row0, int& nrows) {
  m = 0;
  if (P.n_mat > 1 && bt >= P.batch_begin[1]) m = 1;
  if (P.n_mat > 2 && bt >= P.batch_begin[2]) m = 2;
  row0 = (bt - P.batch_begin[m]) * R;
  const int64_t left = P.rows[m] - row0;
  nrows = (int)(left < R ? left : R);
}

// The producer thread: the tiles of every product phase, in phase order.
__device__ void produce_all(const StepArgs& a, uint64_t* full, uint64_t* empty, volatile int* abort_flag,
                            uint8_t* stages) {
  const uint64_t policy = l2_evict_first_policy();
  const int S = a.stages;
  int64_t issued = 0;
  int s = 0;
  uint32_t par = 1;
  bool ok = true;
  for (int ph = 0; ph < a.n_phases && ok; ++ph) {
    const Phase& P = a.phases[ph];
    if (P.kind != PH_GEMV) continue;
    const int R = P.rg * P.rw;
    for (int64_t bt = blockIdx.x; bt < P.total_batches; bt += gridDim.x) {
      if (issued >= S && !mbar_wait(smem_addr(&empty[s]), par, abort_flag)) {
        atomicOr(a.status, DEV_TIMEOUT_EMPTY);
        *abort_flag = 1;
        ok = false;
        break;
      }
      fence_proxy_async_smem();
      int m, nrows;
      int64_t row0;
      phase_batch(P, bt, R, m, row0, nrows);
      uint8_t* dst = stages + (size_t)s * a.stage_bytes;
      const int64_t bytes = (int64_t)nrows * P.row_bytes;
      const uint8_t* src = P.w[m] + row0 * P.row_bytes;
      const uint8_t* srcu = P.pair ? P.up + row0 * P.row_bytes : nullptr;
      const uint32_t bar = smem_addr(&full[s]);
      const uint32_t b0 = gemv::stage_tail(dst, src, bytes);
      const uint32_t b1 = P.pair ? gemv::stage_tail(dst + P.half_bytes, srcu, bytes) : 0u;
      mbar_arrive_expect_tx(bar, b0 + b1);
      gemv::stage_bulk(dst, src, b0, bar, policy);
      if (P.pair) gemv::stage_bulk(dst + P.half_bytes, srcu, b1, bar, policy);
      ++issued;
      if (++s == S) {
        s = 0;
        par ^= 1u;
      }
    }
  }
  // Do not leave while copies into this CTA's shared memory are in flight.
  for (int64_t k = (issued > S ? issued - S : 0); k < issued; ++k)
    if (!mbar_wait(smem_addr(&full[k % S]), (uint32_t)((k / S) & 1), nullptr)) atomicOr(a.status, DEV_TIMEOUT_DRAIN);
}

// Activations of a product into shared memory (f32, K values): the hidden
// state normalised by norm_w (rms_norm_into, x86-order sum), or a buffer.
constexpr int kMaxPerThread = 16;  // K / (kCW * 32) for K <= 6144

__device__ void stage_activations(const StepArgs& a, const Phase& P, float* raw) {
  const int K = P.K, tid = threadIdx.x, nt = gemv::kCW * 32;
  const float* src = P.x ? P.x : a.hidden;
  for (int i = tid; i < K; i += nt) raw[i] = __ldcg(src + i);
  gemv::consumers_sync();
  if (!P.x) {
    __shared__ float scale_s;
    // the norm weights of this thread's columns, loaded while lanes 0-15 sum
    float wv[kMaxPerThread];
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) wv[j] = (tid + j * nt < K) ? P.norm_w[tid + j * nt] : 0.f;
    if (tid < 16) {
      // dot(x, x) in the x86 order (K % 16 == 0): lane tid accumulates
      // columns tid, tid + 16, ... sequentially, from registers loaded 16 at
      // a time
      float acc = 0.f;
      for (int c0 = 0; c0 < K / 16; c0 += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = raw[16 * (c0 + j) + tid];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc = fmaf(v[j], v[j], acc);
      }
      const float d = x86_lane_sum(acc, 0xffffu);
      if (tid == 0) scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)K), a.eps)));
    }
    gemv::consumers_sync();
    const float scale = scale_s;
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) {
      const int i = tid + j * nt;
      if (i < K) raw[i] = __fmul_rn(__fmul_rn(raw[i], scale), wv[j]);
    }
    gemv::consumers_sync();
  }
}

__device__ __forceinline__ void emit(const StepArgs& a, const Phase& P, int m, int64_t row, float out) {
  if (P.residual) {
    a.hidden[row] = __fadd_rn(__ldcg(a.hidden + row), out);  // add (model.rs:1043-1071)
  } else {
    P.y[m][row] = out;
  }
}

template <int FMT, int RW, bool PAIR>
__device__ bool gemv_phase(const StepArgs& a, const Phase& P, uint8_t* smem, uint64_t* full, uint64_t* empty,
                           volatile int* abort_flag, int& s, uint32_t& par, int64_t& it) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* raw = reinterpret_cast<float*>(smem + a.x_raw_off);
  stage_activations(a, P, raw);
  gemv::Params gp{};
  gp.K = P.K;
  gp.U = P.K / 64;
  gp.x_off = a.x_off;
  gp.x_raw_off = 0;
  gp.x_pad_off = a.x_pad_off;
  gp.xmode = gemv::XF32;
  gp.x = raw;
  gp.status = a.status;
  gemv::prepare_x<FMT, 3>(gp, smem);
  const int ks = P.ks, rg = P.rg, R = rg * RW;
  const int ksi = warp % ks, rgi = warp / ks;
  XUnit<3> xu[1];
  int uu[1], ui[1];
  bool uv[1];
  uu[0] = ksi * P.slice + lane;
  uv[0] = lane < P.slice && uu[0] < gp.U;
  ui[0] = uv[0] ? uu[0] : 0;
  gemv::load_x<FMT, 3>(gp, smem, uu[0], uv[0], xu[0]);
  const bool all_units = __all_sync(0xffffffffu, uv[0]);
  const int ridx = gemv::reduce_index<RW>(lane);
  const bool writer = gemv::reduce_writer<RW>(lane);
  const uint32_t stages_s = smem_addr(smem + a.stage_off);
  float* red = reinterpret_cast<float*>(smem + gemv::kRedOffset);
  const int row_bytes = P.row_bytes;
  for (int64_t bt = blockIdx.x; bt < P.total_batches; bt += gridDim.x, ++it) {
    bool ok = mbar_wait(smem_addr(&full[s]), par, abort_flag);
    if (ks > 1) ok = bar_red_and(1 + rgi, ks * 32, ok);
    if (!ok) {
      if (lane == 0) atomicOr(a.status, DEV_TIMEOUT_FULL);
      *abort_flag = 1;
      return false;
    }
    int m, nrows;
    int64_t row0;
    phase_batch(P, bt, R, m, row0, nrows);
    const uint32_t tile = stages_s + (uint32_t)s * (uint32_t)a.stage_bytes;
    const uint32_t base = tile + (uint32_t)(reinterpret_cast<uintptr_t>(P.w[m] + row0 * row_bytes) & 15);
    const uint32_t baseu =
        tile + (uint32_t)P.half_bytes +
        (PAIR ? (uint32_t)(reinterpret_cast<uintptr_t>(P.up + row0 * row_bytes) & 15) : 0u);
    float g[RW], u[RW];
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) g[rr] = u[rr] = 0.f;
    if (all_units && nrows == R)
      gemv::tile_rows<FMT, 3, 1, RW, PAIR, false>(base, baseu, row_bytes, rg, rgi, nrows, ui, uv, xu, g, u);
    else
      gemv::tile_rows<FMT, 3, 1, RW, PAIR, true>(base, baseu, row_bytes, rg, rgi, nrows, ui, uv, xu, g, u);
    gemv::warp_reduce_multi<RW>(g, lane);
    if (PAIR) gemv::warp_reduce_multi<RW>(u, lane);
    const int r = rgi + rg * ridx;
    if (ks == 1) {
      if (writer && r < nrows) {
        float out = g[0];
        if (PAIR) out = (g[0] / (1.0f + expf(-g[0]))) * u[0];  // quant.rs:573-574
        emit(a, P, m, row0 + r, out);
      }
    } else {
      float* rb = red + (it & 1) * (2 * gemv::kCW * 4);
      if (writer) {
        rb[((rgi * RW + ridx) * ks + ksi) * 2] = g[0];
        rb[((rgi * RW + ridx) * ks + ksi) * 2 + 1] = PAIR ? u[0] : 0.f;
      }
      bar_sync_named(1 + rgi, ks * 32);
      if (ksi == 0 && writer && r < nrows) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < ks; ++k) {
          gs += rb[((rgi * RW + ridx) * ks + k) * 2];
          us += rb[((rgi * RW + ridx) * ks + k) * 2 + 1];
        }
        float out = gs;
        if (PAIR) out = (gs / (1.0f + expf(-gs))) * us;
        emit(a, P, m, row0 + r, out);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[s]));
    if (++s == a.stages) {
      s = 0;
      par ^= 1u;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Attention: RoPE + q/k norm (Dense: after RoPE, model.rs:435-446), KV append
// (model.rs:650-667) and attention_into (model.rs:949-1021) in 64-position
// chunks with an on-device combine, as hyq_attention.  Work item = (head,
// chunk); consumer warps 0-3 of a CTA take one item at a time.
// ---------------------------------------------------------------------------
__device__ void rope_norm_warp(float* hs, const float* src, const float* c, const float* sn, const float* nw, int dim,
                               float eps) {
  const int lane = threadIdx.x & 31, half = dim / 2;
  for (int i = lane; i < dim; i += 32) hs[i] = __ldcg(src + i);
  __syncwarp();
  for (int j = lane; j < half; j += 32) {
    const float x0 = hs[j], x1 = hs[j + half];
    hs[j] = __fsub_rn(__fmul_rn(x0, c[j]), __fmul_rn(x1, sn[j]));
    hs[j + half] = __fadd_rn(__fmul_rn(x0, sn[j]), __fmul_rn(x1, c[j]));
  }
  __syncwarp();
  const float d = dot_x86(hs, hs, dim, 0xffffffffu);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)dim), eps)));
  __syncwarp();
  for (int i = lane; i < dim; i += 32) hs[i] = __fmul_rn(__fmul_rn(hs[i], scale), nw[i]);
  __syncwarp();
}

// kc/vc: shared-memory scratch for the chunk's key and value rows
// (kAttnChunk x dim each; the activation words' region, idle in this phase).
__device__ void attention_phase(const StepArgs& a, const Phase& P, float* kc, float* vc) {
  __shared__ float q_s[kAttnMaxDim], k_s[kAttnMaxDim], v_s[kAttnMaxDim];
  __shared__ float e_s[kAttnChunk];
  __shared__ float cw_s[16384 / kAttnChunk];
  __shared__ float bc[2];
  __shared__ int last_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp >= kAttnThreads / 32) return;
  const int dim = a.hd, group = a.heads / a.kv_heads;
  const int pos = *a.pos;
  const int used = (pos + 1 + kAttnChunk - 1) / kAttnChunk;
  const int nsplit = (a.positions + kAttnChunk - 1) / kAttnChunk;
  const size_t width = (size_t)a.kv_heads * dim;
  const float* c = a.cos_tab + (size_t)pos * (dim / 2);
  const float* sn = a.sin_tab + (size_t)pos * (dim / 2);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dim));
  for (int item = blockIdx.x; item < a.heads * used; item += gridDim.x) {
    const int h = item / used, split = item % used, kvh = h / group;
    const bool has_pos = split == used - 1;
    // the rotated, normalised query; the current key and value (the chunk
    // holding this position only), appended to the cache by the first head
    // of the group
    if (warp == 0) rope_norm_warp(q_s, a.q + (size_t)h * dim, c, sn, P.q_norm, dim, a.eps);
    if (warp == 1 && has_pos) {
      rope_norm_warp(k_s, a.k + (size_t)kvh * dim, c, sn, P.k_norm, dim, a.eps);
      for (int i = lane; i < dim; i += 32) v_s[i] = __ldcg(a.v + (size_t)kvh * dim + i);
      __syncwarp();
      if (h % group == 0) {
        for (int i = lane; i < dim; i += 32) {
          P.k_cache[(size_t)pos * width + (size_t)kvh * dim + i] = k_s[i];
          P.v_cache[(size_t)pos * width + (size_t)kvh * dim + i] = v_s[i];
        }
      }
    }
    const int p0 = split * kAttnChunk;
    const int n = min(kAttnChunk, pos + 1 - p0);
    // the chunk's cached key and value rows, coalesced 16-byte loads (rows
    // before this position were written by earlier launches)
    {
      const int vec = dim / 4, rows = has_pos ? n - 1 : n;
      for (int idx = tid; idx < rows * vec; idx += kAttnThreads) {
        const int i = idx / vec, c4 = idx - i * vec;
        const size_t off = (size_t)(p0 + i) * width + (size_t)kvh * dim + 4 * c4;
        reinterpret_cast<float4*>(kc + i * dim)[c4] = *reinterpret_cast<const float4*>(P.k_cache + off);
        reinterpret_cast<float4*>(vc + i * dim)[c4] = *reinterpret_cast<const float4*>(P.v_cache + off);
      }
    }
    bar_sync_named(kAttnBarrier, kAttnThreads);
    if (has_pos)
      for (int d = tid; d < dim; d += kAttnThreads) {
        kc[(n - 1) * dim + d] = k_s[d];
        vc[(n - 1) * dim + d] = v_s[d];
      }
    bar_sync_named(kAttnBarrier, kAttnThreads);
    for (int b0 = 2 * warp; b0 < n; b0 += kAttnThreads / 16) {
      const int i = b0 + (lane >> 4);
      const bool valid = i < n;
      const float d = dot_x86(q_s, kc + (valid ? i : 0) * dim, dim, 0xffffffffu);
      if (valid && (lane & 15) == 0) e_s[i] = __fmul_rn(d, scale);
    }
    bar_sync_named(kAttnBarrier, kAttnThreads);
    if (warp == 0) {
      float mx = -INFINITY;
      for (int i = lane; i < n; i += 32) mx = fmaxf(mx, e_s[i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float l = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float e = expf(__fsub_rn(e_s[i], mx));
        e_s[i] = e;
        l += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) {
        bc[0] = mx;
        bc[1] = l;
      }
    }
    bar_sync_named(kAttnBarrier, kAttnThreads);
    float* w = a.attn_ws + ((size_t)h * nsplit + split) * (2 + dim);
    for (int d = tid; d < dim; d += kAttnThreads) {
      float o = 0.f;
      for (int i = 0; i < n; ++i) o = fmaf(e_s[i], vc[i * dim + d], o);
      w[2 + d] = o;
    }
    if (tid == 0) {
      w[0] = bc[0];
      w[1] = bc[1];
    }
    __threadfence();
    bar_sync_named(kAttnBarrier, kAttnThreads);
    if (tid == 0) last_s = atomicAdd(&a.attn_counters[h], 1u) == (unsigned)(used - 1);
    bar_sync_named(kAttnBarrier, kAttnThreads);
    if (last_s) {
      __threadfence();
      const float* wh = a.attn_ws + (size_t)h * nsplit * (2 + dim);
      const size_t stride = 2 + (size_t)dim;
      if (warp == 0) {
        float mx = -INFINITY;
        for (int i = lane; i < used; i += 32) mx = fmaxf(mx, __ldcg(wh + i * stride));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float l = 0.f;
        for (int i = lane; i < used; i += 32) {
          const float cc = expf(__ldcg(wh + i * stride) - mx);
          cw_s[i] = cc;
          l = fmaf(__ldcg(wh + i * stride + 1), cc, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) bc[1] = 1.0f / l;
      }
      bar_sync_named(kAttnBarrier, kAttnThreads);
      const float inv = bc[1];
      for (int d = tid; d < dim; d += kAttnThreads) {
        float o = 0.f;
        for (int i = 0; i < used; ++i) o = fmaf(__ldcg(wh + i * stride + 2 + d), cw_s[i], o);
        a.attended[(size_t)h * dim + d] = o * inv;
      }
      if (tid == 0) a.attn_counters[h] = 0;  // ready for the next launch
    }
    bar_sync_named(kAttnBarrier, kAttnThreads);
  }
}

// ---------------------------------------------------------------------------
// Embedding row, greedy token (see hyq_model.cu: embed_kernel, argmax_kernel)
// ---------------------------------------------------------------------------
__device__ void embed_phase(const StepArgs& a) {
  const int64_t tok = *a.token;
  if (tok < 0 || tok >= a.vocab) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
    return;
  }
  const uint8_t* row = a.embed + tok * a.embed_row_bytes;
  for (int i = blockIdx.x * gemv::kCW * 32 + threadIdx.x; i < a.H; i += gridDim.x * gemv::kCW * 32) {
    const int b = i / block_len(Q6_K);
    a.hidden[i] = decode_elem<Q6_K>(row + b * block_bytes(Q6_K), i - b * block_len(Q6_K));
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned i) {
  if (isnan(v)) return 0ull;
  unsigned b = __float_as_uint(v == 0.0f ? 0.0f : v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xffffffffu - i);
}

__device__ void argmax_phase(const StepArgs& a) {
  __shared__ unsigned long long wb[gemv::kCW];
  unsigned long long best = 0ull;
  const int nt = gemv::kCW * 32;
  for (int i = blockIdx.x * nt + threadIdx.x; i < a.vocab; i += gridDim.x * nt) {
    const unsigned long long k = argmax_key(__ldcg(a.logits + i), (unsigned)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
  gemv::consumers_sync();
  if (threadIdx.x == 0) {
    for (int w = 1; w < gemv::kCW; ++w) best = wb[w] > best ? wb[w] : best;
    atomicMax(reinterpret_cast<unsigned long long*>(a.sync + 2), best);
  }
}

__device__ void finish_phase(const StepArgs& a) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long k = __ldcg(reinterpret_cast<const unsigned long long*>(a.sync + 2));
    *a.token = k ? (int32_t)(0xffffffffu - (unsigned)(k & 0xffffffffull)) : 0;
    *a.pos += 1;
  }
}

template <int FMT, int RW, bool PAIR>
__device__ bool run_gemv(const StepArgs& a, const Phase& P, uint8_t* smem, uint64_t* full, uint64_t* empty,
                         volatile int* abort_flag, int& s, uint32_t& par, int64_t& it) {
  return gemv_phase<FMT, RW, PAIR>(a, P, smem, full, empty, abort_flag, s, par, it);
}

__global__ void __launch_bounds__(gemv::kThreads, 1) step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + gemv::kMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * gemv::kMaxStages);
  uint8_t* stages = smem + a.stage_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The position comes from device memory (a graph replays the step), so the
  // host cannot check it.  A position outside the cache ends the launch
  // before any phase runs: no cache row, table row or token is touched, pos
  // is not advanced, and HYQ_DEV_BAD_ARGS is raised.  Every thread of every
  // CTA reads pos here, before the first grid barrier; the only write to it
  // (finish_phase) comes after the last one, so all CTAs agree.
  const int pos0 = *a.pos;
  if (pos0 < 0 || pos0 >= a.positions) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), gemv::kCW);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == gemv::kCW) {
    if (lane == 0) produce_all(a, full, empty, abort_flag, stages);
    return;
  }
  unsigned epoch = 0;
  int s = 0;
  uint32_t par = 0;
  int64_t it = 0;
  for (int ph = 0; ph < a.n_phases; ++ph) {
    const Phase& P = a.phases[ph];
    bool ok = true;
    switch (P.kind) {
      case PH_EMBED: embed_phase(a); break;
      case PH_ATTN: {
        float* kc = reinterpret_cast<float*>(smem + a.x_off);
        attention_phase(a, P, kc, kc + kAttnChunk * a.hd);
        break;
      }
      case PH_ARGMAX: argmax_phase(a); break;
      case PH_FINISH: finish_phase(a); break;
      default:
        if (P.fmt == Q6_K) ok = run_gemv<Q6_K, 2, false>(a, P, smem, full, empty, abort_flag, s, par, it);
        else if (P.pair) ok = run_gemv<Q2_0C, 2, true>(a, P, smem, full, empty, abort_flag, s, par, it);
        else if (P.rw == 1) ok = run_gemv<Q2_0C, 1, false>(a, P, smem, full, empty, abort_flag, s, par, it);
        else ok = run_gemv<Q2_0C, 2, false>(a, P, smem, full, empty, abort_flag, s, par, it);
        break;
    }
    if (!ok) atomicExch(&a.sync[1], 1u);
    if (ph + 1 < a.n_phases && !grid_barrier(a, epoch, abort_flag)) break;
  }
}

}  // namespace step
}  // namespace hyq

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
struct hyq_dense_step {
  hyq::step::StepArgs args;
  hyq::step::Phase* phases_dev = nullptr;
  void* scratch = nullptr;  // sync words, attention workspace
  size_t sync_bytes = 0;
  int grid = 0;
  size_t smem = 0;
};

namespace {

struct Mat {
  int dtype = 0;
  int64_t K = 0, N = 0;
  const uint8_t* data = nullptr;
};

int get_mat(const hyq_weight* w, Mat& m, const char* what) {
  int ndim = 0;
  int64_t dims[3] = {};
  const void* data = nullptr;
  if (!w) return hyq::api_fail(HYQ_E_INVALID, "dense_step: null %s", what);
  int rc = hyq_weight_info(w, &m.dtype, &ndim, dims, nullptr, &data);
  if (rc) return rc;
  if (ndim != 2) return hyq::api_fail(HYQ_E_SHAPE, "dense_step: %s is not a matrix", what);
  m.K = dims[0];
  m.N = dims[1];
  m.data = static_cast<const uint8_t*>(data);
  if (reinterpret_cast<uintptr_t>(m.data) & 15) return hyq::api_fail(HYQ_E_ALIGN, "dense_step: %s alignment", what);
  return HYQ_OK;
}

// A product phase: rows over tiles of kCW / ks row groups x rw rows.
hyq::step::Phase gemv_phase_of(int n_mat, const Mat* m, float* const* y, const Mat* up, int rw) {
  using namespace hyq;
  step::Phase P{};
  P.kind = step::PH_GEMV;
  P.fmt = m[0].dtype;
  P.rw = rw;
  P.pair = up != nullptr;
  P.n_mat = n_mat;
  P.K = (int)m[0].K;
  const int U = P.K / 64;
  P.ks = (U + 31) / 32;  // one 64-column unit per lane
  while (gemv::kCW % P.ks) ++P.ks;
  P.rg = gemv::kCW / P.ks;
  P.slice = ((U + P.ks - 1) / P.ks + 3) / 4 * 4;
  P.row_bytes = (int)(m[0].K / block_len(P.fmt) * block_bytes(P.fmt));
  const int R = P.rg * rw;
  P.half_bytes = (int)(((int64_t)R * P.row_bytes + 32 + 15) / 16 * 16);
  for (int i = 0; i < n_mat; ++i) {
    P.w[i] = m[i].data;
    P.rows[i] = m[i].N;
    P.y[i] = y ? y[i] : nullptr;
    P.batch_begin[i] = P.total_batches;
    P.total_batches += (m[i].N + R - 1) / R;
  }
  if (up) P.up = up->data;
  return P;
}

}  // namespace

extern "C" {

int hyq_dense_step_create(const hyq_dense_step_desc* d, hyq_dense_step** out) {
  using namespace hyq;
  if (!d || !out) return api_fail(HYQ_E_INVALID, "dense_step: null pointer");
  *out = nullptr;
  if (d->layers <= 0 || !d->layer || !d->hidden_state || !d->q || !d->k || !d->v || !d->attended || !d->gate ||
      !d->logits || !d->token || !d->pos || !d->cos_tab || !d->sin_tab || !d->output_norm)
    return api_fail(HYQ_E_INVALID, "dense_step: missing buffer");
  const int H = d->hidden, A = d->heads * d->head_dim, KV = d->kv_heads * d->head_dim;
  if (H <= 0 || H % 256 || d->head_dim <= 0 || d->head_dim > step::kAttnMaxDim || (d->head_dim & 1) ||
      d->heads <= 0 || d->kv_heads <= 0 || d->heads % d->kv_heads || d->positions <= 0 || d->positions > 16384 ||
      d->ffn % 256 || d->ffn > 16384 || A % 256)
    return api_fail(HYQ_E_SHAPE, "dense_step: unsupported shape");
  Mat emb;
  int rc = get_mat(d->embed, emb, "embed");
  if (rc) return rc;
  if (emb.dtype != Q6_K || emb.K != H) return api_fail(HYQ_E_UNSUPPORTED, "dense_step: the tied embedding must be Q6_K");
  std::vector<step::Phase> ph;
  step::Phase e{};
  e.kind = step::PH_EMBED;
  ph.push_back(e);
  for (int l = 0; l < d->layers; ++l) {
    const hyq_dense_layer& L = d->layer[l];
    Mat q, k, v, o, g, u, dn;
    if ((rc = get_mat(L.q, q, "q")) || (rc = get_mat(L.k, k, "k")) || (rc = get_mat(L.v, v, "v")) ||
        (rc = get_mat(L.o, o, "o")) || (rc = get_mat(L.gate, g, "gate")) || (rc = get_mat(L.up, u, "up")) ||
        (rc = get_mat(L.down, dn, "down")))
      return rc;
    const Mat* all[7] = {&q, &k, &v, &o, &g, &u, &dn};
    for (const Mat* m : all)
      if (m->dtype != Q2_0C) return api_fail(HYQ_E_UNSUPPORTED, "dense_step: layer products must be Q2_0C");
    if (q.K != H || k.K != H || v.K != H || q.N != A || k.N != KV || v.N != KV || o.K != A || o.N != H ||
        g.K != H || u.K != H || g.N != d->ffn || u.N != d->ffn || dn.K != d->ffn || dn.N != H)
      return api_fail(HYQ_E_SHAPE, "dense_step: layer %d shapes", l);
    if (!L.input_norm || !L.ffn_norm || !L.q_norm || !L.k_norm || !L.k_cache || !L.v_cache)
      return api_fail(HYQ_E_INVALID, "dense_step: layer %d missing norm or cache", l);
    Mat qkv[3] = {q, k, v};
    float* ys[3] = {d->q, d->k, d->v};
    step::Phase P = gemv_phase_of(3, qkv, ys, nullptr, 2);
    P.norm_w = L.input_norm;
    ph.push_back(P);
    step::Phase at{};
    at.kind = step::PH_ATTN;
    at.k_cache = L.k_cache;
    at.v_cache = L.v_cache;
    at.q_norm = L.q_norm;
    at.k_norm = L.k_norm;
    ph.push_back(at);
    P = gemv_phase_of(1, &o, nullptr, nullptr, 1);
    P.x = d->attended;
    P.residual = 1;
    ph.push_back(P);
    float* gy[1] = {d->gate};
    P = gemv_phase_of(1, &g, gy, &u, 2);
    P.norm_w = L.ffn_norm;
    ph.push_back(P);
    P = gemv_phase_of(1, &dn, nullptr, nullptr, 2);
    P.x = d->gate;
    P.residual = 1;
    ph.push_back(P);
  }
  float* ly[1] = {d->logits};
  step::Phase P = gemv_phase_of(1, &emb, ly, nullptr, 2);
  P.norm_w = d->output_norm;
  ph.push_back(P);
  step::Phase am{};
  am.kind = step::PH_ARGMAX;
  ph.push_back(am);
  am.kind = step::PH_FINISH;
  ph.push_back(am);

  // shared memory: the GEMV header, activation words and staged f32 input
  // (largest input: the FFN width), then the ring of stages
  int stage = 0;
  for (const step::Phase& p : ph)
    if (p.kind == step::PH_GEMV) stage = std::max(stage, p.half_bytes * (p.pair ? 2 : 1));
  const int Umax = d->ffn / 64;
  const int x_bytes = (3 * 16 * Umax + 2 * (Umax / 4)) * 4;  // prepare_x: three planes of words, scales
  const int x_off = gemv::kHeaderBytes;
  const int x_raw_off = (x_off + x_bytes + 15) / 16 * 16;
  const int x_pad_off = (x_raw_off + d->ffn * 4 + 15) / 16 * 16;  // prepare_x's padded copy
  const int stage_off = (x_pad_off + Umax * 65 * 4 + 127) / 128 * 128;
  if (stage_off - x_off < 2 * step::kAttnChunk * d->head_dim * 4)
    return api_fail(HYQ_E_UNSUPPORTED, "dense_step: attention scratch does not fit");
  int dev = 0, optin = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaFuncAttributes fa{};
  cudaFuncGetAttributes(&fa, step::step_kernel);  // static shared memory of the phases
  int stages = (optin - (int)fa.sharedSizeBytes - stage_off) / stage;
  if (stages > gemv::kMaxStages) stages = gemv::kMaxStages;
  if (stages < 2) return api_fail(HYQ_E_UNSUPPORTED, "dense_step: shared memory too small");

  hyq_dense_step* st = new (std::nothrow) hyq_dense_step();
  if (!st) return api_fail(HYQ_E_NOMEM, "dense_step: host allocation");
  const int nsplit = (int)((d->positions + step::kAttnChunk - 1) / step::kAttnChunk);
  st->sync_bytes = 256;
  const size_t counters = ((size_t)d->heads * 4 + 255) / 256 * 256;
  const size_t ws = (size_t)d->heads * nsplit * (2 + d->head_dim) * sizeof(float);
  cudaError_t ce = cudaMalloc(&st->phases_dev, ph.size() * sizeof(step::Phase));
  if (ce == cudaSuccess) ce = cudaMalloc(&st->scratch, st->sync_bytes + counters + ws);
  if (ce == cudaSuccess) ce = cudaMemcpy(st->phases_dev, ph.data(), ph.size() * sizeof(step::Phase),
                                         cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = cudaMemset(st->scratch, 0, st->sync_bytes + counters + ws);
  if (ce == cudaSuccess)
    ce = cudaFuncSetAttribute(step::step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              stage_off + stages * stage);
  if (ce != cudaSuccess) {
    hyq_dense_step_free(st);
    return api_fail(HYQ_E_CUDA, "dense_step: %s", cudaGetErrorString(ce));
  }
  step::StepArgs& a = st->args;
  a.phases = st->phases_dev;
  a.n_phases = (int)ph.size();
  a.H = H;
  a.heads = d->heads;
  a.kv_heads = d->kv_heads;
  a.hd = d->head_dim;
  a.positions = (int)d->positions;
  a.vocab = (int)emb.N;
  a.eps = d->eps;
  a.embed = emb.data;
  a.embed_row_bytes = H / block_len(Q6_K) * block_bytes(Q6_K);
  a.cos_tab = d->cos_tab;
  a.sin_tab = d->sin_tab;
  a.hidden = d->hidden_state;
  a.q = d->q;
  a.k = d->k;
  a.v = d->v;
  a.attended = d->attended;
  a.logits = d->logits;
  a.token = d->token;
  a.pos = d->pos;
  a.sync = static_cast<unsigned*>(st->scratch);
  a.attn_counters = reinterpret_cast<unsigned*>(static_cast<char*>(st->scratch) + st->sync_bytes);
  a.attn_ws = reinterpret_cast<float*>(static_cast<char*>(st->scratch) + st->sync_bytes + counters);
  if ((rc = api_status_word(&a.status))) {
    hyq_dense_step_free(st);
    return rc;
  }
  a.stages = stages;
  a.stage_bytes = stage;
  a.stage_off = stage_off;
  a.x_off = x_off;
  a.x_raw_off = x_raw_off;
  a.x_pad_off = x_pad_off;
  st->grid = sms;
  st->smem = (size_t)stage_off + (size_t)stages * stage;
  *out = st;
  return HYQ_OK;
}

int hyq_dense_step_enqueue(hyq_dense_step* st, void* stream) {
  if (!st) return hyq::api_fail(HYQ_E_INVALID, "dense_step: null step");
  cudaStream_t s = (cudaStream_t)stream;
  // barrier arrivals, abort word and argmax key start at zero every launch
  cudaError_t e = cudaMemsetAsync(st->scratch, 0, 16, s);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "dense_step: %s", cudaGetErrorString(e));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (grid-wide barriers)
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)st->grid);
  cfg.blockDim = dim3(hyq::gemv::kThreads);
  cfg.dynamicSmemBytes = st->smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, hyq::step::step_kernel, st->args);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "dense_step: %s", cudaGetErrorString(e));
}

void hyq_dense_step_free(hyq_dense_step* st) {
  if (!st) return;
  if (st->phases_dev) cudaFree(st->phases_dev);
  if (st->scratch) cudaFree(st->scratch);
  delete st;
}

}  // extern "C"
