// Decoder-step kernels around the quantized products: the rest of one
// single-token step of the Dense architecture (Hy-MT2, model.rs:374-547):
// embedding row, RMSNorm, RoPE with the per-head q/k norm, KV-cache append,
// attention over the cache, residual add and greedy argmax.  Every kernel
// that depends on the token position reads it from device memory, so a whole
// step is one CUDA graph replayed for every token.
//
// Numerics follow the reference's x86 branches: the dot products of the
// norms and of the attention scores are summed in the order of dot_avx2
// (quant.rs:2562-2596: two 8-lane FMA accumulators over 16-wide chunks, an
// 8-wide tail, a sequential lane sum from -0, the scalar tail); elementwise
// products are rounded separately as Rust does (no contraction).  Only the
// softmax exponential differs from the reference's libm expf.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "../../include/hyq.h"
#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace model {

// Every kernel here waits for its predecessor grid before touching memory
// (griddepcontrol.wait) and lets its own dependents launch at once.
using hyq::launch_ex;
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  return launch_ex(k, grid, block, smem, st, args...);
}

// Dynamic shared memory of the norm kernels: up to 2 kNormMaxN floats (the
// row and the weights; set once per device and kernel).
template <typename K>
void norm_smem_limit(K k) {
  static int done_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done_dev != dev) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 16384 * (int)sizeof(float));
    done_dev = dev;
  }
}

// RMSNorm of `rows` rows of n floats (rms_norm_into, model.rs:785-830; per
// head, model.rs:832-872): variance = dot(x, x) / n, scale = 1 / sqrt(var +
// eps), out = (x * scale) * w.  One CTA per row; the row and the weights are
// staged in shared memory in one batch of loads (n <= kNormMaxN) so that the
// 16-lane x86-order sum runs from there.
constexpr int kNormMaxN = 16384;

__device__ __forceinline__ float staged_rms_scale(const float* xs, int n, float eps) {
  __shared__ float scale_s;
  if (threadIdx.x < 16) {
    const float d = dot_x86(xs, xs, n, 0xffffu);
    if (threadIdx.x == 0) scale_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)n), eps)));
  }
  __syncthreads();
  return scale_s;
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                        int n, float eps, float* __restrict__ out) {
  grid_dependency_wait();
  allow_dependents_launch();
  extern __shared__ float xs[];  // [n] row, [n] weights
  float* wsm = xs + n;
  const float* xr = x + (size_t)blockIdx.x * n;
  float* orow = out + (size_t)blockIdx.x * n;
#pragma unroll 8
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i], wi = w[i];
    xs[i] = v;
    wsm[i] = wi;
  }
  __syncthreads();
  const float scale = staged_rms_scale(xs, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(__fmul_rn(xs[i], scale), wsm[i]);
}

// Embedding row (Weight::row_into, quant.rs:123-142) of the token held in
// device memory, decoded bit for bit.
template <int T>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t* __restrict__ w, int64_t row_bytes, int64_t n,
                                                     int64_t rows, const int32_t* __restrict__ token,
                                                     float* __restrict__ out, unsigned* status) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int64_t tok = token[blockIdx.y];  // output row blockIdx.y
  if (tok < 0 || tok >= rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(status, DEV_BAD_ARGS);
    return;
  }
  const uint8_t* row = w + tok * row_bytes;
  float* o = out + (size_t)blockIdx.y * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / block_len(T);
    o[i] = decode_elem<T>(row + b * block_bytes(T), (int)(i - b * block_len(T)));
  }
}

// RoPE (rope_with_cache, model.rs:874-913) of q and k with the table row of
// the current position, then (Dense, model.rs:443-446) the per-head RMSNorm
// with q_norm / k_norm; `norm_first` runs the norm before the rotation
// (HyV3, model.rs:425-428).  Also appends k and v to the KV cache at the
// position (KvCache::append, model.rs:650-667).  One warp per head; grid =
// heads + kv_heads.
constexpr int kRopeMaxDim = 256;

struct RopeArgs {
  float* q;
  float* k;
  const float* v;
  int heads, kv_heads, dim;
  const float* cos_tab;  // [positions, dim / 2]
  const float* sin_tab;
  int positions;
  const int32_t* pos;
  const float* q_norm;   // [dim] or null
  const float* k_norm;
  float eps;
  int norm_first;
  void* k_cache;         // [positions, kv_heads * dim], f32 or (kv16) binary16
  void* v_cache;
  int kv16;
  unsigned* status;
  // independent sequences: token t is sequence t at position pos[t], its
  // caches seq_stride floats further per sequence (0: one sequence, token t
  // at position *pos + t)
  int64_t seq_stride;
};

__device__ void head_norm(float* hd, const float* w, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  float scale = 0.f;
  const float d = dot_x86(hd, hd, dim, 0xffffffffu);  // both half-warps compute it
  scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(d, (float)dim), eps)));
  __syncwarp();
  for (int i = lane; i < dim; i += 32) hd[i] = __fmul_rn(__fmul_rn(hd[i], scale), w[i]);
  __syncwarp();
}

__device__ void head_rope(float* hd, const float* c, const float* s, int dim) {
  const int half = dim / 2;
  for (int j = threadIdx.x & 31; j < half; j += 32) {
    const float a = hd[j], b = hd[j + half];
    hd[j] = __fsub_rn(__fmul_rn(a, c[j]), __fmul_rn(b, s[j]));
    hd[j + half] = __fadd_rn(__fmul_rn(a, s[j]), __fmul_rn(b, c[j]));
  }
  __syncwarp();
}

__global__ void __launch_bounds__(32) rope_qk_kernel(const __grid_constant__ RopeArgs a) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int tok = blockIdx.y;
  const int base = a.seq_stride ? a.pos[tok] : *a.pos;
  const int pos = a.seq_stride ? base : base + tok;  // one sequence: token tok at *pos + tok
  if (base < 0 || pos >= a.positions) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
    return;
  }
  const int h = blockIdx.x;
  const bool is_q = h < a.heads;
  const size_t qrow = (size_t)tok * a.heads * a.dim, krow = (size_t)tok * a.kv_heads * a.dim;
  float* hd = is_q ? a.q + qrow + (size_t)h * a.dim : a.k + krow + (size_t)(h - a.heads) * a.dim;
  const float* nw = is_q ? a.q_norm : a.k_norm;
  const float* c = a.cos_tab + (size_t)pos * (a.dim / 2);
  const float* s = a.sin_tab + (size_t)pos * (a.dim / 2);
  // the head, its norm weights, the table row (and for a kv head its value
  // head) staged in shared memory in one batch of loads
  __shared__ float hs[kRopeMaxDim], ws[kRopeMaxDim], cs[kRopeMaxDim / 2], sn[kRopeMaxDim / 2], vs[kRopeMaxDim];
  const int kh = h - a.heads;
  const float* vv = a.v + krow + (size_t)kh * a.dim;
#pragma unroll 4
  for (int i = threadIdx.x; i < a.dim; i += 32) {
    hs[i] = hd[i];
    if (nw) ws[i] = nw[i];
    if (!is_q) vs[i] = vv[i];
    if (i < a.dim / 2) {
      cs[i] = c[i];
      sn[i] = s[i];
    }
  }
  __syncwarp();
  if (a.norm_first && nw) head_norm(hs, ws, a.dim, a.eps);
  head_rope(hs, cs, sn, a.dim);
  if (!a.norm_first && nw) head_norm(hs, ws, a.dim, a.eps);
  for (int i = threadIdx.x; i < a.dim; i += 32) hd[i] = hs[i];
  if (!is_q) {
    const size_t width = (size_t)a.kv_heads * a.dim;
    const size_t seq = a.seq_stride ? (size_t)tok * a.seq_stride : 0;
    const size_t off = seq + (size_t)pos * width + (size_t)kh * a.dim;
    if (a.kv16) {
      // f16 cache: each value rounded to nearest binary16
      __half* kc = static_cast<__half*>(a.k_cache) + off;
      __half* vc = static_cast<__half*>(a.v_cache) + off;
      for (int i = threadIdx.x; i < a.dim; i += 32) {
        kc[i] = __float2half_rn(hs[i]);
        vc[i] = __float2half_rn(vs[i]);
      }
    } else {
      float* kc = static_cast<float*>(a.k_cache) + off;
      float* vc = static_cast<float*>(a.v_cache) + off;
      for (int i = threadIdx.x; i < a.dim; i += 32) {
        kc[i] = hs[i];
        vc[i] = vs[i];
      }
    }
  }
}

// attention_into for one query token (model.rs:949-1021), split over the
// cached positions as in flash decoding.  CTA (split, kv head, token) takes
// positions [64 split, 64 split + 64) of 0..pos for every query head that
// shares the kv head (heads / kv_heads of them), so each K and V row is read
// once: both chunks are staged in shared memory with cp.async (the scores
// start on K while V lands).  Each query head's local max m, exponential sum
// l and unnormalised output go to the workspace, and the last CTA of a (token,
// kv head) to finish combines them per head:
// out = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M).  Scores are dot(q, k) *
// (1 / sqrt(dim)) in the reference's x86 dot order (one thread per position
// and head); the exponentials come from the device expf and the sums follow
// the split tree, so outputs match the reference to rounding, not bit for bit.
constexpr int kMaxPositions = 16384;
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxDim = 256;
constexpr int kAttnMaxGroup = 16;  // query heads per kv head
static_assert(kAttnThreads == 2 * kAttnChunk, "the score phase pairs two threads per position");

// Counters per (token, kv head) at the head of the workspace (sized for
// positions x heads slots), padded to 256 bytes.
inline size_t attn_counter_bytes(int64_t slots) { return ((size_t)slots * sizeof(unsigned) + 255) / 256 * 256; }

// Shared memory of one CTA: K chunk (padded rows), V chunk, the group's query
// heads (same padding), exponentials, combine weights and per-head inverse
// sums.  The K region also holds the V phase's per-group partial outputs.
// (dim % 4 == 0: the row stride in float4 units is 2 mod 8, so the thread
// pairs of the score phase read 8 distinct 4-bank groups per quarter warp)
__host__ __device__ inline int attn_kstride(int dim) { return (dim & 3) ? dim + 1 : dim + 4 * ((10 - (dim >> 2) % 8) % 8); }
inline size_t attn_smem_bytes(int dim, int group, int nsplit) {
  const size_t ks = (size_t)attn_kstride(dim);
  return sizeof(float) * (kAttnChunk * ks + (size_t)kAttnChunk * dim + group * ks + (size_t)group * kAttnChunk +
                          (size_t)group * nsplit + group);
}

// The specialised head-size kernel over an f16 cache keeps the chunk's K and
// V rows in binary16 in shared memory (widened to f32 where they are read):
// K rows padded to a stride of DIM + 8 halves (272 bytes at 128, so the
// score phase's 8-byte reads of 8 rows x 2 threads hit 32 distinct banks),
// V rows unpadded, then the f32 query heads, exponentials and combine
// weights as in the f32 layout.  Half the footprint: more CTAs per SM.
__host__ __device__ constexpr int attn_kstride_h(int dim) { return dim + 8; }
inline size_t attn_smem_bytes_h(int dim, int group, int nsplit) {
  const size_t ks = (size_t)attn_kstride(dim);
  return sizeof(__half) * (size_t)kAttnChunk * (attn_kstride_h(dim) + dim) +
         sizeof(float) * (group * ks + (size_t)group * kAttnChunk + (size_t)group * nsplit + group);
}

// a = x0 * y0 + a, b = x1 * y1 + b in one packed instruction (fma.rn.f32x2:
// each lane rounded as fmaf)
__device__ __forceinline__ void ffma2_into(float& a, float& b, float x0, float x1, float y0, float y1) {
  const float2 r = __ffma2_rn(make_float2(x0, x1), make_float2(y0, y1), make_float2(a, b));
  a = r.x;
  b = r.y;
}

// four binary16 values (one 8-byte shared load) as f32
__device__ __forceinline__ float4 ld_h4(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

struct AttnArgs {
  const float* q;
  const void* k_cache;   // f32, or binary16 in the KV16 kernels
  const void* v_cache;
  int heads, kv_heads, dim;
  const int32_t* pos;
  int positions;
  float* out;
  float* ws;           // [tokens][heads][splits][2 + dim]
  unsigned* counters;  // [tokens][kv_heads], zero between calls
  unsigned* status;
  int64_t seq_stride;  // as RopeArgs: 0 one sequence, else per-token sequences
  // fused RoPE + q/k RMSNorm + KV append (rope_qk of the step's token): the
  // raw q in `q`, the raw key and value rows of each token in k_new / v_new
  // ([tokens, kv_heads * dim]); the caches are written at the position
  int fuse;
  const float* k_new;
  const float* v_new;
  const float* cos_tab;
  const float* sin_tab;
  const float* q_norm;
  const float* k_norm;
  float eps;
  int norm_first;
  float* k_cache_w;
  float* v_cache_w;
};

// RoPE of one head in shared memory with its RMSNorm before or after
// (model.rs:429-446, as rope_qk_kernel); one warp.
__device__ void rope_head(float* hd, const float* nw, const float* c, const float* sn, int dim, float eps,
                          int norm_first) {
  if (norm_first && nw) head_norm(hd, nw, dim, eps);
  head_rope(hd, c, sn, dim);
  if (!norm_first && nw) head_norm(hd, nw, dim, eps);
}


// rows x dim floats from global rows `gstride` apart into shared rows
// `sstride` apart (16-byte copies when every row start is 16-byte aligned).
// DIM > 0: dim == DIM (16-byte copies), rows <= kAttnChunk, loops unrolled.
template <int DIM>
__device__ __forceinline__ void stage_rows(float* dst, int sstride, const float* src, size_t gstride, int rows,
                                           int dim, bool vec) {
  if constexpr (DIM > 0) {
    constexpr int w = DIM / 4, per = kAttnThreads / w;
    static_assert(kAttnThreads % w == 0, "whole rows per pass");
    const int c = threadIdx.x % w, i0 = threadIdx.x / w;
#pragma unroll
    for (int k = 0; k < kAttnChunk / per; ++k) {
      const int i = i0 + k * per;
      if (i < rows) cp_async16(dst + i * sstride + 4 * c, src + i * gstride + 4 * c);
    }
    return;
  }
  // element t = i * w + c of the rows x w copies (w = dim / 4 or dim), walked
  // with one division up front and carries after
  const int w = vec ? dim >> 2 : dim;
  int i = threadIdx.x / w, c = threadIdx.x - (threadIdx.x / w) * w;
  const int di = kAttnThreads / w, dc = kAttnThreads - di * w;
  for (; i < rows;) {
    if (vec) cp_async16(dst + i * sstride + 4 * c, src + i * gstride + 4 * c);
    else cp_async4(dst + i * sstride + c, src + i * gstride + c);
    i += di;
    c += dc;
    if (c >= w) {
      c -= w;
      ++i;
    }
  }
}

// eight binary16 values (one 16-byte load) widened to f32 at dst (16-byte aligned)
__device__ __forceinline__ void widen8(float* d, uint4 u) {
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&u.z));
  const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&u.w));
  *reinterpret_cast<float4*>(d) = make_float4(f0.x, f0.y, f1.x, f1.y);
  *reinterpret_cast<float4*>(d + 4) = make_float4(f2.x, f2.y, f3.x, f3.y);
}

// binary16 cache rows widened to f32 in shared memory: rows x dim halves from
// global rows `gstride` apart into f32 rows `sstride` apart, eight values per
// 16-byte load when `vec` (dim % 8 == 0 and 16-byte aligned rows), else one
// at a time.  Plain loads, complete when the function returns.
template <int DIM>
__device__ __forceinline__ void stage_rows_h(float* dst, int sstride, const __half* src, size_t gstride, int rows,
                                             int dim, bool vec) {
  if (vec) {
    const int w = (DIM ? DIM : dim) >> 3;
    for (int t = threadIdx.x; t < rows * w; t += kAttnThreads) {
      const int i = t / w, c = t - i * w;
      widen8(dst + i * sstride + 8 * c, *reinterpret_cast<const uint4*>(src + i * gstride + 8 * c));
    }
    return;
  }
  for (int t = threadIdx.x; t < rows * dim; t += kAttnThreads) {
    const int i = t / dim, c = t - i * dim;
    dst[i * sstride + c] = __half2float(src[i * gstride + c]);
  }
}

// The end of every attention CTA: once this CTA's partials (max, sum and
// unnormalised output per head, in the workspace) are written, count the
// CTA; the last CTA of a (token, head group) combines the chunks per head:
// out = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M).
__device__ void attn_finish(const AttnArgs& a, int tok, int hblk, int G, int dim, int used, int nsplit, size_t h0,
                            float* cw_s, float* inv_s) {
  __shared__ int last_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int outs = G * dim;
  // the CTA's partials are ordered before the count by the barrier and
  // thread 0's device-scope fence
  __syncthreads();
  unsigned* counter = a.counters + (size_t)tok * gridDim.y + hblk;
  if (threadIdx.x == 0) {
    __threadfence();
    last_s = atomicAdd(counter, 1u) == (unsigned)(used - 1);
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // partials of other CTAs are read past L1 (__ldcg).  The loads of the
  // first eight splits' partial outputs of this thread's first four outputs
  // are issued before the combine weights are computed, and every lane
  // loads the (max, sum) pairs of its splits at once: one round trip to L2
  // for a combine of up to eight splits.
  const size_t stride = 2 + (size_t)dim;
  float pre[4][8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int t = min((int)threadIdx.x + k * kAttnThreads, outs - 1);
    const int g = t / dim;
    const float* src = a.ws + (h0 + g) * nsplit * stride + 2 + (t - g * dim);
#pragma unroll
    for (int j = 0; j < 8; ++j) pre[k][j] = j < used ? __ldcg(src + (size_t)j * stride) : 0.f;
  }
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    const float* wh = a.ws + (h0 + g) * nsplit * stride;
    float* cw = cw_s + g * nsplit;
    float m = -INFINITY, l = 0.f;
    if (used <= 32) {
      // one split per lane: its (max, sum) pair in one load round
      const float mi = lane < used ? __ldcg(wh + lane * stride) : -INFINITY;
      const float li = lane < used ? __ldcg(wh + lane * stride + 1) : 0.f;
      m = mi;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane < used) {
        const float c = expf(mi - m);
        cw[lane] = c;
        l = fmaf(li, c, l);
      }
    } else {
      for (int i = lane; i < used; i += 32) m = fmaxf(m, __ldcg(wh + i * stride));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      for (int i = lane; i < used; i += 32) {
        const float c = expf(__ldcg(wh + i * stride) - m);
        cw[i] = c;
        l = fmaf(__ldcg(wh + i * stride + 1), c, l);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) inv_s[g] = 1.0f / l;
  }
  __syncthreads();
  // four outputs per thread, their partials loaded eight splits at a time
  // (independent loads in flight), accumulated in split order
  for (int t0 = threadIdx.x; t0 < outs; t0 += 4 * kAttnThreads) {
    const float* src[4];
    const float* cw[4];
    float o[4];
    int gk[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = min(t0 + k * kAttnThreads, outs - 1);
      gk[k] = t / dim;
      src[k] = a.ws + (h0 + gk[k]) * nsplit * stride + 2 + (t - gk[k] * dim);
      cw[k] = cw_s + gk[k] * nsplit;
      o[k] = 0.f;
    }
    for (int i0 = 0; i0 < used; i0 += 8) {
      float v[4][8];
      const bool first = t0 == (int)threadIdx.x && i0 == 0;  // the prefetched batch
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[k][j] = first ? pre[k][j] : (i0 + j < used ? __ldcg(src[k] + (size_t)(i0 + j) * stride) : 0.f);
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j < used) o[k] = fmaf(v[k][j], cw[k][i0 + j], o[k]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = t0 + k * kAttnThreads;
      if (t < outs) a.out[(h0 + gk[k]) * dim + (t - gk[k] * dim)] = o[k] * inv_s[gk[k]];
    }
  }
  if (threadIdx.x == 0) *counter = 0;  // ready for the next call
}

// DIM, GRP > 0: a kernel for head size DIM whose CTAs take GRP query heads
// that share a kv head (loops unrolled to constant offsets; GRP may be a
// divisor of the heads per kv head, so that a small launch spreads over more
// CTAs: grid.y = heads / GRP); 0: any shape, a CTA per kv head.  KV16: the
// caches hold binary16 values (widened to f32 as they are staged; the
// arithmetic after that is the same).  Each head's arithmetic does not
// depend on how the heads are grouped.
template <int DIM, int GRP, bool KV16>
__global__ void __launch_bounds__(kAttnThreads, (KV16 && DIM > 0) ? 5 : 3)
    attention_kernel(const __grid_constant__ AttnArgs a) {
  static_assert(DIM == 0 || (DIM % 16 == 0 && kAttnThreads % (DIM / 4) == 0), "specialised head size");
  grid_dependency_wait();
  allow_dependents_launch();
  extern __shared__ __align__(16) float attn_smem[];
  // token tok of the batch sits at position *pos + tok and sees positions
  // 0 ..= it (causal, model.rs:959)
  const int tok = blockIdx.z;
  const int base = a.seq_stride ? a.pos[tok] : *a.pos;
  const int pos = a.seq_stride ? base : base + tok;
  if (base < 0 || pos >= a.positions) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
    return;
  }
  const int visible = pos + 1;
  const int used = (visible + kAttnChunk - 1) / kAttnChunk;  // splits with positions
  const int split = blockIdx.x, hblk = blockIdx.y;  // chunk, head group
  if (split >= used) return;
  const int dim = DIM ? DIM : a.dim, G = GRP ? GRP : a.heads / a.kv_heads, ks = attn_kstride(dim);
  const int kvh = hblk * G / (a.heads / a.kv_heads);  // the group's kv head
  const int nsplit = (a.positions + kAttnChunk - 1) / kAttnChunk;
  // f16 rows in shared memory (KV16, specialised head size), else f32 rows
  constexpr bool kHalf = KV16 && DIM > 0;
  constexpr int ksh = attn_kstride_h(DIM > 0 ? DIM : 8);
  __half* k_h = reinterpret_cast<__half*>(attn_smem);
  __half* v_h = k_h + kAttnChunk * ksh;
  float* k_s = attn_smem;
  float* v_s = k_s + kAttnChunk * ks;
  float* q_s = kHalf ? reinterpret_cast<float*>(v_h + kAttnChunk * (DIM > 0 ? DIM : 8)) : v_s + kAttnChunk * dim;
  float* e_s = q_s + G * ks;
  float* cw_s = e_s + G * kAttnChunk;
  float* inv_s = cw_s + G * nsplit;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t width = (size_t)a.kv_heads * dim;
  const size_t seq = a.seq_stride ? (size_t)tok * a.seq_stride : 0;
  const int p0 = split * kAttnChunk;
  const int n = min(kAttnChunk, visible - p0);
  const size_t c0 = seq + (size_t)p0 * width + (size_t)kvh * dim;  // element offset of the chunk
  const bool fresh = a.fuse && split == used - 1;
  const int n_stage = fresh ? n - 1 : n;
  bool vec;
  if constexpr (KV16) {
    const __half* kg = static_cast<const __half*>(a.k_cache) + c0;
    const __half* vg = static_cast<const __half*>(a.v_cache) + c0;
    const bool v8 = (dim & 7) == 0 && (width & 7) == 0 &&
                    ((reinterpret_cast<uintptr_t>(kg) | reinterpret_cast<uintptr_t>(vg)) & 15) == 0;
    vec = (dim & 3) == 0;
    if constexpr (kHalf) {
      // the host launches this kernel for 16-byte aligned rows only
      if (!v8) {
        if (threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
        return;
      }
      // raw binary16 rows by cp.async, K then V (the scores start on K while V lands)
      constexpr int w = (DIM > 0 ? DIM : 8) / 8, per = kAttnThreads / w;
      static_assert(kAttnThreads % w == 0 && kAttnChunk % per == 0, "whole rows per pass");
      const int c = threadIdx.x % w, i0 = threadIdx.x / w;
#pragma unroll
      for (int k = 0; k < kAttnChunk / per; ++k) {
        const int i = i0 + k * per;
        if (i < n_stage) cp_async16(k_h + i * ksh + 8 * c, kg + i * width + 8 * c);
      }
      cp_async_commit();
#pragma unroll
      for (int k = 0; k < kAttnChunk / per; ++k) {
        const int i = i0 + k * per;
        if (i < n_stage) cp_async16(v_h + i * (DIM > 0 ? DIM : 8) + 8 * c, vg + i * width + 8 * c);
      }
      cp_async_commit();
    } else {
      stage_rows_h<DIM>(k_s, ks, kg, width, n_stage, dim, v8);
      stage_rows_h<DIM>(v_s, dim, vg, width, n_stage, dim, v8);
    }
  } else {
    const float* kg = static_cast<const float*>(a.k_cache) + c0;
    const float* vg = static_cast<const float*>(a.v_cache) + c0;
    vec = (dim & 3) == 0 && (width & 3) == 0 &&
          ((reinterpret_cast<uintptr_t>(kg) | reinterpret_cast<uintptr_t>(vg)) & 15) == 0;
    // (the specialised kernel is launched only for 16-byte aligned caches)
    // fused step: the last chunk ends at the token's own position, whose key
    // and value rows this CTA builds instead of reading them from the cache
    stage_rows<DIM>(k_s, ks, kg, width, n_stage, dim, vec);
    cp_async_commit();
    stage_rows<DIM>(v_s, dim, vg, width, n_stage, dim, vec);
    cp_async_commit();
  }
  const size_t h0 = (size_t)tok * a.heads + (size_t)hblk * G;  // (token, first head of the group)
  const float* qg = a.q + h0 * dim;
  if (vec && (reinterpret_cast<uintptr_t>(qg) & 15) == 0) {
    const int q4 = dim >> 2;
    for (int t = threadIdx.x; t < G * q4; t += kAttnThreads) {
      const int g = t / q4;
      *reinterpret_cast<float4*>(q_s + g * ks + 4 * (t - g * q4)) = *reinterpret_cast<const float4*>(qg + 4 * t);
    }
  } else {
    for (int t = threadIdx.x; t < G * dim; t += kAttnThreads) {
      const int g = t / dim;
      q_s[g * ks + (t - g * dim)] = qg[t];
    }
  }
  if (!KV16 && a.fuse) {
    __syncthreads();  // the raw query heads are in q_s
    const float* c = a.cos_tab + (size_t)pos * (dim / 2);
    const float* sn = a.sin_tab + (size_t)pos * (dim / 2);
    for (int g = warp; g < G; g += kAttnThreads / 32) rope_head(q_s + g * ks, a.q_norm, c, sn, dim, a.eps, a.norm_first);
    // the new key row: a warp without a query head when there is one
    if (fresh && warp == (G < kAttnThreads / 32 ? G : 0)) {
      const size_t row = (size_t)tok * width + (size_t)kvh * dim;
      float* kr = k_s + (size_t)(n - 1) * ks;
      float* vr = v_s + (size_t)(n - 1) * dim;
      for (int i = lane; i < dim; i += 32) {
        kr[i] = a.k_new[row + i];
        vr[i] = a.v_new[row + i];
      }
      __syncwarp();
      rope_head(kr, a.k_norm, c, sn, dim, a.eps, a.norm_first);
      // KV append (no other CTA of this call reads the row; f32 caches
      // only); with several head groups per kv head the first one writes
      if (hblk % ((a.heads / a.kv_heads) / G) == 0) {
        float* kc = a.k_cache_w + seq + (size_t)pos * width + (size_t)kvh * dim;
        float* vc = a.v_cache_w + seq + (size_t)pos * width + (size_t)kvh * dim;
        for (int i = lane; i < dim; i += 32) {
          kc[i] = kr[i];
          vc[i] = vr[i];
        }
      }
    }
  }
  if constexpr (!KV16 || kHalf) cp_async_wait<1>();  // this thread's K copies
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dim));
  if (vec && (dim & 15) == 0) {
    // scores: a thread pair per position, each K row read once for every
    // head of the group.  dot_avx2's 16 accumulator lanes (quant.rs:2562-2596)
    // split as lanes {0-3, 8-11} (first thread: its pairwise sums are lanes
    // 0-3 of the horizontal sum) and {4-7, 12-15} (second: lanes 4-7).
    const int i = threadIdx.x >> 1, hh = threadIdx.x & 1;
    const float* kr = k_s + i * ks + 4 * hh;
    const __half* krh = k_h + i * ksh + 4 * hh;
    for (int g0 = 0; g0 < G; g0 += 4) {
      float acc[4][8];
#pragma unroll
      for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
#pragma unroll
      for (int c = 0; c < (DIM ? DIM : dim); c += 16) {
        const float4 k0 = kHalf ? ld_h4(krh + c) : *reinterpret_cast<const float4*>(kr + c);
        const float4 k1 = kHalf ? ld_h4(krh + c + 8) : *reinterpret_cast<const float4*>(kr + c + 8);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (g0 + g < G) {
            const float* qr = q_s + (g0 + g) * ks + 4 * hh + c;
            const float4 q0 = *reinterpret_cast<const float4*>(qr);
            const float4 q1 = *reinterpret_cast<const float4*>(qr + 8);
            ffma2_into(acc[g][0], acc[g][1], q0.x, q0.y, k0.x, k0.y);
            ffma2_into(acc[g][2], acc[g][3], q0.z, q0.w, k0.z, k0.w);
            ffma2_into(acc[g][4], acc[g][5], q1.x, q1.y, k1.x, k1.y);
            ffma2_into(acc[g][6], acc[g][7], q1.z, q1.w, k1.z, k1.w);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float sm[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) sm[j] = __fadd_rn(acc[g][j], acc[g][4 + j]);  // lanes 4 hh + j
        float h = -0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) h = __fadd_rn(h, sm[j]);
        float hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) hi[j] = __shfl_xor_sync(0xffffffffu, sm[j], 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) h = __fadd_rn(h, hi[j]);
        if (hh == 0 && i < n && g0 + g < G) e_s[(g0 + g) * kAttnChunk + i] = __fmul_rn(__fadd_rn(h, -0.0f), scale);
      }
    }
  } else {
    // scores: one thread per (head, position); a warp shares the head
    for (int t = threadIdx.x; t < G * kAttnChunk; t += kAttnThreads) {
      const int g = t / kAttnChunk, i = t - g * kAttnChunk;
      if (i < n) e_s[t] = __fmul_rn(dot_x86_thread(q_s + g * ks, k_s + i * ks, dim), scale);
    }
  }
  __syncthreads();
  // per head: local max, exponentials, their sum
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float* e = e_s + g * kAttnChunk;
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, e[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float x = expf(__fsub_rn(e[i], m));
      e[i] = x;
      l += x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      float* w = a.ws + ((h0 + g) * nsplit + split) * (2 + dim);
      w[0] = m;
      w[1] = l;
    }
  }
  if constexpr (!KV16 || kHalf) cp_async_wait<0>();
  __syncthreads();
  // unnormalised outputs per (head, dim): sum_i e_i v_i.  Thread (quad dq,
  // group pg) takes four consecutive dims of every head over the positions
  // of its group, in order; the groups' partials are then added in group
  // order (through the K region, free after the scores).
  const int outs = G * dim;
  const int q4 = dim >> 2;
  const int pgs = vec ? kAttnThreads / q4 : 0;  // position groups
  if (vec && q4 * pgs == kAttnThreads && kAttnChunk % pgs == 0 &&
      pgs * G * dim <= (kHalf ? kAttnChunk * ksh / 2 : kAttnChunk * ks)) {
    const int per = kAttnChunk / pgs;
    const int pg = threadIdx.x / q4, dq = threadIdx.x - pg * q4;
    const int i0 = pg * per, i1 = min(i0 + per, n);
    float* red = k_s;  // [pgs][G][dim]
    for (int g0 = 0; g0 < G; g0 += 4) {
      float4 o[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int ii = 0; ii < (DIM ? kAttnChunk / (kAttnThreads / (DIM / 4)) : per); ++ii) {
        const int i = i0 + ii;
        if (i >= i1) break;
        const float4 v = kHalf ? ld_h4(v_h + i * (DIM > 0 ? DIM : 8) + 4 * dq)
                               : *reinterpret_cast<const float4*>(v_s + i * dim + 4 * dq);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (g0 + g < G) {
            const float ei = e_s[(g0 + g) * kAttnChunk + i];
            ffma2_into(o[g].x, o[g].y, ei, ei, v.x, v.y);
            ffma2_into(o[g].z, o[g].w, ei, ei, v.z, v.w);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < 4; ++g)
        if (g0 + g < G) *reinterpret_cast<float4*>(red + ((size_t)pg * G + g0 + g) * dim + 4 * dq) = o[g];
    }
    __syncthreads();
    for (int t = threadIdx.x; t < outs; t += kAttnThreads) {
      float v = red[t];
      for (int z = 1; z < pgs; ++z) v = __fadd_rn(v, red[(size_t)z * outs + t]);
      const int g = t / dim;
      a.ws[((h0 + g) * nsplit + split) * (2 + dim) + 2 + (t - g * dim)] = v;
    }
  } else {
    // any head size: a thread per (head, dim), positions in order
    for (int t0 = threadIdx.x; t0 < outs; t0 += 4 * kAttnThreads) {
      int eo[4], vo[4];
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = min(t0 + j * kAttnThreads, outs - 1);
        const int g = t / dim;
        eo[j] = g * kAttnChunk;
        vo[j] = t - g * dim;
        o[j] = 0.f;
      }
      for (int i = 0; i < n; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = fmaf(e_s[eo[j] + i], v_s[i * dim + vo[j]], o[j]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = t0 + j * kAttnThreads;
        if (t < outs) a.ws[((h0 + t / dim) * nsplit + split) * (2 + dim) + 2 + vo[j]] = o[j];
      }
    }
  }
  attn_finish(a, tok, hblk, G, dim, used, nsplit, h0, cw_s, inv_s);
}

__global__ void __launch_bounds__(256) add_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
  grid_dependency_wait();
  allow_dependents_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __fadd_rn(dst[i], src[i]);
}

// add (model.rs:1043-1071) followed by rms_norm_into (model.rs:785-830) of
// the sum: hidden += delta; out = (hidden * scale) * w.  One CTA; the sum is
// staged in shared memory for the norm.
__global__ void __launch_bounds__(256) add_rms_norm_kernel(float* __restrict__ hidden,
                                                            const float* __restrict__ delta,
                                                            const float* __restrict__ w, int n, float eps,
                                                            float* __restrict__ out) {
  grid_dependency_wait();
  allow_dependents_launch();
  extern __shared__ float xs[];  // [n] row, [n] weights
  float* wsm = xs + n;
  const size_t r = (size_t)blockIdx.x * n;  // one CTA per row
  hidden += r;
  delta += r;
  out += r;
#pragma unroll 8
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float h = hidden[i], d = delta[i], wi = w[i];
    xs[i] = __fadd_rn(h, d);
    wsm[i] = wi;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) hidden[i] = xs[i];
  const float scale = staged_rms_scale(xs, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(xs[i], scale), wsm[i]);
}

// Greedy token (generation.rs:281-290): the first index of the largest value
// (NaN never wins; all-NaN gives 0).  Many CTAs: each reduces its share to a
// 64-bit key (order-preserving value bits, then ~index so that the lowest
// index wins a tie; -0 counts as +0) and folds it into workspace[0] with
// atomicMax; the last CTA to finish (counter in workspace[1]) writes the
// token, advances the position and leaves the workspace zero.
constexpr int kArgmaxThreads = 512;

__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned i) {
  if (isnan(v)) return 0ull;
  unsigned b = __float_as_uint(v == 0.0f ? 0.0f : v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xffffffffu - i);
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ x, int n, int32_t* token,
                                                                int32_t* pos, int pos_step, unsigned long long* ws) {
  grid_dependency_wait();
  allow_dependents_launch();
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(x[i], (unsigned)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  __shared__ unsigned long long wb[kArgmaxThreads / 32];
  __shared__ int last_s;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) wb[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = wb[w] > best ? wb[w] : best;
    atomicMax(&ws[0], best);
    __threadfence();
    last_s = atomicAdd(reinterpret_cast<unsigned*>(&ws[1]), 1u) == gridDim.x - 1;
    if (last_s) {
      __threadfence();
      const unsigned long long k = atomicExch(&ws[0], 0ull);
      atomicExch(reinterpret_cast<unsigned*>(&ws[1]), 0u);
      *token = k ? (int32_t)(0xffffffffu - (unsigned)(k & 0xffffffffull)) : 0;
      if (pos) *pos += pos_step;
    }
  }
}

// Greedy tokens of `rows` independent sequences (generation.rs:281-290 per
// row): one CTA per row, the first index of the largest value (NaN never
// wins, all-NaN gives 0); token[r] and pos[r] += 1.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ x, int n, int32_t* token,
                                                           int32_t* pos) {
  grid_dependency_wait();
  allow_dependents_launch();
  const float* xr = x + (size_t)blockIdx.x * n;
  unsigned long long best = 0ull;
  // float4 loads, four in flight per thread (the maximum does not depend on
  // the order); the unaligned head and the tail one by one
  const int head = min(n, (int)(((16u - (unsigned)(reinterpret_cast<uintptr_t>(xr) & 15u)) & 15u) / 4u));
  const int n4 = (n - head) / 4;
  const float4* x4 = reinterpret_cast<const float4*>(xr + head);
  if ((reinterpret_cast<uintptr_t>(xr) & 3u) == 0) {
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = x4[i];
      const unsigned j = (unsigned)(head + 4 * i);
      unsigned long long k = argmax_key(v.x, j);
      best = k > best ? k : best;
      k = argmax_key(v.y, j + 1);
      best = k > best ? k : best;
      k = argmax_key(v.z, j + 2);
      best = k > best ? k : best;
      k = argmax_key(v.w, j + 3);
      best = k > best ? k : best;
    }
    for (int i = threadIdx.x; i < head; i += blockDim.x) {
      const unsigned long long k = argmax_key(xr[i], (unsigned)i);
      best = k > best ? k : best;
    }
    for (int i = head + 4 * n4 + threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long k = argmax_key(xr[i], (unsigned)i);
      best = k > best ? k : best;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long k = argmax_key(xr[i], (unsigned)i);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  __shared__ unsigned long long wb[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) wb[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = wb[w] > best ? wb[w] : best;
    token[blockIdx.x] = best ? (int32_t)(0xffffffffu - (unsigned)(best & 0xffffffffull)) : 0;
    if (pos) pos[blockIdx.x] += 1;
  }
}

}  // namespace model
}  // namespace hyq

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace {
// SMs of the current device (148 if the query fails)
int sm_count() {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}
}  // namespace

extern "C" {

int hyq_rope_table(int64_t positions, int head_dim, float rope_base, float* cos_out, float* sin_out) {
  if (positions < 0 || head_dim <= 0 || (head_dim & 1) || !cos_out || !sin_out)
    return hyq::api_fail(HYQ_E_INVALID, "rope_table: bad arguments");
  const int half = head_dim / 2;
  for (int j = 0; j < half; ++j) {
    // model.rs:266-272 and 378-391: f32 powf, then (pos * freq).sin_cos()
    const float freq = powf(rope_base, -2.0f * (float)j / (float)head_dim);
    for (int64_t p = 0; p < positions; ++p) {
      const float a = (float)p * freq;
      sin_out[p * half + j] = sinf(a);
      cos_out[p * half + j] = cosf(a);
    }
  }
  return HYQ_OK;
}

int hyq_rms_norm(const float* x, const float* w, int64_t n, int64_t rows, float eps, float* out, void* stream) {
  if (!x || !w || !out) return hyq::api_fail(HYQ_E_INVALID, "rms_norm: null pointer");
  if (n <= 0 || rows <= 0 || n > INT32_MAX || rows > INT32_MAX) return hyq::api_fail(HYQ_E_SHAPE, "rms_norm: shape");
  if (n > hyq::model::kNormMaxN) return hyq::api_fail(HYQ_E_SHAPE, "rms_norm: at most %d columns", hyq::model::kNormMaxN);
  hyq::model::norm_smem_limit(hyq::model::rms_norm_kernel);
  const cudaError_t e =
      hyq::model::launch(hyq::model::rms_norm_kernel, dim3((unsigned)rows), dim3(256), 2 * (size_t)n * sizeof(float),
                         (cudaStream_t)stream, x, w, (int)n, eps, out);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "rms_norm: %s", cudaGetErrorString(e));
}

int hyq_embed(const hyq_weight* w, const int32_t* token, int64_t count, float* out, void* stream) {
  int dtype = 0, ndim = 0;
  int64_t dims[3] = {};
  const void* data = nullptr;
  if (!w || !token || !out) return hyq::api_fail(HYQ_E_INVALID, "embed: null pointer");
  int rc = hyq_weight_info(w, &dtype, &ndim, dims, nullptr, &data);
  if (rc) return rc;
  if (ndim != 2) return hyq::api_fail(HYQ_E_SHAPE, "embed: weight is not a matrix");
  if (count <= 0 || count > 65535) return hyq::api_fail(HYQ_E_SHAPE, "embed: 1 to 65535 tokens");
  unsigned* status = nullptr;
  if ((rc = hyq::api_status_word(&status))) return rc;
  const int64_t n = dims[0], rows = dims[1];
  const int64_t rb = n / hyq::block_len(dtype) * hyq::block_bytes(dtype);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  const uint8_t* wd = static_cast<const uint8_t*>(data);
  cudaError_t e = cudaSuccess;
  switch (dtype) {
    case hyq::F32: e = hyq::model::launch(hyq::model::embed_kernel<hyq::F32>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    case hyq::F16: e = hyq::model::launch(hyq::model::embed_kernel<hyq::F16>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    case hyq::Q4_K: e = hyq::model::launch(hyq::model::embed_kernel<hyq::Q4_K>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    case hyq::Q6_K: e = hyq::model::launch(hyq::model::embed_kernel<hyq::Q6_K>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    case hyq::Q8_0: e = hyq::model::launch(hyq::model::embed_kernel<hyq::Q8_0>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    case hyq::Q2_0C: e = hyq::model::launch(hyq::model::embed_kernel<hyq::Q2_0C>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
    default: e = hyq::model::launch(hyq::model::embed_kernel<hyq::STQ1_0>, dim3(blocks, (unsigned)count), dim3(256), 0, st, wd, rb, n, rows, token, out, status); break;
  }
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "embed: %s", cudaGetErrorString(e));
}

static int rope_qk_impl(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim,
                        const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                        int64_t tokens, const float* q_norm, const float* k_norm, float eps, int norm_first,
                        void* k_cache, void* v_cache, int64_t seq_stride, void* stream, int kv16 = 0) {
  if (!q || !k || !v || !cos_tab || !sin_tab || !pos || !k_cache || !v_cache)
    return hyq::api_fail(HYQ_E_INVALID, "rope_qk: null pointer");
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 || (head_dim & 1) || positions <= 0 ||
      positions > INT32_MAX)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_qk: shape");
  hyq::model::RopeArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.dim = head_dim;
  a.cos_tab = cos_tab;
  a.sin_tab = sin_tab;
  a.positions = (int)positions;
  a.pos = pos;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.eps = eps;
  a.norm_first = norm_first;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv16 = kv16;
  a.seq_stride = seq_stride;
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  if (tokens <= 0 || tokens > 65535 || tokens > positions)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_qk: 1 to %d tokens", (int)(positions < 65535 ? positions : 65535));
  const cudaError_t e = hyq::model::launch(hyq::model::rope_qk_kernel, dim3((unsigned)(heads + kv_heads),
                                           (unsigned)tokens), dim3(32), 0, (cudaStream_t)stream, a);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "rope_qk: %s", cudaGetErrorString(e));
}

int hyq_rope_qk(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                const float* sin_tab, int64_t positions, const int32_t* pos, int64_t tokens, const float* q_norm,
                const float* k_norm, float eps, int norm_first, float* k_cache, float* v_cache, void* stream) {
  return rope_qk_impl(q, k, v, heads, kv_heads, head_dim, cos_tab, sin_tab, positions, pos, tokens, q_norm, k_norm,
                      eps, norm_first, k_cache, v_cache, 0, stream);
}

int hyq_rope_qk_seqs(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                     const float* sin_tab, int64_t positions, const int32_t* pos, int64_t seqs, const float* q_norm,
                     const float* k_norm, float eps, int norm_first, float* k_cache, float* v_cache,
                     int64_t seq_stride, void* stream) {
  if (seq_stride < positions * kv_heads * head_dim)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_qk_seqs: sequences' caches overlap (stride %lld)", (long long)seq_stride);
  return rope_qk_impl(q, k, v, heads, kv_heads, head_dim, cos_tab, sin_tab, positions, pos, seqs, q_norm, k_norm,
                      eps, norm_first, k_cache, v_cache, seq_stride, stream);
}

int hyq_rope_qk_kv16(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                     const float* sin_tab, int64_t positions, const int32_t* pos, int64_t tokens, const float* q_norm,
                     const float* k_norm, float eps, int norm_first, uint16_t* k_cache, uint16_t* v_cache,
                     void* stream) {
  return rope_qk_impl(q, k, v, heads, kv_heads, head_dim, cos_tab, sin_tab, positions, pos, tokens, q_norm, k_norm,
                      eps, norm_first, k_cache, v_cache, 0, stream, 1);
}

int hyq_rope_qk_seqs_kv16(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim,
                          const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                          int64_t seqs, const float* q_norm, const float* k_norm, float eps, int norm_first,
                          uint16_t* k_cache, uint16_t* v_cache, int64_t seq_stride, void* stream) {
  if (seq_stride < positions * kv_heads * head_dim)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_qk_seqs_kv16: sequences' caches overlap (stride %lld)",
                         (long long)seq_stride);
  return rope_qk_impl(q, k, v, heads, kv_heads, head_dim, cos_tab, sin_tab, positions, pos, seqs, q_norm, k_norm,
                      eps, norm_first, k_cache, v_cache, seq_stride, stream, 1);
}

int hyq_attention_workspace_bytes(int heads, int head_dim, int64_t positions, int64_t tokens, size_t* bytes) {
  if (!bytes) return hyq::api_fail(HYQ_E_INVALID, "attention_workspace_bytes: null pointer");
  if (heads <= 0 || head_dim <= 0 || positions <= 0 || tokens <= 0)
    return hyq::api_fail(HYQ_E_SHAPE, "attention_workspace_bytes: shape");
  const int64_t splits = (positions + hyq::model::kAttnChunk - 1) / hyq::model::kAttnChunk;
  // the counter region does not depend on the call's token count (at most
  // `positions`), so calls with different counts share one workspace
  *bytes = hyq::model::attn_counter_bytes(positions * heads) +
           (size_t)tokens * heads * splits * (2 + head_dim) * sizeof(float);
  return HYQ_OK;
}

// RoPE + q/k RMSNorm + KV append folded into the attention launch.
struct AttnFuse {
  const float* k;
  const float* v;
  const float* cos_tab;
  const float* sin_tab;
  const float* q_norm;
  const float* k_norm;
  float eps;
  int norm_first;
  float* k_cache;
  float* v_cache;
};

static int attention_impl(const void* k_cache, const void* v_cache, const float* q, int heads, int kv_heads,
                          int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out,
                          void* workspace, int64_t seq_stride, void* stream, const AttnFuse* fuse, bool kv16) {
  if (!q || !k_cache || !v_cache || !pos || !out || !workspace)
    return hyq::api_fail(HYQ_E_INVALID, "attention: null pointer");
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > hyq::model::kAttnMaxGroup ||
      head_dim <= 0 || head_dim > hyq::model::kAttnMaxDim || positions <= 0 || positions > hyq::model::kMaxPositions)
    return hyq::api_fail(HYQ_E_SHAPE,
                         "attention: shape (head_dim at most %d, at most %d query heads per kv head, at most %d "
                         "positions)",
                         hyq::model::kAttnMaxDim, hyq::model::kAttnMaxGroup, hyq::model::kMaxPositions);
  if (reinterpret_cast<uintptr_t>(workspace) % 16) return hyq::api_fail(HYQ_E_INVALID, "attention: workspace alignment");
  hyq::model::AttnArgs a{};
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.dim = head_dim;
  a.pos = pos;
  a.positions = (int)positions;
  a.out = out;
  a.counters = static_cast<unsigned*>(workspace);
  a.seq_stride = seq_stride;
  if (fuse) {
    if (!fuse->k || !fuse->v || !fuse->cos_tab || !fuse->sin_tab || !fuse->k_cache || !fuse->v_cache)
      return hyq::api_fail(HYQ_E_INVALID, "rope_attention: null pointer");
    if (head_dim & 1) return hyq::api_fail(HYQ_E_SHAPE, "rope_attention: odd head_dim");
    // one sequence: one token (a prompt's tokens would read rows that other
    // CTAs of the launch append; prefill runs hyq_rope_qk + hyq_attention)
    if (!seq_stride && tokens != 1) return hyq::api_fail(HYQ_E_SHAPE, "rope_attention: one token per sequence");
    a.fuse = 1;
    a.k_new = fuse->k;
    a.v_new = fuse->v;
    a.cos_tab = fuse->cos_tab;
    a.sin_tab = fuse->sin_tab;
    a.q_norm = fuse->q_norm;
    a.k_norm = fuse->k_norm;
    a.eps = fuse->eps;
    a.norm_first = fuse->norm_first;
    a.k_cache_w = fuse->k_cache;
    a.v_cache_w = fuse->v_cache;
  }
  if (tokens <= 0 || tokens > 65535 || tokens > positions)
    return hyq::api_fail(HYQ_E_SHAPE, "attention: 1 to %d tokens", (int)(positions < 65535 ? positions : 65535));
  a.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + hyq::model::attn_counter_bytes(positions * heads));
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  const unsigned splits = (unsigned)((positions + hyq::model::kAttnChunk - 1) / hyq::model::kAttnChunk);
  size_t smem = hyq::model::attn_smem_bytes(head_dim, heads / kv_heads, (int)splits);
  // head size 128 with 4 query heads per kv head (the Dense and 7B shapes)
  // over 16-byte aligned caches: the specialised kernel.  A launch with few
  // CTAs (a single request: kv heads x chunks well under the SM count) gives
  // each CTA one query head instead of the kv head's four, so that the
  // scores and values of a chunk are spread over four times the CTAs (the
  // K/V chunk is then read by four CTAs, from L2).
  const bool fixed = head_dim == 128 && heads == 4 * kv_heads &&
                     ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) == 0 &&
                     (seq_stride & (kv16 ? 7 : 3)) == 0;
  const bool single = fixed && tokens * heads * (int64_t)splits <= 2 * (int64_t)sm_count();
  auto kern = kv16 ? (single ? hyq::model::attention_kernel<128, 1, true>
                             : fixed ? hyq::model::attention_kernel<128, 4, true> : hyq::model::attention_kernel<0, 0, true>)
                   : (single ? hyq::model::attention_kernel<128, 1, false>
                             : fixed ? hyq::model::attention_kernel<128, 4, false>
                                     : hyq::model::attention_kernel<0, 0, false>);
  const int group = single ? 1 : heads / kv_heads;  // query heads per CTA
  smem = (kv16 && fixed) ? hyq::model::attn_smem_bytes_h(head_dim, group, (int)splits)
                         : hyq::model::attn_smem_bytes(head_dim, group, (int)splits);
  const int kid = (kv16 ? 3 : 0) + (single ? 2 : fixed ? 1 : 0);
  static int smem_dev[6] = {-1, -1, -1, -1, -1, -1};  // the largest shape's shared memory, allowed once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem_dev[kid] != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)hyq::model::attn_smem_bytes(hyq::model::kAttnMaxDim, hyq::model::kAttnMaxGroup,
                                                          hyq::model::kMaxPositions / hyq::model::kAttnChunk));
    smem_dev[kid] = dev;
  }
  const cudaError_t e = hyq::model::launch(kern, dim3(splits, (unsigned)(heads / group), (unsigned)tokens),
                                           dim3(hyq::model::kAttnThreads), smem, (cudaStream_t)stream, a);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "attention: %s", cudaGetErrorString(e));
}

int hyq_attention(const float* q, const float* k_cache, const float* v_cache, int heads, int kv_heads,
                  int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out, void* workspace,
                  void* stream) {
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, tokens, out, workspace, 0,
                        stream, nullptr, false);
}

int hyq_attention_kv16(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads, int kv_heads,
                       int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out,
                       void* workspace, void* stream) {
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, tokens, out, workspace, 0,
                        stream, nullptr, true);
}

int hyq_attention_seqs_kv16(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads,
                            int kv_heads, int head_dim, int64_t positions, const int32_t* pos, int64_t seqs,
                            int64_t seq_stride, float* out, void* workspace, void* stream) {
  if (seq_stride < positions * kv_heads * head_dim)
    return hyq::api_fail(HYQ_E_SHAPE, "attention_seqs_kv16: sequences' caches overlap (stride %lld)",
                         (long long)seq_stride);
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, seqs, out, workspace,
                        seq_stride, stream, nullptr, true);
}

int hyq_attention_seqs(const float* q, const float* k_cache, const float* v_cache, int heads, int kv_heads,
                       int head_dim, int64_t positions, const int32_t* pos, int64_t seqs, int64_t seq_stride,
                       float* out, void* workspace, void* stream) {
  if (seq_stride < positions * kv_heads * head_dim)
    return hyq::api_fail(HYQ_E_SHAPE, "attention_seqs: sequences' caches overlap (stride %lld)", (long long)seq_stride);
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, seqs, out, workspace,
                        seq_stride, stream, nullptr, false);
}

int hyq_rope_attention(const float* q, const float* k, const float* v, int heads, int kv_heads, int head_dim,
                       const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                       const float* q_norm, const float* k_norm, float eps, int norm_first, float* k_cache,
                       float* v_cache, float* out, void* workspace, void* stream) {
  const AttnFuse f{k, v, cos_tab, sin_tab, q_norm, k_norm, eps, norm_first, k_cache, v_cache};
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, 1, out, workspace, 0, stream,
                        &f, false);
}

int hyq_rope_attention_seqs(const float* q, const float* k, const float* v, int heads, int kv_heads, int head_dim,
                            const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                            int64_t seqs, const float* q_norm, const float* k_norm, float eps, int norm_first,
                            float* k_cache, float* v_cache, int64_t seq_stride, float* out, void* workspace,
                            void* stream) {
  if (seq_stride < positions * kv_heads * head_dim)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_attention_seqs: sequences' caches overlap (stride %lld)",
                         (long long)seq_stride);
  const AttnFuse f{k, v, cos_tab, sin_tab, q_norm, k_norm, eps, norm_first, k_cache, v_cache};
  return attention_impl(k_cache, v_cache, q, heads, kv_heads, head_dim, positions, pos, seqs, out, workspace,
                        seq_stride, stream, &f, false);
}

int hyq_argmax_rows(const float* x, int64_t n, int64_t rows, int32_t* token, int32_t* pos, void* stream) {
  if (!x || !token) return hyq::api_fail(HYQ_E_INVALID, "argmax_rows: null pointer");
  if (n <= 0 || n > INT32_MAX || rows <= 0 || rows > INT32_MAX) return hyq::api_fail(HYQ_E_SHAPE, "argmax_rows: shape");
  const cudaError_t e = hyq::model::launch(hyq::model::argmax_rows_kernel, dim3((unsigned)rows), dim3(1024), 0,
                                           (cudaStream_t)stream, x, (int)n, token, pos);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "argmax_rows: %s", cudaGetErrorString(e));
}

int hyq_add(float* dst, const float* src, int64_t n, void* stream) {
  if (!dst || !src) return hyq::api_fail(HYQ_E_INVALID, "add: null pointer");
  if (n <= 0) return n == 0 ? HYQ_OK : hyq::api_fail(HYQ_E_SHAPE, "add: negative length");
  const cudaError_t e = hyq::model::launch(hyq::model::add_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                                           (cudaStream_t)stream, dst, src, n);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "add: %s", cudaGetErrorString(e));
}

int hyq_add_rms_norm(float* hidden, const float* delta, const float* w, int64_t n, int64_t rows, float eps,
                     float* out, void* stream) {
  if (!hidden || !delta || !w || !out) return hyq::api_fail(HYQ_E_INVALID, "add_rms_norm: null pointer");
  if (n <= 0 || n > hyq::model::kNormMaxN || rows <= 0 || rows > INT32_MAX)
    return hyq::api_fail(HYQ_E_SHAPE, "add_rms_norm: 1 to %d columns", hyq::model::kNormMaxN);
  hyq::model::norm_smem_limit(hyq::model::add_rms_norm_kernel);
  const cudaError_t e = hyq::model::launch(hyq::model::add_rms_norm_kernel, dim3((unsigned)rows), dim3(256),
                                           2 * (size_t)n * sizeof(float), (cudaStream_t)stream, hidden, delta, w, (int)n,
                                           eps, out);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "add_rms_norm: %s", cudaGetErrorString(e));
}

int hyq_argmax(const float* x, int64_t n, int32_t* token, int32_t* pos, int pos_step, void* workspace,
               void* stream) {
  if (!x || !token || !workspace) return hyq::api_fail(HYQ_E_INVALID, "argmax: null pointer");
  if (n <= 0 || n > INT32_MAX) return hyq::api_fail(HYQ_E_SHAPE, "argmax: length");
  if (reinterpret_cast<uintptr_t>(workspace) % 8) return hyq::api_fail(HYQ_E_INVALID, "argmax: workspace alignment");
  // about 2048 values per CTA, at most one CTA per SM
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = (n + 4 * hyq::model::kArgmaxThreads - 1) / (4 * hyq::model::kArgmaxThreads);
  if (blocks > sms) blocks = sms;
  const cudaError_t e = hyq::model::launch(hyq::model::argmax_kernel, dim3((unsigned)blocks),
                                           dim3(hyq::model::kArgmaxThreads), 0, (cudaStream_t)stream, x, (int)n,
                                           token, pos, pos_step, static_cast<unsigned long long*>(workspace));
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "argmax: %s", cudaGetErrorString(e));
}

}  // extern "C"
