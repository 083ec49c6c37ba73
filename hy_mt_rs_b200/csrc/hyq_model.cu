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
#include <cuda_runtime.h>

#include <cmath>

#include "../../include/hyq.h"
#include "hyq_common.cuh"
#include "hyq_formats.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace model {

// Launch with the programmatic-dependent attribute when hyq_set_launch_overlap
// is on: every kernel here waits for its predecessor grid before touching
// memory (griddepcontrol.wait) and lets its own dependents launch at once.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Dynamic shared memory of the norm kernels: up to kNormMaxN floats (set once
// per device and kernel).
template <typename K>
void norm_smem_limit(K k) {
  static int done_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (done_dev != dev) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * (int)sizeof(float));
    done_dev = dev;
  }
}

// RMSNorm of `rows` rows of n floats (rms_norm_into, model.rs:785-830; per
// head, model.rs:832-872): variance = dot(x, x) / n, scale = 1 / sqrt(var +
// eps), out = (x * scale) * w.  One CTA per row; the row is staged in shared
// memory (n <= kNormMaxN) so that the 16-lane x86-order sum runs from there.
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
  extern __shared__ float xs[];
  const float* xr = x + (size_t)blockIdx.x * n;
  float* orow = out + (size_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = xr[i];
  __syncthreads();
  const float scale = staged_rms_scale(xs, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(__fmul_rn(xs[i], scale), w[i]);
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
  float* k_cache;        // [positions, kv_heads * dim]
  float* v_cache;
  unsigned* status;
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
  const int tok = blockIdx.y;  // token tok of the batch sits at position *pos + tok
  const int pos = *a.pos + tok;
  if (*a.pos < 0 || pos >= a.positions) {
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
  __shared__ float hs[kRopeMaxDim];  // the head, worked on in shared memory
  for (int i = threadIdx.x; i < a.dim; i += 32) hs[i] = hd[i];
  __syncwarp();
  if (a.norm_first && nw) head_norm(hs, nw, a.dim, a.eps);
  head_rope(hs, c, s, a.dim);
  if (!a.norm_first && nw) head_norm(hs, nw, a.dim, a.eps);
  for (int i = threadIdx.x; i < a.dim; i += 32) hd[i] = hs[i];
  if (!is_q) {
    const int kh = h - a.heads;
    const size_t width = (size_t)a.kv_heads * a.dim;
    float* kc = a.k_cache + (size_t)pos * width + (size_t)kh * a.dim;
    float* vc = a.v_cache + (size_t)pos * width + (size_t)kh * a.dim;
    const float* vv = a.v + krow + (size_t)kh * a.dim;
    for (int i = threadIdx.x; i < a.dim; i += 32) {
      kc[i] = hs[i];
      vc[i] = vv[i];
    }
  }
}

// attention_into for one query token (model.rs:949-1021), split over the
// cached positions as in flash decoding: CTA (split, head) takes positions
// [64 split, 64 split + 64) of 0..pos, writes its local max m, exponential
// sum l and unnormalised output to the workspace, and the last CTA of a head
// to finish combines them: out = sum_i o_i e^(m_i - M) / sum_i l_i e^(m_i - M).
// Scores are dot(q, k) * (1 / sqrt(dim)) in the reference's x86 dot order;
// the exponentials come from the device expf and the sums follow the split
// tree, so outputs match the reference to rounding, not bit for bit.
constexpr int kMaxPositions = 16384;
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxDim = 256;

// Counters per (token, head) at the head of the workspace, padded to 256 bytes.
inline size_t attn_counter_bytes(int64_t slots) { return ((size_t)slots * sizeof(unsigned) + 255) / 256 * 256; }

struct AttnArgs {
  const float* q;
  const float* k_cache;
  const float* v_cache;
  int heads, kv_heads, dim;
  const int32_t* pos;
  int positions;
  float* out;
  float* ws;           // [tokens][heads][splits][2 + dim]
  unsigned* counters;  // [tokens][heads], zero between calls
  unsigned* status;
};

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnArgs a) {
  grid_dependency_wait();
  allow_dependents_launch();
  __shared__ float q_s[kAttnMaxDim];
  __shared__ float e_s[kAttnChunk];
  __shared__ float cw_s[kMaxPositions / kAttnChunk];
  __shared__ float bc[2];
  __shared__ int last_s;
  // token tok of the batch sits at position *pos + tok and sees positions
  // 0 ..= it (causal, model.rs:959)
  const int tok = blockIdx.z;
  const int pos = *a.pos + tok;
  if (*a.pos < 0 || pos >= a.positions) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(a.status, DEV_BAD_ARGS);
    return;
  }
  const int visible = pos + 1;
  const int used = (visible + kAttnChunk - 1) / kAttnChunk;  // splits with positions
  const int split = blockIdx.x, h = blockIdx.y;
  if (split >= used) return;
  const int dim = a.dim;
  const int kvh = h / (a.heads / a.kv_heads);
  const size_t width = (size_t)a.kv_heads * dim;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dim));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t th = (size_t)tok * a.heads + h;  // (token, head) slot
  for (int d = threadIdx.x; d < dim; d += kAttnThreads) q_s[d] = a.q[th * dim + d];
  __syncthreads();
  const int p0 = split * kAttnChunk;
  const int n = min(kAttnChunk, visible - p0);
  // scores of this chunk in the x86 dot order: a half-warp per position
  for (int base = 2 * warp; base < n; base += kAttnThreads / 16) {
    const int i = base + (lane >> 4);
    const bool valid = i < n;
    const float* kr = a.k_cache + (size_t)(p0 + (valid ? i : 0)) * width + (size_t)kvh * dim;
    const float d = dot_x86(q_s, kr, dim, 0xffffffffu);
    if (valid && (lane & 15) == 0) e_s[i] = __fmul_rn(d, scale);
  }
  __syncthreads();
  // local max and exponentials
  if (warp == 0) {
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, e_s[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(__fsub_rn(e_s[i], m));
      e_s[i] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      bc[0] = m;
      bc[1] = l;
    }
  }
  __syncthreads();
  const int nsplit = (a.positions + kAttnChunk - 1) / kAttnChunk;
  float* w = a.ws + (th * nsplit + split) * (2 + dim);
  for (int d = threadIdx.x; d < dim; d += kAttnThreads) {
    const float* vr = a.v_cache + (size_t)p0 * width + (size_t)kvh * dim + d;
    float o = 0.f;
    for (int i = 0; i < n; ++i) o = fmaf(e_s[i], vr[(size_t)i * width], o);
    w[2 + d] = o;
  }
  if (threadIdx.x == 0) {
    w[0] = bc[0];
    w[1] = bc[1];
  }
  // the last CTA of this head combines the splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atomicAdd(&a.counters[th], 1u) == (unsigned)(used - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // partials of other CTAs are read past L1 (__ldcg)
  const float* wh = a.ws + th * nsplit * (2 + dim);
  const size_t stride = 2 + (size_t)dim;
  if (warp == 0) {
    float m = -INFINITY;
    for (int i = lane; i < used; i += 32) m = fmaxf(m, __ldcg(wh + i * stride));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int i = lane; i < used; i += 32) {
      const float c = expf(__ldcg(wh + i * stride) - m);
      cw_s[i] = c;
      l = fmaf(__ldcg(wh + i * stride + 1), c, l);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) bc[1] = 1.0f / l;
  }
  __syncthreads();
  const float inv = bc[1];
  for (int d = threadIdx.x; d < dim; d += kAttnThreads) {
    float o = 0.f;
    for (int i = 0; i < used; ++i) o = fmaf(__ldcg(wh + i * stride + 2 + d), cw_s[i], o);
    a.out[th * dim + d] = o * inv;
  }
  if (threadIdx.x == 0) a.counters[th] = 0;  // ready for the next call
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
  extern __shared__ float xs[];
  const size_t r = (size_t)blockIdx.x * n;  // one CTA per row
  hidden += r;
  delta += r;
  out += r;
#pragma unroll 4
  for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = __fadd_rn(hidden[i], delta[i]);
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) hidden[i] = xs[i];
  const float scale = staged_rms_scale(xs, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(xs[i], scale), w[i]);
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

}  // namespace model
}  // namespace hyq

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
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
      hyq::model::launch(hyq::model::rms_norm_kernel, dim3((unsigned)rows), dim3(256), (size_t)n * sizeof(float),
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

int hyq_rope_qk(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                const float* sin_tab, int64_t positions, const int32_t* pos, int64_t tokens, const float* q_norm,
                const float* k_norm, float eps, int norm_first, float* k_cache, float* v_cache, void* stream) {
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
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  if (tokens <= 0 || tokens > 65535 || tokens > positions)
    return hyq::api_fail(HYQ_E_SHAPE, "rope_qk: 1 to %d tokens", (int)(positions < 65535 ? positions : 65535));
  const cudaError_t e = hyq::model::launch(hyq::model::rope_qk_kernel, dim3((unsigned)(heads + kv_heads),
                                           (unsigned)tokens), dim3(32), 0, (cudaStream_t)stream, a);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "rope_qk: %s", cudaGetErrorString(e));
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

int hyq_attention(const float* q, const float* k_cache, const float* v_cache, int heads, int kv_heads,
                  int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out, void* workspace,
                  void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !workspace)
    return hyq::api_fail(HYQ_E_INVALID, "attention: null pointer");
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 || head_dim > hyq::model::kAttnMaxDim ||
      positions <= 0 || positions > hyq::model::kMaxPositions)
    return hyq::api_fail(HYQ_E_SHAPE, "attention: shape (head_dim at most %d, at most %d positions)",
                         hyq::model::kAttnMaxDim, hyq::model::kMaxPositions);
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
  if (tokens <= 0 || tokens > 65535 || tokens > positions)
    return hyq::api_fail(HYQ_E_SHAPE, "attention: 1 to %d tokens", (int)(positions < 65535 ? positions : 65535));
  a.ws = reinterpret_cast<float*>(static_cast<char*>(workspace) + hyq::model::attn_counter_bytes(positions * heads));
  int rc = hyq::api_status_word(&a.status);
  if (rc) return rc;
  const unsigned splits = (unsigned)((positions + hyq::model::kAttnChunk - 1) / hyq::model::kAttnChunk);
  const cudaError_t e = hyq::model::launch(hyq::model::attention_kernel, dim3(splits, (unsigned)heads, (unsigned)tokens),
                                           dim3(hyq::model::kAttnThreads), 0, (cudaStream_t)stream, a);
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "attention: %s", cudaGetErrorString(e));
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
                                           (size_t)n * sizeof(float), (cudaStream_t)stream, hidden, delta, w, (int)n,
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
