// Mixture-of-experts layer on the device (Moe::forward, hy-mt-rs
// src/model.rs:688-767): router logits, sigmoid top-k routing, expert
// assignment lists, the grouped expert products on the tensor cores
// (hyq_gemm.cu, expert mode) and the weighted combine.
//
// The reference loops over experts on the host with one small matmul each;
// here every step is one launch over all tokens and experts, and the expert
// token lists stay in device memory (the expert products read them), so a
// MoE layer needs no host round trip.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/hyq.h"
#include "hyq_common.cuh"
#include "hyq_kernels.h"

namespace hyq {
namespace moe {

// Router logits [tokens, experts] of an F32 router (the reference requires
// F32 for the sigmoid router, model.rs:223-227): each logit is the
// reference's batch-1 F32 row product, dot(row, x) in the x86 order
// (quant.rs:225-238, 2562-2596).  One CTA per token with the token row in
// shared memory; a half-warp per group of kRouterChains experts, lane l
// carrying AVX2 accumulator lane l of each expert's dot (four independent
// chains and unrolled loads keep the global reads in flight), then the
// reference's lane sums.
constexpr int kRouterMaxK = 16384;
constexpr int kRouterChains = 4;

__global__ void __launch_bounds__(256) router_kernel(const float* __restrict__ w, const float* __restrict__ x, int K,
                                                     int experts, float* __restrict__ logits) {
  extern __shared__ float xs[];
  const float* xr = x + (size_t)blockIdx.x * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = xr[i];
  __syncthreads();
  const int hw = threadIdx.x >> 4, nhw = blockDim.x >> 4, lane = threadIdx.x & 31, l = lane & 15;
  const unsigned mask = (lane & 16) ? 0xffff0000u : 0x0000ffffu;
  if ((K & 15) == 0) {
    for (int e0 = hw * kRouterChains; e0 < experts; e0 += nhw * kRouterChains) {
      float acc[kRouterChains];
      const float* wr[kRouterChains];
#pragma unroll
      for (int j = 0; j < kRouterChains; ++j) {
        acc[j] = 0.f;
        wr[j] = w + (size_t)min(e0 + j, experts - 1) * K + l;
      }
#pragma unroll 4
      for (int c = 0; c < K / 16; ++c) {
        const float xv = xs[16 * c + l];
#pragma unroll
        for (int j = 0; j < kRouterChains; ++j) acc[j] = fmaf(wr[j][16 * c], xv, acc[j]);
      }
#pragma unroll
      for (int j = 0; j < kRouterChains; ++j) {
        const float d = x86_lane_sum(acc[j], mask);
        if (l == 0 && e0 + j < experts) logits[(size_t)blockIdx.x * experts + e0 + j] = d;
      }
    }
  } else {
    for (int e = hw; e < experts; e += nhw) {
      const float d = dot_x86(w + (size_t)e * K, xs, K, mask);
      if (l == 0) logits[(size_t)blockIdx.x * experts + e] = d;
    }
  }
}

// The same logits with both operands staged: CTA (expert group, token
// group) loads kRouterChains router rows and up to kRouterTokens token rows
// into shared memory with 16-byte loads, all in flight at once, then each
// half-warp computes one token's kRouterChains dots from shared memory in
// the same lane order (bit-identical to router_kernel).  For K a multiple of
// 16 whose rows fit (router_tiled_tokens).
constexpr int kRouterTokens = 16;
constexpr int kRouterSmemBytes = 200 * 1024;

inline int router_tiled_tokens(int64_t K) {
  if (K % 16) return 0;
  const int64_t room = kRouterSmemBytes / (K * (int64_t)sizeof(float)) - kRouterChains;
  return (int)(room < 1 ? 0 : room > kRouterTokens ? kRouterTokens : room);
}

__global__ void __launch_bounds__(256) router_tiled_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                                           int K, int experts, int tokens, int tpc,
                                                           float* __restrict__ logits) {
  extern __shared__ __align__(16) float rs[];  // [kRouterChains][K] router rows, then [tpc][K] token rows
  float* xs = rs + (size_t)kRouterChains * K;
  const int e0 = blockIdx.x * kRouterChains, t0 = blockIdx.y * tpc;
  const int ne = min(kRouterChains, experts - e0), nt = min(tpc, tokens - t0);
  const int k4 = K / 4;
  // asynchronous 16-byte copies: every load of the CTA in flight at once
  for (int r = 0; r < ne + nt; ++r) {
    const float* src = r < ne ? w + (size_t)(e0 + r) * K : x + (size_t)(t0 + r - ne) * K;
    float* dst = r < ne ? rs + (size_t)r * K : xs + (size_t)(r - ne) * K;
    for (int c = threadIdx.x; c < k4; c += blockDim.x) cp_async16(dst + 4 * c, src + 4 * c);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const int hw = threadIdx.x >> 4, lane = threadIdx.x & 31, l = lane & 15;
  const unsigned mask = (lane & 16) ? 0xffff0000u : 0x0000ffffu;
  if (hw >= nt) return;  // whole half-warps leave together
  const float* xr = xs + (size_t)hw * K + l;
  float acc[kRouterChains];
#pragma unroll
  for (int j = 0; j < kRouterChains; ++j) acc[j] = 0.f;
#pragma unroll 4
  for (int c = 0; c < K / 16; ++c) {
    const float xv = xr[16 * c];
#pragma unroll
    for (int j = 0; j < kRouterChains; ++j) acc[j] = fmaf(rs[(size_t)min(j, ne - 1) * K + 16 * c + l], xv, acc[j]);
  }
#pragma unroll
  for (int j = 0; j < kRouterChains; ++j) {
    const float d = x86_lane_sum(acc[j], mask);
    if (l == 0 && j < ne) logits[(size_t)(t0 + hw) * experts + e0 + j] = d;
  }
}

// route (model.rs:728-767) for one token per warp: sigmoid with the
// reference's two branches, order by sigmoid + bias descending under
// f32::total_cmp with ties to the lower index, keep `used`, then weights
// sigmoid / max(sum of the kept sigmoids in that order, f16 MIN_POSITIVE)
// * scale (normalize) or sigmoid * scale.
constexpr int kRouteMaxExperts = 1024;
constexpr float kF16MinPositive = 6.103515625e-05f;

__device__ __forceinline__ int total_order_key(float v) {
  const int b = __float_as_int(v);
  return b ^ ((b >> 31) & 0x7fffffff);
}

__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits, int tokens, int experts,
                                                    const float* __restrict__ bias, int used, int normalize,
                                                    float scale, int32_t* __restrict__ topk_idx,
                                                    float* __restrict__ topk_w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= tokens) return;
  const float* lg = logits + (size_t)t * experts;
  constexpr int kPer = kRouteMaxExperts / 32;
  float sig[kPer];
  int key[kPer];  // total order of sigmoid + bias
  const int per = (experts + 31) / 32;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    sig[j] = 0.f;
    key[j] = INT_MIN;
    if (j < per) {
      const int e = lane + 32 * j;
      if (e < experts) {
        const float xv = lg[e];
        float s;
        if (xv >= 0.f) {
          s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-xv)));
        } else {
          const float ev = expf(xv);
          s = __fdiv_rn(ev, __fadd_rn(1.0f, ev));
        }
        sig[j] = s;
        key[j] = total_order_key(__fadd_rn(s, bias[e]));
      }
    }
  }
  float sum = 0.f;
  uint32_t taken = 0u;  // bit j: expert lane + 32 j is already chosen
  int my_e = 0;
  float my_s = 0.f;
  for (int k = 0; k < used; ++k) {
    // the largest key, then the lowest expert index, among those not taken:
    // one 64-bit value per candidate (order-preserving key bits, then the
    // complemented index), 0 for none, reduced with a maximum
    unsigned long long best = 0ull;
    float mine = 0.f;  // sigmoid of this lane's best candidate
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (j < per) {
        const int e = lane + 32 * j;
        if (e < experts && !((taken >> j) & 1u)) {
          const unsigned long long c =
              ((unsigned long long)((unsigned)key[j] ^ 0x80000000u) << 32) | (0xffffffffu - (unsigned)e);
          if (c > best) {
            best = c;
            mine = sig[j];
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long c = __shfl_xor_sync(0xffffffffu, best, o);
      best = c > best ? c : best;
    }
    const int be = (int)(0xffffffffu - (unsigned)(best & 0xffffffffull));
    // the winner's sigmoid, from the lane whose own best it is
    const float bs = __shfl_sync(0xffffffffu, mine, be & 31);
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    if (lane == k) {
      my_e = be;
      my_s = bs;
    }
    sum = __fadd_rn(sum, bs);  // in the order chosen, as the reference's sum
  }
  if (!normalize) sum = 1.0f;
  else sum = fmaxf(sum, kF16MinPositive);  // f32::max: a NaN sum gives the bound
  if (lane < used) {
    topk_idx[(size_t)t * used + lane] = my_e;
    topk_w[(size_t)t * used + lane] = __fmul_rn(__fdiv_rn(my_s, sum), scale);
  }
}

// Expert assignment lists (model.rs:695-701): for expert e, the tokens that
// chose it in token order, as rows expert_off[e] .. expert_off[e + 1] of the
// grouped activations: row_token (source token), row_weight (its routing
// weight), and token_rows[t * used + k] = the row of token t's k-th choice.
// One CTA, tokens in chunks of kGroupChunk: a per-expert bitmap of the
// chunk's tokens in shared memory gives each assignment its rank among the
// expert's earlier tokens by prefix popcounts (pass 0 counts, pass 1 places).
constexpr int kGroupChunk = 1024;
constexpr int kGroupMaxExperts = 128;
constexpr int kGroupWords = kGroupChunk / 32;

__global__ void __launch_bounds__(1024) group_kernel(const int32_t* __restrict__ topk_idx,
                                                     const float* __restrict__ topk_w, int tokens, int experts,
                                                     int used, int32_t* __restrict__ expert_off,
                                                     int32_t* __restrict__ row_token, float* __restrict__ row_weight,
                                                     int32_t* __restrict__ token_rows) {
  __shared__ uint32_t bits[kGroupMaxExperts * kGroupWords];  // expert-major bitmaps of one chunk
  __shared__ int32_t pre[kGroupMaxExperts * kGroupWords];    // tokens of the expert in earlier words
  __shared__ int32_t base[kGroupMaxExperts + 1];             // rows of the expert placed so far (+ offset)
  const int tid = threadIdx.x, nt = blockDim.x;
  const int nwords = experts * kGroupWords;
  for (int e = tid; e <= experts; e += nt) base[e] = 0;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      __syncthreads();
      if (tid == 0) {
        int run = 0;
        for (int e = 0; e < experts; ++e) {
          const int c = base[e];
          base[e] = run;
          expert_off[e] = run;
          run += c;
        }
        expert_off[experts] = run;
      }
    }
    for (int t0 = 0; t0 < tokens; t0 += kGroupChunk) {
      __syncthreads();
      for (int i = tid; i < nwords; i += nt) bits[i] = 0u;
      __syncthreads();
      const int t = t0 + tid;
      const bool live = tid < kGroupChunk && t < tokens;
      if (live)
        for (int k = 0; k < used; ++k)
          atomicOr(&bits[topk_idx[(size_t)t * used + k] * kGroupWords + (tid >> 5)], 1u << (tid & 31));
      __syncthreads();
      // prefix popcounts over each expert's words (one warp per expert row)
      for (int e = tid >> 5; e < experts; e += nt >> 5) {
        const int lane = tid & 31;
        const int c = __popc(bits[e * kGroupWords + lane]);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        pre[e * kGroupWords + lane] = incl - c;
      }
      __syncthreads();
      if (pass == 1 && live) {
        for (int k = 0; k < used; ++k) {
          const int e = topk_idx[(size_t)t * used + k];
          const int wd = tid >> 5;
          const int rank = pre[e * kGroupWords + wd] + __popc(bits[e * kGroupWords + wd] & ((1u << (tid & 31)) - 1u));
          const int row = base[e] + rank;
          row_token[row] = t;
          row_weight[row] = topk_w[(size_t)t * used + k];
          token_rows[(size_t)t * used + k] = row;
        }
      }
      __syncthreads();
      // this chunk's tokens per expert
      for (int e = tid; e < experts; e += nt)
        base[e] += pre[e * kGroupWords + kGroupWords - 1] + __popc(bits[e * kGroupWords + kGroupWords - 1]);
    }
  }
}

// output = shared; then for each expert in ascending order, output += weight
// * value (model.rs:691, 715-723; separate f32 roundings).  One CTA per
// token.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ shared, const float* __restrict__ y,
                                                      int N, const int32_t* __restrict__ topk_idx,
                                                      const int32_t* __restrict__ token_rows,
                                                      const float* __restrict__ row_weight, int used,
                                                      float* __restrict__ out) {
  __shared__ int32_t ex_s[32], row_s[32], in_e[32], in_r[32];
  __shared__ float w_s[32], in_w[32];
  const int t = blockIdx.x;
  // the token's choices and their weights, loaded by one lane each
  if (threadIdx.x < used) {
    const int r = token_rows[(size_t)t * used + threadIdx.x];
    in_e[threadIdx.x] = topk_idx[(size_t)t * used + threadIdx.x];
    in_r[threadIdx.x] = r;
    in_w[threadIdx.x] = row_weight[r];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // sorted by expert (insertion sort of `used` items)
    for (int k = 0; k < used; ++k) {
      const int e = in_e[k], r = in_r[k];
      const float wk = in_w[k];
      int i = k;
      while (i > 0 && ex_s[i - 1] > e) {
        ex_s[i] = ex_s[i - 1];
        row_s[i] = row_s[i - 1];
        w_s[i] = w_s[i - 1];
        --i;
      }
      ex_s[i] = e;
      row_s[i] = r;
      w_s[i] = wk;
    }
  }
  __syncthreads();
  // out = shared + sum over experts ascending of w * y, eight rows' loads in
  // flight at a time
  for (int c = threadIdx.x; c < N; c += blockDim.x) {
    float acc = shared[(size_t)t * N + c];
    for (int k0 = 0; k0 < used; k0 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = k0 + j < used ? y[(size_t)row_s[k0 + j] * N + c] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (k0 + j < used) acc = __fadd_rn(acc, __fmul_rn(w_s[k0 + j], v[j]));
    }
    out[(size_t)t * N + c] = acc;
  }
}

}  // namespace moe
}  // namespace hyq

extern "C" {

int hyq_moe_router(const hyq_weight* router, const float* x, int64_t tokens, float* logits, void* stream) {
  int dtype = 0, ndim = 0;
  int64_t dims[3] = {};
  const void* data = nullptr;
  if (!router || !x || !logits) return hyq::api_fail(HYQ_E_INVALID, "moe_router: null pointer");
  int rc = hyq_weight_info(router, &dtype, &ndim, dims, nullptr, &data);
  if (rc) return rc;
  if (dtype != HYQ_F32 || ndim != 2) return hyq::api_fail(HYQ_E_UNSUPPORTED, "moe_router: the router must be an F32 matrix");
  const int64_t K = dims[0], E = dims[1];
  if (tokens <= 0 || K <= 0 || K > hyq::moe::kRouterMaxK || E <= 0 || tokens > INT32_MAX)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_router: shape (input width at most %d)", hyq::moe::kRouterMaxK);
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaFuncSetAttribute(hyq::moe::router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         hyq::moe::kRouterMaxK * (int)sizeof(float));
    cudaFuncSetAttribute(hyq::moe::router_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         hyq::moe::kRouterSmemBytes);
    configured = dev;
  }
  const int tpc = hyq::moe::router_tiled_tokens(K);
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(data) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
  if (tpc > 0 && aligned16) {
    const dim3 grid((unsigned)((E + hyq::moe::kRouterChains - 1) / hyq::moe::kRouterChains),
                    (unsigned)((tokens + tpc - 1) / tpc));
    const size_t smem = (size_t)(hyq::moe::kRouterChains + tpc) * K * sizeof(float);
    hyq::moe::router_tiled_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(
        static_cast<const float*>(data), x, (int)K, (int)E, (int)tokens, tpc, logits);
  } else {
    hyq::moe::router_kernel<<<(unsigned)tokens, 256, (size_t)K * sizeof(float), (cudaStream_t)stream>>>(
        static_cast<const float*>(data), x, (int)K, (int)E, logits);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_router: %s", cudaGetErrorString(e));
}

int hyq_moe_route(const float* logits, int64_t tokens, int experts, const float* bias, int used, int normalize,
                  float scale, int32_t* topk_idx, float* topk_w, void* stream) {
  if (!logits || !bias || !topk_idx || !topk_w) return hyq::api_fail(HYQ_E_INVALID, "moe_route: null pointer");
  if (tokens <= 0 || tokens > INT32_MAX || experts <= 0 || experts > hyq::moe::kRouteMaxExperts || used <= 0 ||
      used > experts || used > 32)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_route: shape (at most %d experts, 32 used)", hyq::moe::kRouteMaxExperts);
  const unsigned blocks = (unsigned)((tokens + 7) / 8);
  hyq::moe::route_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(logits, (int)tokens, experts, bias, used,
                                                                   normalize, scale, topk_idx, topk_w);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_route: %s", cudaGetErrorString(e));
}

int hyq_moe_group(const int32_t* topk_idx, const float* topk_w, int64_t tokens, int experts, int used,
                  int32_t* expert_off, int32_t* row_token, float* row_weight, int32_t* token_rows, void* stream) {
  if (!topk_idx || !topk_w || !expert_off || !row_token || !row_weight || !token_rows)
    return hyq::api_fail(HYQ_E_INVALID, "moe_group: null pointer");
  if (tokens <= 0 || tokens * used > INT32_MAX || experts <= 0 || experts > hyq::moe::kGroupMaxExperts || used <= 0 ||
      used > 32)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_group: shape (at most %d experts)", hyq::moe::kGroupMaxExperts);
  hyq::moe::group_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(
      topk_idx, topk_w, (int)tokens, experts, used, expert_off, row_token, row_weight, token_rows);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_group: %s", cudaGetErrorString(e));
}

int hyq_moe_combine(const float* shared, const float* expert_out, int64_t tokens, int64_t n, const int32_t* topk_idx,
                    const int32_t* token_rows, const float* row_weight, int used, float* out, void* stream) {
  if (!shared || !expert_out || !topk_idx || !token_rows || !row_weight || !out)
    return hyq::api_fail(HYQ_E_INVALID, "moe_combine: null pointer");
  if (tokens <= 0 || tokens > INT32_MAX || n <= 0 || n > INT32_MAX || used <= 0 || used > 32)
    return hyq::api_fail(HYQ_E_SHAPE, "moe_combine: shape");
  hyq::moe::combine_kernel<<<(unsigned)tokens, 256, 0, (cudaStream_t)stream>>>(shared, expert_out, (int)n, topk_idx,
                                                                              token_rows, row_weight, used, out);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HYQ_OK : hyq::api_fail(HYQ_E_CUDA, "moe_combine: %s", cudaGetErrorString(e));
}

}  // extern "C"
