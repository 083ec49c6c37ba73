/*
 * hyq.h -- C ABI of the B200 block-quantized GEMV/GEMM library (libhyq.so).
 *
 * Drop-in boundary for the quantized linear-algebra path of hy-mt-rs
 * (src/quant.rs).  Every entry point names the reference routine it replaces.
 * Conventions:
 *   - plain pointers and sizes; device pointers unless a name says host;
 *   - weights are packed GGUF blocks, uploaded unchanged; dims follow GGUF
 *     order: dims[0] = K (contiguous input width), dims[1] = N (output rows),
 *     dims[2] = number of experts (optional);
 *   - outputs of batched products are [batch, N] row-major (quant.rs:337-343);
 *   - every call is ordered on `stream` (a cudaStream_t, NULL = legacy default
 *     stream) and returns HYQ_OK or a negative HYQ_E_* code; nothing aborts;
 *     hyq_last_error() describes the last failure of the calling thread;
 *   - calls on different streams may run concurrently; a weight handle may be
 *     shared by any number of threads (it is immutable after creation).
 */
#ifndef HYQ_H_
#define HYQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Packed tensor types, in the order of DType (quant.rs:19-27). */
typedef enum hyq_dtype {
  HYQ_F32 = 0,
  HYQ_F16 = 1,
  HYQ_Q4_K = 2,
  HYQ_Q6_K = 3,
  HYQ_Q8_0 = 4,
  HYQ_Q2_0C = 5,  /* Tencent Q2_0C: 512 weights per 130-byte block */
  HYQ_STQ1_0 = 6  /* Tencent STQ1 stride-16 sparse ternary: 256 weights per 42 bytes */
} hyq_dtype;

/* GGUF type-id profiles (gguf.rs:17-27, Profile).  Auto (hyq_gguf_open only)
 * resolves to Standard, or for files with legacy ids 40/42 to the Tencent
 * profile whose known export the file's SHA-256 matches. */
typedef enum hyq_profile {
  HYQ_PROFILE_AUTO = 0,
  HYQ_PROFILE_STANDARD = 1,
  HYQ_PROFILE_TENCENT_Q2_0C = 2,
  HYQ_PROFILE_TENCENT_STQ1 = 3
} hyq_profile;

#define HYQ_OK 0
#define HYQ_E_INVALID (-1)     /* null pointer, unknown dtype/profile, bad argument */
#define HYQ_E_SHAPE (-2)       /* shape or byte count mismatch (the reference's ensure! checks) */
#define HYQ_E_ALIGN (-3)       /* a device pointer is not aligned to its element size */
#define HYQ_E_CUDA (-4)        /* CUDA runtime error; see hyq_last_error() */
#define HYQ_E_DEVICE (-5)      /* a kernel's bounded wait expired (see hyq_device_status) */
#define HYQ_E_UNSUPPORTED (-6) /* combination the library does not implement */
#define HYQ_E_NOMEM (-7)       /* device allocation failed */

/* Device status bits returned by hyq_device_status. */
#define HYQ_DEV_TIMEOUT_FULL 1u  /* a consumer gave up waiting for a tile copy */
#define HYQ_DEV_TIMEOUT_EMPTY 2u /* a producer gave up waiting for a free stage */
#define HYQ_DEV_TIMEOUT_DRAIN 4u /* exit path gave up waiting for copies in flight */
#define HYQ_DEV_BAD_ARGS 8u      /* a kernel saw arguments the host should have rejected */
#define HYQ_DEV_TIMEOUT_PEER 16u /* a peer all-reduce or exchange gave up waiting for another rank */
#define HYQ_DEV_TIMEOUT_GRID 32u /* hyq_dense_step_enqueue's kernel gave up at a grid-wide barrier */

typedef struct hyq_weight hyq_weight;

/* Message for the last failing call on this thread ("" if none). */
const char* hyq_last_error(void);

/* DType::block_len / block_bytes (quant.rs:43-62).  0 for an unknown dtype. */
int hyq_block_len(int dtype);
int hyq_block_bytes(int dtype);

/* DType::from_id (quant.rs:30-41): GGUF tensor type id -> dtype under a
 * profile.  IDs 40/42 are only valid under their Tencent profile. */
int hyq_dtype_from_id(uint32_t type_id, int profile, int* dtype_out);

/* Weight (quant.rs:65-97): copy `byte_len` packed bytes from host memory
 * (e.g. a memory-mapped GGUF tensor) to a new device buffer, unchanged.
 * byte_len must equal dims[1] * (dims[2] or 1) * dims[0] / block_len * block_bytes. */
int hyq_upload(const void* packed_host, size_t byte_len, int dtype, int ndim, const int64_t* dims,
               hyq_weight** out);

/* As hyq_upload, but borrow packed bytes that already live in device memory
 * (the caller keeps them alive while the handle is used). */
int hyq_weight_wrap(const void* packed_device, size_t byte_len, int dtype, int ndim, const int64_t* dims,
                    hyq_weight** out);

/* Weight::expert (quant.rs:144-154): view of expert `index` of a rank-3
 * weight [K, N, E] as a [K, N] matrix (byte offset index * byte_len / E). */
int hyq_weight_expert(const hyq_weight* w, int64_t index, hyq_weight** out);

/* Tensor-parallel shard of a [K, N] matrix (no counterpart in the CPU
 * reference; the split a dense tensor-parallel 7B layer uses: column-parallel
 * QKV / gate / up / lm_head, row-parallel O / down).
 *   axis 0 (column-parallel: QKV, gate/up, lm_head): output rows
 *     [part*N/parts, (part+1)*N/parts), a view of the parent's bytes (the
 *     parent must outlive it); N % parts == 0.
 *   axis 1 (row-parallel: O, down): input columns [part*K/parts, ...) of every
 *     row, on whole blocks, gathered into a new device buffer by one strided
 *     copy ordered on `stream`; the partial products of all parts sum to the
 *     full product.  K/parts must be a multiple of the block length
 *     (HYQ_E_SHAPE otherwise, e.g. Q2_0C K=6144 at parts=8). */
int hyq_weight_shard(const hyq_weight* w, int axis, int64_t part, int64_t parts, void* stream, hyq_weight** out);

/* Shape/type/buffer of a handle (any output pointer may be NULL; dims needs 3). */
int hyq_weight_info(const hyq_weight* w, int* dtype, int* ndim, int64_t* dims, size_t* byte_len,
                    const void** device_ptr);

/* Release a handle (frees the device buffer only if hyq_upload made it). */
void hyq_free(hyq_weight* w);

/* decode (quant.rs:1066-1079): `byte_len` packed bytes -> `out_len` f32, bit
 * for bit as decode_unchecked (quant.rs:2405-2486). */
int hyq_decode(int dtype, const void* bytes, size_t byte_len, float* out, size_t out_len, void* stream);

/* Weight::row_into (quant.rs:123-142): decode one row (embedding lookup). */
int hyq_weight_row_into(const hyq_weight* w, int64_t row, float* out, int64_t out_len, void* stream);

/* dot (quant.rs:2500): *out = sum a[i]*b[i] (f32; summation order differs). */
int hyq_dot(const float* a, const float* b, size_t n, float* out, void* stream);

/* Weight::matmul (quant.rs:159-344): out[batch, N] = input[batch, K] . W^T
 * with f32 activations.  From batch 16 the tensor-core path takes a
 * stream-ordered workspace (fp16 activations, split-K partials) from a memory
 * pool the library creates per device; freed workspace stays cached in that
 * pool until the process exits.  The device's default memory pool is not
 * touched.  Under stream capture the workspace is a graph allocation. */
int hyq_matmul(const hyq_weight* w, const float* input, int64_t batch, float* out, void* stream);

/* Weight::gemv_qkv (quant.rs:658-721): three batch-1 projections of one
 * input in one launch. */
int hyq_gemv_qkv(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input,
                 float* q_out, float* k_out, float* v_out, void* stream);

/* Weight::matmul_gate_up_silu (quant.rs:724-841): out = silu(gate.x) * up.x. */
int hyq_matmul_gate_up_silu(const hyq_weight* gate, const hyq_weight* up, const float* input, float* out,
                            void* stream);

/* Batch-1 products fused with the decoder's residual-stream steps (the
 * per-token chain of model.rs:1007-1041: rms_norm_into, a projection, add).
 * Each is one launch of the batch-1 product whose activation prologue or
 * output step does the extra work, with the same arithmetic as the separate
 * calls (results bit-identical to hyq_rms_norm / hyq_add + the plain product):
 *   _norm forms: the product of RMSNorm(hidden) * norm_w (rms_norm_into,
 *     model.rs:785-830; hidden[K] is not modified);
 *   hyq_gemv_residual: hidden[N] += W . input (add, model.rs:1043-1071).
 * `act` picks the product's activations, as the reference's two decode
 * branches do (model.rs:395-529):
 *   HYQ_ACT_F32: f32 activations (x86: gemv_qkv, matmul, matmul_gate_up_silu);
 *   HYQ_ACT_Q8: the (normalised) input quantized to Q8 inside the kernel
 *     exactly as Q8::quantize_into, then the SDOT-order product (aarch64:
 *     gemv_qkv_fast, gemv_q8_fast, matmul_gate_up_silu_fast; the same
 *     results as hyq_q8_quantize followed by the _q8 entry points).
 * They need the streaming engine with staged f32 activations: a packed
 * format (not F32/F16), K a multiple of 256 and at most 6144, 16-byte aligned
 * weights and input; HYQ_E_UNSUPPORTED otherwise.  hyq_gemv_fusable reports
 * whether a weight qualifies (*out = 1) for 16-byte aligned activations. */
#define HYQ_ACT_F32 0
#define HYQ_ACT_Q8 1
int hyq_gemv_qkv_norm(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* hidden,
                      const float* norm_w, float eps, int act, float* q_out, float* k_out, float* v_out,
                      void* stream);
int hyq_gemv_gate_up_silu_norm(const hyq_weight* gate, const hyq_weight* up, const float* hidden,
                               const float* norm_w, float eps, int act, float* out, void* stream);
int hyq_gemv_norm(const hyq_weight* w, const float* hidden, const float* norm_w, float eps, int act, float* out,
                  void* stream);
int hyq_gemv_residual(const hyq_weight* w, const float* input, int act, float* hidden, void* stream);
int hyq_gemv_fusable(const hyq_weight* w, int* out);

/* Batched Weight::gemv_qkv: q/k/v_out[batch, N_q|N_k|N_v] = input[batch, K] .
 * {Q,K,V}^T.  The reference runs gemv_qkv per token (quant.rs:658-721) and
 * three Weight::matmul calls for prefill (model.rs:559-565); here one
 * tensor-core launch covers all three matrices (the activations are
 * converted once) from 16 tokens up, batch-1 products below. */
int hyq_matmul_qkv(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input, int64_t batch,
                   float* q_out, float* k_out, float* v_out, void* stream);

/* Batched matmul_gate_up_silu (quant.rs:724-841 per token; for batches
 * DenseFfn::forward runs gate and up through Weight::matmul and combines
 * them elementwise, model.rs:678-682):
 * out[batch, N] = silu(input . gate^T) * (input . up^T), silu(g) = g/(1+e^-g).
 * From 16 tokens up one tensor-core launch computes matching gate and up rows
 * in the same tile and writes only the combined output. */
int hyq_matmul_gate_up_silu_batch(const hyq_weight* gate, const hyq_weight* up, const float* input, int64_t batch,
                                  float* out, void* stream);

/* Batched products fused with the residual-stream steps in front of them
 * (the batched forward, model.rs:569-616): hidden [batch, K] += delta (when
 * delta is not NULL; add, model.rs:1043-1071, written back to hidden), then
 * the product of RMSNorm(hidden rows) * norm_w (rms_norm_into,
 * model.rs:785-830).  From 16 rows the tensor-core path does the add and the
 * norm in its activation conversion (one CTA per row, K at most 16384);
 * below that, and for shapes it does not take, the separate add + norm
 * kernel writes a pool buffer that the plain forms read.  Either way the
 * results and hidden are bit-identical to hyq_add_rms_norm / hyq_rms_norm
 * followed by hyq_matmul_qkv, hyq_matmul_gate_up_silu_batch or hyq_matmul. */
int hyq_matmul_qkv_norm(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, float* hidden,
                        const float* delta, const float* norm_w, float eps, int64_t batch, float* q_out,
                        float* k_out, float* v_out, void* stream);
int hyq_matmul_gate_up_silu_norm(const hyq_weight* gate, const hyq_weight* up, float* hidden, const float* delta,
                                 const float* norm_w, float eps, int64_t batch, float* out, void* stream);
int hyq_matmul_norm(const hyq_weight* w, float* hidden, const float* delta, const float* norm_w, float eps,
                    int64_t batch, float* out, void* stream);

/* Q8::quantize_into (quant.rs:904-922): int8 activations, one f32 scale per
 * 256 values, and the Q2_0C de-interleaved copy (values_q2c may be NULL).
 * Bit-exact with the reference.  scales has ceil(len/256) entries. */
int hyq_q8_quantize(const float* input, int64_t len, int8_t* values, float* scales, int8_t* values_q2c,
                    void* stream);

/* gemv_q8_fast (quant.rs:353-357): batch-1 product on pre-quantized
 * activations (values/scales from hyq_q8_quantize; values_q2c may be NULL). */
int hyq_gemv_q8(const hyq_weight* w, const int8_t* values, const float* scales, const int8_t* values_q2c,
                float* out, void* stream);

/* gemv_qkv_fast (quant.rs:441-538). */
int hyq_gemv_qkv_q8(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const int8_t* values,
                    const float* scales, const int8_t* values_q2c, float* q_out, float* k_out, float* v_out,
                    void* stream);

/* matmul_gate_up_silu_fast (quant.rs:540-651). */
int hyq_matmul_gate_up_silu_q8(const hyq_weight* gate, const hyq_weight* up, const int8_t* values,
                               const float* scales, const int8_t* values_q2c, float* out, void* stream);

/* Batch-1 product through int8 activations, quantized inside the kernel
 * exactly as Q8::quantize would (the aarch64 path of Weight::matmul:
 * quant.rs:169-178 -> gemv_q8 :346-351).  Same result as hyq_q8_quantize
 * followed by hyq_gemv_q8, in one launch and without the Q8 buffers.
 * K must be a multiple of 256 unless the buffers are 16-byte aligned. */
int hyq_gemv_int8(const hyq_weight* w, const float* input, float* out, void* stream);

/* Weight::gemv_qkv through int8 activations (quant.rs:673-714). */
int hyq_gemv_qkv_int8(const hyq_weight* q, const hyq_weight* k, const hyq_weight* v, const float* input,
                      float* q_out, float* k_out, float* v_out, void* stream);

/* Weight::matmul_gate_up_silu through int8 activations (quant.rs:735-766). */
int hyq_matmul_gate_up_silu_int8(const hyq_weight* gate, const hyq_weight* up, const float* input, float* out,
                                 void* stream);

/* Overlapped launches (no counterpart in the reference, which runs on the
 * host).  With `enable` != 0, every later batch-1 product (hyq_matmul with
 * batch 1..15, hyq_gemv_*, hyq_matmul_gate_up_silu*) launches as a
 * programmatic dependent of the preceding grid in its stream: it is scheduled
 * while that grid is still running and starts streaming its packed weights,
 * and waits for that grid to complete before it reads activations or writes
 * outputs.  This hides launch latency and the first weight fetch in chains of
 * products (a decode step).  Contract: no kernel still in flight on the stream
 * when a product is issued may write that product's weights (upload or wrap
 * the weights, then order them before use, e.g. by a stream synchronization).
 * Process-wide; default 0 (plain stream order). */
int hyq_set_launch_overlap(int enable);

/* Arithmetic of the batched tensor-core products (hyq_matmul and
 * hyq_matmul_noalloc from batch 16, hyq_matmul_qkv, the batched gate/up, the
 * expert products).  No counterpart in the reference, whose batched path is
 * an f32 GEMM on the host (quant.rs:272-311, Candle).
 *   HYQ_GEMM_FP16 (default): activations and decoded weights rounded to fp16,
 *     f32 accumulation; about 1e-3 relative L2 against an f64 product.
 *   HYQ_GEMM_F32: split operands -- each activation and each weight (decoded
 *     exactly in f32) as hi + lo / 2^11, both fp16; three MMAs per K chunk
 *     (hi.hi, hi.lo, lo.hi) into f32 accumulators -- which keeps 22
 *     significant bits of every operand: products agree with an f32 GEMM to
 *     about 1e-6 relative, at about three times the tensor-core instructions
 *     and twice the activation bytes (token tiles of at most 128, no 2-SM
 *     form).  The gate/up SiLU then uses expf and IEEE division, as the
 *     batch-1 products do.  Activations must stay below 65504 in magnitude.
 * Process-wide, read when a call is issued: a captured CUDA graph keeps the
 * precision its calls were captured with. */
#define HYQ_GEMM_FP16 0
#define HYQ_GEMM_F32 1
int hyq_set_gemm_precision(int precision);

/* Bytes of the fixed device scratch behind hyq_matmul_noalloc (64 MiB). */
#define HYQ_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* hyq_matmul with no device allocation: same arguments, checks and result
 * (the same kernels run), but the tensor-core path keeps its fp16 activation
 * copy and split-K partial sums in a device array of
 * HYQ_NOALLOC_SCRATCH_BYTES that belongs to the library's module image (every
 * GPU that loads the library holds it until the process exits), instead of a
 * stream-ordered allocation.  No counterpart in the reference, whose matmul
 * works in host memory.  It serves callers that may not allocate device
 * memory per call: a server that hands all free HBM to its own cache at
 * start-up (where a per-call allocation could fail mid request), and hosts
 * that account for every byte of device memory themselves (hyq_matmul's
 * workspace pool keeps freed workspace cached until the process exits, out of
 * that host's sight).
 * Limits:
 *   - a batch whose scratch would exceed HYQ_NOALLOC_SCRATCH_BYTES
 *     (K * batch * 2 bytes plus split-K partials) fails with HYQ_E_SHAPE;
 *   - the first call on each device looks up the array's device address with
 *     that device current; make that first call before any stream capture;
 *   - every call on a device shares the one array, so calls that overlap on
 *     the GPU (different streams, no ordering between them) race: keep them
 *     on one stream or order them with events. */
int hyq_matmul_noalloc(const hyq_weight* w, const float* input, int64_t batch, float* out, void* stream);

/* --- Single-token decoder step around the products ----------------------
 * The rest of Model::forward_into for one token (Dense architecture,
 * model.rs:374-547), so that a whole step runs on the device and replays as
 * one CUDA graph: kernels that depend on the position read it from `pos`
 * (device int32), the embedding reads the token from `token` (device int32),
 * and hyq_argmax writes the next token there and advances `pos`.  Norms and
 * attention scores sum in the reference's x86 dot order; the softmax uses the
 * device exponential. */

/* Rotary tables on the host (model.rs:266-272, 378-391): cos/sin[p * hd/2 + j]
 * = (p * base^(-2j/hd)).sin_cos() in f32, for p < positions. */
int hyq_rope_table(int64_t positions, int head_dim, float rope_base, float* cos_out, float* sin_out);

/* rms_norm_into (model.rs:785-830) of `rows` rows of n floats (rows > 1: the
 * per-head q/k norm, model.rs:832-872): out = x * (1/sqrt(mean(x^2)+eps)) * w.
 * n is at most 16384 (the row is staged in shared memory). */
int hyq_rms_norm(const float* x, const float* w, int64_t n, int64_t rows, float eps, float* out, void* stream);

/* Weight::row_into (quant.rs:123-142) of rows token[0 .. count) (device
 * int32) into out [count, K] (the embedding rows of a prompt chunk,
 * model.rs:373-376). */
int hyq_embed(const hyq_weight* w, const int32_t* token, int64_t count, float* out, void* stream);

/* RoPE of q [tokens, heads, hd] and k [tokens, kv_heads, hd], token i at
 * position *pos + i (rope, model.rs:919-947; tables from
 * hyq_rope_table, on the device), the per-head RMSNorm with q_norm/k_norm
 * after it (Dense, model.rs:435-446) or before it (norm_first: HyV3,
 * model.rs:425-434; NULL norms skip it), then KvCache::append of k and v
 * (model.rs:650-667) into row *pos of k_cache/v_cache [positions, kv_heads*hd]. */
int hyq_rope_qk(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                const float* sin_tab, int64_t positions, const int32_t* pos, int64_t tokens, const float* q_norm,
                const float* k_norm, float eps, int norm_first, float* k_cache, float* v_cache, void* stream);

/* attention_into (model.rs:949-1021) for q [tokens, heads, hd]: token i sits
 * at position *pos + i and attends to cache rows 0 ..= *pos + i (causal;
 * grouped-query: head h reads kv head h / (heads / kv_heads)); out [tokens,
 * heads, hd].  positions is the cache capacity (at most 16384), head_dim at
 * most 256.  The cached positions are split into chunks of 64 whose partial
 * softmax sums are combined on the device; `workspace` holds those partials
 * and one counter per (token, head): hyq_attention_workspace_bytes bytes for
 * the largest token count used, zero before the first call (every call leaves
 * it zero again; calls with fewer tokens share it).  Calls that share a
 * workspace must not overlap in time. */
int hyq_attention_workspace_bytes(int heads, int head_dim, int64_t positions, int64_t tokens, size_t* bytes);
int hyq_attention(const float* q, const float* k_cache, const float* v_cache, int heads, int kv_heads,
                  int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out, void* workspace,
                  void* stream);

/* The same for `seqs` independent sequences decoding one token each
 * (concurrent requests: separate Sessions over one shared Model,
 * README.md:139-141; per sequence, rope_with_cache model.rs:874-913 and
 * attention_into model.rs:949-1021): token t is sequence t at position pos[t] (device
 * int32 [seqs]) with its caches at k_cache/v_cache + t * seq_stride floats
 * (seq_stride >= positions * kv_heads * head_dim); seqs <= positions.  The
 * attention workspace is hyq_attention_workspace_bytes(..., positions, seqs). */
int hyq_rope_qk_seqs(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                     const float* sin_tab, int64_t positions, const int32_t* pos, int64_t seqs, const float* q_norm,
                     const float* k_norm, float eps, int norm_first, float* k_cache, float* v_cache,
                     int64_t seq_stride, void* stream);
int hyq_attention_seqs(const float* q, const float* k_cache, const float* v_cache, int heads, int kv_heads,
                       int head_dim, int64_t positions, const int32_t* pos, int64_t seqs, int64_t seq_stride,
                       float* out, void* workspace, void* stream);

/* One decode step's RoPE + q/k RMSNorm + KV append (hyq_rope_qk;
 * model.rs:429-446, 874-913) and attention (hyq_attention; model.rs:949-1021)
 * in one launch, bit-identical to the two calls:
 * q, k and v are the step's raw projections (q [heads * head_dim], k and v
 * [kv_heads * head_dim]; left unchanged), the position is read from `pos`,
 * the rotated key and the value are appended to the caches at it, and the
 * attention output goes to `out`.  One token of one sequence (a prompt's
 * tokens use hyq_rope_qk and hyq_attention).  Workspace as hyq_attention
 * with tokens = 1. */
int hyq_rope_attention(const float* q, const float* k, const float* v, int heads, int kv_heads, int head_dim,
                       const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                       const float* q_norm, const float* k_norm, float eps, int norm_first, float* k_cache,
                       float* v_cache, float* out, void* workspace, void* stream);

/* The same for `seqs` independent sequences, one token each (as
 * hyq_rope_qk_seqs + hyq_attention_seqs: q [seqs, heads * head_dim], k and v
 * [seqs, kv_heads * head_dim], sequence t at position pos[t] with its caches
 * t * seq_stride floats further). */
int hyq_rope_attention_seqs(const float* q, const float* k, const float* v, int heads, int kv_heads, int head_dim,
                            const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                            int64_t seqs, const float* q_norm, const float* k_norm, float eps, int norm_first,
                            float* k_cache, float* v_cache, int64_t seq_stride, float* out, void* workspace,
                            void* stream);
/* The same calls over an f16 KV cache (BASELINE config 4 asks for one; the
 * reference's KvCache is f32, model.rs:116-120): k_cache / v_cache hold IEEE
 * binary16 values (uint16_t bit patterns) in the same [positions, kv_heads *
 * head_dim] layout, seq_stride counts elements.  The append rounds each
 * rotated key and value to the nearest binary16; attention widens the
 * cached rows to f32 as it loads them and computes as the f32 calls do, so
 * the only difference is that rounding.  Half the cache bytes per step. */
int hyq_rope_qk_kv16(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim, const float* cos_tab,
                     const float* sin_tab, int64_t positions, const int32_t* pos, int64_t tokens, const float* q_norm,
                     const float* k_norm, float eps, int norm_first, uint16_t* k_cache, uint16_t* v_cache,
                     void* stream);
int hyq_rope_qk_seqs_kv16(float* q, float* k, const float* v, int heads, int kv_heads, int head_dim,
                          const float* cos_tab, const float* sin_tab, int64_t positions, const int32_t* pos,
                          int64_t seqs, const float* q_norm, const float* k_norm, float eps, int norm_first,
                          uint16_t* k_cache, uint16_t* v_cache, int64_t seq_stride, void* stream);
int hyq_attention_kv16(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads, int kv_heads,
                       int head_dim, int64_t positions, const int32_t* pos, int64_t tokens, float* out,
                       void* workspace, void* stream);
int hyq_attention_seqs_kv16(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, int heads,
                            int kv_heads, int head_dim, int64_t positions, const int32_t* pos, int64_t seqs,
                            int64_t seq_stride, float* out, void* workspace, void* stream);

/* Greedy token of each of `rows` rows of n logits (generation.rs:281-290):
 * token[r]; pos[r] += 1 when pos is not NULL. */
int hyq_argmax_rows(const float* x, int64_t n, int64_t rows, int32_t* token, int32_t* pos, void* stream);

/* add (model.rs:1043-1071): dst += src. */
int hyq_add(float* dst, const float* src, int64_t n, void* stream);

/* The residual add followed by the next rms_norm_into (model.rs:1043-1071,
 * 785-830) in one launch: hidden += delta; out = hidden * scale * w, with
 * scale from the updated hidden. */
int hyq_add_rms_norm(float* hidden, const float* delta, const float* w, int64_t n, int64_t rows, float eps,
                     float* out, void* stream);

/* Greedy token (generation.rs:281-290: first index of the largest value)
 * into *token; when pos is not NULL, *pos += pos_step.  `workspace`: 16 bytes,
 * 8-byte aligned, zero before the first call (every call leaves it zero);
 * calls that share one must not overlap in time. */
#define HYQ_ARGMAX_WORKSPACE_BYTES 16
int hyq_argmax(const float* x, int64_t n, int32_t* token, int32_t* pos, int pos_step, void* workspace,
               void* stream);

/* --- GGUF v3 model files (gguf.rs:50-210) --------------------------------
 * hyq_gguf_open maps the file read-only and checks it as the reference does
 * (header bounds, metadata types, alignment, tensor table, Tencent legacy
 * profiles, truncated or overlapping tensors); errors are HYQ_E_* codes with
 * the reason in hyq_last_error.  Tensor dims are in GGUF order (contiguous
 * input first); offsets are absolute file offsets.  hyq_gguf_upload copies a
 * tensor's packed bytes unchanged to a new device weight (hyq_upload).
 * Metadata getters follow the reference's typed access: integers of any
 * GGUF integer type that fit u64, floats of any numeric type, booleans,
 * strings; array lengths.  The file must not change while it is open. */
typedef struct hyq_gguf hyq_gguf;
int hyq_gguf_open(const char* path, int profile, hyq_gguf** out);
void hyq_gguf_close(hyq_gguf* g);
int hyq_gguf_profile(const hyq_gguf* g);
int64_t hyq_gguf_tensor_count(const hyq_gguf* g);
int hyq_gguf_tensor_name(const hyq_gguf* g, int64_t index, const char** name);
int hyq_gguf_tensor_info(const hyq_gguf* g, const char* name, int* dtype, uint32_t* type_id, int* ndim,
                         int64_t* dims /* [4] */, uint64_t* offset, uint64_t* byte_len);
int hyq_gguf_tensor_data(const hyq_gguf* g, const char* name, const void** data, size_t* bytes);
int hyq_gguf_upload(const hyq_gguf* g, const char* name, hyq_weight** out);
int64_t hyq_gguf_meta_count(const hyq_gguf* g);
int hyq_gguf_meta_key(const hyq_gguf* g, int64_t index, const char** key, int* type);
int hyq_gguf_meta_u64(const hyq_gguf* g, const char* key, uint64_t* out);
int hyq_gguf_meta_f64(const hyq_gguf* g, const char* key, double* out);
int hyq_gguf_meta_bool(const hyq_gguf* g, const char* key, int* out);
int hyq_gguf_meta_str(const hyq_gguf* g, const char* key, const char** s, size_t* len);
int hyq_gguf_meta_array_len(const hyq_gguf* g, const char* key, int64_t* n);

/* --- The whole Dense decoder token step as one persistent kernel --------
 * model.rs:374-547 for one token: embedding row, per layer RMSNorm -> QKV ->
 * RoPE + q/k norm + KV append -> attention -> O + residual -> RMSNorm ->
 * gate/up-SiLU -> down + residual, then the output norm, the tied lm_head and
 * the greedy token, in one cooperative launch (one CTA per SM; a grid-wide
 * barrier between dependent phases instead of ~8 launches per layer).  Same
 * arithmetic as the per-call entry points (x86-order norms, exact f32
 * products).  Supported: Q2_0C layer products and a Q6_K tied embedding (the
 * 1.8B architecture).  The step reads the token and position from device
 * ints and writes the next token and position + 1 there, so a CUDA graph
 * can replay it.  No reference counterpart as one call (the reference runs
 * these steps on the host). */
typedef struct hyq_dense_layer {
  const hyq_weight *q, *k, *v, *o, *gate, *up, *down;
  const float *input_norm, *ffn_norm, *q_norm, *k_norm;  /* device f32 */
  float *k_cache, *v_cache;                              /* [positions, kv_heads * head_dim] */
} hyq_dense_layer;

typedef struct hyq_dense_step_desc {
  int layers, hidden, heads, kv_heads, head_dim, ffn;
  int64_t positions;                 /* KV-cache capacity, at most 16384 */
  float eps;
  const hyq_dense_layer* layer;      /* host array of `layers` */
  const hyq_weight* embed;           /* Q6_K [hidden, vocab], tied lm_head */
  const float* output_norm;
  const float *cos_tab, *sin_tab;    /* hyq_rope_table, on the device */
  /* device activations: hidden_state [hidden], q [heads*hd], k, v [kv*hd],
   * attended [heads*hd], gate [ffn], logits [vocab]; token, pos: one int32 */
  float *hidden_state, *q, *k, *v, *attended, *gate, *logits;
  int32_t *token, *pos;
} hyq_dense_step_desc;

typedef struct hyq_dense_step hyq_dense_step;
int hyq_dense_step_create(const hyq_dense_step_desc* desc, hyq_dense_step** out);
/* One token step on `stream` (a zeroing copy of the step's 16-byte sync
 * words, then the kernel).  Steps of one handle must not overlap in time.
 * The kernel checks the device position first: when *pos is outside
 * [0, positions) (e.g. a graph replayed past the cache's capacity) the step
 * does nothing -- no cache row, rotary row or token is touched and *pos is
 * not advanced -- and raises HYQ_DEV_BAD_ARGS (see hyq_device_status). */
int hyq_dense_step_enqueue(hyq_dense_step* step, void* stream);
void hyq_dense_step_free(hyq_dense_step* step);

/* --- Mixture-of-experts layer (Moe::forward, model.rs:688-767) ----------
 * The reference routes on the host and loops over experts with one small
 * matmul each; these steps keep the routing, the expert token lists and the
 * expert products on the device (no host round trip), in the reference's
 * order of results:
 *   hyq_moe_router      logits [tokens, experts] = x . router (F32 router,
 *                       model.rs:223-227; each logit the batch-1 F32 row
 *                       product, quant.rs:225-238, x86 dot order)
 *   hyq_moe_route       route (model.rs:728-767) per token: sigmoid, top
 *                       `used` of sigmoid + bias (f32::total_cmp, ties to the
 *                       lower index), weights sigmoid / max(sum, f16
 *                       MIN_POSITIVE) * scale (normalize) or sigmoid * scale;
 *                       topk_idx/topk_w [tokens, used] in that order
 *   hyq_moe_group       assignments (model.rs:695-701): the tokens of each
 *                       expert in token order as rows expert_off[e] ..
 *                       expert_off[e+1] of a grouped matrix (expert_off:
 *                       experts + 1 ints, at most 128 experts; row_token, row_weight: tokens * used
 *                       each; token_rows[t * used + k]: the row of token t's
 *                       k-th choice)
 *   hyq_matmul_experts_gate_up_silu / hyq_matmul_experts
 *                       the expert FFN (DenseFfn::forward, model.rs:673-685)
 *                       over the grouped rows on the tensor cores: weights are
 *                       [K, N, experts] tensors (Weight::expert,
 *                       quant.rs:144-154, gives expert e's slice); row i of
 *                       the input is input row input_rows[i] (NULL: row i);
 *                       output [rows, N] grouped; max_rows bounds any
 *                       expert's rows (e.g. tokens).  fp16 operands, f32
 *                       accumulation, as hyq_matmul at batch >= 16.
 *   hyq_moe_combine     out = shared; out += weight * value per expert in
 *                       ascending expert order (model.rs:691, 715-723). */
int hyq_moe_router(const hyq_weight* router, const float* x, int64_t tokens, float* logits, void* stream);
int hyq_moe_route(const float* logits, int64_t tokens, int experts, const float* bias, int used, int normalize,
                  float scale, int32_t* topk_idx, float* topk_w, void* stream);
int hyq_moe_group(const int32_t* topk_idx, const float* topk_w, int64_t tokens, int experts, int used,
                  int32_t* expert_off, int32_t* row_token, float* row_weight, int32_t* token_rows, void* stream);
int hyq_matmul_experts_gate_up_silu(const hyq_weight* gate, const hyq_weight* up, const float* input,
                                    const int32_t* input_rows, int64_t rows, const int32_t* expert_off,
                                    int64_t max_rows, float* out, void* stream);
int hyq_matmul_experts(const hyq_weight* w, const float* input, const int32_t* input_rows, int64_t rows,
                       const int32_t* expert_off, int64_t max_rows, float* out, void* stream);
int hyq_moe_combine(const float* shared, const float* expert_out, int64_t tokens, int64_t n, const int32_t* topk_idx,
                    const int32_t* token_rows, const float* row_weight, int used, float* out, void* stream);

/* --- Tensor-parallel all-reduce over NVLink peer memory ------------------
 * No counterpart in the reference (CPU only).  Sums the row-parallel partial
 * products (O, down) of a tensor-parallel layer across the ranks of one node
 * with plain peer loads and stores, no multicast.  Each rank owns a peer
 * region: HYQ_PEER_DATA_OFFSET bytes of flags, then its partial product.
 * hyq_peer_alloc: cudaMalloc a zeroed region for `data_bytes` of partials and
 *   return its CUDA IPC handle (64 bytes) for the other ranks;
 * hyq_peer_open / hyq_peer_close: map / unmap another rank's region;
 * hyq_peer_allreduce: regions[q] = rank q's region as mapped in this process
 *   (regions[rank] = the own one); out[0..n) = sum of the n partials at
 *   region + HYQ_PEER_DATA_OFFSET over all ranks, in rank order (identical on
 *   every rank).  Every rank makes the same sequence of calls; a call waits
 *   (bounded, 5 s unless hyq_set_peer_timeout_ms says otherwise ->
 *   HYQ_DEV_TIMEOUT_PEER) for the other ranks' flags, so the
 *   ranks' streams must all reach it.  At most 8 ranks; the partial may be
 *   rewritten once the call has completed on the stream.
 *   After HYQ_DEV_TIMEOUT_PEER on any rank, `out` of that call is undefined on
 *   every rank, and so are the results of all later calls on the same regions:
 *   a rank that gave up has left its flags for that epoch behind, so a late
 *   peer may sum a partial its owner has since overwritten.  Free and
 *   re-create the regions on every rank (hyq_peer_free / hyq_peer_alloc /
 *   hyq_peer_open) before the next call.  */
#define HYQ_PEER_DATA_OFFSET 1024
int hyq_peer_alloc(size_t data_bytes, void** region, void* ipc_handle);
int hyq_peer_open(const void* ipc_handle, void** region);
int hyq_peer_close(void* region);
int hyq_peer_free(void* region);
int hyq_peer_allreduce(const uint64_t* regions, int rank, int world, int64_t n, float* out, void* stream);
/* Expert-parallel row exchange over the same kind of regions (no
 * counterpart in the reference; it replaces the NCCL all-to-all of the
 * expert-parallel MoE layer).  send = [world][rows][row_floats] floats, block
 * q for rank q; rows [0, valid[q]) of block q (all rows when valid is NULL)
 * and, with last_row, the block's last row are stored into rank q's region
 * at HYQ_PEER_DATA_OFFSET + 4 * rank * slot_floats bytes, at the same row
 * offsets.  When the call has completed on the stream, this rank's region
 * holds every source's block (source s at slot s).  region_data_bytes = the
 * data_bytes every rank passed to hyq_peer_alloc, at least world *
 * slot_floats * 4; slot_floats >= rows * row_floats.  Two launches: the
 * first waits (bounded, as hyq_peer_allreduce) until every rank has reached
 * the same call, so no rank overwrites data a peer has not consumed; the
 * second pushes and waits for every peer's push.  Use its own regions (not
 * shared with hyq_peer_allreduce); every rank makes the same calls in the
 * same order; after HYQ_DEV_TIMEOUT_PEER the regions must be re-created. */
int hyq_peer_exchange(const uint64_t* regions, int rank, int world, size_t region_data_bytes, const float* send,
                      int rows, int row_floats, const int32_t* valid, int last_row, int64_t slot_floats,
                      void* stream);
/* Expert parallelism of the MoE layer over such regions (no counterpart in
 * the reference: Moe::forward, model.rs:688-767, runs one process), the
 * index work of the exchange done inside it.  Slots hold (cap + 1) rows of
 * `hidden` floats, cap = tokens x experts used per token (the most rows a
 * rank can send anywhere); every rank passes the same tokens and cap.
 * hyq_moe_ep_dispatch: this rank's grouped rows for rank q's experts (off /
 *   row_token from hyq_moe_group, experts_per_rank = E / world; rows
 *   row_token[off[q El] + i] of x) go into q's region, slot = rank, with a
 *   count row (row cap: the int32 row counts of q's experts);
 * hyq_moe_ep_plan: from the count rows in this rank's region, the
 *   expert-major gather index perm [world cap] (rows of the region data, as
 *   hyq_matmul_experts* take it), expert_off [El + 1], the inverse inv
 *   [world cap] and back_rows [world] (rows received from each source);
 * hyq_moe_ep_return: the expert outputs y [world cap, hidden] (expert-major)
 *   go back, rows inv[s cap + i] for i < back_rows[s] into source s's
 *   region at slot = rank;
 * hyq_moe_ep_home: the returned rows into out (the grouped-row outputs,
 *   row off[q El] + i from slot q).
 * Dispatch and return are exchanges (two launches each, bounded waits, as
 * hyq_peer_exchange); plan and home are local. */
int hyq_moe_ep_dispatch(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                        const float* x, int tokens, int hidden, const int32_t* off, const int32_t* row_token,
                        int experts_per_rank, int cap, void* stream);
int hyq_moe_ep_plan(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                    int hidden, int cap, int experts_per_rank, int32_t* perm, int32_t* expert_off, int32_t* inv,
                    int32_t* back_rows, void* stream);
int hyq_moe_ep_return(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                      const float* y, int hidden, const int32_t* inv, const int32_t* back_rows, int cap,
                      void* stream);
int hyq_moe_ep_home(const uint64_t* regions, int rank, int world, size_t region_data_bytes, int64_t slot_floats,
                    int hidden, const int32_t* off, int experts_per_rank, int cap, float* out, void* stream);
/* How long hyq_peer_allreduce waits for the other ranks' flags before it
 * gives up with HYQ_DEV_TIMEOUT_PEER: 1 .. 600000 ms, 5000 by default;
 * process-wide, read when a call is issued. */
int hyq_set_peer_timeout_ms(int ms);

/* Synchronize `stream`, then return (and clear) the device status word of
 * the current device: 0, or HYQ_DEV_* bits from kernels whose bounded waits
 * expired. */
int hyq_device_status(void* stream, uint32_t* status_out);

#ifdef __cplusplus
}
#endif

#endif /* HYQ_H_ */
