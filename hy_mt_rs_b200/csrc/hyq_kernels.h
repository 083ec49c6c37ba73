// Internal host-side launch interface between the C ABI layer (hyq_api.cu)
// and the kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace hyq {

cudaError_t launch_decode(int dtype, const void* src, float* dst, int64_t n_out, cudaStream_t st);
cudaError_t launch_dot(const float* a, const float* b, int64_t n, float* out, cudaStream_t st);
cudaError_t launch_q8_quantize(const float* x, int64_t len, int8_t* values, float* scales, int8_t* values_q2c,
                               cudaStream_t st);

// One fused matrix-vector launch over up to three matrices that share the
// input width K and the packed type (QKV), or over a gate/up pair whose rows
// are combined as silu(gate) * up.
struct GemvJob {
  int dtype = 0;
  int n_mat = 1;                  // 1..3
  const uint8_t* w[3] = {};       // packed rows, device
  float* y[3] = {};               // outputs, device
  int64_t rows[3] = {};
  const uint8_t* up = nullptr;    // gate/up mode: up rows (same shape as w[0])
  int64_t K = 0;
  // Activations: exactly one of (x) or (xq, xs) is set.
  const float* x = nullptr;       // f32 [K]
  const int8_t* xq = nullptr;     // int8 [K] (natural order, as Q8::values)
  const float* xs = nullptr;      // f32 [ceil(K/256)] (Q8::scales)
  // With x set: quantize it to Q8 inside the kernel (gemv_q8, quant.rs:348)
  // instead of multiplying the f32 values.
  bool quantize_q8 = false;
  // Fused forms (see gemv_fusable): normalise x in the prologue
  // (RMSNorm with these weights and eps), add every output into y.
  const float* norm_w = nullptr;
  float eps = 0.f;
  bool residual = false;
  unsigned* status = nullptr;     // device status word (bounded-wait failures)
  // Launch as a programmatic dependent of the preceding grid in the stream
  // (hyq_set_launch_overlap); weights must not be written by work in flight.
  bool overlap = false;
};

cudaError_t launch_gemv(const GemvJob& job, cudaStream_t st);

// Which engine launch_gemv picks for a job (for tests and the bench):
// 0 = streaming bulk-copy kernel, 1 = per-element fallback.
int gemv_engine(const GemvJob& job);
// Whether the fused forms (norm_w / residual) accept a job: the streaming
// engine with f32 activations staged in shared memory, K <= 6144.
bool gemv_fusable(const GemvJob& job);

// Batched products (Weight::matmul, batch >= 2) on tcgen05 tensor cores.
// The activations are first rounded to fp16 into `workspace`
// (gemm_workspace_bytes bytes, 256-byte aligned), which also holds split-K
// partial sums when the grid is small.
// Several matrices of one type sharing K and the activations (QKV: their
// outputs are separate), or a gate/up pair with out = silu(gate x) * (up x).
struct GemmJob {
  int dtype = 0;
  int n_mat = 1;                // 1..3, or 2 with gate_up
  bool gate_up = false;
  const uint8_t* w[3] = {};     // packed rows, 16-byte aligned
  int64_t rows[3] = {};
  float* y[3] = {};             // [M, rows[m]]; gate_up: y[0] only
  int64_t K = 0, M = 0;
  const float* x = nullptr;     // f32 [M, K]
  unsigned* status = nullptr;
  // Expert mode (Moe::forward, model.rs:688-726): w[m] hold `experts`
  // matrices of rows[m] rows each, back to back (a GGUF [K, rows, experts]
  // tensor), and the M activation rows are grouped by expert: those of expert
  // e are rows expert_off[e] .. expert_off[e + 1] (device memory, written by
  // an earlier kernel in the stream; at most expert_max_rows per expert).
  // Row i of the activations is row x_rows[i] of x (x_rows null: row i).
  int experts = 0;
  const int32_t* expert_off = nullptr;
  int64_t expert_max_rows = 0;
  const int32_t* x_rows = nullptr;
  // Split-operand form (hi + lo fp16 operands, three MMAs per K chunk, f32
  // accuracy); the workspace then holds two activation copies.
  bool split = false;
  // Fused input (not with experts or x_rows): with norm_w set the product
  // reads RMSNorm(norm_x rows) * norm_w; with norm_delta set too, norm_x +=
  // norm_delta first (written back).  K at most 16384.
  float* norm_x = nullptr;
  const float* norm_delta = nullptr;
  const float* norm_w = nullptr;
  float norm_eps = 0.f;
};
bool gemm_job_supported(const GemmJob& job);
size_t gemm_job_workspace_bytes(const GemmJob& job);
cudaError_t launch_gemm_job(const GemmJob& job, void* workspace, cudaStream_t st);

bool gemm_supported(int dtype, int64_t K, int64_t N, int64_t M, const void* w);
size_t gemm_workspace_bytes(int dtype, int64_t K, int64_t N, int64_t M, bool split);
cudaError_t launch_gemm(int dtype, const uint8_t* w, int64_t K, int64_t N, const float* x, int64_t M, float* y,
                        void* workspace, unsigned* status, cudaStream_t st, bool split);

// hyq_set_gemm_precision's switch (HYQ_GEMM_F32: split-operand products),
// read once per call by the entry points that launch batched products.
bool gemm_split();

// C-ABI plumbing (hyq_api.cu): set the calling thread's hyq_last_error text
// and return `code`; the current device's status word.
int api_fail(int code, const char* fmt, ...);
int api_status_word(unsigned** out);
// hyq_set_launch_overlap's switch, read at launch time.
bool launch_overlap();

// Launch with the programmatic-dependent attribute when launch_overlap() is
// on: such kernels wait for their predecessor grid (griddepcontrol.wait)
// before touching memory, and let their own dependents launch early.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
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

}  // namespace hyq
