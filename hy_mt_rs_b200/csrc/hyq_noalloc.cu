// hyq_matmul_noalloc: Weight::matmul (hy-mt-rs src/quant.rs:159-344) on the
// same kernels as hyq_matmul, with the tensor-core path's scratch in a fixed
// device array instead of a stream-ordered allocation.
//
// Some callers cannot take a device allocation on every product: a serving
// process that gives all free HBM to its own cache when it starts (an
// allocation in the middle of a request could then fail), or a host that
// accounts for every byte of device memory itself and so cannot accept the
// workspace pool hyq_matmul keeps cached until the process exits.  This entry
// point allocates nothing: the array below belongs to the module image, and
// every GPU that loads the module holds it until the process exits.
//
// Limits: one call's scratch is at most HYQ_NOALLOC_SCRATCH_BYTES; every call
// on a device uses the same array, so two calls that overlap on the GPU race.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/hyq.h"
#include "hyq_kernels.h"

namespace {

// fp16 activation copy followed by the split-K partial sums of one call.  The
// array keeps whatever the previous call left, and nothing in it has to start
// at zero: each byte a call reads was written earlier in the same call (the
// conversion kernel writes the whole fp16 copy, and every split-K slice
// stores its whole partial tile before the reduction reads it).
static __device__ __align__(256) unsigned char g_scratch[HYQ_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Set-up, once per device, by the first call made with that device current.
// Host code sees g_scratch only as a host-side stand-in, so the kernels get
// the device address of this device's copy of the array.
int scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hyq::api_fail(HYQ_E_CUDA, "matmul_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return hyq::api_fail(HYQ_E_UNSUPPORTED, "matmul_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_scratch);
    if (e != cudaSuccess)
      return hyq::api_fail(HYQ_E_CUDA, "matmul_noalloc: cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return HYQ_OK;
}

// Batches from this size up take the tensor-core GEMM, as in hyq_matmul.
constexpr int64_t kGemmMinBatch = 16;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

extern "C" int hyq_matmul_noalloc(const hyq_weight* w, const float* input, int64_t batch, float* out,
                                  void* stream) {
  if (!w) return hyq::api_fail(HYQ_E_INVALID, "matmul_noalloc: null weight");
  int dtype = 0, ndim = 0;
  int64_t dims[3] = {};
  const void* data = nullptr;
  int rc = hyq_weight_info(w, &dtype, &ndim, dims, nullptr, &data);
  if (rc) return rc;
  if (ndim != 2) return hyq::api_fail(HYQ_E_SHAPE, "matmul_noalloc: weight is not a matrix");
  if (batch <= 0) return hyq::api_fail(HYQ_E_SHAPE, "invalid activation shape");
  if (!input || !out) return hyq::api_fail(HYQ_E_INVALID, "matmul_noalloc: null pointer");
  if (!aligned(input, 4)) return hyq::api_fail(HYQ_E_ALIGN, "matmul_noalloc: input not 4-byte aligned");
  void* scratch = nullptr;
  if ((rc = scratch_ptr(&scratch))) return rc;
  const int64_t K = dims[0], N = dims[1];
  cudaStream_t st = (cudaStream_t)stream;
  if (batch >= kGemmMinBatch && hyq::gemm_supported(dtype, K, N, batch, data) && aligned(input, 16)) {
    const bool split = hyq::gemm_split();
    const size_t need = hyq::gemm_workspace_bytes(dtype, K, N, batch, split);
    if (need > HYQ_NOALLOC_SCRATCH_BYTES)
      return hyq::api_fail(HYQ_E_SHAPE,
                           "matmul_noalloc: batch %lld x K %lld (N %lld) needs %zu bytes of scratch, more than the "
                           "fixed %zu (HYQ_NOALLOC_SCRATCH_BYTES); split the batch or use hyq_matmul",
                           (long long)batch, (long long)K, (long long)N, need, (size_t)HYQ_NOALLOC_SCRATCH_BYTES);
    unsigned* status = nullptr;
    if ((rc = hyq::api_status_word(&status))) return rc;
    const cudaError_t e =
        hyq::launch_gemm(dtype, static_cast<const uint8_t*>(data), K, N, input, batch, out, scratch, status, st, split);
    if (e != cudaSuccess)
      return hyq::api_fail(HYQ_E_CUDA, "matmul_noalloc (tensor-core GEMM): %s", cudaGetErrorString(e));
    return HYQ_OK;
  }
  // Other batches run batch-1 products, which use no scratch.
  for (int64_t b = 0; b < batch; ++b)
    if ((rc = hyq_matmul(w, input + b * K, 1, out + b * N, stream))) return rc;
  return HYQ_OK;
}
