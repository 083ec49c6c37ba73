// Streaming GEMV kernels for STQ1_0 (see hyq_gemv_impl.cuh).
#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace gemv {
template cudaError_t dispatch_fmt<STQ1_0>(const Params&, const Plan&, bool, cudaStream_t);
}  // namespace gemv
}  // namespace hyq
