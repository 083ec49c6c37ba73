// Streaming GEMV kernels for Q8_0 (see hyq_gemv_impl.cuh).
#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace gemv {
template cudaError_t dispatch_fmt<Q8_0>(const Params&, const Plan&, bool, cudaStream_t);
}  // namespace gemv
}  // namespace hyq
