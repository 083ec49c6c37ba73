// Streaming GEMV kernels for Q2_0C (see hyq_gemv_impl.cuh).
#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace gemv {
template cudaError_t dispatch_fmt<Q2_0C>(const Params&, const Plan&, bool, cudaStream_t);
}  // namespace gemv
}  // namespace hyq
