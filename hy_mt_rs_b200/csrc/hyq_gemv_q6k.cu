// Streaming GEMV kernels for Q6_K (see hyq_gemv_impl.cuh).
#include "hyq_gemv_impl.cuh"

namespace hyq {
namespace gemv {
template cudaError_t dispatch_fmt<Q6_K>(const Params&, const Plan&, bool, cudaStream_t);
}  // namespace gemv
}  // namespace hyq
