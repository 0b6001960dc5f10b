// ql_gemv_q50.cu -- GEMV engine instantiations for Q5_0.
#include "ql_gemv_impl.cuh"

namespace ql {
template cudaError_t gemv_launch_fmt<kQ5_0>(int, const GemvArgs &, int, bool, int, cudaStream_t);
}  // namespace ql
