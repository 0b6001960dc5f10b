// ql_gemv_q40.cu -- GEMV engine instantiations for Q4_0.
#include "ql_gemv_impl.cuh"

namespace ql {
template cudaError_t gemv_launch_fmt<kQ4_0>(int, const GemvArgs &, int, bool, int, cudaStream_t);
}  // namespace ql
