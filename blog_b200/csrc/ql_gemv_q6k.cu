// ql_gemv_q6k.cu -- GEMV engine instantiations for Q6_K.
#include "ql_gemv_impl.cuh"

namespace ql {
template cudaError_t gemv_launch_fmt<kQ6_K>(int, const GemvArgs &, int, bool, int, cudaStream_t);
}  // namespace ql
