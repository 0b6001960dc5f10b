// ql_gemv_q4k.cu -- GEMV engine instantiations for Q4_K.
#include "ql_gemv_impl.cuh"

namespace ql {
template cudaError_t gemv_launch_fmt<kQ4_K>(int, const GemvArgs &, int, bool, int, cudaStream_t);
}  // namespace ql
