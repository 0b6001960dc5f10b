// ql_gemv.cu -- format dispatch of the streaming GEMV engine (see ql_gemv.cuh).
#include "ql_gemv.cuh"

namespace ql {

template <int FMT>
cudaError_t gemv_launch_fmt(int kind, const GemvArgs &a, int MT, bool tma, int smem, cudaStream_t s);

cudaError_t gemv_launch(int fmt, int kind, const GemvArgs &a, int MT, bool tma, int smem, cudaStream_t s) {
    switch (fmt) {
    case kQ4_K: return gemv_launch_fmt<kQ4_K>(kind, a, MT, tma, smem, s);
    case kQ8_0: return gemv_launch_fmt<kQ8_0>(kind, a, MT, tma, smem, s);
    case kQ4_0: return gemv_launch_fmt<kQ4_0>(kind, a, MT, tma, smem, s);
    case kQ5_0: return gemv_launch_fmt<kQ5_0>(kind, a, MT, tma, smem, s);
    case kQ6_K: return gemv_launch_fmt<kQ6_K>(kind, a, MT, tma, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace ql
