// Opt-in int8 activation path (ql_q81.cu): Q8_1 activation quantizer and Q8_1 GEMV.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace ql {

struct Q81MmArgs {
    const uint8_t *w;      // [out_dim][rb] weights (16-byte-aligned base)
    size_t rb;
    const uint8_t *xq;     // [m][q81_row_bytes(in_dim)] Q8_1 activation rows
    float *y;              // [m][out_dim]
    int out_dim, in_dim, m;
    int row_pitch;         // shared-memory bytes per staged weight row (q81_mm_row_pitch)
    int *err;
};

size_t q81_row_bytes(int in_dim);
size_t q81_mmq_row_bytes(int in_dim);
int q81_mm_row_pitch(size_t row_bytes);
cudaError_t matmul_q81_launch(int fmt, const Q81MmArgs &a, bool mmq, cudaStream_t s);
cudaError_t quantize_q81_launch(const float *x, uint8_t *xq, int in_dim, int m, bool store_raw_sum, bool mmq,
                                cudaStream_t s);
cudaError_t gemv_q81_launch(int fmt, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int out_dim, int in_dim,
                            cudaStream_t s);

}  // namespace ql
