// ref_shim.cpp -- test infrastructure (oracle side), not product code.
//
// extern "C" entry points over the reference's own C++ launch functions so the
// tests can call the reference's CUDA kernels (AI/codes/local-llm/src/backend/
// cuda/ops/{kernel.cu,launch.cu}, compiled unchanged for sm_100a into
// oracle/_ref by oracle/Makefile) through ctypes.  Every function forwards its
// arguments verbatim; the reference launches on its process-global current
// stream (common.cpp:12-17), which ref_set_stream sets.
#include "backend/cuda/common.h"
#include "backend/cuda/ops/kernel.cuh"

#include <cuda_runtime.h>

extern "C" {

int ref_set_stream(void *stream) {
    set_current_cuda_stream(static_cast<cudaStream_t>(stream));
    return 0;
}

int ref_last_error(void) { return static_cast<int>(cudaGetLastError()); }

// kernel.cuh:34-35
void ref_quant_gemv(int t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim, int m) {
    launch_quant_gemv(static_cast<DType>(t), w, rb, x, y, out_dim, in_dim, m);
}
// kernel.cuh:37-38
void ref_quant_gemv_add(int t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim) {
    launch_quant_gemv_add(static_cast<DType>(t), w, rb, x, y, out_dim, in_dim);
}
// kernel.cuh:42-43
void ref_quant_matmul(int t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim, int m) {
    launch_quant_matmul(static_cast<DType>(t), w, rb, x, y, out_dim, in_dim, m);
}
// kernel.cuh:65-67
void ref_quant_swiglu(int t, const uint8_t *g, const uint8_t *u, size_t grb, size_t urb, const float *x, float *act,
                      int ffn_dim, int in_dim) {
    launch_quant_swiglu(static_cast<DType>(t), g, u, grb, urb, x, act, ffn_dim, in_dim);
}
// kernel.cuh:72-76
void ref_quant_swiglu_indexed(int t, const uint8_t *g, const uint8_t *u, size_t geb, size_t ueb, size_t grb,
                              size_t urb, const float *x, const int *ids, float *act, int k, int ffn_dim,
                              int in_dim) {
    launch_quant_swiglu_indexed(static_cast<DType>(t), g, u, geb, ueb, grb, urb, x, ids, act, k, ffn_dim, in_dim);
}
// kernel.cuh:125-129
void ref_quant_down_ordered(int t, const uint8_t *d, size_t deb, size_t drb, const float *act, const int *ids,
                            const float *rw, float *out, int k, int hidden, int ffn_dim) {
    launch_quant_down_f32_indexed_accum_ordered(static_cast<DType>(t), d, deb, drb, act, ids, rw, out, k, hidden,
                                                ffn_dim);
}
// kernel.cuh:335-336
void ref_moe_router_topk(const float *logits, int *idx, float *w, int tokens, int n_experts, int k, float scale) {
    launch_moe_router_topk(logits, idx, w, tokens, n_experts, k, scale);
}
// kernel.cuh:141-142
void ref_quant_embedding(int t, const int *ids, float *out, const uint8_t *table, size_t rb, int hidden, int n) {
    launch_quant_embedding(static_cast<DType>(t), ids, out, table, rb, hidden, n);
}
// kernel.cuh:347
void ref_argmax(const float *logits, int n, int *out_idx) { launch_argmax(logits, n, out_idx); }
// kernel.cuh:244-253
void ref_dequantize_q4k(const uint8_t *src, uint16_t *out, int64_t n) { launch_dequantize_q4k_to_f16(src, out, n); }
void ref_dequantize_q80(const uint8_t *src, uint16_t *out, int64_t n) { launch_dequantize_q80_to_f16(src, out, n); }
void ref_dequantize_q50(const uint8_t *src, uint16_t *out, int64_t n) { launch_dequantize_q50_to_f16(src, out, n); }
void ref_dequantize_q6k(const uint8_t *src, uint16_t *out, int64_t n) { launch_dequantize_q6k_to_f16(src, out, n); }

// kernel.cuh:186-189
void ref_full_attention_attend(const float *q, const float *gate, const void *k, const void *v, int kv_bf16,
                               float *attn, int n_heads, int kv_heads, int head_dim, int max_seq_len,
                               const int *pos_dev) {
    launch_full_attention_attend(q, gate, k, v, kv_bf16 != 0, attn, n_heads, kv_heads, head_dim, max_seq_len,
                                 pos_dev);
}
// kernel.cuh:191-194
void ref_full_attention_attend_batch(const float *q, const float *gate, const void *k, const void *v, int kv_bf16,
                                     float *attn, int tokens, int n_heads, int kv_heads, int head_dim,
                                     int max_seq_len, int start_pos) {
    launch_full_attention_attend_batch(q, gate, k, v, kv_bf16 != 0, attn, tokens, n_heads, kv_heads, head_dim,
                                       max_seq_len, start_pos);
}

// kernel.cuh:48-49
void ref_quantize_q8_1(const float *x, uint8_t *xq, int in_dim, int m, int store_raw_sum) {
    launch_quantize_q8_1(x, xq, in_dim, m, store_raw_sum != 0);
}
// kernel.cuh:50-52
void ref_quant_gemv_q8_1(int t, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int out_dim, int in_dim) {
    launch_quant_gemv_q8_1(static_cast<DType>(t), w, rb, xq, y, out_dim, in_dim);
}

// kernel.cuh:53-55
void ref_quant_matmul_q8_1(int t, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int out_dim, int in_dim,
                           int m) {
    launch_quant_matmul_q8_1(static_cast<DType>(t), w, rb, xq, y, out_dim, in_dim, m);
}

// kernel.cuh:57-61
void ref_quantize_q8_1_mmq(const float *x, uint8_t *xq, int in_dim, int m, int store_raw_sum) {
    launch_quantize_q8_1_mmq(x, xq, in_dim, m, store_raw_sum != 0);
}
void ref_quant_matmul_q8_1_mmq(int t, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int out_dim,
                               int in_dim, int m) {
    launch_quant_matmul_q8_1_mmq(static_cast<DType>(t), w, rb, xq, y, out_dim, in_dim, m);
}

}  // extern "C"
