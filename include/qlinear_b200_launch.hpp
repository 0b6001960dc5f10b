// qlinear_b200_launch.hpp -- drop-in C++ replacements for the quantized launch
// functions of the local-llm engine (AI/codes/local-llm/src/backend/cuda/ops/
// kernel.cuh), implemented on libqlinear_b200.so.
//
// Include this header in the reference build AFTER "tensor/TensorCommon.h" and
// "backend/cuda/common.h" (it uses their DType and get_current_cuda_stream).
// In exactly one translation unit define QLINEAR_B200_DEFINE_LAUNCH before the
// include: that unit then holds the out-of-line definitions matching the
// declarations in kernel.cuh (whose definitions in launch.cu are removed).
// Without the macro the functions are inline.  Signatures are exactly the reference's; each call launches on the
// reference's current stream, and an error throws std::runtime_error (the
// reference's convention for host-side failures, common.cpp:19-29) instead of
// the reference's silent no-op on unsupported dtypes (launch.cu:57-58).
#ifndef QLINEAR_B200_LAUNCH_HPP
#define QLINEAR_B200_LAUNCH_HPP

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "qlinear_b200.h"

#ifndef LOCAL_LLM_TENSORCOMMON_H
#error "include tensor/TensorCommon.h (the reference's DType) before qlinear_b200_launch.hpp"
#endif

#ifdef QLINEAR_B200_DEFINE_LAUNCH
#define QLB200_LINKAGE
#else
#define QLB200_LINKAGE inline
#endif

namespace qlinear_b200_detail {
inline void check(int status, const char *what) {
    if (status != QL_OK) throw std::runtime_error(std::string(what) + ": " + ql_last_error());
}
inline int32_t code(DType t) { return static_cast<int32_t>(t); }
inline void bind_stream() { ql_set_stream(static_cast<void *>(get_current_cuda_stream())); }
}  // namespace qlinear_b200_detail

// kernel.cuh:34-35
QLB200_LINKAGE void launch_quant_gemv(DType quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                              int out_dim, int in_dim, int m) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(
        ql_quant_gemv(qlinear_b200_detail::code(quant_type), weight, row_bytes, x, y, out_dim, in_dim, m),
        "launch_quant_gemv");
}
// kernel.cuh:37-38
QLB200_LINKAGE void launch_quant_gemv_add(DType quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                                  int out_dim, int in_dim) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(
        ql_quant_gemv_add(qlinear_b200_detail::code(quant_type), weight, row_bytes, x, y, out_dim, in_dim),
        "launch_quant_gemv_add");
}
// kernel.cuh:42-43
QLB200_LINKAGE void launch_quant_matmul(DType quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                                int out_dim, int in_dim, int m) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(
        ql_quant_matmul(qlinear_b200_detail::code(quant_type), weight, row_bytes, x, y, out_dim, in_dim, m),
        "launch_quant_matmul");
}
// kernel.cuh:65-67
QLB200_LINKAGE void launch_quant_swiglu(DType quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                                size_t gate_row_bytes, size_t up_row_bytes, const float *x, float *act, int ffn_dim,
                                int in_dim) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_quant_swiglu(qlinear_b200_detail::code(quant_type), gate_weight, up_weight,
                                               gate_row_bytes, up_row_bytes, x, act, ffn_dim, in_dim),
                               "launch_quant_swiglu");
}
// kernel.cuh:72-76
QLB200_LINKAGE void launch_quant_swiglu_indexed(DType quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                                        size_t gate_expert_bytes, size_t up_expert_bytes, size_t gate_row_bytes,
                                        size_t up_row_bytes, const float *x, const int *expert_ids, float *act, int k,
                                        int ffn_dim, int in_dim) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(
        ql_quant_swiglu_indexed(qlinear_b200_detail::code(quant_type), gate_weight, up_weight, gate_expert_bytes,
                                up_expert_bytes, gate_row_bytes, up_row_bytes, x, expert_ids, act, k, ffn_dim, in_dim),
        "launch_quant_swiglu_indexed");
}
// kernel.cuh:125-129
QLB200_LINKAGE void launch_quant_down_f32_indexed_accum_ordered(DType quant_type, const uint8_t *down_weight,
                                                        size_t down_expert_bytes, size_t down_row_bytes,
                                                        const float *act, const int *expert_ids,
                                                        const float *route_weights, float *out, int k,
                                                        int hidden_size, int ffn_dim) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(
        ql_quant_down_f32_indexed_accum_ordered(qlinear_b200_detail::code(quant_type), down_weight, down_expert_bytes,
                                                down_row_bytes, act, expert_ids, route_weights, out, k, hidden_size,
                                                ffn_dim),
        "launch_quant_down_f32_indexed_accum_ordered");
}
// kernel.cuh:141-142
QLB200_LINKAGE void launch_quant_embedding(DType quant_type, const int *input, float *output, const uint8_t *table,
                                   size_t row_bytes, int hidden_size, int input_size) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_quant_embedding(qlinear_b200_detail::code(quant_type), input, output, table,
                                                  row_bytes, hidden_size, input_size),
                               "launch_quant_embedding");
}
// kernel.cuh:244-253
QLB200_LINKAGE void launch_dequantize_q4k_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_dequantize_q4k_to_f16(src, out, num_elements), "launch_dequantize_q4k_to_f16");
}
QLB200_LINKAGE void launch_dequantize_q80_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_dequantize_q80_to_f16(src, out, num_elements), "launch_dequantize_q80_to_f16");
}
QLB200_LINKAGE void launch_dequantize_q50_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_dequantize_q50_to_f16(src, out, num_elements), "launch_dequantize_q50_to_f16");
}
QLB200_LINKAGE void launch_dequantize_q6k_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_dequantize_q6k_to_f16(src, out, num_elements), "launch_dequantize_q6k_to_f16");
}
// kernel.cuh:335-336
QLB200_LINKAGE void launch_moe_router_topk(const float *router_logits, int *top_idx, float *top_w, int tokens, int n_experts,
                                   int k, float routed_scaling) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_moe_router_topk(router_logits, top_idx, top_w, tokens, n_experts, k, routed_scaling),
                               "launch_moe_router_topk");
}
// kernel.cuh:347
QLB200_LINKAGE void launch_argmax(const float *logits, int n, int *out_idx) {
    qlinear_b200_detail::bind_stream();
    qlinear_b200_detail::check(ql_argmax(logits, n, out_idx), "launch_argmax");
}

#endif  // QLINEAR_B200_LAUNCH_HPP
