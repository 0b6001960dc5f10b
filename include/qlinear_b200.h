/*
 * qlinear_b200.h -- C ABI of libqlinear_b200.so, the B200 (sm_100a) block-quantized
 * linear path of the local-llm engine (allenzhang61/blog, AI/codes/local-llm).
 *
 * Every entry point below is the C twin of one reference launch function in
 * src/backend/cuda/ops/kernel.cuh (cited per function): same argument order and
 * meaning, raw GGUF weight bytes as uploaded unchanged by CudaWeightPool
 * (CudaWeightPool.cpp:148-175), fp32 activations, launches on the library's
 * current stream (the reference's process-global stream, common.cpp:12-17).
 * Differences from the reference, by design:
 *   - each function returns a status instead of void; an unsupported dtype or
 *     an invalid shape returns QL_EINVAL instead of silently doing nothing
 *     (the reference's launchers fall through `default: break;`, launch.cu:57-58);
 *   - Q4_0 is supported (the reference parses it but has no arithmetic for it);
 *   - all pointers are device pointers unless stated otherwise.
 * A C++ header-only shim with the reference's exact C++ signatures
 * (DType enum, void return, throw on error) is in qlinear_b200_launch.hpp.
 */
#ifndef QLINEAR_B200_H
#define QLINEAR_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QL_API __attribute__((visibility("default")))
#else
#define QL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type codes, equal to the reference's DType (src/tensor/TensorCommon.h:15-33). */
#define QL_F32 0
#define QL_F16 1
#define QL_Q4_0 2
#define QL_Q5_0 6
#define QL_Q8_0 8
#define QL_Q4_K 12
#define QL_Q6_K 14

/* Status codes. */
#define QL_OK 0
#define QL_EINVAL 1   /* bad argument: dtype, shape, block multiple, null pointer */
#define QL_ECUDA 2    /* CUDA runtime error (see ql_last_error) */
#define QL_EDEVICE 3  /* a kernel gave up a bounded wait and recorded an error */

/* ---- runtime -------------------------------------------------------------------- */
/* set/get the stream every launch uses (reference set/get_current_cuda_stream,
 * common.h:40-44).  NULL = the legacy default stream. */
QL_API int ql_set_stream(void *stream);
QL_API void *ql_get_stream(void);
/* Allocate the per-device workspace (stream-K partials, arrival counters, argmax
 * partials, error word) for `device`.  Called implicitly by the first launch on a
 * device; call it explicitly before capturing launches into a CUDA graph. */
QL_API int ql_init(int device);
/* Human-readable description of the last error returned by this thread. */
QL_API const char *ql_last_error(void);
/* Synchronize the current stream and read (and clear) the device error word. */
QL_API int ql_check_device(void);

/* ---- quantized linear (reference kernel.cuh:34-43) ------------------------------- */
/* y[m, o] = sum_k W[o, k] * x[m, k].  W: out_dim rows of row_bytes GGUF bytes.
 * x: [m, in_dim] f32, y: [m, out_dim] f32, row-major.  kernel.cuh:34-35. */
QL_API int ql_quant_gemv(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                  int out_dim, int in_dim, int m);
/* y[o] += W[o, :] . x  (m = 1).  kernel.cuh:37-38. */
QL_API int ql_quant_gemv_add(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                      int out_dim, int in_dim);
/* Same contract as ql_quant_gemv, intended for m > 1 (prefill).  kernel.cuh:42-43. */
QL_API int ql_quant_matmul(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x, float *y,
                    int out_dim, int in_dim, int m);
/* Prefill GEMM with a selectable path and fused extras (no reference twin; the
 * reference runs prefill as launch_quant_matmul, kernel.cuh:42-43, or as
 * dequantize-to-f16 + cuBLAS, TensorTool.cpp:127-144):
 *   y[m, o] (+)= scale_m * sum_k W[o, k] * g[k] * x[m, k] + bias[o]
 * with x rows x_stride floats apart, y rows y_stride apart, optional fused RMSNorm
 * (gamma != NULL: scale_m = 1/sqrt(mean_k x[m,k]^2 + eps), g = gamma; else 1),
 * optional bias, accumulate != 0 adds into y.  path: QL_PATH_AUTO picks by shape;
 * QL_PATH_GEMV forces the CUDA-core streaming engine (fp32 activations, exact
 * decode); QL_PATH_TENSOR forces the tcgen05 tensor-core GEMM (Q4_K, Q4_0 or Q8_0, in_dim
 * a multiple of 256; activations and dequantized weights rounded to f16, fp32
 * accumulation; QL_EINVAL when the shape or dtype does not qualify). */
#define QL_PATH_AUTO 0
#define QL_PATH_GEMV 1
#define QL_PATH_TENSOR 2
QL_API int ql_quant_matmul_ex(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x,
                              int64_t x_stride, float *y, int64_t y_stride, int out_dim, int in_dim, int m,
                              const float *gamma, float eps, const float *bias, int accumulate, int path);
/* Greedy LM head (fused GEMV/GEMM + argmax, no separate argmax launch): for each token m,
 * out_idx[m] = index_offset + argmax_o y[m, o] with y as ql_quant_matmul_ex (plain store,
 * optional fused RMSNorm), lowest index on ties, NaN never wins (reference argmax,
 * kernel.cu:3531-3592).  logits (nullable) also receives y.  out_key (nullable) receives
 * an order-preserving 64-bit key per token (larger = better, ties to the lower index);
 * the maximum key over vocabulary shards, each launched with its own index_offset,
 * selects the same token as an argmax over the whole vocabulary.  m <= 4096. */
QL_API int ql_quant_gemv_argmax_ex(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x,
                                   int64_t x_stride, float *logits, int64_t logits_stride, int out_dim, int in_dim,
                                   int m, const float *gamma, float eps, int index_offset, int *out_idx,
                                   uint64_t *out_key);
/* ---- a chain of single-token GEMVs in one persistent launch ----------------------
 * A decode step's projections (q/k/v, o + residual, gate/up SwiGLU, down + residual,
 * ..., LM head + argmax) as one cooperative kernel: the weight stream runs across op
 * boundaries and each op waits at a grid barrier for the previous op's output.  Q4_K,
 * one token, in_dim a multiple of 256 and >= 1792, 16-byte aligned weights with
 * row_bytes % 16 == 0 and >= 32 rows per source.  Op semantics equal the per-op entry
 * points: STORE y = (RMSNorm?)(x) . W^T + bias over 1..3 stacked sources (all but the
 * last a multiple of 32 rows), optionally with a greedy argmax (argmax_idx, device int,
 * index + argmax_offset; y may then be NULL); ADD y += ...; SWIGLU y = SiLU(g) * u with
 * w[0] = gate, w[1] = up.  Every op may read what any earlier op wrote.  The chain keeps
 * the pointers: buffers must outlive it.  ql_gemv_chain_run enqueues one launch on the
 * current stream (graph-capturable). */
#define QL_OP_STORE 0
#define QL_OP_ADD 1
#define QL_OP_SWIGLU 2
/* MLP (one GPU): y += down . (SiLU(gate . x^) * (up . x^)), x^ = RMSNorm(x) with gamma, as SWIGLU
 * then ADD in one op without the grid barrier between them: w[0] = gate, w[1] = up (rows[0] =
 * rows[1] = FFN width, a multiple of 256), w[2] = down (rows[2] = len(y), in FFN blocks).  The
 * down projection is split over the FFN (two SMs per 256-row chunk) and its partial sums are
 * added in 64-bit fixed point (2^-32 resolution, |y| < 2^31; deterministic).  y must be last
 * written by an ADD op of the chain (same y and rows), and the next op must not be an ADD into
 * y or another MLP.  The SwiGLU activations are not stored. */
#define QL_OP_MLP 3
typedef struct ql_chain_op {
    int32_t kind;
    int32_t quant_type;
    int32_t nsrc;
    const uint8_t *w[3];
    size_t row_bytes[3];
    int32_t rows[3];
    int32_t in_dim;
    const float *x;
    const float *gamma;
    float eps;
    const float *bias;
    float *y;
    int *argmax_idx;
    int32_t argmax_offset;
    int32_t reduce; /* tensor parallel ADD: y += sum over ranks of this op's partial (no bias) */
    /* batched chains only (ql_gemv_chain_create_batch): floats between consecutive tokens' rows of
     * x and of y; 0 = rows packed (in_dim, resp. the op's total output rows) */
    int64_t x_stride;
    int64_t y_stride;
    /* RoPE fused into a STORE op (no reference twin as a fusion; the reference rotates q and k in
     * its attention kernels, kernel.cu:186-260): output rows [0, rope_rows) -- whole heads of
     * head_dim rows, e.g. the q and k rows of a stacked q/k/v -- are rotated after bias, pairing
     * rows i and i + head_dim/2 of each head: (x1, x2) -> (x1 c - x2 s, x2 c + x1 s), angle =
     * pos / rope_theta^(2i / head_dim).  rope_pos: device int32, the position (batched chains: one
     * per token).  rope_rows = 0 disables it; head_dim a multiple of 32, at most 128 in batched
     * chains; no argmax on a RoPE op. */
    const int32_t *rope_pos;
    float rope_theta;
    int32_t rope_rows;
    int32_t head_dim;
} ql_chain_op;
QL_API int ql_gemv_chain_create(const ql_chain_op *ops, int nops, void **chain);
/* Tensor-parallel chain: ops with reduce != 0 (row-parallel ADD projections) sum their
 * partials over ranks inside the kernel through peer memory (each rank's exchange buffer,
 * ql_gemv_chain_exchange_bytes bytes, zeroed, mapped into every rank: exchange[r] for
 * rank r, e.g. with ql_ipc_alloc / ql_ipc_open); an argmax op (vocabulary shard with
 * argmax_offset) combines the ranks' keys the same way.  Every rank must create and run
 * the same chain; a rank that never arrives makes the others give up after ~5 s with an
 * error in the device error word. */
QL_API size_t ql_gemv_chain_exchange_bytes(const ql_chain_op *ops, int nops, int world);
QL_API int ql_gemv_chain_create_tp(const ql_chain_op *ops, int nops, int rank, int world, void *const *exchange,
                                   void **chain);
/* Device allocation shareable with other processes (zeroed), its CUDA IPC handle, and the
 * peer side: map / unmap another process's allocation. */
QL_API int ql_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle);
QL_API int ql_ipc_free(void *ptr);
QL_API int ql_ipc_open(const uint8_t *handle, void **ptr);
QL_API int ql_ipc_close(void *ptr);
/* Batched chain (no reference twin; the reference runs batched decode as quant_matmul_kernel,
 * kernel.cu:1253-1279, one warp per (token, row) on the CUDA cores): the same op list for
 * `tokens` (1..32) tokens in one persistent launch on the tensor cores.  x and y are [tokens, *]
 * row-major with the ops' x_stride / y_stride; RMSNorm, bias, residual add and SwiGLU apply per
 * token; an argmax op writes one index per token (argmax_idx[0..tokens)).  Kinds STORE, ADD,
 * SWIGLU (no MLP, no tensor-parallel reduce); Q4_K; stacked sources but the last a multiple of
 * 128 rows; x rows 16-byte aligned.  Weights and x * gamma are rounded to f16 (|x * gamma| <
 * 65504), accumulation is fp32.  ql_gemv_chain_run / ql_gemv_chain_destroy run and free it. */
QL_API int ql_gemv_chain_create_batch(const ql_chain_op *ops, int nops, int tokens, void **chain);
QL_API int ql_gemv_chain_run(void *chain);
QL_API int ql_gemv_chain_destroy(void *chain);

/* Reserve the tensor-core path's scratch (f16 activations, row scales, split-K
 * partial tiles) on the current device for up to max_tokens x max_in_dim, so later
 * prefill calls of at most that size allocate nothing (e.g. inside graph capture).
 * Larger calls grow the scratch with cudaMalloc. */
QL_API int ql_reserve_prefill(int max_tokens, int max_in_dim);

/* ---- tensor-parallel exchange over NVLink peer memory ------------------------------
 * One-shot all-reduce for the decode step's row-parallel projections (no reference
 * twin: the reference engine is single-GPU).  Setup, once per rank:
 *   ql_comm_alloc   allocates this rank's zeroed exchange buffer on the current device
 *                   and returns its CUDA IPC handle (QL_IPC_HANDLE_BYTES bytes);
 *   (exchange the handles between ranks by any host channel, in rank order)
 *   ql_comm_create  maps every peer's buffer (handles: world x QL_IPC_HANDLE_BYTES).
 * Per step: the same sequence of ql_allreduce_f32 calls on every rank, each naming
 * its call site with a distinct slot < slots, then one ql_comm_step.  Everything is
 * enqueued on the current stream and may be captured into a CUDA graph.  A peer that
 * never arrives makes the call give up after ~5 s with an error in the device error
 * word (ql_check_device returns QL_EDEVICE). */
#define QL_IPC_HANDLE_BYTES 64
QL_API size_t ql_comm_bytes(int world, int max_floats, int slots);
QL_API int ql_comm_alloc(int world, int max_floats, int slots, void **exchange, uint8_t *handle);
QL_API int ql_comm_create(int rank, int world, int max_floats, int slots, void *exchange, const uint8_t *handles,
                          void **comm);
QL_API int ql_comm_destroy(void *comm);
/* buf[0..n) (device, n <= max_floats) := sum over ranks, bit-identical on every rank. */
QL_API int ql_allreduce_f32(void *comm, float *buf, int n, int slot);
QL_API int ql_comm_step(void *comm);

/* act[f] = SiLU(Wg[f] . x) * (Wu[f] . x).  kernel.cuh:65-67. */
QL_API int ql_quant_swiglu(int32_t quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                    size_t gate_row_bytes, size_t up_row_bytes, const float *x, float *act, int ffn_dim,
                    int in_dim);

/* ---- MoE (reference kernel.cuh:72-76, 125-129, 335-336) -------------------------- */
/* act[r, f] = SiLU(Wg[e_r][f] . x) * (Wu[e_r][f] . x), e_r = expert_ids[r] (device);
 * e_r < 0 writes zeros.  Expert e's rows start at weight + e * expert_bytes. */
QL_API int ql_quant_swiglu_indexed(int32_t quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                            size_t gate_expert_bytes, size_t up_expert_bytes, size_t gate_row_bytes,
                            size_t up_row_bytes, const float *x, const int *expert_ids, float *act, int k,
                            int ffn_dim, int in_dim);
/* out[h] += sum_r route_weights[r] * (Wd[e_r][h] . act[r, :]) over routes with e_r >= 0,
 * in a fixed (deterministic) order. */
QL_API int ql_quant_down_f32_indexed_accum_ordered(int32_t quant_type, const uint8_t *down_weight,
                                            size_t down_expert_bytes, size_t down_row_bytes, const float *act,
                                            const int *expert_ids, const float *route_weights, float *out, int k,
                                            int hidden_size, int ffn_dim);
/* Per token: softmax over n_experts (<= 64) logits, top-k by logit (lowest id on
 * ties, non-finite = -inf), top_w = p * routed_scaling. */
QL_API int ql_moe_router_topk(const float *router_logits, int *top_idx, float *top_w, int tokens, int n_experts, int k,
                       float routed_scaling);

/* Grouped routed experts for a batch of tokens (no reference twin: the reference runs
 * ql_quant_swiglu_indexed and ql_quant_down_f32_indexed_accum_ordered once per token,
 * RoutedExperts.cpp:80-118).  Every expert's rows are read once per call for all the tokens
 * routed to it.  Route (t, r) has expert id expert_ids[t * k + r]; it belongs to this call when
 * e = id - expert_begin is in [0, n_experts) (expert e's rows start expert_bytes * e past the
 * weight pointer: one expert-parallel shard of experts), and is skipped otherwise.
 *   act[t * k + r][f] = SiLU(Wg[e][f] . x_t) * (Wu[e][f] . x_t), 0 for a skipped route,
 * x_t = x + t * x_stride, act rows ffn_dim floats apart.  Numerics as QL_PATH_TENSOR: each
 * activation row (times a power of two) and each dequantized weight rounded to f16, fp32
 * accumulation on the tensor cores.  Q4_0, Q5_0, Q8_0, Q4_K; rows up to ~3.5 KB and up to 256
 * experts per call run grouped (16 rows per warp in shared memory), others run the per-token
 * indexed launches. */
QL_API int ql_moe_swiglu_grouped(int32_t quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                                 size_t gate_expert_bytes, size_t up_expert_bytes, size_t gate_row_bytes,
                                 size_t up_row_bytes, const float *x, int64_t x_stride, const int *expert_ids,
                                 int expert_begin, int n_experts, float *act, int tokens, int k, int ffn_dim,
                                 int in_dim);
/* out[t][h] += total_t,h with total = fmaf(Wd[e][h] . act[t * k + r], route_weights[t * k + r],
 * total) over t's routes r = 0..k-1 that belong to this call, in route order (the reference
 * combine, kernel.cu:2252-2287); out rows out_stride floats apart.  Same numerics and limits
 * as ql_moe_swiglu_grouped. */
QL_API int ql_moe_down_grouped_accum_ordered(int32_t quant_type, const uint8_t *down_weight, size_t down_expert_bytes,
                                             size_t down_row_bytes, const float *act, const int *expert_ids,
                                             int expert_begin, int n_experts, const float *route_weights,
                                             float *out, int64_t out_stride, int tokens, int k, int hidden,
                                             int ffn_dim);

/* ---- decode attention around the projections (reference kernel.cuh:185-194) ------- */
/* Causal attention with an output gate for the token at position *pos_dev (device int, so a
 * captured launch replays at every step): for query head h (kv head h / (n_heads / kv_heads)),
 *   attn_h = softmax_j((q_h . k_j) / sqrt(head_dim)) . v_j * sigmoid(gate_h),  j = 0..pos,
 * q, gate, attn [n_heads * head_dim]; key_cache / value_cache [max_seq_len][kv_heads][head_dim],
 * bf16 when kv_bf16 != 0, else f32 (launch_full_attention_attend, launch.cu:676-692).  Keys are
 * split over CTAs per KV head (each K/V tile read once for the head's whole query group) and the
 * splits merged by a second launch.  head_dim <= 256. */
QL_API int ql_full_attention_attend(const float *q, const float *gate, const void *key_cache,
                                    const void *value_cache, int kv_bf16, float *attn, int n_heads, int kv_heads,
                                    int head_dim, int max_seq_len, const int *pos_dev);
/* The same for `tokens` queries at positions start_pos .. start_pos + tokens - 1, rows
 * n_heads * head_dim apart (launch_full_attention_attend_batch, launch.cu:694-709). */
QL_API int ql_full_attention_attend_batch(const float *q, const float *gate, const void *key_cache,
                                          const void *value_cache, int kv_bf16, float *attn, int tokens, int n_heads,
                                          int kv_heads, int head_dim, int max_seq_len, int start_pos);

/* ---- opt-in int8 activation path, Q8_1 (reference kernel.cuh:47-52) -------------------
 * Changes numerics (activations rounded to int8 per 32), as in the reference, which keeps it off
 * by default (TensorTool.cpp:159-161).  Bytes of one Q8_1 row of in_dim activations (36 per 32). */
QL_API size_t ql_q8_1_row_bytes(int in_dim);
/* x [m][in_dim] (rows in_dim apart) -> x_q8_1 [m][ql_q8_1_row_bytes(in_dim)]: per 32 activations
 * f16 d = max|x| / 127, f16 sum (sum of x when store_raw_sum, else d * sum q), 32 int8 q; the same
 * bytes as launch_quantize_q8_1 (launch.cu:201-207). */
QL_API int ql_quantize_q8_1(const float *x, uint8_t *x_q8_1, int in_dim, int m, int store_raw_sum);
/* y[out_dim] = W . x for one Q8_1 activation row: integer dot products per 32-element block with
 * the block scales in fp32 (launch_quant_gemv_q8_1, launch.cu:222-245); Q4_K, Q6_K, Q5_0, Q8_0. */
QL_API int ql_quant_gemv_q8_1(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const uint8_t *x_q8_1,
                              float *y, int out_dim, int in_dim);
/* y[m][out_dim] for m Q8_1 activation rows (ql_q8_1_row_bytes(in_dim) apart), the GEMV's per-block
 * formula for every (token, output row), on the integer tensor cores (launch_quant_matmul_q8_1,
 * launch.cu:512-531); Q4_K, Q6_K, Q5_0, Q8_0. */
QL_API int ql_quant_matmul_q8_1(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const uint8_t *x_q8_1,
                                float *y, int out_dim, int in_dim, int m);
/* The reference's packed (MMQ) Q8_1 layout (kernel.cuh:56-61): 144-byte groups of 4 blocks
 * {4 x (f16 d, f16 sum), 4 x 32 int8}, group-major ([group][row]); ql_q8_1_mmq_row_bytes(in_dim)
 * per row.  The quantizer's bytes equal launch_quantize_q8_1_mmq's; the matmul computes
 * ql_quant_matmul_q8_1's result from that layout (Q4_K, Q6_K, as launch_quant_matmul_q8_1_mmq). */
QL_API size_t ql_q8_1_mmq_row_bytes(int in_dim);
QL_API int ql_quantize_q8_1_mmq(const float *x, uint8_t *x_q8_1_mmq, int in_dim, int m, int store_raw_sum);
QL_API int ql_quant_matmul_q8_1_mmq(int32_t quant_type, const uint8_t *weight, size_t row_bytes,
                                    const uint8_t *x_q8_1_mmq, float *y, int out_dim, int in_dim, int m);

/* ---- embedding, dequant, argmax (reference kernel.cuh:141-142, 244-253, 347) ----- */
QL_API int ql_quant_embedding(int32_t quant_type, const int *input, float *output, const uint8_t *table, size_t row_bytes,
                       int hidden_size, int input_size);
/* Whole-tensor dequant to IEEE f16 bits, num_elements a multiple of the block size. */
QL_API int ql_dequantize_to_f16(int32_t quant_type, const uint8_t *src, uint16_t *out, int64_t num_elements);
QL_API int ql_dequantize_q4k_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements);
QL_API int ql_dequantize_q80_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements);
QL_API int ql_dequantize_q50_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements);
QL_API int ql_dequantize_q6k_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements);
QL_API int ql_dequantize_q40_to_f16(const uint8_t *src, uint16_t *out, int64_t num_elements);
/* out_idx[0] = argmax(logits[0..n)), lowest index on ties. */
QL_API int ql_argmax(const float *logits, int n, int *out_idx);

/* Same result as ql_argmax, without ever allocating device memory.  No
 * counterpart in the reference.  For callers that cannot let a library call
 * cudaMalloc: a server whose HBM is owned by its own pool or budgeted once at
 * start-up (weights, KV cache), or code under an allocation ban after start-up.
 * The partials live in a fixed 8 KB array inside the library's device image: n
 * is limited to 16,777,216 (larger n returns QL_EINVAL); calls that overlap on
 * the GPU race on the shared array; the first call on a device performs a
 * one-time set-up (resolving the array's address) and should come before any
 * stream capture; do not use it on a device after cudaDeviceReset. */
QL_API int ql_argmax_noalloc(const float *logits, int n, int *out_idx);

/* ---- fused forms (no reference counterpart; fusions the reference runs as
 *      separate rms_norm / add kernels, kernel.cu:80-84,112-147) ------------------ */
/* y[m*y_stride + o] (=|+=) W[o] . rmsnorm(x[m*x_stride + :]) (+ bias[o]).
 * norm_gamma == NULL skips the norm; bias may be NULL; accumulate != 0 adds into y. */
QL_API int ql_quant_gemv_ex(int32_t quant_type, const uint8_t *weight, size_t row_bytes, const float *x, int64_t x_stride,
                     float *y, int64_t y_stride, int out_dim, int in_dim, int m, const float *norm_gamma, float eps,
                     const float *bias, int accumulate);
/* Fused projections sharing one activation (e.g. q, k and v): the outputs of
 * nsrc (1..3) matrices, stacked by rows, y[m*y_stride + r] for r < sum(rows),
 * with one optional RMSNorm and a stacked bias.  Every source but the last must
 * have a multiple of 32 rows.  w, row_bytes and rows are host arrays of nsrc. */
QL_API int ql_quant_gemv_stacked_ex(int32_t quant_type, int nsrc, const uint8_t *const *weights,
                                    const size_t *row_bytes, const int *rows, const float *x, int64_t x_stride,
                                    float *y, int64_t y_stride, int in_dim, int m, const float *norm_gamma, float eps,
                                    const float *bias);
/* act[m*act_stride + f] = SiLU(Wg[f] . n(x_m)) * (Wu[f] . n(x_m)), n = optional RMSNorm. */
QL_API int ql_quant_swiglu_ex(int32_t quant_type, const uint8_t *gate_weight, const uint8_t *up_weight,
                       size_t gate_row_bytes, size_t up_row_bytes, const float *x, int64_t x_stride, float *act,
                       int64_t act_stride, int ffn_dim, int in_dim, int m, const float *norm_gamma, float eps);
/* y = x * rsqrt(mean(x^2) + eps) * gamma (gamma f32, may be NULL), rows x hidden. */
QL_API int ql_rms_norm_f32(const float *x, float *y, const float *gamma, int rows, int hidden, float eps);

/* ---- GGUF loader (reference GgufFile, src/format/gguf/GgufFile.cpp:152-250, and
 *      MF::validate, src/format/MF.cpp:43-84) --------------------------------------
 * ql_gguf_open maps a GGUF v2/v3 file read-only and parses its metadata and tensor table
 * (QL_EINVAL with a message on any format error; every length is checked against the file).
 * Tensor shapes are reported outermost-first (the file stores dims innermost-first); data
 * points into the mapping (host memory, valid until ql_gguf_close); nbytes follows the ggml
 * block traits.  The data section starts at the end of the tensor table rounded up to
 * general.alignment (default 32).  ql_gguf_find_tensor returns the index or -1.
 * ql_gguf_metadata_type returns the GGUF value type (0..12) or -1 when the key is absent;
 * integer, bool and float values convert between the int and float getters.
 * ql_gguf_validate applies MF::validate's container checks (tensors present, names non-empty
 * and unique, shapes non-empty with positive dims, data present) and admits the types this
 * library computes with: F32, F16, BF16, Q4_0, Q4_K, Q5_0, Q6_K, Q8_0 (the reference's
 * validator leaves Q4_0 out although its parser reads it). */
QL_API int ql_gguf_open(const char *path, void **file);
QL_API int ql_gguf_close(void *file);
QL_API int ql_gguf_version(void *file);
QL_API int64_t ql_gguf_tensor_count(void *file);
QL_API int64_t ql_gguf_find_tensor(void *file, const char *name);
QL_API int ql_gguf_tensor_info(void *file, int64_t index, const char **name, int32_t *quant_type, int32_t *n_dims,
                               int64_t *shape /* [8] */, const uint8_t **data, size_t *nbytes);
QL_API int ql_gguf_metadata_type(void *file, const char *key);
QL_API int ql_gguf_metadata_int(void *file, const char *key, int64_t *out);
QL_API int ql_gguf_metadata_float(void *file, const char *key, double *out);
QL_API int ql_gguf_metadata_string(void *file, const char *key, const char **out);
QL_API int64_t ql_gguf_metadata_array_len(void *file, const char *key);
QL_API int ql_gguf_metadata_array_int(void *file, const char *key, int64_t index, int64_t *out);
QL_API int ql_gguf_metadata_array_float(void *file, const char *key, int64_t index, double *out);
QL_API int ql_gguf_metadata_array_string(void *file, const char *key, int64_t index, const char **out);
QL_API int ql_gguf_validate(void *file);
/* Weight upload (reference CudaWeightPool::cached_weight, CudaWeightPool.cpp:119-175, which
 * uploads the raw blocks unchanged): copies rows [row0, row0 + nrows) of a host matrix whose
 * rows are row_bytes apart, bytes [byte0, byte0 + nbytes_per_row) of each row, to dst (device,
 * rows packed nbytes_per_row apart), as one pitched copy on the current stream.  A whole matrix
 * is byte0 = 0, nbytes_per_row = row_bytes; a column-parallel shard a row range; a row-parallel
 * shard whole blocks of every row (byte0 and nbytes_per_row multiples of the block bytes).  The
 * kernels read the raw GGUF layout, so no repack is needed.  Pinned host memory makes the copy
 * asynchronous; pageable memory makes it synchronous. */
QL_API int ql_weight_upload(const uint8_t *host, size_t row_bytes, int64_t row0, int64_t nrows, size_t byte0,
                            size_t nbytes_per_row, uint8_t *dst);

/* ---- synthetic weights (benchmarks; no reference counterpart) -------------------- */
/* dst[rows x row_bytes] = quantize(N(0, std) with seed), generated on the device. */
QL_API int ql_synth_quantized(int32_t quant_type, uint64_t seed, int64_t rows, int in_dim, float std, uint8_t *dst);

/* ---- introspection ------------------------------------------------------------- */
/* Bytes per row of `in_dim` elements of `quant_type` (0 if not a block multiple). */
QL_API size_t ql_row_bytes(int32_t quant_type, int in_dim);
/* Number of kernel launches the last call on this thread issued. */
QL_API int ql_last_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* QLINEAR_B200_H */
