// ql_gemm.cuh -- prefill GEMM on the 5th-generation tensor cores (tcgen05).
//
// y[m][n] = sum_k x[m][k] * W(n, k) for a GGUF Q4_K weight W [N][K] and fp32
// activations x [M][K] (reference quant_matmul_kernel, kernel.cu:1253-1279,
// and the dequantize-then-GEMM prefill path, TensorTool.cpp:127-144).
//
// Two launches:
//  1. xprep: each activation row (times the RMSNorm weight, when a norm is
//     fused) is scaled by a power of two s_m (its largest
//     magnitude lands in [2^13, 2^14), so no row overflows or loses precision
//     to f16 subnormals), rounded to f16 and written K-major with a fixed
//     permutation inside every 8-element group (the order in which the
//     dequantizer below emits nibbles: positions 0..7 hold elements
//     0,2,1,3,4,6,5,7).  1/s_m is kept per row.
//  2. qgemm: one CTA per 128 x 256 accumulator tile; when the grid would
//     underfill the GPU, the K range is split over a thread-block cluster of up
//     to 8 CTAs whose partial tiles are summed through distributed shared memory
//     in a fixed order (deterministic).  Warp roles, 320 threads:
//       warp 0   -- one thread issues TMA: raw Q4_K super-blocks {144 B, 1, 256 rows}
//                   and 128 x 64 f16 activation tiles (128-byte swizzle);
//       warp 1   -- allocates 256 TMEM columns; one thread issues
//                   tcgen05.mma.kind::f16 (M 128, N 256, K 16; fp32 accumulate in TMEM)
//                   and tcgen05.commit to release ring slots;
//       warps 2-9 -- dequantize: thread r owns weight row r of the tile and writes
//                   its 64 f16 values per chunk straight into the canonical
//                   K-major 128-byte-swizzled layout the MMA reads; then the same
//                   warps drain TMEM (tcgen05.ld) in the epilogue.
//     Dequantized weights: f16(d*sc*q - dmin*m) computed in f16 arithmetic
//     (exact nibble, one rounding of d*sc and dmin*m, one rounding of the
//     fused multiply-add), i.e. within about one f16 ulp of the reference's
//     dequantize_q4k_to_f16 (kernel.cu:954-975).
#pragma once

#include <cudaTypedefs.h>

#include "ql_common.cuh"

namespace ql {

constexpr int kGemmBM = 128;   // output rows (tokens) per CTA tile = MMA M
constexpr int kGemmBN = 256;   // output columns (weight rows) per CTA tile = MMA N
constexpr int kGemmBK = 64;    // K per pipeline chunk: one 128-byte swizzle row of f16
constexpr int kGemmNA = 4;     // activation chunk ring
constexpr int kGemmNB = 2;     // dequantized weight chunk ring
constexpr int kGemmNR = 2;     // raw super-block ring
constexpr int kGemmDqWarps = 16;                         // dequantizer warps (8 or 16)
constexpr int kGemmThreads = 64 + 32 * kGemmDqWarps;
constexpr int kGemmABytes = kGemmBM * kGemmBK * 2;  // 16 KB
constexpr int kGemmBBytes = kGemmBN * kGemmBK * 2;  // 32 KB
constexpr int kGemmRBytes = kGemmBN * 144;          // 36 KB
constexpr int kGemmSmem = kGemmNA * kGemmABytes + kGemmNB * kGemmBBytes + kGemmNR * kGemmRBytes + 256 + 1024;
constexpr int kGemmTileFloats = kGemmBM * kGemmBN;
constexpr int kGemmRedPitch = kGemmBN * 4 + 16;  // bytes per row of the epilogue's fp32 tile in shared memory
constexpr int kGemmMaxSplit = 8;

// Epilogues: plain (scale, optional bias, optional accumulate) over 256-column
// tiles of one or several stacked weight sources, or SwiGLU over 128-column
// tiles of a gate/up pair (the MMA's 256 columns are 128 gate + 128 up rows).
enum GemmEpi : int { kGemmPlain = 1, kGemmSwiglu = 2 };

struct GemmArgs {
    CUtensorMap tm_x;      // f16 [M][K] activations (permuted), box {64, 128}, 128-byte swizzle
    CUtensorMap tm_w[3];   // Q4_K sources viewed as uint8 {144, K/256, rows}; box {144, 1, 256} (plain)
                           // or {144, 1, 128} (SwiGLU: tm_w[0] gate, tm_w[1] up)
    int src_end[3];        // plain: cumulative row ends of the stacked sources (multiples of 256 but the last)
    const float *rinv;     // [M] 1/s_m (times the row's RMSNorm factor when one is fused)
    const float *bias;     // [N] or null (plain)
    float *y;              // [M][y_stride]
    int64_t y_stride;
    int accumulate;        // plain: y += result
    int vec;               // y, y_stride and bias allow 16-byte stores
    int M, N, K;           // N = output columns (plain: all sources' rows; SwiGLU: FFN rows)
    int nsb;               // K / 256
    int ksplit;            // K ranges per output tile = cluster size along z (<= 8)
    int *err;
    AmaxOut amax;          // fused greedy argmax over the output columns (plain; amax.amax null = off)
    int fmt;               // kQ4_K (tm_w 3-D views) or kQ4_0 (tm_w 2-D byte views {row_bytes, rows},
                           // box {144, 256 or 128}: 8 blocks per 256 inputs)
};

bool gemv_pdl_enabled();  // programmatic dependent launch (always on)
cudaError_t gemm_xprep_launch(const float *x, int64_t x_stride, const float *gamma, float eps, __half *xh,
                              float *rinv, int M, int K, cudaStream_t s);
cudaError_t gemm_q4k_launch(const GemmArgs &a, int epi, cudaStream_t s);
// Prefill GEMM with the weights as the MMA's M side (A in tensor memory): tiles of 128 weight rows
// (SwiGLU: 64 + 64) x ntok tokens (128 or 256); tm_w boxes of 128 (SwiGLU: 64) rows, tm_x boxes
// {64, ntok}; no K split, no fused argmax.
int gemm_ta_tokens(int M, int row_tiles, int sms);
cudaError_t gemm_ta_launch(const GemmArgs &a, int epi, int ntok, cudaStream_t s);

}  // namespace ql
