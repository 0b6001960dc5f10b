// Grouped routed experts (ql_moe.cu): launch arguments and host entry points.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace ql {

struct MoeArgs {
    const uint8_t *w[2];  // SwiGLU: gate, up; down: the down matrix (w[1] unused)
    size_t eb[2];         // bytes between consecutive experts
    size_t rb[2];         // bytes per weight row
    int row_pitch;        // shared-memory bytes per staged row (moe_row_pitch)
    int rows;             // rows per expert (ffn_dim for SwiGLU, hidden for down)
    int K;                // input dimension
    const uint4 *xq;      // activations from moe_xprep: two f16 limbs, K / 4 words per row
    const float *rinv;    // per activation row: 1 / its power-of-two scale
    const float *bsum;    // per activation row: K / 32 block sums of the scaled row
    const int *ids;       // [npairs] expert id of route (t, r) at t * k + r
    const int *bucket_off;  // [n_experts + 2] from moe_bucket: expert e's pairs are bucket[off[e] .. off[e + 1])
    const int *bucket;      // [npairs] pair indices t * k + r grouped by expert (bucket n_experts: skipped)
    int e_begin;          // expert id of this call's first expert
    int n_experts;        // experts this call holds (packed eb apart from w)
    int npairs;           // tokens * k
    int k;                // routes per token
    float *y;             // SwiGLU: act [(t, r)][rows]; down: per-pair rows [(t, r)][rows]
    int64_t y_stride;
    int *err;
};

int moe_row_pitch(size_t row_bytes);
int moe_max_row_pitch();
cudaError_t moe_grouped_launch(const MoeArgs &a, int fmt, bool swiglu, cudaStream_t s);
cudaError_t moe_xprep_launch(const float *x, int64_t x_stride, uint4 *xq, float *rinv, float *bsum, int rows, int K,
                             cudaStream_t s);
cudaError_t moe_bucket_launch(const int *ids, int npairs, int e_begin, int n_experts, int *off, int *list,
                              cudaStream_t s);
int moe_max_experts();
cudaError_t moe_local_ids_launch(const int *ids, int e_begin, int n_experts, int *out, int n, cudaStream_t s);
cudaError_t moe_combine_launch(const float *y, const int *ids, int e_begin, int n_experts, const float *rw,
                               float *out, int64_t out_stride, int tokens, int k, int H, cudaStream_t s);

}  // namespace ql
