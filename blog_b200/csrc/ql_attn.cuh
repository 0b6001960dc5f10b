// Causal gated decode attention over a KV cache (ql_attn.cu): launch arguments.
#pragma once
#include <cuda_runtime.h>
#include <cstddef>

namespace ql {

struct AttnArgs {
    const float *q;            // [tokens][n_heads * head_dim]
    const float *gate;         // [tokens][n_heads * head_dim]
    const void *key_cache;     // [max_seq_len][kv_heads][head_dim], f32 or bf16
    const void *value_cache;
    float *attn;               // [tokens][n_heads * head_dim]
    const int *pos_dev;        // single token: position on the device (nullptr: start_pos + token)
    int start_pos;
    int tokens, n_heads, kv_heads, head_dim, max_seq_len;
    int splits;                // key splits per (token, KV head)
    float *part_ml;            // [tokens][n_heads][splits][2]: running max, running sum
    float *part_acc;           // [tokens][n_heads][splits][head_dim]
};

size_t attn_smem_bytes(int group, int head_dim);
int attn_tile();
int attn_ctas_per_sm(int head_dim);  // resident split CTAs per SM
int attn_max_splits();
cudaError_t attn_launch(const AttnArgs &a, bool kv_bf16, cudaStream_t s);

}  // namespace ql
