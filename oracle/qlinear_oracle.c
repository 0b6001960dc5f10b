/*
 * qlinear_oracle.c -- CPU ORACLE (test infrastructure, not product code).
 *
 * A plain-C restatement of the block-quantized linear path of the local-llm
 * engine in allenzhang61/blog (AI/codes/local-llm).  The reference has no CPU
 * implementation of this path (its only device is CUDA,
 * src/backend/common.h:8), so this file restates the arithmetic of its CUDA
 * kernels in C.  It is used only by tests/, by __graft_entry__.smoke() as the
 * checker, and by bench.py's cpu_baseline leg / reference arm as the timed CPU
 * baseline.  Nothing in the product library links or calls it.
 *
 * Parity pins (see tests/test_oracle_golden.py):
 *   - the hand-built known-answer blocks of test/LaunchAddTest.cpp
 *     (Q8_0 matmul :186-240, Q4_K w=14 :711-756, Q6_K w=6 :758-803,
 *      MoE down / SwiGLU fixtures :301-677);
 *   - gguf-py 0.19.0 (third-party, pinned in tests/golden/make_golden.py)
 *     dequantize/quantize vectors for Q8_0/Q4_0/Q5_0/Q4_K/Q6_K;
 *   - on a GPU, the reference's own CUDA kernels compiled from the reference
 *     sources into oracle/_ref (tests/test_ref_cuda_pin.py): dequant and the
 *     lane-ordered GEMV must agree bit for bit.
 * Q4_0 arithmetic does not exist in the reference (it is parsed,
 * GgufFile.cpp:40, but never computed): its pin is gguf-py only.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* GGML type codes == reference DType values (src/tensor/TensorCommon.h:15-33). */
enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

/* ------------------------------------------------------------------------ */
/* f16 <-> f32, bit level (restates test/LaunchAddTest.cpp:38-65 for decode; */
/* encode is IEEE round-to-nearest-even, the rounding of __float2half).      */
/* ------------------------------------------------------------------------ */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x03ffu;
    uint32_t out;
    if (exp == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            exp = 1;
            while ((mant & 0x0400u) == 0) { mant <<= 1; --exp; }
            mant &= 0x03ffu;
            out = sign | ((exp + 127 - 15) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        out = sign | 0x7f800000u | (mant << 13);
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    }
    float v;
    memcpy(&v, &out, 4);
    return v;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf / nan */
        if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (absx < 0x38800000u) { /* result is subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign;           /* < 2^-25 -> 0 */
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 + (113 - e) */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 112;
    uint32_t m = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    return (uint16_t)(sign | q);
}

static inline float h2f(const uint8_t *p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
static inline void put_h(uint8_t *p, uint16_t h) { p[0] = (uint8_t)(h & 0xff); p[1] = (uint8_t)(h >> 8); }

/* ------------------------------------------------------------------------ */
/* Block traits (GgufFile.cpp:35-55).                                       */
/* ------------------------------------------------------------------------ */
int orc_block_elems(int t) {
    switch (t) {
    case T_F32: case T_F16: return 1;
    case T_Q4_0: case T_Q5_0: case T_Q8_0: return 32;
    case T_Q4_K: case T_Q6_K: return 256;
    default: return 0;
    }
}
int orc_block_bytes(int t) {
    switch (t) {
    case T_F32: return 4;
    case T_F16: return 2;
    case T_Q4_0: return 18;
    case T_Q5_0: return 22;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q6_K: return 210;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* Element decode: restates kernel.cu:913-921 (q4k_scale_min) and           */
/* kernel.cu:1090-1185 (q4k_at, q6k_at, q50_at, q80_at).  Q4_0 is new: GGUF  */
/* block {f16 d, u8 qs[16]}, element i<16 = low nibble of qs[i], element    */
/* i>=16 = high nibble of qs[i-16], value d*(q-8).                          */
/* ------------------------------------------------------------------------ */
static inline void q4k_scale_min(int j, const uint8_t *s, uint8_t *sc, uint8_t *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

static inline float q4k_at(const uint8_t *row, int idx) {
    const uint8_t *b = row + (size_t)(idx >> 8) * 144;
    int in = idx & 255, j = in >> 5, inner = in & 31;
    float d = h2f(b), dmin = h2f(b + 2);
    uint8_t sc, m;
    q4k_scale_min(j, b + 4, &sc, &m);
    uint8_t q = b[16 + (j >> 1) * 32 + inner];
    int nib = (j & 1) ? (q >> 4) : (q & 0x0F);
    /* kernel.cu:1118: d * sc * nib - dmin * m (every product is exact in fp32) */
    return d * (float)sc * (float)nib - dmin * (float)m;
}

static inline float q6k_at(const uint8_t *row, int idx) {
    const uint8_t *b = row + (size_t)(idx >> 8) * 210;
    int in = idx & 255, half = in >> 7, n = half * 128, within = in & 127;
    int grp = within >> 5, l = within & 31, is = l / 16;
    const uint8_t *ql = b + n / 2, *qh = b + 128 + n / 4;
    const int8_t *sc = (const int8_t *)(b + 192) + n / 16;
    float d = h2f(b + 208);
    int q, si;
    if (grp == 0) { q = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32; si = is + 0; }
    else if (grp == 1) { q = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32; si = is + 2; }
    else if (grp == 2) { q = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32; si = is + 4; }
    else { q = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32; si = is + 6; }
    return d * (float)sc[si] * (float)q;
}

static inline float q50_at(const uint8_t *row, int idx) {
    const uint8_t *b = row + (size_t)(idx >> 5) * 22;
    int in = idx & 31;
    float d = h2f(b);
    uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
    const uint8_t *qs = b + 6;
    int q;
    if (in < 16) q = (qs[in] & 0x0F) | (((qh >> in) & 1) << 4);
    else q = (qs[in - 16] >> 4) | (((qh >> in) & 1) << 4);
    return d * (float)(q - 16);
}

static inline float q80_at(const uint8_t *row, int idx) {
    const uint8_t *b = row + (size_t)(idx >> 5) * 34;
    return h2f(b) * (float)(int8_t)b[2 + (idx & 31)];
}

static inline float q40_at(const uint8_t *row, int idx) {
    const uint8_t *b = row + (size_t)(idx >> 5) * 18;
    int in = idx & 31;
    int q = (in < 16) ? (b[2 + in] & 0x0F) : (b[2 + in - 16] >> 4);
    return h2f(b) * (float)(q - 8);
}

static inline float w_at(int t, const uint8_t *row, int idx) {
    switch (t) {
    case T_Q4_K: return q4k_at(row, idx);
    case T_Q6_K: return q6k_at(row, idx);
    case T_Q5_0: return q50_at(row, idx);
    case T_Q8_0: return q80_at(row, idx);
    case T_Q4_0: return q40_at(row, idx);
    case T_F16: return h2f(row + 2 * (size_t)idx);
    case T_F32: { float v; memcpy(&v, row + 4 * (size_t)idx, 4); return v; }
    default: return NAN;
    }
}

/* Dequantize `rows` rows of K elements each to fp32. */
int orc_dequant_rows_f32(int t, const uint8_t *w, size_t row_bytes, int64_t rows, int K, float *out) {
    if (orc_block_elems(t) == 0 || K % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int k = 0; k < K; ++k) out[r * K + k] = w_at(t, w + r * row_bytes, k);
    return 0;
}

/* Whole-tensor dequant to f16 bits: restates dequantize_*_to_f16_kernel
 * (kernel.cu:954-1063): value in fp32, then one round-to-nearest-even. */
int orc_dequant_f16(int t, const uint8_t *src, int64_t n, uint16_t *out) {
    int be = orc_block_elems(t), bb = orc_block_bytes(t);
    if (be == 0 || n % be != 0) return 1;
    int64_t nb = n / be;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; ++b)
        for (int i = 0; i < be; ++i) out[b * be + i] = orc_f32_to_f16(w_at(t, src + b * bb, i));
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Dot products.  order 0 restates the summation order of the reference's    */
/* warp-per-row kernels (kernel.cu:1191-1215 and siblings): lane l sums       */
/* fmaf(w[k], x[k], acc) for k = l, l+32, ... ; then the __shfl_down_sync     */
/* tree with offsets 16, 8, 4, 2, 1; lane 0 holds the result.  order 1 is a   */
/* double-precision accumulation rounded once (an accuracy reference).        */
/* ------------------------------------------------------------------------ */
static float dot_ref_order(int t, const uint8_t *row, const float *x, int K) {
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int k = l; k < K; k += 32) acc = fmaf(w_at(t, row, k), x[k], acc);
        lane[l] = acc;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + ((l + off < 32) ? lane[l + off] : lane[l]);
        memcpy(lane, nxt, sizeof(lane));
    }
    return lane[0];
}

static float dot_f64(int t, const uint8_t *row, const float *x, int K) {
    double acc = 0.0;
    for (int k = 0; k < K; ++k) acc += (double)w_at(t, row, k) * (double)x[k];
    return (float)acc;
}

static inline float dot_any(int order, int t, const uint8_t *row, const float *x, int K) {
    return order == 0 ? dot_ref_order(t, row, x, K) : dot_f64(t, row, x, K);
}

/* y[m][o] = W[o,:] . x[m,:]   (launch_quant_gemv / launch_quant_matmul, kernel.cuh:34-43) */
int orc_gemv(int t, const uint8_t *w, size_t row_bytes, const float *x, float *y, int N, int K, int M, int order) {
    if (orc_block_elems(t) == 0 || K % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < N; ++o)
        for (int m = 0; m < M; ++m)
            y[(size_t)m * N + o] = dot_any(order, t, w + (size_t)o * row_bytes, x + (size_t)m * K, K);
    return 0;
}

/* y[o] += W[o,:] . x   (quant_gemv_add_kernel, kernel.cu:1222-1244) */
int orc_gemv_add(int t, const uint8_t *w, size_t row_bytes, const float *x, float *y, int N, int K, int order) {
    if (orc_block_elems(t) == 0 || K % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static)
    for (int o = 0; o < N; ++o) y[o] += dot_any(order, t, w + (size_t)o * row_bytes, x, K);
    return 0;
}

/* act[f] = SiLU(Wg[f].x) * (Wu[f].x), SiLU(g) = g / (1 + exp(-g))
 * (quant_swiglu_kernel, kernel.cu:1288-1328). */
int orc_swiglu(int t, const uint8_t *gw, const uint8_t *uw, size_t grb, size_t urb, const float *x,
               float *act, int F, int K, int order) {
    if (orc_block_elems(t) == 0 || K % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static)
    for (int f = 0; f < F; ++f) {
        float g = dot_any(order, t, gw + (size_t)f * grb, x, K);
        float u = dot_any(order, t, uw + (size_t)f * urb, x, K);
        act[f] = g / (1.0f + expf(-g)) * u;
    }
    return 0;
}

/* Indexed SwiGLU over k routes (quant_swiglu_indexed_kernel, kernel.cu:1339-1385):
 * expert e = ids[r]; e < 0 writes 0 for the whole route. */
int orc_swiglu_indexed(int t, const uint8_t *gw, const uint8_t *uw, size_t g_eb, size_t u_eb, size_t grb,
                       size_t urb, const float *x, const int *ids, float *act, int k, int F, int K, int order) {
    if (orc_block_elems(t) == 0 || K % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static) collapse(2)
    for (int r = 0; r < k; ++r)
        for (int f = 0; f < F; ++f) {
            int e = ids[r];
            if (e < 0) { act[(size_t)r * F + f] = 0.0f; continue; }
            float g = dot_any(order, t, gw + (size_t)e * g_eb + (size_t)f * grb, x, K);
            float u = dot_any(order, t, uw + (size_t)e * u_eb + (size_t)f * urb, x, K);
            act[(size_t)r * F + f] = g / (1.0f + expf(-g)) * u;
        }
    return 0;
}

/* Ordered routed down + combine (quant_down_f32_indexed_accum_ordered_kernel,
 * kernel.cu:2252-2287): total = fmaf(dot(Wd[e_r][h], act[r]), w[r], total) in
 * route order, skipping e_r < 0; then out[h] += total. */
int orc_down_indexed_ordered(int t, const uint8_t *dw, size_t d_eb, size_t drb, const float *act, const int *ids,
                             const float *rw, float *out, int k, int H, int F, int order) {
    if (orc_block_elems(t) == 0 || F % orc_block_elems(t) != 0) return 1;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; ++h) {
        float total = 0.0f;
        for (int r = 0; r < k; ++r) {
            int e = ids[r];
            if (e < 0) continue;
            float acc = dot_any(order, t, dw + (size_t)e * d_eb + (size_t)h * drb, act + (size_t)r * F, F);
            total = fmaf(acc, rw[r], total);
        }
        out[h] += total;
    }
    return 0;
}

/* Router: softmax over all experts, top-k by logit scanning e ascending with
 * strict '>', non-finite logits treated as -inf, weight = exp(best-max)/denom *
 * routed_scaling (moe_router_topk_kernel, kernel.cu:3463-3511).  The reference
 * uses the __expf intrinsic; this restatement uses expf, so weights agree to a
 * few ulp while indices agree exactly. */
int orc_router_topk(const float *logits, int *top_idx, float *top_w, int T, int E, int k, float scale) {
    if (E > 64 || k > E || k <= 0) return 1;
    for (int tok = 0; tok < T; ++tok) {
        const float *lg = logits + (size_t)tok * E;
        float maxv = -INFINITY;
        for (int e = 0; e < E; ++e) { float v = isfinite(lg[e]) ? lg[e] : -INFINITY; maxv = fmaxf(maxv, v); }
        float denom = 0.0f;
        if (isfinite(maxv))
            for (int e = 0; e < E; ++e) { float v = isfinite(lg[e]) ? lg[e] : -INFINITY; denom += expf(v - maxv); }
        int used[64] = {0};
        for (int r = 0; r < k; ++r) {
            float best = -INFINITY;
            int be = -1;
            for (int e = 0; e < E; ++e) {
                if (used[e]) continue;
                float v = isfinite(lg[e]) ? lg[e] : -INFINITY;
                if (v > best) { best = v; be = e; }
            }
            if (be < 0) be = r < E ? r : 0;
            used[be] = 1;
            float prob = (denom > 0.0f && isfinite(best)) ? expf(best - maxv) / denom : 0.0f;
            top_idx[(size_t)tok * k + r] = be;
            top_w[(size_t)tok * k + r] = prob * scale;
        }
    }
    return 0;
}

/* argmax, lowest index on ties (argmax_partial/final_kernel, kernel.cu:3531-3592;
 * host Sampler strict '>' rule, Sampler.cpp:24-50).  NaN never wins. */
/* Causal decode attention with an output gate (full_attn_attend_head, kernel.cu:355-430, one
 * head per block): for query head h of token t at position pos, kv head kh = h / (n_heads /
 * kv_heads), scores s_j = (q_h . k_j) / sqrt(head_dim) over keys j = 0..pos, p = softmax(s),
 * out_h = (sum_j p_j v_j) * sigmoid(gate_h).  The cache is [max_seq][kv_heads][head_dim], f32 or
 * bf16 (kv_bf16: 16-bit values, the top half of an f32).  The reference keeps an online softmax
 * in f32 with __expf; this restatement evaluates the softmax directly in double. */
static inline double kv_at(const void *cache, int bf16, size_t i) {
    if (bf16) {
        const uint32_t b = (uint32_t)((const uint16_t *)cache)[i] << 16;
        float f;
        memcpy(&f, &b, 4);
        return (double)f;
    }
    return (double)((const float *)cache)[i];
}
int orc_attention_attend(const float *q, const float *gate, const void *kc, const void *vc, int kv_bf16, float *out,
                         int tokens, int n_heads, int kv_heads, int head_dim, int start_pos) {
    if (n_heads <= 0 || kv_heads <= 0 || n_heads % kv_heads || head_dim <= 0 || start_pos < 0) return 1;
    const int group = n_heads / kv_heads;
    const double scale = 1.0 / sqrt((double)head_dim);
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < tokens; ++t)
        for (int h = 0; h < n_heads; ++h) {
            const int n_keys = start_pos + t + 1, kh = h / group;
            const float *qh = q + ((size_t)t * n_heads + h) * head_dim;
            double *s = (double *)malloc(sizeof(double) * (size_t)n_keys);
            double mx = -INFINITY, den = 0.0;
            for (int j = 0; j < n_keys; ++j) {
                double dot = 0.0;
                for (int d = 0; d < head_dim; ++d)
                    dot += (double)qh[d] * kv_at(kc, kv_bf16, ((size_t)j * kv_heads + kh) * head_dim + d);
                s[j] = dot * scale;
                if (s[j] > mx) mx = s[j];
            }
            for (int j = 0; j < n_keys; ++j) {
                s[j] = exp(s[j] - mx);
                den += s[j];
            }
            for (int d = 0; d < head_dim; ++d) {
                double acc = 0.0;
                for (int j = 0; j < n_keys; ++j)
                    acc += s[j] * kv_at(vc, kv_bf16, ((size_t)j * kv_heads + kh) * head_dim + d);
                const size_t o = ((size_t)t * n_heads + h) * head_dim + d;
                out[o] = (float)(acc / den / (1.0 + exp(-(double)gate[o])));
            }
            free(s);
        }
    return 0;
}

/* Q8_1 activation blocks (quantize_q8_1_kernel, kernel.cu:1679-1720): per 32 activations (zeros
 * past in_dim), d = max|x| / 127, q = round-half-even(x * (1 / d)) clamped to +-127, f16 d, f16 sum
 * (the warp-tree sum of x when store_raw_sum, else d * sum q), 32 x int8.  The tree adds lane
 * l + 16, then + 8, + 4, + 2, + 1 into lane l; lane 0 holds the block sum. */
int orc_quantize_q8_1(const float *x, uint8_t *out, int in_dim, int m, int store_raw_sum) {
    if (in_dim <= 0 || m < 0) return 1;
    const int bpr = (in_dim + 31) / 32;
    for (int r = 0; r < m; ++r)
        for (int b = 0; b < bpr; ++b) {
            float v[32], t[32];
            float amax = 0.0f;
            for (int l = 0; l < 32; ++l) {
                const int k = b * 32 + l;
                v[l] = k < in_dim ? x[(size_t)r * in_dim + k] : 0.0f;
                t[l] = v[l];
                amax = fmaxf(amax, fabsf(v[l]));
            }
            const float d = amax > 0.0f ? amax / 127.0f : 0.0f;
            const float id = d > 0.0f ? 1.0f / d : 0.0f;
            for (int o = 16; o > 0; o >>= 1)
                for (int l = 0; l < o; ++l) t[l] = t[l] + t[l + o];
            uint8_t *dst = out + ((size_t)r * bpr + b) * 36;
            int qsum = 0;
            for (int l = 0; l < 32; ++l) {
                const float p = v[l] * id;
                int q = (int)lrintf(p);
                q = q < -127 ? -127 : q > 127 ? 127 : q;
                qsum += q;
                dst[4 + l] = (uint8_t)(int8_t)q;
            }
            put_h(dst, orc_f32_to_f16(d));
            put_h(dst + 2, orc_f32_to_f16(store_raw_sum ? t[0] : d * (float)qsum));
        }
    return 0;
}

/* GEMV against one Q8_1 activation row (quant_gemv_q8_1_kernel, kernel.cu:1767-1865), per block b
 * in order: Q4_K acc = fmaf(d sc dx, qdot, acc) - dmin m sum_x; Q6_K acc = fmaf(d dx, s0 qdot_lo +
 * s1 qdot_hi, acc); Q5_0 / Q8_0 acc += w_k * (dx q_k) per element (the reference's float form). */
int orc_gemv_q8_1(int t, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int N, int K) {
    if (t != 12 && t != 14 && t != 6 && t != 8) return 1;
    const int bpr = (K + 31) / 32;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const uint8_t *row = w + (size_t)n * rb;
        float acc = 0.0f;
        for (int b = 0; b < bpr; ++b) {
            const uint8_t *xb = xq + (size_t)b * 36;
            const float dx = h2f(xb), sx = h2f(xb + 2);
            const int8_t *qx = (const int8_t *)(xb + 4);
            if (t == 12) {
                const uint8_t *base = row + (size_t)(b >> 3) * 144;
                const int j = b & 7;
                int dot = 0;
                for (int l = 0; l < 32; ++l) {
                    const uint8_t pk = base[16 + (j >> 1) * 32 + l];
                    dot += ((j & 1) ? (pk >> 4) : (pk & 15)) * qx[l];
                }
                uint8_t sc, mn;
                q4k_scale_min(j, base + 4, &sc, &mn);
                acc = fmaf(h2f(base) * (float)sc * dx, (float)dot, acc);
                acc -= h2f(base + 2) * (float)mn * sx;
            } else if (t == 14) {
                const uint8_t *base = row + (size_t)(b >> 3) * 210;
                const int sub = b & 7, hf = sub >> 2, grp = sub & 3;
                const uint8_t *ql = base + 64 * hf, *qh = base + 128 + 32 * hf;
                const int8_t *sc = (const int8_t *)(base + 192) + 8 * hf;
                int d0 = 0, d1 = 0;
                for (int l = 0; l < 32; ++l) {
                    const int lo = (grp & 1) ? ql[l + 32] : ql[l];
                    const int q = (((grp >> 1) ? (lo >> 4) : (lo & 15)) | (((qh[l] >> (2 * grp)) & 3) << 4)) - 32;
                    if (l < 16) d0 += q * qx[l];
                    else d1 += q * qx[l];
                }
                acc = fmaf(h2f(base + 208) * dx, (float)sc[2 * grp] * (float)d0 + (float)sc[2 * grp + 1] * (float)d1,
                           acc);
            } else {
                for (int l = 0; l < 32; ++l) {
                    const int k = b * 32 + l;
                    if (k >= K) break;
                    const float wv = t == 6 ? q50_at(row, k) : q80_at(row, k);
                    acc = fmaf(wv, dx * (float)qx[l], acc);
                }
            }
        }
        y[n] = acc;
    }
    return 0;
}

int orc_argmax(const float *v, int n) {
    int bi = 0;
    float bv = -INFINITY;
    for (int i = 0; i < n; ++i)
        if (v[i] > bv) { bv = v[i]; bi = i; }
    return bi;
}

/* RMSNorm y = x * rsqrt(mean(x^2) + eps) * gamma (rms_norm_kernel, kernel.cu:112-147),
 * accumulated in double. */
void orc_rmsnorm(const float *x, float *y, const float *gamma, int rows, int H, float eps) {
    for (int r = 0; r < rows; ++r) {
        double ss = 0.0;
        for (int j = 0; j < H; ++j) ss += (double)x[(size_t)r * H + j] * x[(size_t)r * H + j];
        float inv = (float)(1.0 / sqrt(ss / H + (double)eps));
        for (int j = 0; j < H; ++j) y[(size_t)r * H + j] = x[(size_t)r * H + j] * inv * (gamma ? gamma[j] : 1.0f);
    }
}

/* Quantized embedding rows (quant_embedding_kernel, kernel.cu:2677-2693). */
int orc_embedding(int t, const int *ids, float *out, const uint8_t *table, size_t row_bytes, int H, int T) {
    if (orc_block_elems(t) == 0 || H % orc_block_elems(t) != 0) return 1;
    for (int i = 0; i < T; ++i)
        for (int k = 0; k < H; ++k) out[(size_t)i * H + k] = w_at(t, table + (size_t)ids[i] * row_bytes, k);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Quantizers (float -> GGUF blocks).  The reference only consumes GGUF      */
/* files, so these are not a restatement of it.  Q8_0 / Q4_0 / Q5_0 follow   */
/* the published ggml reference quantizers (as restated by gguf-py 0.19.0    */
/* quants.py:220-330,378-393; checked bit for bit in the tests).  Q4_K uses  */
/* this build's own min/max fit (gguf-py has no Q4_K quantizer).             */
/* ------------------------------------------------------------------------ */
static float roundf_away(float v) { return roundf(v); } /* C roundf rounds half away from zero */

static void quant_q8_0_block(const float *x, uint8_t *b) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_h(b, orc_f32_to_f16(d));
    for (int i = 0; i < 32; ++i) b[2 + i] = (uint8_t)(int8_t)roundf_away(x[i] * id);
}

static void quant_q4_0_block(const float *x, uint8_t *b) {
    float amax = 0.0f, maxv = 0.0f;
    for (int i = 0; i < 32; ++i)
        if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); maxv = x[i]; }
    float d = maxv / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_h(b, orc_f32_to_f16(d));
    uint8_t q[32];
    for (int i = 0; i < 32; ++i) {
        float v = truncf(x[i] * id + 8.5f);
        int iv = (int)v;
        q[i] = (uint8_t)(iv < 0 ? 0 : (iv > 15 ? 15 : iv));
    }
    for (int i = 0; i < 16; ++i) b[2 + i] = (uint8_t)(q[i] | (q[i + 16] << 4));
}

static void quant_q5_0_block(const float *x, uint8_t *b) {
    float amax = 0.0f, maxv = 0.0f;
    for (int i = 0; i < 32; ++i)
        if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); maxv = x[i]; }
    float d = maxv / -16.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_h(b, orc_f32_to_f16(d));
    uint8_t q[32];
    uint32_t qh = 0;
    for (int i = 0; i < 32; ++i) {
        float v = truncf(x[i] * id + 16.5f);
        int iv = (int)v;
        q[i] = (uint8_t)(iv < 0 ? 0 : (iv > 31 ? 31 : iv));
        qh |= (uint32_t)((q[i] >> 4) & 1) << i;
    }
    b[2] = (uint8_t)(qh & 0xff); b[3] = (uint8_t)((qh >> 8) & 0xff);
    b[4] = (uint8_t)((qh >> 16) & 0xff); b[5] = (uint8_t)(qh >> 24);
    for (int i = 0; i < 16; ++i) b[6 + i] = (uint8_t)((q[i] & 0x0F) | ((q[i + 16] & 0x0F) << 4));
}

/* Q4_K: per 32-element sub-block j, an affine fit x ~= D_j*q - M_j with q in
 * [0,15], D_j = d*sc_j, M_j = dmin*m_j, sc_j/m_j 6-bit.  Layout as decoded by
 * q4k_at / q4k_scale_min (kernel.cu:913-921,1090-1119). */
static void quant_q4_k_block(const float *x, uint8_t *b) {
    float scale[8], minv[8];
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = 0.0f;
        for (int i = 0; i < 32; ++i) { lo = fminf(lo, x[32 * j + i]); hi = fmaxf(hi, x[32 * j + i]); }
        scale[j] = (hi - lo) / 15.0f;
        minv[j] = -lo; /* >= 0 */
    }
    float smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) { smax = fmaxf(smax, scale[j]); mmax = fmaxf(mmax, minv[j]); }
    float d = smax / 63.0f, dmin = mmax / 63.0f;
    uint16_t dh = orc_f32_to_f16(d), dmh = orc_f32_to_f16(dmin);
    float dq = orc_f16_to_f32(dh), dmq = orc_f16_to_f32(dmh);
    uint8_t sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        int s = dq > 0.0f ? (int)lrintf(scale[j] / dq) : 0;
        int mm = dmq > 0.0f ? (int)lrintf(minv[j] / dmq) : 0;
        sc[j] = (uint8_t)(s < 0 ? 0 : (s > 63 ? 63 : s));
        m[j] = (uint8_t)(mm < 0 ? 0 : (mm > 63 ? 63 : mm));
    }
    put_h(b, dh);
    put_h(b + 2, dmh);
    uint8_t *s = b + 4;
    memset(s, 0, 12);
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
    }
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
        float D = dq * (float)sc[j], M = dmq * (float)m[j];
        for (int i = 0; i < 32; ++i) {
            int v = D > 0.0f ? (int)lrintf((x[32 * j + i] + M) / D) : 0;
            q[32 * j + i] = (uint8_t)(v < 0 ? 0 : (v > 15 ? 15 : v));
        }
    }
    for (int p = 0; p < 4; ++p)
        for (int i = 0; i < 32; ++i) b[16 + 32 * p + i] = (uint8_t)(q[64 * p + i] | (q[64 * p + 32 + i] << 4));
}

int orc_quantize_rows(int t, const float *src, int64_t rows, int K, uint8_t *dst) {
    int be = orc_block_elems(t), bb = orc_block_bytes(t);
    if (be <= 1 || K % be != 0) return 1;
    if (t != T_Q8_0 && t != T_Q4_0 && t != T_Q5_0 && t != T_Q4_K) return 2;
    int64_t nbr = K / be;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t i = 0; i < nbr; ++i) {
            const float *xb = src + r * K + i * be;
            uint8_t *ob = dst + (r * nbr + i) * bb;
            if (t == T_Q8_0) quant_q8_0_block(xb, ob);
            else if (t == T_Q4_0) quant_q4_0_block(xb, ob);
            else if (t == T_Q5_0) quant_q5_0_block(xb, ob);
            else quant_q4_k_block(xb, ob);
        }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Seeded normal generator: splitmix64 counter stream + Box-Muller.         */
/* Element i of stream (seed) is a pure function of (seed, i).              */
/* ------------------------------------------------------------------------ */
static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void orc_randn(uint64_t seed, uint64_t offset, int64_t n, float std, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint64_t c = offset + (uint64_t)i;
        uint64_t a = splitmix64(seed * 0x100000001B3ull ^ (c >> 1) * 2);
        uint64_t b = splitmix64(a ^ 0xD1B54A32D192ED03ull);
        double u1 = ((a >> 11) + 1.0) * (1.0 / 9007199254740993.0); /* (0,1] */
        double u2 = (b >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        double v = (c & 1) ? r * sin(6.283185307179586 * u2) : r * cos(6.283185307179586 * u2);
        out[i] = (float)(v * std);
    }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads of the OpenMP loops (a launcher such as torchrun sets OMP_NUM_THREADS=1). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
