// ql_misc.cu -- element-wise and routing kernels around the quantized linear.
//
//  * dequant_f16_kernel: whole-tensor GGUF block -> f16 (bit-exact with the
//    reference's dequantize_*_to_f16_kernel, kernel.cu:954-1063; adds Q4_0).
//  * embedding_kernel: quantized row gather (quant_embedding_kernel,
//    kernel.cu:2677-2693).
//  * argmax: two-stage, lowest index on ties (kernel.cu:3531-3592).
//  * router_topk_kernel: softmax + top-k, one warp per token
//    (moe_router_topk_kernel, kernel.cu:3463-3511, which runs on one thread).
//  * rmsnorm_kernel: f32 RMSNorm (rms_norm_kernel, kernel.cu:112-147).
//  * synth_kernel: seeded N(0, std) weights quantized in place on the device
//    (synthetic models for benchmarks; not part of the reference).
#include "ql_common.cuh"

namespace ql {

// Element decode shared by the dequant and embedding kernels (restates
// q4k_at / q6k_at / q50_at / q80_at, kernel.cu:1090-1185, plus Q4_0).
template <int T>
__device__ __forceinline__ float elem_at(const uint8_t *row, int idx) {
    if (T == kQ4_K) {
        const uint8_t *b = row + (size_t)(idx >> 8) * 144;
        const int in = idx & 255, j = in >> 5, inner = in & 31;
        const float d = half_bits_to_float(b[0] | (b[1] << 8)), dmin = half_bits_to_float(b[2] | (b[3] << 8));
        const uint8_t *s = b + 4;
        uint32_t sc, m;
        if (j < 4) {
            sc = s[j] & 63;
            m = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const uint8_t q = b[16 + (j >> 1) * 32 + inner];
        const int nib = (j & 1) ? (q >> 4) : (q & 0x0F);
        return d * (float)sc * (float)nib - dmin * (float)m;
    } else if (T == kQ6_K) {
        const uint8_t *b = row + (size_t)(idx >> 8) * 210;
        const int in = idx & 255, n = (in >> 7) * 128, within = in & 127, grp = within >> 5, l = within & 31;
        const int is = l / 16;
        const uint8_t *ql = b + n / 2, *qh = b + 128 + n / 4;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192) + n / 16;
        const float d = half_bits_to_float(b[208] | (b[209] << 8));
        int q, si;
        if (grp == 0) { q = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32; si = is; }
        else if (grp == 1) { q = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32; si = is + 2; }
        else if (grp == 2) { q = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32; si = is + 4; }
        else { q = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32; si = is + 6; }
        return d * (float)sc[si] * (float)q;
    } else if (T == kQ5_0) {
        const uint8_t *b = row + (size_t)(idx >> 5) * 22;
        const int in = idx & 31;
        const float d = half_bits_to_float(b[0] | (b[1] << 8));
        const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        const int q = (in < 16) ? ((b[6 + in] & 0x0F) | (((qh >> in) & 1) << 4))
                                : ((b[6 + in - 16] >> 4) | (((qh >> in) & 1) << 4));
        return d * (float)(q - 16);
    } else if (T == kQ8_0) {
        const uint8_t *b = row + (size_t)(idx >> 5) * 34;
        return half_bits_to_float(b[0] | (b[1] << 8)) * (float)(int8_t)b[2 + (idx & 31)];
    } else {  // Q4_0
        const uint8_t *b = row + (size_t)(idx >> 5) * 18;
        const int in = idx & 31;
        const int q = (in < 16) ? (b[2 + in] & 0x0F) : (b[2 + in - 16] >> 4);
        return half_bits_to_float(b[0] | (b[1] << 8)) * (float)(q - 8);
    }
}

template <int T>
__global__ void dequant_f16_kernel(const uint8_t *src, uint16_t *out, int64_t nblocks) {
    constexpr int BE = block_elems(T), BB = block_bytes(T);
    const int64_t blk = blockIdx.x;
    if (blk >= nblocks) return;
    const uint8_t *b = src + blk * BB;
    for (int i = threadIdx.x; i < BE; i += blockDim.x)
        out[blk * BE + i] = __half_as_ushort(__float2half_rn(elem_at<T>(b, i)));
}

template <int T>
__global__ void embedding_kernel(const int *ids, float *out, const uint8_t *table, size_t row_bytes, int hidden,
                                 int n) {
    const int tok = blockIdx.x;
    if (tok >= n) return;
    const uint8_t *row = table + (size_t)ids[tok] * row_bytes;
    float *o = out + (size_t)tok * hidden;
    for (int k = threadIdx.x; k < hidden; k += blockDim.x) o[k] = elem_at<T>(row, k);
}

// ---- argmax: lowest index wins ties; NaN never wins ------------------------
__device__ __forceinline__ void amax_merge(float &v, int &i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
__device__ __forceinline__ void amax_warp(float &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
        amax_merge(v, i, v2, i2);
    }
}
__global__ void argmax_partial_kernel(const float *x, int n, float *pv, int *pi) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) {
        const float a = x[k];
        if (a > v) { v = a; i = k; }  // ascending k: strict '>' keeps the lowest index
    }
    amax_warp(v, i);
    __shared__ float sv[32];
    __shared__ int si[32];
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = v; si[threadIdx.x >> 5] = i; }
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < blockDim.x / 32 ? sv[threadIdx.x] : -INFINITY;
        i = threadIdx.x < blockDim.x / 32 ? si[threadIdx.x] : 0x7fffffff;
        amax_warp(v, i);
        if (threadIdx.x == 0) { pv[blockIdx.x] = v; pi[blockIdx.x] = i; }
    }
}
__global__ void argmax_final_kernel(const float *pv, const int *pi, int np, int *out) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int k = threadIdx.x; k < np; k += 32) amax_merge(v, i, pv[k], pi[k]);
    amax_warp(v, i);
    if (threadIdx.x == 0) out[0] = (i == 0x7fffffff) ? 0 : i;
}

// ---- MoE router: one warp per token ------------------------------------------
// Selection is the reference's: k rounds of "largest finite logit, lowest
// expert id on ties" (its serial strict-'>' scan), a fallback of id r when no
// finite logit remains, weight = __expf(best - max) / denom * routed_scaling
// with denom summed over experts in ascending order as the reference does.
__global__ void router_topk_kernel(const float *logits, int *top_idx, float *top_w, int tokens, int E, int k,
                                   float scale) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= tokens) return;
    const float *lg = logits + (size_t)warp * E;
    float v0 = -INFINITY, v1 = -INFINITY;  // experts lane and lane + 32
    if (lane < E) { const float t = lg[lane]; v0 = isfinite(t) ? t : -INFINITY; }
    if (lane + 32 < E) { const float t = lg[lane + 32]; v1 = isfinite(t) ? t : -INFINITY; }
    float mx = fmaxf(v0, v1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float denom = 0.f;
    if (isfinite(mx)) {
        const float e0 = (lane < E) ? __expf(v0 - mx) : 0.f;
        const float e1 = (lane + 32 < E) ? __expf(v1 - mx) : 0.f;
        for (int e = 0; e < E; ++e) {  // ascending-order sum, like the reference's single thread
            const float t = __shfl_sync(0xffffffffu, e < 32 ? e0 : e1, e & 31);
            denom += t;
        }
    }
    bool used0 = false, used1 = false;
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        if (lane < E && !used0 && v0 > -INFINITY) { bv = v0; bi = lane; }
        if (lane + 32 < E && !used1 && v1 > -INFINITY && (v1 > bv)) { bv = v1; bi = lane + 32; }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
            if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
        }
        int be = (bi == 0x7fffffff) ? -1 : bi;
        if (be < 0) be = r < E ? r : 0;
        if (be == lane) used0 = true;
        if (be == lane + 32) used1 = true;
        if (lane == 0) {
            const float prob = (denom > 0.f && isfinite(bv)) ? __expf(bv - mx) / denom : 0.f;
            top_idx[(size_t)warp * k + r] = be;
            top_w[(size_t)warp * k + r] = prob * scale;
        }
    }
}

// ---- RMSNorm (f32 gamma), one CTA per row ------------------------------------
__global__ void rmsnorm_kernel(const float *x, float *y, const float *gamma, int H, float eps) {
    const float *xr = x + (size_t)blockIdx.x * H;
    float *yr = y + (size_t)blockIdx.x * H;
    float ss = 0.f;
    for (int j = threadIdx.x; j < H; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    __shared__ float sh[32];
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        ss = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (threadIdx.x == 0) sh[0] = rsqrtf(ss / (float)H + eps);
    }
    __syncthreads();
    const float inv = sh[0];
    for (int j = threadIdx.x; j < H; j += blockDim.x) yr[j] = xr[j] * inv * (gamma ? gamma[j] : 1.0f);
}

// ---- synthetic weights: seeded N(0, std), quantized per block ----------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float gauss(uint64_t seed, uint64_t i) {
    const uint64_t a = mix64(seed * 0x100000001B3ull ^ (i >> 1) * 2), b = mix64(a ^ 0xD1B54A32D192ED03ull);
    const float u1 = ((a >> 40) + 1.0f) * (1.0f / 16777217.0f), u2 = (b >> 40) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    return (i & 1) ? r * sinpif(2.0f * u2) : r * cospif(2.0f * u2);
}

__device__ __forceinline__ void put_f16(uint8_t *p, float v) {
    const uint16_t h = __half_as_ushort(__float2half_rn(v));
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

// One thread per block.  Q8_0 / Q4_0 / Q5_0 follow the ggml reference
// quantizers; Q4_K uses a min/max fit with 6-bit scales and mins.
template <int T>
__global__ void synth_kernel(uint64_t seed, int64_t nblocks, int blocks_per_row, int K, float std, uint8_t *dst) {
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= nblocks) return;
    constexpr int BE = block_elems(T), BB = block_bytes(T);
    const int64_t row = blk / blocks_per_row, col0 = (blk % blocks_per_row) * BE;
    float x[BE];
    for (int i = 0; i < BE; ++i) x[i] = std * gauss(seed, (uint64_t)(row * K + col0 + i));
    uint8_t *b = dst + blk * BB;
    if (T == kQ8_0) {
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
        const float d = amax / 127.0f, id = d != 0.f ? 1.0f / d : 0.f;
        put_f16(b, d);
        for (int i = 0; i < 32; ++i) b[2 + i] = (uint8_t)(int8_t)roundf(x[i] * id);
    } else if (T == kQ4_0 || T == kQ5_0) {
        float amax = 0.f, mx = 0.f;
        for (int i = 0; i < 32; ++i)
            if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); mx = x[i]; }
        const float d = mx / (T == kQ4_0 ? -8.0f : -16.0f), id = d != 0.f ? 1.0f / d : 0.f;
        put_f16(b, d);
        uint8_t q[32];
        uint32_t qh = 0;
        for (int i = 0; i < 32; ++i) {
            const int v = (int)truncf(x[i] * id + (T == kQ4_0 ? 8.5f : 16.5f));
            const int hi = T == kQ4_0 ? 15 : 31;
            q[i] = (uint8_t)(v < 0 ? 0 : (v > hi ? hi : v));
            qh |= (uint32_t)((q[i] >> 4) & 1) << i;
        }
        if (T == kQ4_0) {
            for (int i = 0; i < 16; ++i) b[2 + i] = (uint8_t)(q[i] | (q[i + 16] << 4));
        } else {
            b[2] = qh & 0xff; b[3] = (qh >> 8) & 0xff; b[4] = (qh >> 16) & 0xff; b[5] = qh >> 24;
            for (int i = 0; i < 16; ++i) b[6 + i] = (uint8_t)((q[i] & 0xF) | ((q[i + 16] & 0xF) << 4));
        }
    } else {  // Q4_K
        float scale[8], minv[8], smax = 0.f, mmax = 0.f;
        for (int j = 0; j < 8; ++j) {
            float lo = 0.f, hi = 0.f;
            for (int i = 0; i < 32; ++i) { lo = fminf(lo, x[32 * j + i]); hi = fmaxf(hi, x[32 * j + i]); }
            scale[j] = (hi - lo) / 15.0f;
            minv[j] = -lo;
            smax = fmaxf(smax, scale[j]);
            mmax = fmaxf(mmax, minv[j]);
        }
        const __half dh = __float2half_rn(smax / 63.0f), dmh = __float2half_rn(mmax / 63.0f);
        const float dq = __half2float(dh), dmq = __half2float(dmh);
        uint8_t sc[8], mm[8];
        for (int j = 0; j < 8; ++j) {
            const int s = dq > 0.f ? __float2int_rn(scale[j] / dq) : 0;
            const int m = dmq > 0.f ? __float2int_rn(minv[j] / dmq) : 0;
            sc[j] = (uint8_t)min(63, max(0, s));
            mm[j] = (uint8_t)min(63, max(0, m));
        }
        const uint16_t dhb = __half_as_ushort(dh), dmb = __half_as_ushort(dmh);
        b[0] = dhb & 0xff; b[1] = dhb >> 8; b[2] = dmb & 0xff; b[3] = dmb >> 8;
        for (int j = 0; j < 4; ++j) {
            b[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            b[8 + j] = (uint8_t)((mm[j] & 63) | ((mm[j + 4] >> 4) << 6));
            b[12 + j] = (uint8_t)((sc[j + 4] & 0x0F) | ((mm[j + 4] & 0x0F) << 4));
        }
        for (int p = 0; p < 4; ++p)
            for (int i = 0; i < 32; ++i) {
                uint8_t qq[2];
                for (int h = 0; h < 2; ++h) {
                    const int j = 2 * p + h;
                    const float D = dq * (float)sc[j], M = dmq * (float)mm[j];
                    const int v = D > 0.f ? __float2int_rn((x[32 * j + i] + M) / D) : 0;
                    qq[h] = (uint8_t)min(15, max(0, v));
                }
                b[16 + 32 * p + i] = (uint8_t)(qq[0] | (qq[1] << 4));
            }
    }
}

// ----------------------------------------------------------------------------
// Host-side launchers used by the C ABI layer.
// ----------------------------------------------------------------------------
cudaError_t dequant_f16_launch(int t, const uint8_t *src, uint16_t *out, int64_t n, cudaStream_t s) {
    const int64_t nb = n / block_elems(t);
    if (nb == 0) return cudaSuccess;
    switch (t) {
    case kQ4_K: dequant_f16_kernel<kQ4_K><<<(unsigned)nb, 128, 0, s>>>(src, out, nb); break;
    case kQ6_K: dequant_f16_kernel<kQ6_K><<<(unsigned)nb, 128, 0, s>>>(src, out, nb); break;
    case kQ5_0: dequant_f16_kernel<kQ5_0><<<(unsigned)nb, 32, 0, s>>>(src, out, nb); break;
    case kQ8_0: dequant_f16_kernel<kQ8_0><<<(unsigned)nb, 32, 0, s>>>(src, out, nb); break;
    case kQ4_0: dequant_f16_kernel<kQ4_0><<<(unsigned)nb, 32, 0, s>>>(src, out, nb); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t embedding_launch(int t, const int *ids, float *out, const uint8_t *table, size_t rb, int hidden, int n,
                             cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    switch (t) {
    case kQ4_K: embedding_kernel<kQ4_K><<<n, 256, 0, s>>>(ids, out, table, rb, hidden, n); break;
    case kQ6_K: embedding_kernel<kQ6_K><<<n, 256, 0, s>>>(ids, out, table, rb, hidden, n); break;
    case kQ5_0: embedding_kernel<kQ5_0><<<n, 256, 0, s>>>(ids, out, table, rb, hidden, n); break;
    case kQ8_0: embedding_kernel<kQ8_0><<<n, 256, 0, s>>>(ids, out, table, rb, hidden, n); break;
    case kQ4_0: embedding_kernel<kQ4_0><<<n, 256, 0, s>>>(ids, out, table, rb, hidden, n); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t argmax_launch(const float *x, int n, int *out, float *pv, int *pi, int max_parts, cudaStream_t s) {
    int blocks = (n + 1023) / 1024;
    if (blocks > max_parts) blocks = max_parts;
    if (blocks < 1) blocks = 1;
    argmax_partial_kernel<<<blocks, 256, 0, s>>>(x, n, pv, pi);
    argmax_final_kernel<<<1, 32, 0, s>>>(pv, pi, blocks, out);
    return cudaGetLastError();
}

cudaError_t router_launch(const float *logits, int *idx, float *w, int tokens, int E, int k, float scale,
                          cudaStream_t s) {
    if (tokens == 0) return cudaSuccess;
    const int warps_per_block = 4;
    router_topk_kernel<<<(tokens + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(
        logits, idx, w, tokens, E, k, scale);
    return cudaGetLastError();
}

cudaError_t rmsnorm_launch(const float *x, float *y, const float *gamma, int rows, int H, float eps,
                           cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    rmsnorm_kernel<<<rows, 256, 0, s>>>(x, y, gamma, H, eps);
    return cudaGetLastError();
}

cudaError_t synth_launch(int t, uint64_t seed, int64_t rows, int K, float std, uint8_t *dst, cudaStream_t s) {
    const int bpr = K / block_elems(t);
    const int64_t nb = rows * bpr;
    if (nb == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((nb + 127) / 128);
    switch (t) {
    case kQ4_K: synth_kernel<kQ4_K><<<grid, 128, 0, s>>>(seed, nb, bpr, K, std, dst); break;
    case kQ8_0: synth_kernel<kQ8_0><<<grid, 128, 0, s>>>(seed, nb, bpr, K, std, dst); break;
    case kQ4_0: synth_kernel<kQ4_0><<<grid, 128, 0, s>>>(seed, nb, bpr, K, std, dst); break;
    case kQ5_0: synth_kernel<kQ5_0><<<grid, 128, 0, s>>>(seed, nb, bpr, K, std, dst); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ql
