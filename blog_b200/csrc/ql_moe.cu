// Grouped routed experts for a batch of tokens.
//
// The reference runs a batch's routed experts one token at a time: per token one
// quant_swiglu_indexed launch over its k routes, then one quant_down_f32_indexed_accum_ordered
// launch (RoutedExperts.cpp:80-118; kernel.cu:1339-1385, 2252-2287), so an expert chosen by n
// tokens is read n times.  Here each expert's rows are read once per layer for all the tokens
// routed to it:
//   1. moe_xprep: token rows -> two f16 limbs with a power-of-two row scale, 32-element block sums;
//   2. moe_bucket_kernel: the (token, route) pairs grouped by expert, in routing-table order;
//      moe_grouped_kernel<SwiGLU>: CTA = (expert, 32 gate + 32 up rows); it multiplies its weight
//      rows with its expert's tokens on the tensor cores, and writes act[(t, r), f] = SiLU(g) * u;
//   3. moe_xprep over the act rows, and the buckets again;
//   4. moe_grouped_kernel<down>: CTA = (expert, 64 rows of the hidden size); writes each pair's
//      down projection (fp32) to a scratch row;
//   5. moe_combine_kernel: out[t, h] += sum over t's routes in route order (fmaf(y, w, total)),
//      the reference combine's order.
//
// Weight rows stream into shared memory one row per bulk copy (TMA engine), from the 16-byte
// boundary at or before the row's first byte plus plain loads of its last < 16 bytes, into slots
// whose pitch is 16 mod 32 bytes (the 8 rows a lane quad reads at once fall in distinct banks).
// This works for any row length, including the 32-element formats whose rows are not 16-byte
// multiples (Q5_0 with K = 1408: 968 B rows).  A CTA has 8 warps: 4 slabs of 16 rows, each slab
// shared by two warps that take one half of K each (their sums meet in shared memory).  Each thread
// decodes its MMA A fragment straight from the raw bytes (no dequantized tile): mma.sync m16n8k16
// with the k order of the activation layout (elements 0, 2, 1, 3 | 4, 6, 5, 7 of each group of 8),
// so lane (g, c) of a 16-element step needs quants 4c..4c+3 of rows g and g + 8: one 32-bit word of
// nibbles per row, masked into exact integer f16 pairs with the magic-number conversion.  Tokens are
// the MMA's n = 8 columns, up to 16 per pass over the staged rows (decode at batch 64: ~6 tokens per
// expert, one n-tile).
#include "ql_common.cuh"
#include "ql_gemm.cuh"
#include "ql_moe.cuh"

namespace ql {
namespace {

constexpr int kMoeThreads = 256;  // 4 slabs of 16 weight rows x 2 warps (one per half of K)
constexpr int kMoePass = 16;      // tokens per pass (2 MMA n-tiles)

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
// 32-bit word at a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t *p) {
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Quants of one 32-element block as exact small integers in f16 (the MMA's A operand), with the
// block's scale (and Q4_K's min) returned in fp32 and applied to the block's MMA result: the
// weights enter the tensor cores without rounding.  Rows g (row0) and g + 8 (row1), lane quad c:
// A0 = elements 0..15 of the block, A1 = 16..31; registers {row g: (4c, 4c+2)}, {row g+8: same},
// {row g: (4c+1, 4c+3)}, {row g+8: same} (the activation layout's k order).
struct BlockScale {
    float d[2];  // rows g, g + 8: value = d * q - m
    float m[2];
};
// Small unsigned integers at bits 0.. and 16.. (< 1024) minus `bias` -> exact f16 pair.
__device__ __forceinline__ uint32_t int_pair(uint32_t n, __half2 bias) { return h2u(__hsub2(u2h(n | 0x64006400u), bias)); }

template <int FMT>
__device__ __forceinline__ void decode_block(const uint8_t *row0, const uint8_t *row1, int kb, int c,
                                             uint32_t (&A0)[4], uint32_t (&A1)[4], BlockScale &sc) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint8_t *rp = h ? row1 : row0;
        uint32_t r00, r01, r10, r11;  // (step 0, pair 0), (step 0, pair 1), (step 1, pair 0), (step 1, pair 1)
        if (FMT == kQ4_0) {  // d * (q - 8)
            const uint8_t *blk = rp + 18 * kb;
            const __half2 B = __float2half2_rn(1032.f);
            sc.d[h] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
            sc.m[h] = 0.f;
            const uint32_t w = lds_u32_a2(blk + 2 + 4 * c);  // low nibbles: elements 4c.., high: 16 + 4c..
            r00 = int_pair(w & 0x000F000Fu, B);
            r01 = int_pair((w >> 8) & 0x000F000Fu, B);
            r10 = int_pair((w >> 4) & 0x000F000Fu, B);
            r11 = int_pair((w >> 12) & 0x000F000Fu, B);
        } else if (FMT == kQ5_0) {  // d * (q - 16), q = nibble | fifth bit << 4
            const uint8_t *blk = rp + 22 * kb;
            const __half2 B = __float2half2_rn(1040.f);
            sc.d[h] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
            sc.m[h] = 0.f;
            const uint32_t qh = lds_u32_a2(blk + 2);
            const uint32_t w = lds_u32_a2(blk + 6 + 4 * c);
            const uint32_t h0 = qh >> (4 * c), h1 = qh >> (16 + 4 * c);  // fifth bits of 4c.. and 16 + 4c..
            r00 = int_pair((w & 0x000F000Fu) | ((h0 & 1u) << 4) | ((h0 & 4u) << 18), B);
            r01 = int_pair(((w >> 8) & 0x000F000Fu) | ((h0 & 2u) << 3) | ((h0 & 8u) << 17), B);
            r10 = int_pair(((w >> 4) & 0x000F000Fu) | ((h1 & 1u) << 4) | ((h1 & 4u) << 18), B);
            r11 = int_pair(((w >> 12) & 0x000F000Fu) | ((h1 & 2u) << 3) | ((h1 & 8u) << 17), B);
        } else if (FMT == kQ8_0) {  // d * q, q signed: (q + 128) - 128
            const uint8_t *blk = rp + 34 * kb;
            const __half2 B = __float2half2_rn(1152.f);
            sc.d[h] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
            sc.m[h] = 0.f;
            const uint32_t w0 = lds_u32_a2(blk + 2 + 4 * c) ^ 0x80808080u;
            const uint32_t w1 = lds_u32_a2(blk + 18 + 4 * c) ^ 0x80808080u;
            r00 = int_pair(w0 & 0x00FF00FFu, B);
            r01 = int_pair((w0 >> 8) & 0x00FF00FFu, B);
            r10 = int_pair(w1 & 0x00FF00FFu, B);
            r11 = int_pair((w1 >> 8) & 0x00FF00FFu, B);
        } else {  // Q4_K: sub-block j of super-block sb, d * sc * q - dmin * m (rows on 16 bytes)
            const int sb = kb >> 3, j = kb & 7;
            const uint8_t *blk = rp + 144 * sb;
            const __half2 B = __float2half2_rn(1024.f);
            const uint32_t dd = *reinterpret_cast<const uint32_t *>(blk);
            const uint8_t *s = blk + 4;
            uint32_t scv, mnv;  // q4k_scale_min (reference kernel.cu:913-921)
            if (j < 4) {
                scv = s[j] & 63u;
                mnv = s[j + 4] & 63u;
            } else {
                scv = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
                mnv = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
            }
            sc.d[h] = half_bits_to_float(dd) * (float)scv;  // exact: 11-bit x 6-bit
            sc.m[h] = half_bits_to_float(dd >> 16) * (float)mnv;
            const uint8_t *q = blk + 16 + 32 * (j >> 1) + 4 * c;
            const int sh = 4 * (j & 1);
            const uint32_t w0 = *reinterpret_cast<const uint32_t *>(q) >> sh;
            const uint32_t w1 = *reinterpret_cast<const uint32_t *>(q + 16) >> sh;
            r00 = int_pair(w0 & 0x000F000Fu, B);
            r01 = int_pair((w0 >> 8) & 0x000F000Fu, B);
            r10 = int_pair(w1 & 0x000F000Fu, B);
            r11 = int_pair((w1 >> 8) & 0x000F000Fu, B);
        }
        A0[h] = r00;
        A0[2 + h] = r01;
        A1[h] = r10;
        A1[2 + h] = r11;
    }
}

// Activation prep (one CTA per row): s = 2^k with max|x| * s in [2^13, 2^14) (the tensor-core
// GEMM's rule), x * s split into two f16 limbs hi = f16(x s), lo = f16(x s - hi) (together exact
// to ~2^-22), stored per 16-element step and lane quad c as one 16-byte word {hi of elements
// 4c, 4c+2 | 4c+1, 4c+3 | lo of the same}; rinv = 1 / s; bsum = sum of x * s over each 32-element
// block (fp32), for the Q4_K min term.
__global__ void __launch_bounds__(256) moe_xprep_kernel(const float *__restrict__ x, int64_t x_stride,
                                                        uint4 *__restrict__ xq, float *__restrict__ rinv,
                                                        float *__restrict__ bsum, int K) {
    const int m = blockIdx.x;
    const float *xr = x + (size_t)m * x_stride;
    float mx = 0.f;
    bool nan = false;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(xr)[i];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        nan = nan || v.x != v.x || v.y != v.y || v.z != v.z || v.w != v.w;
    }
    if (nan) mx = __int_as_float(0x7f800000);
    __shared__ float red[8];
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    int k = 0;
    if (mx > 0.f && mx < __int_as_float(0x7f800000)) {
        int ex;
        frexpf(mx, &ex);
        k = 14 - ex;
        k = k > 126 ? 126 : k;
    }
    const float s = __int_as_float((127 + k) << 23);
    if (threadIdx.x == 0) rinv[m] = __int_as_float((127 - k) << 23);
    // thread = (16-element step, lane quad c): elements 16 G + 4c .. + 3; 8 threads per 32-block
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(xr)[i];
        const float a0 = v.x * s, a1 = v.y * s, a2 = v.z * s, a3 = v.w * s;
        const __half2 h02 = __floats2half2_rn(a0, a2), h13 = __floats2half2_rn(a1, a3);
        const float2 f02 = __half22float2(h02), f13 = __half22float2(h13);
        uint4 o;
        o.x = h2u(h02);
        o.y = h2u(h13);
        o.z = h2u(__floats2half2_rn(a0 - f02.x, a2 - f02.y));
        o.w = h2u(__floats2half2_rn(a1 - f13.x, a3 - f13.y));
        xq[(size_t)m * (K / 4) + i] = o;
        float bs = (a0 + a1) + (a2 + a3);  // the 8 threads of a 32-block are 8 consecutive lanes
        bs += __shfl_xor_sync(__activemask(), bs, 1);
        bs += __shfl_xor_sync(__activemask(), bs, 2);
        bs += __shfl_xor_sync(__activemask(), bs, 4);
        if ((i & 7) == 0) bsum[(size_t)m * (K / 32) + (i >> 3)] = bs;
    }
}

// One pass over the warp's 16 staged rows for NT token tiles: per 32-element block, the exact
// integer quants times both activation limbs on the tensor cores (4 MMAs per tile), then the
// block's fp32 scale (and Q4_K's min times the block sum) into the accumulators.  The activation
// words and block sums of block kb + PF load while block kb computes (they come from L2, and an
// SM holds only 12 of these warps).
template <int FMT, int NT>
__device__ __forceinline__ void pass_blocks(const uint8_t *row0, const uint8_t *row1, int kb_lo, int nkb, int c,
                                            const uint4 *const (&xr)[2], const float *const (&bsr)[2][2],
                                            float (&acc)[2][4]) {
    constexpr int PF = NT == 1 ? 6 : 3;
    uint4 b[PF][NT][2];
    float bs[PF][NT][2];
    auto load = [&](int p, int kb) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            b[p][j][0] = xr[j][8 * kb];      // step 0 of the block: 4 words per 16 elements
            b[p][j][1] = xr[j][8 * kb + 4];  // step 1
            if (FMT == kQ4_K) {
                bs[p][j][0] = bsr[j][0][kb];
                bs[p][j][1] = bsr[j][1][kb];
            }
        }
    };
#pragma unroll
    for (int p = 0; p < PF; ++p)
        if (kb_lo + p < nkb) load(p, kb_lo + p);
    for (int kb0 = kb_lo; kb0 < nkb; kb0 += PF) {
#pragma unroll
        for (int p = 0; p < PF; ++p) {
            const int kb = kb0 + p;
            if (kb < nkb) {
                uint32_t A0[4], A1[4];
                BlockScale bsc;
                decode_block<FMT>(row0, row1, kb, c, A0, A1, bsc);
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    float t[4] = {0.f, 0.f, 0.f, 0.f};  // this block's integer-weight dot products
                    mma16816(t, A0, b[p][j][0].x, b[p][j][0].y);
                    mma16816(t, A0, b[p][j][0].z, b[p][j][0].w);
                    mma16816(t, A1, b[p][j][1].x, b[p][j][1].y);
                    mma16816(t, A1, b[p][j][1].z, b[p][j][1].w);
                    acc[j][0] = fmaf(bsc.d[0], t[0], acc[j][0]);
                    acc[j][1] = fmaf(bsc.d[0], t[1], acc[j][1]);
                    acc[j][2] = fmaf(bsc.d[1], t[2], acc[j][2]);
                    acc[j][3] = fmaf(bsc.d[1], t[3], acc[j][3]);
                    if (FMT == kQ4_K) {
                        acc[j][0] = fmaf(-bsc.m[0], bs[p][j][0], acc[j][0]);
                        acc[j][1] = fmaf(-bsc.m[0], bs[p][j][1], acc[j][1]);
                        acc[j][2] = fmaf(-bsc.m[1], bs[p][j][0], acc[j][2]);
                        acc[j][3] = fmaf(-bsc.m[1], bs[p][j][1], acc[j][3]);
                    }
                }
                if (kb + PF < nkb) load(p, kb + PF);
            }
        }
    }
}

// Q4_K pass: per super-block, each row's header (d, dmin, 12 scale bytes) is loaded once as 4
// words and each 32-bit word of quants once per sub-block pair (low nibbles: sub-block 2p, high:
// 2p + 1); the unrolled sub-block index makes the scale/min extraction constant shifts.  Rows are
// 16-byte multiples (144 B per 256 inputs), so every load is aligned.
template <int NT>
__device__ __forceinline__ void pass_q4k(const uint8_t *row0, const uint8_t *row1, int kb_lo, int nkb, int c,
                                         const uint4 *const (&xr)[2], const float *const (&bsr)[2][2],
                                         float (&acc)[2][4]) {
    constexpr int PF = NT == 1 ? 4 : 2;  // divides 8 and the start (a multiple of 8): slot = sub-block % PF
    uint4 b[PF][NT][2];
    float bs[PF][NT][2];
    auto load = [&](int p, int kb) {
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            b[p][j][0] = xr[j][8 * kb];
            b[p][j][1] = xr[j][8 * kb + 4];
            bs[p][j][0] = bsr[j][0][kb];
            bs[p][j][1] = bsr[j][1][kb];
        }
    };
#pragma unroll
    for (int p = 0; p < PF; ++p)
        if (kb_lo + p < nkb) load(p, kb_lo + p);
    const __half2 B = __float2half2_rn(1024.f);
    for (int sb = kb_lo / 8; sb < nkb / 8; ++sb) {
        uint4 hd[2];  // rows g, g + 8: {d | dmin << 16, scales 0-3, 4-7, 8-11}
        hd[0] = *reinterpret_cast<const uint4 *>(row0 + 144 * sb);
        hd[1] = *reinterpret_cast<const uint4 *>(row1 + 144 * sb);
        // the 4 lanes of a quad share rows g and g + 8: lane c decodes one of the 4 per-sub-block
        // values (c = 0: d sc of row g, 1: dmin m of row g, 2 / 3: the same for row g + 8), which a
        // quad shuffle then hands to the others
        const uint4 &hsel = (c & 2) ? hd[1] : hd[0];
        const bool is_min = c & 1;
        const uint32_t lo6 = is_min ? hsel.z : hsel.y;  // 6-bit values of sub-blocks 0-3, top bits of 4-7
        const uint32_t hi4 = hsel.w >> (is_min ? 4 : 0);  // low 4 bits of sub-blocks 4-7
        const float sup = half_bits_to_float(is_min ? (hsel.x >> 16) : hsel.x);
        const int qbase = (threadIdx.x & 31) & ~3;
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            uint32_t w[2][2];  // rows x (bytes 4c.., bytes 16 + 4c..) of sub-blocks 2pr, 2pr + 1
            w[0][0] = *reinterpret_cast<const uint32_t *>(row0 + 144 * sb + 16 + 32 * pr + 4 * c);
            w[0][1] = *reinterpret_cast<const uint32_t *>(row0 + 144 * sb + 32 + 32 * pr + 4 * c);
            w[1][0] = *reinterpret_cast<const uint32_t *>(row1 + 144 * sb + 16 + 32 * pr + 4 * c);
            w[1][1] = *reinterpret_cast<const uint32_t *>(row1 + 144 * sb + 32 + 32 * pr + 4 * c);
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
                const int j = 2 * pr + hb, kb = 8 * sb + j, slot = j % PF;
                uint32_t A0[4], A1[4];
                uint32_t v6;  // q4k_scale_min (reference kernel.cu:913-921) for this lane's value
                if (j < 4) v6 = (lo6 >> (8 * j)) & 63u;
                else v6 = ((hi4 >> (8 * (j - 4))) & 0xFu) | (((lo6 >> (8 * (j - 4) + 6)) & 3u) << 4);
                const float mine = sup * (float)v6;  // exact: 11-bit x 6-bit
                float dsc[2], msc[2];
                dsc[0] = __shfl_sync(0xffffffffu, mine, qbase);
                msc[0] = __shfl_sync(0xffffffffu, mine, qbase + 1);
                dsc[1] = __shfl_sync(0xffffffffu, mine, qbase + 2);
                msc[1] = __shfl_sync(0xffffffffu, mine, qbase + 3);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t w0 = w[h][0] >> (4 * hb), w1 = w[h][1] >> (4 * hb);
                    A0[h] = int_pair(w0 & 0x000F000Fu, B);
                    A0[2 + h] = int_pair((w0 >> 8) & 0x000F000Fu, B);
                    A1[h] = int_pair(w1 & 0x000F000Fu, B);
                    A1[2 + h] = int_pair((w1 >> 8) & 0x000F000Fu, B);
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    float r[4] = {0.f, 0.f, 0.f, 0.f};
                    mma16816(r, A0, b[slot][t][0].x, b[slot][t][0].y);
                    mma16816(r, A0, b[slot][t][0].z, b[slot][t][0].w);
                    mma16816(r, A1, b[slot][t][1].x, b[slot][t][1].y);
                    mma16816(r, A1, b[slot][t][1].z, b[slot][t][1].w);
                    acc[t][0] = fmaf(dsc[0], r[0], fmaf(-msc[0], bs[slot][t][0], acc[t][0]));
                    acc[t][1] = fmaf(dsc[0], r[1], fmaf(-msc[0], bs[slot][t][1], acc[t][1]));
                    acc[t][2] = fmaf(dsc[1], r[2], fmaf(-msc[1], bs[slot][t][0], acc[t][2]));
                    acc[t][3] = fmaf(dsc[1], r[3], fmaf(-msc[1], bs[slot][t][1], acc[t][3]));
                }
                if (kb + PF < nkb) load(slot, kb + PF);
            }
        }
    }
}

// Stable bucketing of the (token, route) pairs by expert, one CTA of 1024 threads: bucket e in
// [0, n) holds the pairs of this call's expert e, bucket n the pairs routed elsewhere, each in
// routing-table order; off[b] .. off[b + 1] is bucket b's range of `list`.  Chunks of 1024
// pairs: a pair's place = its bucket's running base + the same-bucket pairs of earlier warps in
// the chunk + those of earlier lanes in its warp (__match_any_sync).
constexpr int kBucketMax = 257;  // n_experts <= 256, plus the skipped bucket
__global__ void __launch_bounds__(1024) moe_bucket_kernel(const int *__restrict__ ids, int npairs, int e_begin,
                                                          int n, int *__restrict__ off, int *__restrict__ list) {
    __shared__ int base[kBucketMax + 1];
    __shared__ unsigned short wcnt[32][kBucketMax];  // per warp of a chunk: pairs per bucket
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = n + 1;
    auto bucket_of = [&](int i) {
        const int le = ids[i] - e_begin;
        return (le >= 0 && le < n) ? le : n;
    };
    for (int b = tid; b <= nb; b += blockDim.x) base[b] = 0;
    __syncthreads();
    for (int i = tid; i < npairs; i += blockDim.x) atomicAdd(&base[bucket_of(i) + 1], 1);  // counts
    __syncthreads();
    if (tid == 0) {  // exclusive offsets
        for (int b = 1; b <= nb; ++b) base[b] += base[b - 1];
        for (int b = 0; b <= nb; ++b) off[b] = base[b];
    }
    __syncthreads();
    for (int c0 = 0; c0 < npairs; c0 += blockDim.x) {
        const int i = c0 + tid;
        const bool valid = i < npairs;
        const int b = valid ? bucket_of(i) : nb;  // nb: not a pair
        for (int x = tid; x < 32 * nb; x += blockDim.x) wcnt[x / nb][x % nb] = 0;
        __syncthreads();
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (valid && rank == 0) wcnt[warp][b] = (unsigned short)__popc(peers);
        __syncthreads();
        if (valid) {
            int before = 0;
            for (int w = 0; w < warp; ++w) before += wcnt[w][b];
            list[base[b] + before + rank] = i;
        }
        __syncthreads();
        for (int bb = tid; bb < nb; bb += blockDim.x) {
            int total = 0;
            for (int w = 0; w < 32; ++w) total += wcnt[w][bb];
            base[bb] += total;
        }
        __syncthreads();
    }
}

template <int FMT, bool SWIGLU>
__global__ void __launch_bounds__(kMoeThreads, 2) moe_grouped_kernel(const __grid_constant__ MoeArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];  // [4 slabs][16 rows][row_pitch] raw weight rows
    __shared__ float red[4][32][8];                  // second K half's partial sums, per slab and lane
    __shared__ float su[32][kMoePass + 1];           // SwiGLU: up rows handed to the gate warps
    __shared__ int plist[8][kMoePass];               // per warp: the pass's (token, route) pairs
    __shared__ uint64_t bar[4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slab_i = warp & 3, khalf = warp >> 2;  // warps w and w + 4 share slab w, one K half each
    const int g = lane >> 2, c = lane & 3;
    const int e = blockIdx.y;
    constexpr int RT = SWIGLU ? 32 : 64;  // output rows per CTA
    const int row_base = blockIdx.x * RT;

    const int lbeg = a.bucket_off[e], lend = a.bucket_off[e + 1];  // this expert's pairs in a.bucket
    if (SWIGLU && e == a.n_experts) {
        // zero act[(t, r), row_base ..] for the routes that go to no expert of this call
        for (int l = lbeg + warp; l < lend; l += 8)
            if (row_base + lane < a.rows) a.y[(size_t)a.bucket[l] * a.y_stride + row_base + lane] = 0.f;
        return;
    }
    if (lbeg == lend) return;  // no route chose this expert (nothing is in flight yet)
    // ---- slab s: 16 rows, one bulk copy per row into a slot of a.row_pitch bytes (warp s issues) ----
    // (pitch = 16 mod 32: rows g = 0..7 of a quad's 4-byte loads fall in 32 distinct banks)
    const int mat = SWIGLU ? (slab_i >> 1) : 0;
    const int wrow0 = row_base + 16 * (SWIGLU ? (slab_i & 1) : slab_i);
    int nr = min(16, a.rows - wrow0);
    const size_t rb = a.rb[mat];
    const int P = a.row_pitch;
    uint8_t *slab = smem + (size_t)slab_i * 16 * P;
    const uint8_t *wbase = a.w[mat] + (size_t)e * a.eb[mat] + (size_t)wrow0 * rb;
    uintptr_t lo = 0, hi = 0, end = 0;
    if (khalf == 0 && nr > 0) {
        // lane r < nr copies row r: [floor16(start), floor16(end)) by the TMA engine, the < 16 bytes
        // after that by plain loads
        if (lane < nr) {
            const uintptr_t st = reinterpret_cast<uintptr_t>(wbase + (size_t)lane * rb);
            lo = st & ~uintptr_t(15);
            end = st + rb;
            hi = end & ~uintptr_t(15);
        }
        const uint32_t tx = __reduce_add_sync(0xffffffffu, (uint32_t)(hi - lo));
        if (lane == 0) {
            mbar_init(&bar[slab_i], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            mbar_arrive_expect_tx(&bar[slab_i], tx);
        }
    }
    __syncthreads();  // barriers initialised before the other K half waits on them
    if (khalf == 0 && lane < nr) {
        uint8_t *dst = slab + (size_t)lane * P;
        if (hi > lo)
            bulk_g2s(dst, reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &bar[slab_i],
                     l2_evict_first_policy());
        for (uintptr_t q = hi; q < end; ++q) dst[q - lo] = *reinterpret_cast<const uint8_t *>(q);
    }
    __syncthreads();  // the tails' plain stores, for both K halves
    if (nr > 0 && !mbar_wait(&bar[slab_i], 0u, a.err, kErrWaitFull)) {
        mbar_wait(&bar[slab_i], 0u, nullptr, 0);  // never leave with the copies in flight
        nr = 0;                                   // rows not staged: nothing is computed or stored
    }
    const int sh0 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)g * rb) & 15);
    const int sh1 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)(g + 8) * rb) & 15);
    const uint8_t *row0 = slab + (size_t)g * P + sh0, *row1 = slab + (size_t)(g + 8) * P + sh1;
    const int nkb = a.K / 32;
    // K halves (Q4_K on super-block boundaries)
    const int unit = FMT == kQ4_K ? 8 : 1;
    const int kmid = ((nkb / unit) / 2) * unit;
    const int kb_lo = khalf ? kmid : 0, kb_hi = khalf ? nkb : kmid;

    // ---- passes of up to 16 (token, route) pairs of expert e, in routing-table order ----
    for (int l0 = lbeg; l0 < lend; l0 += kMoePass) {
        const int cnt = min(kMoePass, lend - l0);
        if (lane < cnt) plist[warp][lane] = a.bucket[l0 + lane];
        __syncwarp();
        const int nt = (cnt + 7) >> 3;
        const uint4 *xr[2];     // B operand rows: token slot 8j + g
        const float *bsr[2][2];  // block sums of the accumulator's token slots 8j + 2c, 8j + 2c + 1
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int p = plist[warp][min(8 * j + g, cnt - 1)];
            xr[j] = a.xq + (size_t)(SWIGLU ? p / a.k : p) * (a.K / 4) + c;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int p2 = plist[warp][min(8 * j + 2 * c + q, cnt - 1)];
                bsr[j][q] = a.bsum + (size_t)(SWIGLU ? p2 / a.k : p2) * (a.K / 32);
            }
        }
        float acc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        if (nr > 0 && kb_lo < kb_hi) {
            if (FMT == kQ4_K) {
                if (nt == 1) pass_q4k<1>(row0, row1, kb_lo, kb_hi, c, xr, bsr, acc);
                else pass_q4k<2>(row0, row1, kb_lo, kb_hi, c, xr, bsr, acc);
            } else {
                if (nt == 1) pass_blocks<FMT, 1>(row0, row1, kb_lo, kb_hi, c, xr, bsr, acc);
                else pass_blocks<FMT, 2>(row0, row1, kb_lo, kb_hi, c, xr, bsr, acc);
            }
        }
        // ---- the second K half's partial sums join the first's (fixed order: deterministic) ----
        if (khalf) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) red[slab_i][lane][4 * j + q] = acc[j][q];
        }
        __syncthreads();
        if (!khalf) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[j][q] += red[slab_i][lane][4 * j + q];
        }
        // ---- epilogue (first-half warps): acc[j] = rows (g, g + 8) x token slots (8j + 2c, 8j + 2c + 1) ----
        if (SWIGLU) {
            if (warp == 2 || warp == 3) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    su[16 * (warp & 1) + g][8 * j + 2 * c] = acc[j][0];
                    su[16 * (warp & 1) + g][8 * j + 2 * c + 1] = acc[j][1];
                    su[16 * (warp & 1) + g + 8][8 * j + 2 * c] = acc[j][2];
                    su[16 * (warp & 1) + g + 8][8 * j + 2 * c + 1] = acc[j][3];
                }
            }
            __syncthreads();
            if (warp < 2) {
#pragma unroll
                for (int j = 0; j < 2; ++j)
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int slot = 8 * j + 2 * c + (q & 1), rr = g + 8 * (q >> 1);
                        if (slot < cnt && rr < nr) {
                            const int p = plist[warp][slot];
                            const float sc = a.rinv[p / a.k];
                            const float gv = acc[j][q] * sc, uv = su[16 * warp + rr][slot] * sc;
                            a.y[(size_t)p * a.y_stride + wrow0 + rr] = gv / (1.0f + expf(-gv)) * uv;
                        }
                    }
            }
        } else if (!khalf) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int slot = 8 * j + 2 * c + (q & 1), rr = g + 8 * (q >> 1);
                    if (slot < cnt && rr < nr) {
                        const int p = plist[warp][slot];
                        a.y[(size_t)p * a.y_stride + wrow0 + rr] = acc[j][q] * a.rinv[p];
                    }
                }
        }
        __syncthreads();  // red, su and plist are rewritten by the next pass
    }
}

// out[t, h] += total, total = fmaf(y[(t, r), h], w[t, r], total) over t's routes in order.
__global__ void moe_combine_kernel(const float *__restrict__ y, const int *__restrict__ ids, int e_begin,
                                   int n_experts, const float *__restrict__ rw, float *__restrict__ out,
                                   int64_t out_stride, int k, int H) {
    const int t = blockIdx.x;
    for (int h = blockIdx.y * blockDim.x + threadIdx.x; h < H; h += gridDim.y * blockDim.x) {
        float total = 0.f;
        for (int r = 0; r < k; ++r) {
            const int i = t * k + r, le = ids[i] - e_begin;
            if (le >= 0 && le < n_experts) total = fmaf(y[(size_t)i * H + h], rw[i], total);
        }
        out[(size_t)t * out_stride + h] += total;
    }
}

// ids relative to this call's experts: id - e_begin when in [0, n_experts), else -1.
__global__ void moe_local_ids_kernel(const int *__restrict__ ids, int e_begin, int n_experts, int *__restrict__ out,
                                     int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const int le = ids[i] - e_begin;
        out[i] = (le >= 0 && le < n_experts) ? le : -1;
    }
}

template <int FMT, bool SWIGLU>
cudaError_t grouped_launch_t(const MoeArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)4 * 16 * a.row_pitch;  // 4 slabs of 16 rows
    cudaError_t e = cudaFuncSetAttribute(moe_grouped_kernel<FMT, SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    constexpr int RT = SWIGLU ? 32 : 64;
    const dim3 grid((a.rows + RT - 1) / RT, a.n_experts + (SWIGLU ? 1 : 0));
    moe_grouped_kernel<FMT, SWIGLU><<<grid, kMoeThreads, smem, s>>>(a);
    return cudaGetLastError();
}
}  // namespace

cudaError_t moe_xprep_launch(const float *x, int64_t x_stride, uint4 *xq, float *rinv, float *bsum, int rows, int K,
                             cudaStream_t s) {
    moe_xprep_kernel<<<rows, 256, 0, s>>>(x, x_stride, xq, rinv, bsum, K);
    return cudaGetLastError();
}

cudaError_t moe_bucket_launch(const int *ids, int npairs, int e_begin, int n_experts, int *off, int *list,
                              cudaStream_t s) {
    moe_bucket_kernel<<<1, 1024, 0, s>>>(ids, npairs, e_begin, n_experts, off, list);
    return cudaGetLastError();
}
int moe_max_experts() { return kBucketMax - 1; }

cudaError_t moe_local_ids_launch(const int *ids, int e_begin, int n_experts, int *out, int n, cudaStream_t s) {
    moe_local_ids_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, e_begin, n_experts, out, n);
    return cudaGetLastError();
}

// Shared-memory slot of one staged row: the row plus up to 15 bytes of alignment shift, rounded
// to 16 bytes and made = 16 mod 32 (bank spread of the 8 rows a quad of lanes reads at once).
int moe_row_pitch(size_t row_bytes) {
    int p = (int)((row_bytes + 15 + 15) & ~size_t(15));
    if (p % 32 == 0) p += 16;
    return p;
}
int moe_max_row_pitch() { return (232448 - 8192) / 64; }  // 4 warps x 16 rows of dynamic shared memory

cudaError_t moe_grouped_launch(const MoeArgs &a, int fmt, bool swiglu, cudaStream_t s) {
    switch (fmt) {
    case kQ4_0: return swiglu ? grouped_launch_t<kQ4_0, true>(a, s) : grouped_launch_t<kQ4_0, false>(a, s);
    case kQ5_0: return swiglu ? grouped_launch_t<kQ5_0, true>(a, s) : grouped_launch_t<kQ5_0, false>(a, s);
    case kQ8_0: return swiglu ? grouped_launch_t<kQ8_0, true>(a, s) : grouped_launch_t<kQ8_0, false>(a, s);
    case kQ4_K: return swiglu ? grouped_launch_t<kQ4_K, true>(a, s) : grouped_launch_t<kQ4_K, false>(a, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t moe_combine_launch(const float *y, const int *ids, int e_begin, int n_experts, const float *rw,
                               float *out, int64_t out_stride, int tokens, int k, int H, cudaStream_t s) {
    const dim3 grid(tokens, (H + 255) / 256);
    moe_combine_kernel<<<grid, 256, 0, s>>>(y, ids, e_begin, n_experts, rw, out, out_stride, k, H);
    return cudaGetLastError();
}

}  // namespace ql
