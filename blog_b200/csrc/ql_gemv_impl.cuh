// ql_gemv_impl.cuh -- kernel body of the streaming GEMV engine (see ql_gemv.cuh);
// included once per format by ql_gemv_<fmt>.cu so formats compile in parallel.
#pragma once
#include "ql_gemv.cuh"

namespace ql {

// Bit position p at which element k's weight sits after the decoder's single
// AND (see the unit decoders below).  Activations are staged as x * 2^(96-p).
// Q8_0 and Q6_K are decoded to ordinary floats, so their activations are
// staged unscaled (p = 96).
template <int FMT>
__device__ __forceinline__ int weight_bitpos(int k) {
    if (FMT == kQ4_K || FMT == kQ4_0 || FMT == kQ5_0) {
        // low nibble of byte b of a 32-bit word: b0 -> 0, b1 -> 8, b2 -> 16, b3 -> 12 (after >> 12)
        // high nibble:                          b0 -> 4, b1 -> 12, b2 -> 8 (after >> 12), b3 -> 16 (after >> 12)
        const bool hi = (FMT == kQ4_K) ? ((k >> 5) & 1) : ((k >> 4) & 1);
        const uint32_t tab = hi ? 0x10080C04u : 0x0C100800u;
        return (int)((tab >> (8 * (k & 3))) & 0xffu);
    }
    return 96;
}
__device__ __forceinline__ float pow2_dev(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }
__device__ __forceinline__ float dn(uint32_t bits) { return __uint_as_float(bits); }

// ----------------------------------------------------------------------------
// Unit decoders: one GGUF block of one row (this lane) of each of NMAT matrices
// (gate and up share the activation, which is loaded once), against MT tokens.
// ----------------------------------------------------------------------------
// Two bytes of a packed word -> the pair of floats (exact: byte | 2^23 bit pattern, minus 2^23).
__device__ __forceinline__ float2 byte_pair_f(uint32_t w, int b0) {
    const float2 t = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + b0)),
                                 __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + b0 + 1)));
    return fadd2(t, make_float2(-8388608.0f, -8388608.0f));
}

template <int MT, int NMAT>
__device__ __forceinline__ void unit_q4k(const uint8_t *const (&blk)[NMAT], const float *xs, int K, const float *xsum,
                                         int nblk, int k0, float (&acc)[NMAT][MT]) {
    // Per matrix, once per block: d, dmin and the eight 6-bit scales / mins (q4k_scale_min,
    // reference kernel.cu:913-921) as packed bytes: sub-blocks 0-3 in sc03/m03, 4-7 in sc47/m47.
    float2 d2[NMAT], dm2[NMAT];
    uint32_t scw[NMAT][2], mw[NMAT][2];
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat) {
        const uint4 h = *reinterpret_cast<const uint4 *>(blk[mat]);
        const float d = half_bits_to_float(h.x) * pow2f(53), dmin = half_bits_to_float(h.x >> 16);
        d2[mat] = make_float2(d, d);
        dm2[mat] = make_float2(dmin, dmin);
        scw[mat][0] = h.y & 0x3F3F3F3Fu;
        mw[mat][0] = h.z & 0x3F3F3F3Fu;
        scw[mat][1] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        mw[mat][1] = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        // sub-blocks 2p, 2p+1: D = d*sc, M = dmin*m (packed multiplies, the same products as scalar ones)
        float2 D[NMAT], Mn[NMAT];
#pragma unroll
        for (int mat = 0; mat < NMAT; ++mat) {
            D[mat] = fmul2(d2[mat], byte_pair_f(scw[mat][p >> 1], 2 * (p & 1)));
            Mn[mat] = fmul2(dm2[mat], byte_pair_f(mw[mat][p >> 1], 2 * (p & 1)));
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float4 xl[8], xh[8];
            const float4 *xp = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0 + 64 * p);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                xl[i] = xp[i];
                xh[i] = xp[8 + i];
            }
            const float X0 = xsum[(size_t)m * nblk + (k0 >> 5) + 2 * p];
            const float X1 = xsum[(size_t)m * nblk + (k0 >> 5) + 2 * p + 1];
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                // Two packed accumulators (fma.rn.f32x2): a = sub-block 2p, b = 2p+1;
                // each lane of a pair sums every other element, as two scalar chains would.
                const uint4 qa = *reinterpret_cast<const uint4 *>(blk[mat] + 16 + 32 * p);
                const uint4 qb = *reinterpret_cast<const uint4 *>(blk[mat] + 32 + 32 * p);
                const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t w = wq[i], w2 = w >> 12;
                    ffma2(a, make_float2(dn(w & 0x0000000Fu), dn(w & 0x00000F00u)), make_float2(xl[i].x, xl[i].y));
                    ffma2(a, make_float2(dn(w & 0x000F0000u), dn(w2 & 0x0000F000u)), make_float2(xl[i].z, xl[i].w));
                    ffma2(b, make_float2(dn(w & 0x000000F0u), dn(w & 0x0000F000u)), make_float2(xh[i].x, xh[i].y));
                    ffma2(b, make_float2(dn(w2 & 0x00000F00u), dn(w2 & 0x000F0000u)), make_float2(xh[i].z, xh[i].w));
                }
                float r = acc[mat][m];
                r = fmaf(D[mat].x, a.x + a.y, r);
                r = fmaf(D[mat].y, b.x + b.y, r);
                r = fmaf(-Mn[mat].x, X0, r);
                r = fmaf(-Mn[mat].y, X1, r);
                acc[mat][m] = r;
            }
        }
    }
}

// Loads `NW` 32-bit words starting at a 2-byte-aligned shared address.
template <int NW>
__device__ __forceinline__ void load_words_u16aligned(const uint8_t *p, uint32_t (&out)[NW]) {
    const uint32_t *b4 = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3u) * 8u;
    uint32_t r[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) r[i] = b4[i];
#pragma unroll
    for (int i = 0; i < NW; ++i) out[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// Q8_0: value d * q, q a signed byte.  q + 128 is placed in the low byte of the
// float 2^23 (0x4B000000): that float is 2^23 + q + 128 exactly, and one
// subtraction of 2^23 + 128 yields q exactly.  Activations are staged unscaled.
template <int MT, int NMAT>
__device__ __forceinline__ void unit_q80(const uint8_t *const (&blk)[NMAT], const float *xs, int K, const float *,
                                         int, int k0, float (&acc)[NMAT][MT]) {
    float4 xv[MT][8];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[m][i] = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0)[i];
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk[mat]));
        uint32_t wq[8];
        load_words_u16aligned<8>(blk[mat] + 2, wq);
        float e[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = wq[i] ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                e[4 * i + b] = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u + b)) - 8388736.0f;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                a0 = fmaf(e[4 * i + 0], xv[m][i].x, a0);
                a1 = fmaf(e[4 * i + 1], xv[m][i].y, a1);
                a2 = fmaf(e[4 * i + 2], xv[m][i].z, a2);
                a3 = fmaf(e[4 * i + 3], xv[m][i].w, a3);
            }
            acc[mat][m] = fmaf(d, (a0 + a1) + (a2 + a3), acc[mat][m]);
        }
    }
}

// Q4_0: value d * (q - 8), element i < 16 the low nibble of qs[i], i >= 16 the
// high nibble of qs[i - 16] (GGUF block layout; no reference arithmetic).
template <int MT, int NMAT>
__device__ __forceinline__ void unit_q40(const uint8_t *const (&blk)[NMAT], const float *xs, int K, const float *xsum,
                                         int nblk, int k0, float (&acc)[NMAT][MT]) {
    float4 xl[MT][4], xh[MT][4];
    float X[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const float4 *xp = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            xl[m][i] = xp[i];
            xh[m][i] = xp[4 + i];
        }
        X[m] = xsum[(size_t)m * nblk + (k0 >> 5)];
    }
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk[mat]));
        uint32_t wq[4];
        load_words_u16aligned<4>(blk[mat] + 2, wq);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = wq[i], w2 = w >> 12;
                ffma2(a, make_float2(dn(w & 0x0000000Fu), dn(w & 0x00000F00u)), make_float2(xl[m][i].x, xl[m][i].y));
                ffma2(a, make_float2(dn(w & 0x000F0000u), dn(w2 & 0x0000F000u)), make_float2(xl[m][i].z, xl[m][i].w));
                ffma2(b, make_float2(dn(w & 0x000000F0u), dn(w & 0x0000F000u)), make_float2(xh[m][i].x, xh[m][i].y));
                ffma2(b, make_float2(dn(w2 & 0x00000F00u), dn(w2 & 0x000F0000u)), make_float2(xh[m][i].z, xh[m][i].w));
            }
            float r = fmaf(d * pow2f(53), (a.x + a.y) + (b.x + b.y), acc[mat][m]);
            acc[mat][m] = fmaf(-8.0f * d, X[m], r);
        }
    }
}

// Q5_0: q = low nibble | (qh bit k) << 4, value d * (q - 16)  (reference q50_at,
// kernel.cu:1159-1174).  The high bit is moved to bit p+4 next to the nibble at
// bit p, so the 5-bit field decodes as one denormal like Q4_0.
template <int MT, int NMAT>
__device__ __forceinline__ void unit_q50(const uint8_t *const (&blk)[NMAT], const float *xs, int K, const float *xsum,
                                         int nblk, int k0, float (&acc)[NMAT][MT]) {
    float4 xv[MT][8];
    float X[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[m][i] = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0)[i];
        X[m] = xsum[(size_t)m * nblk + (k0 >> 5)];
    }
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat) {
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk[mat]));
        uint32_t wv[5];
        load_words_u16aligned<5>(blk[mat] + 2, wv);
        const uint32_t qh = wv[0];
        float q[32];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = wv[1 + i], w2 = w >> 12;
            const uint32_t nib_lo[4] = {w & 0x0000000Fu, w & 0x00000F00u, w & 0x000F0000u, w2 & 0x0000F000u};
            const uint32_t nib_hi[4] = {w & 0x000000F0u, w & 0x0000F000u, w2 & 0x00000F00u, w2 & 0x000F0000u};
            const int plo[4] = {0, 8, 16, 12}, phi[4] = {4, 12, 8, 16};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int kl = 4 * i + b, kh = 16 + 4 * i + b;  // element indices within the block
                const int tl = plo[b] + 4, th = phi[b] + 4;      // target bit of the high bit
                const uint32_t hl = (tl >= kl ? (qh << (tl - kl)) : (qh >> (kl - tl))) & (1u << tl);
                const uint32_t hh = (th >= kh ? (qh << (th - kh)) : (qh >> (kh - th))) & (1u << th);
                q[kl] = dn(nib_lo[b] | hl);
                q[kh] = dn(nib_hi[b] | hh);
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                a0 = fmaf(q[4 * i + 0], xv[m][i].x, a0);
                a1 = fmaf(q[4 * i + 1], xv[m][i].y, a1);
                a2 = fmaf(q[4 * i + 2], xv[m][i].z, a2);
                a3 = fmaf(q[4 * i + 3], xv[m][i].w, a3);
            }
            float r = fmaf(d * pow2f(53), (a0 + a1) + (a2 + a3), acc[mat][m]);
            acc[mat][m] = fmaf(-16.0f * d, X[m], r);
        }
    }
}

// Q6_K: reference q6k_at (kernel.cu:1122-1156); byte-granular (block starts are
// only 2-byte aligned).  Activations are staged unscaled for this format.
template <int MT, int NMAT>
__device__ __forceinline__ void unit_q6k(const uint8_t *const (&blk)[NMAT], const float *xs, int K, const float *,
                                         int, int k0, float (&acc)[NMAT][MT]) {
#pragma unroll
    for (int mat = 0; mat < NMAT; ++mat) {
        const uint8_t *ql = blk[mat], *qh = blk[mat] + 128;
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk[mat] + 192);
        const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk[mat] + 208));
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
            const int n = half * 128;
#pragma unroll 1
            for (int is = 0; is < 2; ++is) {
                float s[MT][4];
#pragma unroll
                for (int m = 0; m < MT; ++m) s[m][0] = s[m][1] = s[m][2] = s[m][3] = 0.f;
#pragma unroll 4
                for (int l = 16 * is; l < 16 * is + 16; ++l) {
                    const uint32_t a = ql[n / 2 + l], b = ql[n / 2 + l + 32], c = qh[n / 4 + l];
                    const float q1 = (float)((int)((a & 0xF) | ((c & 3) << 4)) - 32);
                    const float q2 = (float)((int)((b & 0xF) | (((c >> 2) & 3) << 4)) - 32);
                    const float q3 = (float)((int)((a >> 4) | (((c >> 4) & 3) << 4)) - 32);
                    const float q4 = (float)((int)((b >> 4) | (((c >> 6) & 3) << 4)) - 32);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const float *x = xs + (size_t)m * K + k0 + n + l;
                        s[m][0] = fmaf(q1, x[0], s[m][0]);
                        s[m][1] = fmaf(q2, x[32], s[m][1]);
                        s[m][2] = fmaf(q3, x[64], s[m][2]);
                        s[m][3] = fmaf(q4, x[96], s[m][3]);
                    }
                }
                const int8_t *scg = sc + n / 16 + is;
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int g = 0; g < 4; ++g) acc[mat][m] = fmaf(d * (float)scg[2 * g], s[m][g], acc[mat][m]);
            }
        }
    }
}

template <int FMT, int MT, int NMAT>
__device__ __forceinline__ void unit_dispatch(const uint8_t *const (&blk)[NMAT], const float *xs, int K,
                                              const float *xsum, int nblk, int k0, float (&acc)[NMAT][MT]) {
    if (FMT == kQ4_K) unit_q4k<MT, NMAT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ8_0) unit_q80<MT, NMAT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ4_0) unit_q40<MT, NMAT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ5_0) unit_q50<MT, NMAT>(blk, xs, K, xsum, nblk, k0, acc);
    else unit_q6k<MT, NMAT>(blk, xs, K, xsum, nblk, k0, acc);
}

// Copies n bytes global -> shared with the widest accesses the (shared)
// alignment allows; source and destination have equal address mod 16.
__device__ __forceinline__ void copy_ragged(uint8_t *dst, const uint8_t *src, int n) {
    while (n > 0) {
        const uintptr_t ad = reinterpret_cast<uintptr_t>(src);
        if ((ad & 7) == 0 && n >= 8) {
            *reinterpret_cast<uint64_t *>(dst) = __ldg(reinterpret_cast<const unsigned long long *>(src));
            dst += 8; src += 8; n -= 8;
        } else if ((ad & 3) == 0 && n >= 4) {
            *reinterpret_cast<uint32_t *>(dst) = __ldg(reinterpret_cast<const unsigned int *>(src));
            dst += 4; src += 4; n -= 4;
        } else if ((ad & 1) == 0 && n >= 2) {
            *reinterpret_cast<uint16_t *>(dst) = __ldg(reinterpret_cast<const unsigned short *>(src));
            dst += 2; src += 2; n -= 2;
        } else {
            *dst = __ldg(src);
            dst += 1; src += 1; n -= 1;
        }
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int FMT, int MT, int NMAT, int SRC, int EPI, bool TMA>
__global__ void __launch_bounds__(kGemvThreads, 1) qgemv_kernel(const __grid_constant__ GemvArgs a) {
    // Warp roles.  TMA: warp 0 produces (one thread), warp 1 finishes row groups,
    // warps 2..15 consume.  cp.async: warps 0..3 produce, warp 4 finishes, 5..15 consume.
    constexpr int NPW = gemv_producer_warps(TMA), EW = NPW, CW0 = NPW + 1;
    constexpr int W = gemv_consumer_warps(TMA);
    constexpr int SEG = stage_seg(FMT, TMA), PITCH = stage_pitch(FMT, TMA);
    constexpr int BB = block_bytes(FMT), BE = block_elems(FMT);
    constexpr int STAGE_BYTES = NMAT * kRowGroup * PITCH;
    constexpr int RED = W * MT * NMAT * kRowGroup;  // floats per reduction buffer
    extern __shared__ __align__(1024) uint8_t smem[];

    const int NST = a.nst;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);       // [kGemvStages]
    uint64_t *empty = full + kGemvStages;                        // [kGemvStages]
    uint64_t *red_full = empty + kGemvStages;                    // [2]
    uint64_t *red_empty = red_full + 2;                          // [2]
    uint64_t *x_ready = red_empty + 2;                           // [1] activations staged
    int *abort_flag = reinterpret_cast<int *>(x_ready + 1);
    float *inv_rms = reinterpret_cast<float *>(smem + 112);      // [kGemvMaxTokens]
    float *ss_part = reinterpret_cast<float *>(smem + 128);      // [W][kGemvMaxTokens] sums of squares
    const int K = a.K, nblk = K / 32;
    size_t off = kGemvHeaderBytes;
    float *xs = reinterpret_cast<float *>(smem + off);
    off += ((size_t)MT * K * 4 + 127) / 128 * 128;
    float *xsum = reinterpret_cast<float *>(smem + off);
    off += ((size_t)MT * nblk * 4 + 127) / 128 * 128;
    float *red = reinterpret_cast<float *>(smem + off);  // [2][W][MT][NMAT][32]
    off += ((size_t)2 * RED * 4 + 127) / 128 * 128;
    uint8_t *stages = smem + off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t t0 = plan_start(a.plan, blockIdx.x), t1 = plan_start(a.plan, blockIdx.x + 1);
    const int U = a.U;
    const int upr = (SRC == kSrcIndexedK) ? a.units_per_route : 0;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            // cp.async: every producer lane arrives twice; TMA: one expect-tx arrival
            mbar_init(&full[s], TMA ? 1 : 64 * NPW);
            mbar_init(&empty[s], W);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&red_full[b], W);
            mbar_init(&red_empty[b], 1);
        }
        mbar_init(x_ready, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Let the next kernel in the stream start its weight prefetch early; every
    // read of data another kernel writes (activations, expert ids, outputs,
    // workspace) happens after griddepcontrol.wait below.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (TMA && warp < NPW) {
        // ---------------------------- producer (TMA) ----------------------------
        // One thread issues one box per matrix per stage (Q4_K: 3-D; 32-element formats: 2-D from the
        // 16-byte boundary at or before the stage's first block).
        if (lane != 0) return;
        if (SRC != kSrcPlain) asm volatile("griddepcontrol.wait;" ::: "memory");  // expert ids
        int64_t t = t0;
        Stage st;
        int it = 0;
        constexpr uint32_t BOX = kRowGroup * PITCH;
        while (next_stage(t, t1, U, SEG, upr, st)) {
            const int slot = it % NST;
            const uint32_t ph = (uint32_t)(it / NST) & 1u;
            // After the first pre_x stages, let the activation loads go first.
            if (it == a.pre_x && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(x_ready, 0u, a.err, kErrWaitFull)) *abort_flag = 1;
            }
            if (it >= NST && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&empty[slot], ph ^ 1u, a.err, kErrWaitEmpty)) *abort_flag = 1;
            }
            const bool aborted = *reinterpret_cast<volatile int *>(abort_flag) != 0;
            int row0 = st.g * kRowGroup, blk0 = st.us, map = 0;
            bool live = !aborted;
            if (SRC == kSrcStacked) {
                map = stacked_source(a, row0, &row0);
            } else if (SRC == kSrcIndexedRows) {  // a row group never straddles a route here
                const int r = row0 / a.rows_per_route, e = a.ids[r];
                live = live && e >= 0;
                row0 = e * a.rows_per_route + (row0 - r * a.rows_per_route);
            } else if (SRC == kSrcIndexedK) {
                const int r = st.us / a.units_per_route, e = a.ids[r];
                live = live && e >= 0;
                row0 = e * a.rows + row0;
                blk0 = st.us - r * a.units_per_route;
            }
            mbar_arrive_expect_tx(&full[slot], live ? NMAT * BOX : 0u);
            if (live) {
                uint8_t *sbase = stages + slot * STAGE_BYTES;
#pragma unroll
                for (int mat = 0; mat < NMAT; ++mat) {
                    if (FMT == kQ4_K)
                        tma_load_3d(sbase + mat * BOX, &a.tmap[SRC == kSrcStacked ? map : mat], 0, blk0, row0,
                                    &full[slot]);
                    else if (!a.tma_pair)  // x in 8-byte elements: the 16-byte chunk holding the stage's first byte
                        tma_box2d(sbase + mat * BOX, &a.tmap[SRC == kSrcStacked ? map : mat], ((blk0 * BB) >> 4) << 1,
                                  row0, &full[slot]);
                    else {  // super-rows of two rows: even rows from the stage's offset, odd rows one row later
                        const int src = SRC == kSrcStacked ? map : mat;
                        const int rb = (int)a.row_bytes[src];
                        tma_box2d(sbase + mat * BOX, &a.tmap[src], ((blk0 * BB) >> 4) << 1, row0 >> 1, &full[slot]);
                        tma_box2d(sbase + mat * BOX + (BOX >> 1), &a.tmap[src], ((rb + blk0 * BB) >> 4) << 1, row0 >> 1,
                                  &full[slot]);
                    }
                }
            }
            ++it;
        }
        for (int j = (it > NST ? it - NST : 0); j < it; ++j)
            mbar_wait(&full[j % NST], (uint32_t)(j / NST) & 1u, nullptr, 0);
        return;
    }

    if (!TMA && warp < NPW) {
        // ------------------------------- producer -------------------------------
        // Each row's run of blocks is copied with coalesced 16-byte cp.async
        // (consecutive threads take consecutive 16-byte chunks); the ragged
        // head/tail bytes of unaligned runs are copied by warp 0, lane = row.
        // Every producer lane arrives twice per stage on the stage's full
        // barrier: once when its cp.asyncs land, once after its plain stores.
        if (SRC != kSrcPlain) asm volatile("griddepcontrol.wait;" ::: "memory");  // expert ids
        const uint64_t pol = l2_evict_first_policy();
        int64_t t = t0;
        Stage st;
        int it = 0;
        while (next_stage(t, t1, U, SEG, upr, st)) {
            const int slot = it % NST;
            const uint32_t ph = (uint32_t)(it / NST) & 1u;
            // After the first pre_x stages, let the activation loads go first.
            if (it == a.pre_x && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(x_ready, 0u, a.err, kErrWaitFull)) *abort_flag = 1;
            }
            if (it >= NST && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&empty[slot], ph ^ 1u, a.err, kErrWaitEmpty)) *abort_flag = 1;
            }
            const bool aborted = *reinterpret_cast<volatile int *>(abort_flag) != 0;
            uint8_t *sbase = stages + slot * STAGE_BYTES;
            const int len = (st.ue - st.us) * BB;
            if (!aborted) {
                const int NC = len >> 4;  // no row's aligned interior exceeds len / 16 chunks
#pragma unroll
                for (int mat = 0; mat < NMAT; ++mat) {
                    // this lane's row (lane = row): source, aligned interior, ragged bytes
                    const int v = st.g * kRowGroup + lane;
                    const uint8_t *src = v < a.rows ? gemv_block_ptr<SRC, FMT>(a, a.ids, mat, v, st.us) : nullptr;
                    const uintptr_t A = reinterpret_cast<uintptr_t>(src);
                    const uintptr_t lo = (A + 15) & ~uintptr_t(15), hi = (A + len) & ~uintptr_t(15);
                    const int nch = (src != nullptr && hi > lo) ? (int)((hi - lo) >> 4) : 0;
                    uint8_t *rowbase = sbase + (mat * kRowGroup + lane) * PITCH;  // byte A at rowbase + (A & 15)
                    const uint32_t dlo = smem_u32(rowbase + (lo - (A & ~uintptr_t(15))));
                    // interior: chunk idx = r * NC + c over all rows, consecutive threads -> consecutive chunks
                    constexpr int PT = 32 * NPW;
                    const int ptid = warp * 32 + lane;
                    int r = ptid / (NC > 0 ? NC : 1), c = ptid - r * (NC > 0 ? NC : 1);
                    for (int idx0 = warp * 32; idx0 < kRowGroup * NC; idx0 += PT) {
                        const uintptr_t lo_r = __shfl_sync(0xffffffffu, lo, r);
                        const uint32_t d_r = __shfl_sync(0xffffffffu, dlo, r);
                        const int n_r = __shfl_sync(0xffffffffu, nch, r);
                        if (c < n_r)
                            asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(
                                             d_r + 16u * (uint32_t)c),
                                         "l"(lo_r + 16 * (uintptr_t)c), "l"(pol)
                                         : "memory");
                        c += PT;
                        while (c >= NC) { c -= NC; ++r; }
                    }
                    if (src != nullptr && warp == 0) {
                        uint8_t *row = rowbase + (A & 15);
                        if (hi > lo) {
                            copy_ragged(row, src, (int)(lo - A));
                            copy_ragged(row + (hi - A), src + (hi - A), (int)(A + len - hi));
                        } else {
                            copy_ragged(row, src, len);
                        }
                    }
                }
            }
            cp_async_mbar_arrive(&full[slot]);
            mbar_arrive(&full[slot]);
            ++it;
        }
        // Drain: never leave the CTA with copies in flight.
        for (int j = (it > NST ? it - NST : 0); j < it; ++j)
            mbar_wait(&full[j % NST], (uint32_t)(j / NST) & 1u, nullptr, 0);
        return;
    }

    if (warp == EW) {
        // ---------------------------- row-group finisher ----------------------------
        // Sums the consumer warps' partials of each row group in fixed warp order,
        // then stores the result (single-CTA group) or runs the stream-K fixup:
        // the last CTA to finish a shared group sums all parts in K order.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        int gi = 0;
        for (int64_t gg = t0 / U; gg * U < t1; ++gg, ++gi) {
            const int g = (int)gg;
            const int bsel = gi & 1;
            bool ok = !*reinterpret_cast<volatile int *>(abort_flag);
            if (ok && !mbar_wait(&red_full[bsel], (uint32_t)(gi >> 1) & 1u, a.err, kErrWaitFull)) {
                *abort_flag = 1;
                ok = false;
            }
            float val[NMAT][MT];
            const float *rb = red + bsel * RED;
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    float sum = 0.f;
                    for (int w = 0; w < W; ++w) sum += rb[((w * MT + m) * NMAT + mat) * kRowGroup + lane];
                    val[mat][m] = sum;
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_empty[bsel]);
            const int64_t gs = (int64_t)g * U, ge = gs + U;
            bool finish = ok;
            if (ok && (gs < t0 || ge > t1)) {
                const int si = (g == (int)(t0 / U)) ? 0 : 1;
                float *pp = a.part + ((size_t)blockIdx.x * 2 + si) * (MT * NMAT * kRowGroup);
#pragma unroll
                for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                    for (int m = 0; m < MT; ++m) pp[(m * NMAT + mat) * kRowGroup + lane] = val[mat][m];
                __threadfence();
                __syncwarp();
                const int cf = plan_cta_of(a.plan, gs), cl = plan_cta_of(a.plan, ge - 1);
                unsigned prev = 0;
                if (lane == 0) prev = atomicAdd(&a.counters[g], 1u);
                prev = __shfl_sync(0xffffffffu, prev, 0);
                finish = (prev == (unsigned)(cl - cf));
                if (finish) {
                    __threadfence();
#pragma unroll
                    for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                        for (int m = 0; m < MT; ++m) val[mat][m] = 0.f;
                    for (int c = cf; c <= cl; ++c) {
                        const int sj = (g == (int)(plan_start(a.plan, c) / U)) ? 0 : 1;
                        const float *qp = a.part + ((size_t)c * 2 + sj) * (MT * NMAT * kRowGroup);
#pragma unroll
                        for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                            for (int m = 0; m < MT; ++m)
                                val[mat][m] += __ldcg(qp + (m * NMAT + mat) * kRowGroup + lane);
                    }
                    if (lane == 0) a.counters[g] = 0u;
                }
            }
            const int v = g * kRowGroup + lane;
            if (finish && v < a.rows) {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    float *yp = a.y + (size_t)m * a.y_stride + v;
                    const float nrm = a.gamma != nullptr ? inv_rms[m] : 1.0f;  // fused RMSNorm factor
                    if (EPI == kEpiSwiglu) {
                        const float gv = val[0][m] * nrm, uv = val[NMAT - 1][m] * nrm;
                        float o = gv / (1.0f + expf(-gv)) * uv;
                        if (SRC == kSrcIndexedRows && a.ids[v / a.rows_per_route] < 0) o = 0.f;
                        *yp = o;
                    } else {
                        float o = val[0][m] * nrm;
                        if (a.bias != nullptr) o += a.bias[v];
                        if (EPI == kEpiAdd) *yp += o;
                        else if (a.y != nullptr) *yp = o;
                        val[0][m] = o;
                    }
                }
            }
            if (EPI == kEpiStore && a.amax.amax != nullptr && finish) {  // fused greedy argmax
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    unsigned long long k = v < a.rows ? amax_key(val[0][m], (uint32_t)(v + a.amax.offset)) : 0ull;
                    k = warp_max_u64(k);
                    if (lane == 0 && k != 0ull) atomicMax(&a.amax.amax[m], k);
                }
            }
        }
        if (EPI == kEpiStore && a.amax.amax != nullptr && lane == 0) amax_cta_done(a.amax, a.M);
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int cw = warp - CW0;
    const int nthr = W * 32;
    const int ctid = tid - 32 * CW0;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // activations come from the previous kernel

    // Prologue, one pass over x: stage x * g * 2^(96-p) (float4 per thread, loads
    // issued in batches) and the 32-element block sums of x * g (8-lane reduce).
    // With a fused RMSNorm the pass also sums x^2; the norm factor
    // 1/sqrt(mean(x^2) + eps) is one scalar per token, so the finisher applies it
    // to the finished dot products and nothing here waits for it.
    constexpr int B = 12;  // float4 loads in flight per thread: K <= 21504 stages in one round trip
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) ss[m] = 0.f;
    {
        const int nch = MT * (K / 4);
        // The loop bound is warp-uniform (the shuffles below need every lane);
        // lanes past the end are masked by `ok`.
        for (int j0 = ctid; j0 - lane < nch; j0 += B * nthr) {
            float4 v[B], gv[B];
#pragma unroll
            for (int u = 0; u < B; ++u) {
                const int j = j0 + u * nthr;
                v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                gv[u] = make_float4(1.f, 1.f, 1.f, 1.f);
                if (j < nch) {
                    const int m = j / (K / 4), k = 4 * (j - m * (K / 4));
                    if (a.gamma != nullptr) gv[u] = *reinterpret_cast<const float4 *>(a.gamma + k);  // with x: one round trip
                    if (SRC == kSrcIndexedK) {
                        const int F = a.units_per_route * BE;
                        const int r = k / F;
                        if (a.ids[r] >= 0) {
                            v[u] = *reinterpret_cast<const float4 *>(a.x + (size_t)r * a.x_stride + (k - r * F));
                            const float rw = a.route_w[r];
                            v[u].x *= rw; v[u].y *= rw; v[u].z *= rw; v[u].w *= rw;
                        }
                    } else {
                        v[u] = *reinterpret_cast<const float4 *>(a.x + (size_t)m * a.x_stride + k);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < B; ++u) {
                const int j = j0 + u * nthr;
                const bool ok = j < nch;
                const int m = ok ? j / (K / 4) : 0, k = ok ? 4 * (j - m * (K / 4)) : 0;
                float4 xv = v[u];
                if (ok && a.gamma != nullptr) {
                    const float q = fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, fmaf(xv.z, xv.z, xv.w * xv.w)));
#pragma unroll
                    for (int mm = 0; mm < MT; ++mm)
                        if (mm == m) ss[mm] += q;
                    const float4 g = gv[u];
                    xv.x *= g.x; xv.y *= g.y; xv.z *= g.z; xv.w *= g.w;
                }
                float bs = (xv.x + xv.y) + (xv.z + xv.w);
                bs += __shfl_xor_sync(0xffffffffu, bs, 1);
                bs += __shfl_xor_sync(0xffffffffu, bs, 2);
                bs += __shfl_xor_sync(0xffffffffu, bs, 4);
                if (ok) {
                    float4 o;
                    o.x = xv.x * pow2_dev(96 - weight_bitpos<FMT>(k + 0));
                    o.y = xv.y * pow2_dev(96 - weight_bitpos<FMT>(k + 1));
                    o.z = xv.z * pow2_dev(96 - weight_bitpos<FMT>(k + 2));
                    o.w = xv.w * pow2_dev(96 - weight_bitpos<FMT>(k + 3));
                    *reinterpret_cast<float4 *>(xs + (size_t)m * K + k) = o;
                    if ((k & 31) == 0) xsum[(size_t)m * nblk + (k >> 5)] = bs;
                }
            }
        }
    }
    if (a.gamma != nullptr) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float w = warp_sum(ss[m]);
            if (lane == 0) ss_part[cw * kGemvMaxTokens + m] = w;
        }
    }
    named_bar_sync(1, nthr);
    if (ctid == 0) mbar_arrive(x_ready);  // the producer may issue the rest of its stages
    if (a.gamma != nullptr && cw == 0) {
        for (int m = 0; m < MT; ++m) {
            const float tsum = warp_sum(lane < W ? ss_part[lane * kGemvMaxTokens + m] : 0.f);
            if (lane == 0) inv_rms[m] = rsqrtf(tsum / (float)K + a.eps);
        }
    }

    float acc[NMAT][MT];
#pragma unroll
    for (int i = 0; i < NMAT; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.f;

    int64_t t = t0;
    Stage st;
    int it = 0, ucount = 0, gi = 0;
    while (next_stage(t, t1, U, SEG, upr, st)) {
        const int slot = it % NST;
        const uint32_t ph = (uint32_t)(it / NST) & 1u;
        if (!*reinterpret_cast<volatile int *>(abort_flag)) {
            if (!mbar_wait(&full[slot], ph, a.err, kErrWaitFull)) *abort_flag = 1;
        }
        const int n = st.ue - st.us;
        const int v = st.g * kRowGroup + lane;
        const bool aborted = *reinterpret_cast<volatile int *>(abort_flag) != 0;
        if (!aborted && v < a.rows) {
            const int first = ((cw - ucount) % W + W) % W;
            const uint8_t *rowp[NMAT];
            bool live = true;
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                const uint8_t *rs = gemv_block_ptr<SRC, FMT>(a, a.ids, mat, v, st.us);
                live = live && (rs != nullptr);
                // row slot of this lane: paired tensor-map stages hold the even rows, then the odd rows
                const int rsl = (TMA && FMT != kQ4_K && a.tma_pair) ? ((lane & 1) << 4) | (lane >> 1) : lane;
                rowp[mat] = stages + slot * STAGE_BYTES + (mat * kRowGroup + rsl) * PITCH +
                            (reinterpret_cast<uintptr_t>(rs) & 15);
            }
            if (live) {
                for (int lu = first; lu < n; lu += W) {
                    const uint8_t *bp[NMAT];
#pragma unroll
                    for (int mat = 0; mat < NMAT; ++mat) bp[mat] = rowp[mat] + lu * BB;
                    unit_dispatch<FMT, MT, NMAT>(bp, xs, K, xsum, nblk, (st.us + lu) * BE, acc);
                }
            }
        }
        ucount += n;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++it;

        if (st.last_in_group) {
            // hand the partials to the finisher warp (double-buffered)
            const int bsel = gi & 1;
            if (gi >= 2 && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&red_empty[bsel], (uint32_t)((gi >> 1) - 1) & 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
            }
            float *rb = red + bsel * RED;
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    rb[((cw * MT + m) * NMAT + mat) * kRowGroup + lane] = acc[mat][m];
                    acc[mat][m] = 0.f;
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_full[bsel]);
            ++gi;
        }
    }
}

// ----------------------------------------------------------------------------
// Host launchers for one format.  Indexed sources run one token (decode).
// ----------------------------------------------------------------------------
template <int FMT, int MT, int NMAT, int SRC, int EPI, bool TMA>
static cudaError_t launch_typed(const GemvArgs &a, int smem, cudaStream_t stream) {
    auto k = qgemv_kernel<FMT, MT, NMAT, SRC, EPI, TMA>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    // Programmatic dependent launch: this kernel may start while the previous
    // kernel in the stream drains (it waits with griddepcontrol.wait before
    // reading anything that kernel writes).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.plan.C);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = gemv_pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, a);
}

template <int FMT, int MT, int NMAT, int SRC, int EPI>
static cudaError_t launch_tma(const GemvArgs &a, bool tma, int smem, cudaStream_t s) {
    if (tma_format(FMT) && tma) return launch_typed<FMT, MT, NMAT, SRC, EPI, true>(a, smem, s);
    return launch_typed<FMT, MT, NMAT, SRC, EPI, false>(a, smem, s);
}

template <int FMT, int NMAT, int SRC, int EPI>
static cudaError_t launch_mt(const GemvArgs &a, int MT, bool tma, int smem, cudaStream_t s) {
    switch (MT) {
    case 1: return launch_tma<FMT, 1, NMAT, SRC, EPI>(a, tma, smem, s);
    case 2: return launch_tma<FMT, 2, NMAT, SRC, EPI>(a, tma, smem, s);
    case 3: return launch_tma<FMT, 3, NMAT, SRC, EPI>(a, tma, smem, s);
    default: return launch_tma<FMT, 4, NMAT, SRC, EPI>(a, tma, smem, s);
    }
}

// kind: 0 plain store, 1 plain add, 2 plain SwiGLU pair, 3 indexed-rows SwiGLU
// pair (MT = 1), 4 indexed-K add (MT = 1), 5 stacked sources store.  `tma` selects tensor-map staging
// (Q4_K, Q4_0, Q5_0, Q8_0; the caller has filled a.tmap).
template <int FMT>
cudaError_t gemv_launch_fmt(int kind, const GemvArgs &a, int MT, bool tma, int smem, cudaStream_t s) {
    switch (kind) {
    case 0: return launch_mt<FMT, 1, kSrcPlain, kEpiStore>(a, MT, tma, smem, s);
    case 1: return launch_mt<FMT, 1, kSrcPlain, kEpiAdd>(a, MT, tma, smem, s);
    case 2: return launch_mt<FMT, 2, kSrcPlain, kEpiSwiglu>(a, MT, tma, smem, s);
    case 3: return MT == 1 ? launch_tma<FMT, 1, 2, kSrcIndexedRows, kEpiSwiglu>(a, tma, smem, s) : cudaErrorInvalidValue;
    case 4: return MT == 1 ? launch_tma<FMT, 1, 1, kSrcIndexedK, kEpiAdd>(a, tma, smem, s) : cudaErrorInvalidValue;
    case 5: return launch_mt<FMT, 1, kSrcStacked, kEpiStore>(a, MT, tma, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace ql
