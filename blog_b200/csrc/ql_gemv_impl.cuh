// ql_gemv_impl.cuh -- kernel body of the streaming GEMV engine (see ql_gemv.cuh);
// included once per format by ql_gemv_<fmt>.cu so formats compile in parallel.
#pragma once
#include "ql_gemv.cuh"

namespace ql {

// Bit position p at which element k's weight sits after the decoder's single
// AND (see the unit decoders below).  Activations are staged as x * 2^(96-p).
// Q6_K is decoded to ordinary floats, so its activations are staged unscaled.
template <int FMT>
__device__ __forceinline__ int weight_bitpos(int k) {
    if (FMT == kQ8_0) return 8 * (k & 1);
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
// Unit decoders: one GGUF block of one row (lane) against MT staged tokens.
// ----------------------------------------------------------------------------
template <int MT>
__device__ __forceinline__ void unit_q4k(const uint8_t *blk, const float *xs, int K, const float *xsum, int nblk,
                                         int k0, float *acc) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const float d = half_bits_to_float(h.x) * pow2f(53);
    const float dmin = half_bits_to_float(h.x >> 16);
    const uint32_t sA = h.y, sB = h.z, sC = h.w;  // scale bytes 0-3, 4-7, 8-11
#pragma unroll
    for (int p = 0; p < 4; ++p) {
        // q4k_scale_min (reference kernel.cu:913-921) for sub-blocks 2p and 2p+1
        uint32_t sc0, m0, sc1, m1;
        if (p < 2) {
            const int j0 = 2 * p, j1 = 2 * p + 1;
            sc0 = (sA >> (8 * j0)) & 63u; m0 = (sB >> (8 * j0)) & 63u;
            sc1 = (sA >> (8 * j1)) & 63u; m1 = (sB >> (8 * j1)) & 63u;
        } else {
            const int j0 = 2 * p - 4, j1 = 2 * p - 3;  // j - 4
            sc0 = ((sC >> (8 * j0)) & 0x0Fu) | (((sA >> (8 * j0 + 6)) & 3u) << 4);
            m0 = ((sC >> (8 * j0 + 4)) & 0x0Fu) | (((sB >> (8 * j0 + 6)) & 3u) << 4);
            sc1 = ((sC >> (8 * j1)) & 0x0Fu) | (((sA >> (8 * j1 + 6)) & 3u) << 4);
            m1 = ((sC >> (8 * j1 + 4)) & 0x0Fu) | (((sB >> (8 * j1 + 6)) & 3u) << 4);
        }
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
        const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        float lo[32], hi[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = wq[i], w2 = w >> 12;
            lo[4 * i + 0] = dn(w & 0x0000000Fu);
            lo[4 * i + 1] = dn(w & 0x00000F00u);
            lo[4 * i + 2] = dn(w & 0x000F0000u);
            lo[4 * i + 3] = dn(w2 & 0x0000F000u);
            hi[4 * i + 0] = dn(w & 0x000000F0u);
            hi[4 * i + 1] = dn(w & 0x0000F000u);
            hi[4 * i + 2] = dn(w2 & 0x00000F00u);
            hi[4 * i + 3] = dn(w2 & 0x000F0000u);
        }
        const float D0 = d * (float)sc0, D1 = d * (float)sc1;
        const float M0 = dmin * (float)m0, M1 = dmin * (float)m1;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float4 *xl = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0 + 64 * p);
            const float4 *xh = xl + 8;
            float2 aL0 = make_float2(0.f, 0.f), aL1 = aL0, aH0 = aL0, aH1 = aL0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 a = xl[i], b = xh[i];
                ffma2(aL0, make_float2(lo[4 * i], lo[4 * i + 1]), make_float2(a.x, a.y));
                ffma2(aL1, make_float2(lo[4 * i + 2], lo[4 * i + 3]), make_float2(a.z, a.w));
                ffma2(aH0, make_float2(hi[4 * i], hi[4 * i + 1]), make_float2(b.x, b.y));
                ffma2(aH1, make_float2(hi[4 * i + 2], hi[4 * i + 3]), make_float2(b.z, b.w));
            }
            const float SL = (aL0.x + aL0.y) + (aL1.x + aL1.y);
            const float SH = (aH0.x + aH0.y) + (aH1.x + aH1.y);
            const float *X = xsum + (size_t)m * nblk + (k0 >> 5) + 2 * p;
            acc[m] = fmaf(D0, SL, acc[m]);
            acc[m] = fmaf(D1, SH, acc[m]);
            acc[m] = fmaf(-M0, X[0], acc[m]);
            acc[m] = fmaf(-M1, X[1], acc[m]);
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

template <int MT>
__device__ __forceinline__ void unit_q80(const uint8_t *blk, const float *xs, int K, const float *xsum, int nblk,
                                         int k0, float *acc) {
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
    const float dD = d * pow2f(53);
    uint32_t wq[8];
    load_words_u16aligned<8>(blk + 2, wq);
    float e[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = wq[i] ^ 0x80808080u, w2 = w >> 16;  // q + 128 as unsigned bytes
        e[4 * i + 0] = dn(w & 0xFFu);
        e[4 * i + 1] = dn(w & 0xFF00u);
        e[4 * i + 2] = dn(w2 & 0xFFu);
        e[4 * i + 3] = dn(w2 & 0xFF00u);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const float4 *xv = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0);
        float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = xv[i];
            ffma2(a0, make_float2(e[4 * i], e[4 * i + 1]), make_float2(a.x, a.y));
            ffma2(a1, make_float2(e[4 * i + 2], e[4 * i + 3]), make_float2(a.z, a.w));
        }
        const float S = (a0.x + a0.y) + (a1.x + a1.y);
        acc[m] = fmaf(dD, S, acc[m]);
        acc[m] = fmaf(-128.0f * d, xsum[(size_t)m * nblk + (k0 >> 5)], acc[m]);
    }
}

template <int MT>
__device__ __forceinline__ void unit_q40(const uint8_t *blk, const float *xs, int K, const float *xsum, int nblk,
                                         int k0, float *acc) {
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
    const float dD = d * pow2f(53);
    uint32_t wq[4];
    load_words_u16aligned<4>(blk + 2, wq);
    float lo[16], hi[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t w = wq[i], w2 = w >> 12;
        lo[4 * i + 0] = dn(w & 0x0000000Fu);
        lo[4 * i + 1] = dn(w & 0x00000F00u);
        lo[4 * i + 2] = dn(w & 0x000F0000u);
        lo[4 * i + 3] = dn(w2 & 0x0000F000u);
        hi[4 * i + 0] = dn(w & 0x000000F0u);
        hi[4 * i + 1] = dn(w & 0x0000F000u);
        hi[4 * i + 2] = dn(w2 & 0x00000F00u);
        hi[4 * i + 3] = dn(w2 & 0x000F0000u);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const float4 *xl = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0);
        const float4 *xh = xl + 4;
        float2 a0 = make_float2(0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = xl[i], b = xh[i];
            ffma2(a0, make_float2(lo[4 * i], lo[4 * i + 1]), make_float2(a.x, a.y));
            ffma2(a1, make_float2(lo[4 * i + 2], lo[4 * i + 3]), make_float2(a.z, a.w));
            ffma2(a2, make_float2(hi[4 * i], hi[4 * i + 1]), make_float2(b.x, b.y));
            ffma2(a3, make_float2(hi[4 * i + 2], hi[4 * i + 3]), make_float2(b.z, b.w));
        }
        const float S = ((a0.x + a0.y) + (a1.x + a1.y)) + ((a2.x + a2.y) + (a3.x + a3.y));
        acc[m] = fmaf(dD, S, acc[m]);
        acc[m] = fmaf(-8.0f * d, xsum[(size_t)m * nblk + (k0 >> 5)], acc[m]);
    }
}

// Q5_0: q = low nibble | (qh bit k) << 4, value d * (q - 16)  (reference q50_at,
// kernel.cu:1159-1174).  The high bit is moved to bit p+4 next to the nibble at
// bit p, so the 5-bit field decodes as one denormal like Q4_0.
template <int MT>
__device__ __forceinline__ void unit_q50(const uint8_t *blk, const float *xs, int K, const float *xsum, int nblk,
                                         int k0, float *acc) {
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
    const float dD = d * pow2f(53);
    uint32_t wv[5];
    load_words_u16aligned<5>(blk + 2, wv);
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
        const float4 *xv = reinterpret_cast<const float4 *>(xs + (size_t)m * K + k0);
        float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = xv[i];
            ffma2(a0, make_float2(q[4 * i], q[4 * i + 1]), make_float2(a.x, a.y));
            ffma2(a1, make_float2(q[4 * i + 2], q[4 * i + 3]), make_float2(a.z, a.w));
        }
        const float S = (a0.x + a0.y) + (a1.x + a1.y);
        acc[m] = fmaf(dD, S, acc[m]);
        acc[m] = fmaf(-16.0f * d, xsum[(size_t)m * nblk + (k0 >> 5)], acc[m]);
    }
}

// Q6_K: reference q6k_at (kernel.cu:1122-1156); byte-granular (block starts are
// only 2-byte aligned).  Activations are staged unscaled for this format.
template <int MT>
__device__ __forceinline__ void unit_q6k(const uint8_t *blk, const float *xs, int K, const float *, int, int k0,
                                         float *acc) {
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192);
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk + 208));
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
                for (int g = 0; g < 4; ++g) acc[m] = fmaf(d * (float)scg[2 * g], s[m][g], acc[m]);
        }
    }
}

template <int FMT, int MT>
__device__ __forceinline__ void unit_dispatch(const uint8_t *blk, const float *xs, int K, const float *xsum, int nblk,
                                              int k0, float *acc) {
    if (FMT == kQ4_K) unit_q4k<MT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ8_0) unit_q80<MT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ4_0) unit_q40<MT>(blk, xs, K, xsum, nblk, k0, acc);
    else if (FMT == kQ5_0) unit_q50<MT>(blk, xs, K, xsum, nblk, k0, acc);
    else unit_q6k<MT>(blk, xs, K, xsum, nblk, k0, acc);
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

template <int FMT, int MT, int NMAT, int SRC, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) qgemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int W = kGemvConsumerWarps;
    constexpr int SEG = gemv_seg(FMT), PITCH = gemv_pitch(FMT), BB = block_bytes(FMT), BE = block_elems(FMT);
    constexpr int STAGE_BYTES = NMAT * kRowGroup * PITCH;
    extern __shared__ __align__(1024) uint8_t smem[];

    const int NST = a.nst;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kGemvStages;
    float *inv_rms = reinterpret_cast<float *>(smem + 2 * kGemvStages * 8);  // MT floats
    int *abort_flag = reinterpret_cast<int *>(smem + 2 * kGemvStages * 8 + 4 * kGemvMaxTokens);
    const int K = a.K, nblk = K / 32;
    size_t off = 128;
    float *xs = reinterpret_cast<float *>(smem + off);
    off += ((size_t)MT * K * 4 + 127) / 128 * 128;
    float *xsum = reinterpret_cast<float *>(smem + off);
    off += ((size_t)MT * nblk * 4 + 127) / 128 * 128;
    float *red = reinterpret_cast<float *>(smem + off);
    off += ((size_t)W * MT * NMAT * kRowGroup * 4 + 127) / 128 * 128;
    uint8_t *stages = smem + off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t t0 = plan_start(a.plan, blockIdx.x), t1 = plan_start(a.plan, blockIdx.x + 1);
    const int U = a.U;
    const int upr = (SRC == kSrcIndexedK) ? a.units_per_route : 0;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 64);  // 32 producer lanes x 2 arrivals
            mbar_init(&empty[s], W);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------- producer -------------------------------
        const uint64_t pol = l2_evict_first_policy();
        int64_t t = t0;
        Stage st;
        int it = 0;
        while (next_stage(t, t1, U, SEG, upr, st)) {
            const int slot = it % NST;
            const uint32_t ph = (uint32_t)(it / NST) & 1u;
            if (it >= NST && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&empty[slot], ph ^ 1u, a.err, kErrWaitEmpty)) *abort_flag = 1;
            }
            const bool aborted = *reinterpret_cast<volatile int *>(abort_flag) != 0;
            uint8_t *sbase = stages + slot * STAGE_BYTES;
            const int v = st.g * kRowGroup + lane;
            const int len = (st.ue - st.us) * BB;
            const uint8_t *src[NMAT];
            uint32_t bulk_bytes = 0;
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                src[mat] = (!aborted && v < a.rows) ? gemv_block_ptr<SRC, FMT>(a, a.ids, mat, v, st.us) : nullptr;
                if (src[mat]) {
                    const uintptr_t A = reinterpret_cast<uintptr_t>(src[mat]);
                    const uintptr_t lo = (A + 15) & ~uintptr_t(15), hi = (A + len) & ~uintptr_t(15);
                    if (hi > lo) bulk_bytes += (uint32_t)(hi - lo);
                }
            }
            mbar_arrive_expect_tx(&full[slot], bulk_bytes);
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                if (!src[mat]) continue;
                const uintptr_t A = reinterpret_cast<uintptr_t>(src[mat]);
                const uintptr_t lo = (A + 15) & ~uintptr_t(15), hi = (A + len) & ~uintptr_t(15);
                uint8_t *row = sbase + (mat * kRowGroup + lane) * PITCH;  // holds byte A at row + (A & 15)
                if (hi > lo) bulk_g2s(row + (lo - (A & ~uintptr_t(15))), reinterpret_cast<const void *>(lo),
                                      (uint32_t)(hi - lo), &full[slot], pol);
            }
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                if (!src[mat]) continue;
                const uintptr_t A = reinterpret_cast<uintptr_t>(src[mat]);
                const uintptr_t lo = (A + 15) & ~uintptr_t(15), hi = (A + len) & ~uintptr_t(15);
                uint8_t *row = sbase + (mat * kRowGroup + lane) * PITCH + (A & 15);
                if (hi > lo) {
                    copy_ragged(row, src[mat], (int)(lo - A));
                    copy_ragged(row + (hi - A), src[mat] + (hi - A), (int)(A + len - hi));
                } else {
                    copy_ragged(row, src[mat], len);
                }
            }
            mbar_arrive(&full[slot]);
            ++it;
        }
        // Drain: never leave the CTA with bulk copies in flight.
        for (int j = (it > NST ? it - NST : 0); j < it; ++j)
            mbar_wait(&full[j % NST], (uint32_t)(j / NST) & 1u, nullptr, 0);
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int cw = warp - 1;
    const int nthr = W * 32;
    const int ctid = tid - 32;

    // Prologue: optional RMSNorm, then stage x * 2^(96-p) and 32-element block sums.
    if (a.gamma != nullptr) {
        for (int m = 0; m < MT; ++m) {
            float ss = 0.f;
            for (int k = ctid; k < K; k += nthr) {
                const float v = a.x[(size_t)m * a.x_stride + k];
                ss = fmaf(v, v, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[cw] = ss;
            named_bar_sync(1, nthr);
            if (cw == 0) {
                float tsum = lane < W ? red[lane] : 0.f;
                tsum = warp_sum(tsum);
                if (lane == 0) inv_rms[m] = rsqrtf(tsum / (float)K + a.eps);
            }
            named_bar_sync(1, nthr);
        }
    }
    for (int idx = cw; idx < MT * nblk; idx += W) {
        const int m = idx / nblk, b = idx - m * nblk, k = 32 * b + lane;
        float xv;
        if (SRC == kSrcIndexedK) {
            const int F = a.units_per_route * BE;
            const int r = k / F;
            const int e = a.ids[r];
            xv = e >= 0 ? a.x[(size_t)r * a.x_stride + (k - r * F)] * a.route_w[r] : 0.f;
        } else {
            xv = a.x[(size_t)m * a.x_stride + k];
        }
        if (a.gamma != nullptr) xv = xv * inv_rms[m] * a.gamma[k];
        xs[(size_t)m * K + k] = xv * pow2_dev(96 - weight_bitpos<FMT>(k));
        const float s = warp_sum(xv);
        if (lane == 0) xsum[(size_t)m * nblk + b] = s;
    }
    named_bar_sync(1, nthr);

    float acc[NMAT][MT];
#pragma unroll
    for (int i = 0; i < NMAT; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.f;

    int64_t t = t0;
    Stage st;
    int it = 0, ucount = 0;
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
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
                const uint8_t *rs = gemv_block_ptr<SRC, FMT>(a, a.ids, mat, v, st.us);
                if (rs == nullptr) continue;
                const uint8_t *row = stages + slot * STAGE_BYTES + (mat * kRowGroup + lane) * PITCH +
                                     (reinterpret_cast<uintptr_t>(rs) & 15);
                for (int lu = first; lu < n; lu += W)
                    unit_dispatch<FMT, MT>(row + lu * BB, xs, K, xsum, nblk, (st.us + lu) * BE, acc[mat]);
            }
        }
        ucount += n;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        ++it;

        if (st.last_in_group) {
            // Cross-warp reduction in fixed warp order, then epilogue or stream-K fixup.
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                for (int m = 0; m < MT; ++m) red[((cw * MT + m) * NMAT + mat) * kRowGroup + lane] = acc[mat][m];
            named_bar_sync(1, nthr);
            if (cw == 0) {
                float val[NMAT][MT];
#pragma unroll
                for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        float s = 0.f;
                        for (int w = 0; w < W; ++w) s += red[((w * MT + m) * NMAT + mat) * kRowGroup + lane];
                        val[mat][m] = s;
                    }
                const int g = st.g;
                const int64_t gs = (int64_t)g * U, ge = gs + U;
                bool finish = true;
                if (gs < t0 || ge > t1) {
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
                if (finish && v < a.rows && !aborted) {
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        float *yp = a.y + (size_t)m * a.y_stride + v;
                        if (EPI == kEpiSwiglu) {
                            const float gv = val[0][m], uv = val[NMAT - 1][m];
                            float o = gv / (1.0f + expf(-gv)) * uv;
                            if (SRC == kSrcIndexedRows && a.ids[v / a.rows_per_route] < 0) o = 0.f;
                            *yp = o;
                        } else {
                            float o = val[0][m];
                            if (a.bias != nullptr) o += a.bias[v];
                            if (EPI == kEpiAdd) *yp += o;
                            else *yp = o;
                        }
                    }
                }
            }
            named_bar_sync(1, nthr);
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat)
#pragma unroll
                for (int m = 0; m < MT; ++m) acc[mat][m] = 0.f;
        }
    }
}

// ----------------------------------------------------------------------------
// Host launchers for one format.  Indexed sources run one token (decode).
// ----------------------------------------------------------------------------
template <int FMT, int MT, int NMAT, int SRC, int EPI>
static cudaError_t launch_typed(const GemvArgs &a, int smem, cudaStream_t stream) {
    auto k = qgemv_kernel<FMT, MT, NMAT, SRC, EPI>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    k<<<a.plan.C, kGemvThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

template <int FMT, int NMAT, int SRC, int EPI>
static cudaError_t launch_mt(const GemvArgs &a, int MT, int smem, cudaStream_t s) {
    switch (MT) {
    case 1: return launch_typed<FMT, 1, NMAT, SRC, EPI>(a, smem, s);
    case 2: return launch_typed<FMT, 2, NMAT, SRC, EPI>(a, smem, s);
    case 3: return launch_typed<FMT, 3, NMAT, SRC, EPI>(a, smem, s);
    default: return launch_typed<FMT, 4, NMAT, SRC, EPI>(a, smem, s);
    }
}

// kind: 0 plain store, 1 plain add, 2 plain SwiGLU pair, 3 indexed-rows SwiGLU
// pair (MT = 1), 4 indexed-K add (MT = 1).
template <int FMT>
cudaError_t gemv_launch_fmt(int kind, const GemvArgs &a, int MT, int smem, cudaStream_t s) {
    switch (kind) {
    case 0: return launch_mt<FMT, 1, kSrcPlain, kEpiStore>(a, MT, smem, s);
    case 1: return launch_mt<FMT, 1, kSrcPlain, kEpiAdd>(a, MT, smem, s);
    case 2: return launch_mt<FMT, 2, kSrcPlain, kEpiSwiglu>(a, MT, smem, s);
    case 3: return MT == 1 ? launch_typed<FMT, 1, 2, kSrcIndexedRows, kEpiSwiglu>(a, smem, s) : cudaErrorInvalidValue;
    case 4: return MT == 1 ? launch_typed<FMT, 1, 1, kSrcIndexedK, kEpiAdd>(a, smem, s) : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace ql
