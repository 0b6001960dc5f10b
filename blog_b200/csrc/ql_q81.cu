// Opt-in int8 activation path (Q8_1), the reference's llama.cpp-style alternative to fp32
// activations (kernel.cu:1679-1865, launch.cu:191-240; the engine keeps it off by default because
// it changes numerics, TensorTool.cpp:159-161).
//
// Q8_1 block (36 bytes per 32 activations): f16 d = max|x| / 127, f16 sum (sum of x, or d * sum of q),
// 32 x int8 q = round(x / d) clamped to +-127.  The quantizer reproduces the reference's bytes
// exactly: the same per-block arithmetic (IEEE divide, round-half-even conversion) and the same
// warp tree for the sum (lane l adds lane l + 16, then + 8, + 4, + 2, + 1), eight blocks per CTA.
//
// The GEMV takes one Q8_1 activation row: a warp per weight row, lane = one 32-element block at a
// time (32 adjacent blocks per warp pass: coalesced row reads), the block's integer dot product
// with 8 dp4a, then the block's scale terms in fp32:
//   Q4_K: acc += (d_w sc d_x) qdot - dmin_w m sum_x      (the min folded through the block sum)
//   Q6_K: acc += (d_w d_x) (s0 qdot_lo16 + s1 qdot_hi16)  (two 16-element scale groups)
//   Q5_0 / Q8_0: acc += (d_w d_x) qdot
// and a warp reduction.  The reference sums blocks in order on one lane (Q4_K / Q6_K) or per
// element in floats (Q5_0 / Q8_0); the results agree to float rounding (~1e-7 relative).
#include "ql_common.cuh"
#include "ql_q81.cuh"

namespace ql {
namespace {

constexpr int kQ81Warps = 8;

// MMQ: the reference's packed layout (quantize_q8_1_mmq_kernel, kernel.cu:1724-1765): 144-byte groups
// of 4 consecutive blocks, group-major ([group][row]), each {4 x (f16 d, f16 sum), 4 x 32 int8}.
template <bool MMQ>
__global__ void __launch_bounds__(32 * kQ81Warps) quantize_q81_kernel(const float *__restrict__ x,
                                                                     uint8_t *__restrict__ xq, int in_dim, int m,
                                                                     int bpr, int store_raw_sum) {
    const int lane = threadIdx.x & 31;
    const long long blk = (long long)blockIdx.x * kQ81Warps + (threadIdx.x >> 5);
    if (blk >= (long long)m * bpr) return;
    const int row = (int)(blk / bpr), qb = (int)(blk - (long long)row * bpr);
    const int k = qb * 32 + lane;
    const float v = k < in_dim ? x[(size_t)row * in_dim + k] : 0.0f;
    float amax = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_down_sync(0xffffffffu, amax, o));
    amax = __shfl_sync(0xffffffffu, amax, 0);
    const float d = amax > 0.0f ? amax / 127.0f : 0.0f;
    const float id = d > 0.0f ? 1.0f / d : 0.0f;
    float raw = v;  // lane 0 ends with the tree sum ((v0 + v16) + (v8 + v24)) + ...
    for (int o = 16; o > 0; o >>= 1) raw += __shfl_down_sync(0xffffffffu, raw, o);
    int q = __float2int_rn(v * id);
    q = max(-127, min(127, q));
    int qs = q;
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_down_sync(0xffffffffu, qs, o);
    uint8_t *ds, *qd;
    if (MMQ) {
        uint8_t *grp = xq + ((size_t)(qb >> 2) * m + row) * 144;
        ds = grp + 4 * (qb & 3);
        qd = grp + 16 + 32 * (qb & 3);
    } else {
        ds = xq + (size_t)blk * 36;
        qd = ds + 4;
    }
    if (lane == 0) {
        *reinterpret_cast<uint16_t *>(ds) = __half_as_ushort(__float2half(d));
        const float s = store_raw_sum ? raw : d * (float)qs;
        *reinterpret_cast<uint16_t *>(ds + 2) = __half_as_ushort(__float2half(s));
    }
    reinterpret_cast<int8_t *>(qd)[lane] = (int8_t)q;
}

__device__ __forceinline__ uint32_t ld_u16_pair(const uint8_t *p) {  // 4 bytes at a 2-byte-aligned address
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}
// Spread bits 0..3 of h to bit 4 of bytes 0..3.
__device__ __forceinline__ uint32_t bits_to_byte4(uint32_t h) { return ((h * 0x00204081u) & 0x01010101u) << 4; }

template <int FMT>
__global__ void __launch_bounds__(32 * kQ81Warps) gemv_q81_kernel(const uint8_t *__restrict__ w, size_t rb,
                                                                 const uint8_t *__restrict__ xq, float *__restrict__ y,
                                                                 int out_dim, int bpr) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kQ81Warps + (threadIdx.x >> 5);
    if (row >= out_dim) return;
    const uint8_t *rp = w + (size_t)row * rb;
    float acc = 0.f;
    for (int b = lane; b < bpr; b += 32) {
        const uint8_t *xb = xq + (size_t)b * 36;
        const uint32_t dh = *reinterpret_cast<const uint32_t *>(xb);
        const float dx = half_bits_to_float(dh), sx = half_bits_to_float(dh >> 16);
        const int *qx = reinterpret_cast<const int *>(xb + 4);
        if (FMT == kQ4_K) {
            const int sb = b >> 3, j = b & 7;
            const uint8_t *base = rp + 144 * sb;
            const uint4 q0 = *reinterpret_cast<const uint4 *>(base + 16 + 32 * (j >> 1));
            const uint4 q1 = *reinterpret_cast<const uint4 *>(base + 32 + 32 * (j >> 1));
            const uint32_t W[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            const int sh = 4 * (j & 1);
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = __dp4a((int)((W[i] >> sh) & 0x0F0F0F0Fu), qx[i], dot);
            const uint8_t *s = base + 4;  // q4k_scale_min (reference kernel.cu:913-921)
            uint32_t sc, mn;
            if (j < 4) {
                sc = s[j] & 63u;
                mn = s[j + 4] & 63u;
            } else {
                sc = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
                mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
            }
            const uint32_t dd = *reinterpret_cast<const uint32_t *>(base);
            acc = fmaf(half_bits_to_float(dd) * (float)sc * dx, (float)dot, acc);
            acc -= half_bits_to_float(dd >> 16) * (float)mn * sx;
        } else if (FMT == kQ6_K) {
            const int sb = b >> 3, sub = b & 7, hf = sub >> 2, grp = sub & 3;
            const uint8_t *base = rp + 210 * sb;
            const uint8_t *ql = base + 64 * hf + ((grp & 1) ? 32 : 0), *qh = base + 128 + 32 * hf;
            const int8_t *scl = reinterpret_cast<const int8_t *>(base + 192) + 8 * hf + 2 * grp;
            const int lsh = (grp >> 1) ? 4 : 0, hsh = 2 * grp;
            int dot0 = 0, dot1 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {  // elements 4i .. 4i + 3: 6-bit values minus 32 as signed bytes
                const uint32_t l = ld_u16_pair(ql + 4 * i), h = ld_u16_pair(qh + 4 * i);
                const uint32_t v6 = ((l >> lsh) & 0x0F0F0F0Fu) | (((h >> hsh) & 0x03030303u) << 4);
                const int q = (int)__vsub4(v6, 0x20202020u);
                if (i < 4) dot0 = __dp4a(q, qx[i], dot0);
                else dot1 = __dp4a(q, qx[i], dot1);
            }
            const float dwx = half_bits_to_float(*reinterpret_cast<const uint16_t *>(base + 208)) * dx;
            acc = fmaf(dwx, (float)scl[0] * (float)dot0 + (float)scl[1] * (float)dot1, acc);
        } else if (FMT == kQ5_0) {
            const uint8_t *base = rp + 22 * b;
            const uint32_t qh = ld_u16_pair(base + 2);
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t l = ld_u16_pair(base + 6 + 4 * i);
                const int lo = (int)__vsub4((l & 0x0F0F0F0Fu) | bits_to_byte4((qh >> (4 * i)) & 0xFu), 0x10101010u);
                const int hi =
                    (int)__vsub4(((l >> 4) & 0x0F0F0F0Fu) | bits_to_byte4((qh >> (16 + 4 * i)) & 0xFu), 0x10101010u);
                dot = __dp4a(lo, qx[i], dot);
                dot = __dp4a(hi, qx[4 + i], dot);
            }
            acc = fmaf(half_bits_to_float(*reinterpret_cast<const uint16_t *>(base)) * dx, (float)dot, acc);
        } else {  // Q8_0
            const uint8_t *base = rp + 34 * b;
            int dot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = __dp4a((int)ld_u16_pair(base + 2 + 4 * i), qx[i], dot);
            acc = fmaf(half_bits_to_float(*reinterpret_cast<const uint16_t *>(base)) * dx, (float)dot, acc);
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[row] = acc;
}
// ---------------------------------------------------------------------------------------------
// Q8_1 matmul for m token rows (the reference's quant_matmul_q8_1_kernel, kernel.cu:2304-2400:
// the GEMV's per-block formula for every (token, output row)) on the integer tensor cores.  CTA =
// 64 weight rows (4 warps x 16) x up to 64 tokens; each warp's 16 rows are staged once in shared
// memory (one bulk copy per row into a slot whose pitch is 16 mod 32 bytes: the 8 rows a quad reads
// fall in distinct banks); per 32-element block the quants are an exact int8 A fragment, the Q8_1
// activations the int8 B fragment, one mma.sync.m16n8k32.s8 per 8 tokens (Q6_K: two k16 MMAs, one
// per 16-element scale group), then acc(row, token) = fmaf(d_w sc d_x, qdot, acc) (- dmin m sum_x)
// in block order, the reference's expression for each output.
// ---------------------------------------------------------------------------------------------
constexpr int kMmThreads = 128;
constexpr int kMmTokens = 64;  // tokens per CTA: 4 passes of 16 (two n-tiles of 8)

__device__ __forceinline__ void imma_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void imma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

struct MmBlock {
    uint32_t a[4];  // int8 quants: {row g: k 4c.., row g+8: k 4c.., row g: k 16 + 4c.., row g+8: k 16 + 4c..}
    float s[2][2];  // per row (g, g + 8): Q4_K {d sc, dmin m}; Q6_K {d s0, d s1}; Q5_0 / Q8_0 {d, -}
};

template <int FMT>
__device__ __forceinline__ void mm_decode(const uint8_t *row0, const uint8_t *row1, int b, int c, MmBlock &o) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint8_t *rp = h ? row1 : row0;
        if (FMT == kQ4_K) {
            const int sb = b >> 3, j = b & 7;
            const uint8_t *base = rp + 144 * sb;
            const int sh = 4 * (j & 1);
            o.a[h] = (*reinterpret_cast<const uint32_t *>(base + 16 + 32 * (j >> 1) + 4 * c) >> sh) & 0x0F0F0F0Fu;
            o.a[2 + h] = (*reinterpret_cast<const uint32_t *>(base + 32 + 32 * (j >> 1) + 4 * c) >> sh) & 0x0F0F0F0Fu;
            const uint8_t *s = base + 4;  // q4k_scale_min (reference kernel.cu:913-921)
            uint32_t sc, mn;
            if (j < 4) {
                sc = s[j] & 63u;
                mn = s[j + 4] & 63u;
            } else {
                sc = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
                mn = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
            }
            const uint32_t dd = *reinterpret_cast<const uint32_t *>(base);
            o.s[h][0] = half_bits_to_float(dd) * (float)sc;
            o.s[h][1] = half_bits_to_float(dd >> 16) * (float)mn;
        } else if (FMT == kQ6_K) {
            const int sb = b >> 3, sub = b & 7, hf = sub >> 2, grp = sub & 3;
            const uint8_t *base = rp + 210 * sb;
            const uint8_t *ql = base + 64 * hf + ((grp & 1) ? 32 : 0), *qh = base + 128 + 32 * hf;
            const int lsh = (grp >> 1) ? 4 : 0, hsh = 2 * grp;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int e = 16 * half + 4 * c;
                const uint32_t l = ld_u16_pair(ql + e), hh = ld_u16_pair(qh + e);
                o.a[2 * half + h] = __vsub4(((l >> lsh) & 0x0F0F0F0Fu) | (((hh >> hsh) & 0x03030303u) << 4), 0x20202020u);
            }
            const int8_t *scl = reinterpret_cast<const int8_t *>(base + 192) + 8 * hf + 2 * grp;
            const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(base + 208));
            o.s[h][0] = dw;
            o.s[h][1] = 0.f;
            (void)scl;
        } else if (FMT == kQ5_0) {
            const uint8_t *base = rp + 22 * b;
            const uint32_t qh = ld_u16_pair(base + 2), l = ld_u16_pair(base + 6 + 4 * c);
            o.a[h] = __vsub4((l & 0x0F0F0F0Fu) | bits_to_byte4((qh >> (4 * c)) & 0xFu), 0x10101010u);
            o.a[2 + h] = __vsub4(((l >> 4) & 0x0F0F0F0Fu) | bits_to_byte4((qh >> (16 + 4 * c)) & 0xFu), 0x10101010u);
            o.s[h][0] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(base));
            o.s[h][1] = 0.f;
        } else {  // Q8_0
            const uint8_t *base = rp + 34 * b;
            o.a[h] = ld_u16_pair(base + 2 + 4 * c);
            o.a[2 + h] = ld_u16_pair(base + 18 + 4 * c);
            o.s[h][0] = half_bits_to_float(*reinterpret_cast<const uint16_t *>(base));
            o.s[h][1] = 0.f;
        }
    }
}

template <int FMT, bool MMQ>
__global__ void __launch_bounds__(kMmThreads) q81_matmul_kernel(const __grid_constant__ Q81MmArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t bar[4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int wrow0 = blockIdx.x * 64 + 16 * warp, tok0 = blockIdx.y * kMmTokens;
    int nr = min(16, a.out_dim - wrow0);
    const int P = a.row_pitch, bpr = (a.in_dim + 31) / 32;
    uint8_t *slab = smem + (size_t)warp * 16 * P;
    const uint8_t *wbase = a.w + (size_t)wrow0 * a.rb;
    if (nr > 0) {
        uintptr_t lo = 0, hi = 0, end = 0;
        if (lane < nr) {
            const uintptr_t st = reinterpret_cast<uintptr_t>(wbase + (size_t)lane * a.rb);
            lo = st & ~uintptr_t(15);
            end = st + a.rb;
            hi = end & ~uintptr_t(15);
        }
        const uint32_t tx = __reduce_add_sync(0xffffffffu, (uint32_t)(hi - lo));
        if (lane == 0) {
            mbar_init(&bar[warp], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            mbar_arrive_expect_tx(&bar[warp], tx);
        }
        __syncwarp();
        if (lane < nr) {
            uint8_t *dst = slab + (size_t)lane * P;
            if (hi > lo)
                bulk_g2s(dst, reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &bar[warp],
                         l2_evict_first_policy());
            for (uintptr_t q = hi; q < end; ++q) dst[q - lo] = *reinterpret_cast<const uint8_t *>(q);
        }
        __syncwarp();
        if (!mbar_wait(&bar[warp], 0u, a.err, kErrWaitFull)) {
            mbar_wait(&bar[warp], 0u, nullptr, 0);  // never leave with the copies in flight
            nr = 0;
        }
    }
    if (nr <= 0) return;
    const int sh0 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)g * a.rb) & 15);
    const int sh1 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)(g + 8) * a.rb) & 15);
    const uint8_t *row0 = slab + (size_t)g * P + sh0, *row1 = slab + (size_t)(g + 8) * P + sh1;
    // all of the CTA's tokens (up to 8 tiles of 8) per weight block: the block is decoded once and the
    // tiles' activation loads go out together
    const size_t xrb = (size_t)bpr * 36;
    const int ntile = (min(kMmTokens, a.m - tok0) + 7) >> 3;
    int xrow[8], srow[8][2];  // token rows of the B operand (8j + g) and of the scales (8j + 2c, + 1)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        xrow[j] = min(tok0 + 8 * j + g, a.m - 1);
        srow[j][0] = min(tok0 + 8 * j + 2 * c, a.m - 1);
        srow[j][1] = min(tok0 + 8 * j + 2 * c + 1, a.m - 1);
    }
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int b = 0; b < bpr; ++b) {
        MmBlock blk;
        mm_decode<FMT>(row0, row1, b, c, blk);
        const int8_t *scl[2] = {nullptr, nullptr};
        if (FMT == kQ6_K) {
            const int sb = b >> 3, sub = b & 7, hf = sub >> 2, grp = sub & 3;
            scl[0] = reinterpret_cast<const int8_t *>(row0 + 210 * sb + 192) + 8 * hf + 2 * grp;
            scl[1] = reinterpret_cast<const int8_t *>(row1 + 210 * sb + 192) + 8 * hf + 2 * grp;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j < ntile) {
                // plain rows: block b at b * 36 of the token's row; MMQ: group b / 4 of the token, sub-block b % 4
                const uint8_t *bb = MMQ ? a.xq + ((size_t)(b >> 2) * a.m + xrow[j]) * 144 + 16 + 32 * (b & 3)
                                        : a.xq + (size_t)xrow[j] * xrb + (size_t)b * 36 + 4;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(bb + 4 * c);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(bb + 16 + 4 * c);
                float dx[2], sx[2];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint8_t *dsp = MMQ ? a.xq + ((size_t)(b >> 2) * a.m + srow[j][q]) * 144 + 4 * (b & 3)
                                             : a.xq + (size_t)srow[j][q] * xrb + (size_t)b * 36;
                    const uint32_t ds = *reinterpret_cast<const uint32_t *>(dsp);
                    dx[q] = half_bits_to_float(ds);
                    sx[q] = half_bits_to_float(ds >> 16);
                }
                if (FMT == kQ6_K) {
                    int t0v[4] = {0, 0, 0, 0}, t1v[4] = {0, 0, 0, 0};
                    imma_k16(t0v, blk.a[0], blk.a[1], b0);
                    imma_k16(t1v, blk.a[2], blk.a[3], b1);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int h = q >> 1;
                        acc[j][q] = fmaf(blk.s[h][0] * dx[q & 1],
                                         (float)scl[h][0] * (float)t0v[q] + (float)scl[h][1] * (float)t1v[q], acc[j][q]);
                    }
                } else {
                    int t[4] = {0, 0, 0, 0};
                    imma_k32(t, blk.a, b0, b1);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int h = q >> 1;
                        acc[j][q] = fmaf(blk.s[h][0] * dx[q & 1], (float)t[q], acc[j][q]);
                        if (FMT == kQ4_K) acc[j][q] -= blk.s[h][1] * sx[q & 1];
                    }
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int tok = tok0 + 8 * j + 2 * c + (q & 1), r = g + 8 * (q >> 1);
            if (j < ntile && tok < a.m && r < nr) a.y[(size_t)tok * a.out_dim + wrow0 + r] = acc[j][q];
        }
}
}  // namespace

int q81_mm_row_pitch(size_t row_bytes) {
    int p = (int)((row_bytes + 15 + 15) & ~size_t(15));
    if (p % 32 == 0) p += 16;
    return p;
}

namespace {
// Staged variant (in_dim a multiple of 128): 8 warps, warps w and w + 4 share slab w and split the
// K range; each half streams its 128-element activation chunks (64 tokens x 144 bytes: 4 plain blocks
// or one MMQ group, 16-byte aligned) into shared memory with cp.async, double-buffered, so the B
// fragments come from shared memory (token records 144 B apart: the 8 tokens x 4 lanes of a load hit
// 32 distinct banks) instead of an L2 round trip per token tile; the halves' sums meet in shared memory.
constexpr int kMmsThreads = 256;
constexpr int kChunk = 64 * 144;  // one activation chunk: 64 tokens x 128 activations

__device__ __forceinline__ void cp_async16_cg(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int FMT, bool MMQ>
__global__ void __launch_bounds__(kMmsThreads, 1) q81_matmul_staged_kernel(const __grid_constant__ Q81MmArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t bar[4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int slab_i = warp & 3, kh = warp >> 2, gtid = threadIdx.x & 127;
    const int wrow0 = blockIdx.x * 64 + 16 * slab_i, tok0 = blockIdx.y * kMmTokens;
    int nr = min(16, a.out_dim - wrow0);
    const int P = a.row_pitch, bpr = a.in_dim / 32, nch = bpr / 4;
    uint8_t *slab = smem + (size_t)slab_i * 16 * P;
    uint8_t *act = smem + (size_t)64 * P + (size_t)kh * 2 * kChunk;  // this half's two chunk buffers
    const uint8_t *wbase = a.w + (size_t)wrow0 * a.rb;
    uintptr_t lo = 0, hi = 0, end = 0;
    if (kh == 0 && nr > 0) {
        if (lane < nr) {
            const uintptr_t st = reinterpret_cast<uintptr_t>(wbase + (size_t)lane * a.rb);
            lo = st & ~uintptr_t(15);
            end = st + a.rb;
            hi = end & ~uintptr_t(15);
        }
        const uint32_t tx = __reduce_add_sync(0xffffffffu, (uint32_t)(hi - lo));
        if (lane == 0) {
            mbar_init(&bar[slab_i], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            mbar_arrive_expect_tx(&bar[slab_i], tx);
        }
    }
    __syncthreads();  // the slab barriers exist before the other half waits on them
    if (kh == 0 && lane < nr) {
        uint8_t *dst = slab + (size_t)lane * P;
        if (hi > lo)
            bulk_g2s(dst, reinterpret_cast<const void *>(lo), (uint32_t)(hi - lo), &bar[slab_i], l2_evict_first_policy());
        for (uintptr_t q = hi; q < end; ++q) dst[q - lo] = *reinterpret_cast<const uint8_t *>(q);
    }
    // this half's chunks [c0, c1) (Q4_K: whole super-blocks of 2 chunks)
    const int unit = FMT == kQ4_K || FMT == kQ6_K ? 2 : 1;
    const int cmid = (nch / unit) / 2 * unit, c0 = kh ? cmid : 0, c1 = kh ? nch : cmid;
    const size_t xrb = (size_t)bpr * 36;
    auto issue = [&](int ch, int buf) {
        uint8_t *dstb = act + (size_t)buf * kChunk;
        for (int i = gtid; i < 64 * 9; i += 128) {
            const int slot = i / 9, piece = i - slot * 9, tok = min(tok0 + slot, a.m - 1);
            const uint8_t *src = MMQ ? a.xq + ((size_t)ch * a.m + tok) * 144 : a.xq + (size_t)tok * xrb + (size_t)ch * 144;
            cp_async16_cg(dstb + slot * 144 + 16 * piece, src + 16 * piece);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (c0 < c1) issue(c0, 0);
    __syncthreads();  // the tails' plain stores, for both halves
    if (nr > 0 && !mbar_wait(&bar[slab_i], 0u, a.err, kErrWaitFull)) {
        mbar_wait(&bar[slab_i], 0u, nullptr, 0);  // never leave with the copies in flight
        nr = 0;
    }
    const int sh0 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)g * a.rb) & 15);
    const int sh1 = (int)(reinterpret_cast<uintptr_t>(wbase + (size_t)(g + 8) * a.rb) & 15);
    const uint8_t *row0 = slab + (size_t)g * P + sh0, *row1 = slab + (size_t)(g + 8) * P + sh1;
    const int ntile = (min(kMmTokens, a.m - tok0) + 7) >> 3;
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int ch = c0; ch < c1; ++ch) {
        if (ch + 1 < c1) issue(ch + 1, (ch + 1 - c0) & 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // chunk ch has landed
        named_bar_sync(1 + kh, 128);
        const uint8_t *buf = act + (size_t)((ch - c0) & 1) * kChunk;
        if (nr > 0) {
#pragma unroll
            for (int bi = 0; bi < 4; ++bi) {
                const int b = 4 * ch + bi;
                MmBlock blk;
                mm_decode<FMT>(row0, row1, b, c, blk);
                const int8_t *scl[2] = {nullptr, nullptr};
                if (FMT == kQ6_K) {
                    const int sb = b >> 3, sub = b & 7, hf = sub >> 2, grp = sub & 3;
                    scl[0] = reinterpret_cast<const int8_t *>(row0 + 210 * sb + 192) + 8 * hf + 2 * grp;
                    scl[1] = reinterpret_cast<const int8_t *>(row1 + 210 * sb + 192) + 8 * hf + 2 * grp;
                }
                const int qoff = MMQ ? 16 + 32 * bi : 36 * bi + 4, doff = MMQ ? 4 * bi : 36 * bi;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (j < ntile) {
                        const uint8_t *rb_ = buf + (8 * j + g) * 144 + qoff;
                        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(rb_ + 4 * c);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(rb_ + 16 + 4 * c);
                        float dx[2], sx[2];
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const uint32_t ds = *reinterpret_cast<const uint32_t *>(buf + (8 * j + 2 * c + q) * 144 + doff);
                            dx[q] = half_bits_to_float(ds);
                            sx[q] = half_bits_to_float(ds >> 16);
                        }
                        if (FMT == kQ6_K) {
                            int t0v[4] = {0, 0, 0, 0}, t1v[4] = {0, 0, 0, 0};
                            imma_k16(t0v, blk.a[0], blk.a[1], b0);
                            imma_k16(t1v, blk.a[2], blk.a[3], b1);
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int h = q >> 1;
                                acc[j][q] = fmaf(blk.s[h][0] * dx[q & 1],
                                                 (float)scl[h][0] * (float)t0v[q] + (float)scl[h][1] * (float)t1v[q],
                                                 acc[j][q]);
                            }
                        } else {
                            int t[4] = {0, 0, 0, 0};
                            imma_k32(t, blk.a, b0, b1);
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int h = q >> 1;
                                acc[j][q] = fmaf(blk.s[h][0] * dx[q & 1], (float)t[q], acc[j][q]);
                                if (FMT == kQ4_K) acc[j][q] -= blk.s[h][1] * sx[q & 1];
                            }
                        }
                    }
                }
            }
        }
        named_bar_sync(1 + kh, 128);  // this buffer is refilled two chunks later
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // both halves done with their chunk buffers: they now hold the second half's sums
    float *red = reinterpret_cast<float *>(smem + (size_t)64 * P);  // [4 slabs][32 lanes][32]
    if (kh) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) red[(slab_i * 32 + lane) * 32 + 4 * j + q] = acc[j][q];
    }
    __syncthreads();
    if (!kh && nr > 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int tok = tok0 + 8 * j + 2 * c + (q & 1), r = g + 8 * (q >> 1);
                if (j < ntile && tok < a.m && r < nr)
                    a.y[(size_t)tok * a.out_dim + wrow0 + r] = acc[j][q] + red[(slab_i * 32 + lane) * 32 + 4 * j + q];
            }
    }
}

template <int FMT, bool MMQ>
cudaError_t mm_launch_t(const Q81MmArgs &a, size_t smem, dim3 grid, cudaStream_t s) {
    cudaError_t e =
        cudaFuncSetAttribute(q81_matmul_kernel<FMT, MMQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    q81_matmul_kernel<FMT, MMQ><<<grid, kMmThreads, smem, s>>>(a);
    return cudaGetLastError();
}
template <int FMT, bool MMQ>
cudaError_t mms_launch_t(const Q81MmArgs &a, size_t smem, dim3 grid, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(q81_matmul_staged_kernel<FMT, MMQ>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    q81_matmul_staged_kernel<FMT, MMQ><<<grid, kMmsThreads, smem, s>>>(a);
    return cudaGetLastError();
}
template <bool MMQ>
cudaError_t mm_launch_fmt(int fmt, const Q81MmArgs &a, size_t smem, dim3 grid, bool staged, cudaStream_t s) {
    switch (fmt) {
    case kQ4_K: return staged ? mms_launch_t<kQ4_K, MMQ>(a, smem, grid, s) : mm_launch_t<kQ4_K, MMQ>(a, smem, grid, s);
    case kQ6_K: return staged ? mms_launch_t<kQ6_K, MMQ>(a, smem, grid, s) : mm_launch_t<kQ6_K, MMQ>(a, smem, grid, s);
    case kQ5_0: return staged ? mms_launch_t<kQ5_0, MMQ>(a, smem, grid, s) : mm_launch_t<kQ5_0, MMQ>(a, smem, grid, s);
    case kQ8_0: return staged ? mms_launch_t<kQ8_0, MMQ>(a, smem, grid, s) : mm_launch_t<kQ8_0, MMQ>(a, smem, grid, s);
    default: return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t matmul_q81_launch(int fmt, const Q81MmArgs &a, bool mmq, cudaStream_t s) {
    const size_t wsm = (size_t)4 * 16 * a.row_pitch;
    const size_t ssm = wsm + 4 * (size_t)kChunk;  // + two chunk buffers per K half (also the halves' sums)
    const bool staged = a.in_dim % 128 == 0 && ssm <= 232448 - 1024;
    const size_t smem = staged ? ssm : wsm;
    const dim3 grid((a.out_dim + 63) / 64, (a.m + kMmTokens - 1) / kMmTokens);
    return mmq ? mm_launch_fmt<true>(fmt, a, smem, grid, staged, s) : mm_launch_fmt<false>(fmt, a, smem, grid, staged, s);
}

size_t q81_row_bytes(int in_dim) { return (size_t)((in_dim + 31) / 32) * 36; }

size_t q81_mmq_row_bytes(int in_dim) { return (size_t)((in_dim + 127) / 128) * 144; }

cudaError_t quantize_q81_launch(const float *x, uint8_t *xq, int in_dim, int m, bool store_raw_sum, bool mmq,
                                cudaStream_t s) {
    const int bpr = mmq ? (in_dim + 127) / 128 * 4 : (in_dim + 31) / 32;  // MMQ: every block of every group
    const long long blocks = ((long long)m * bpr + kQ81Warps - 1) / kQ81Warps;
    if (mmq)
        quantize_q81_kernel<true><<<(unsigned)blocks, 32 * kQ81Warps, 0, s>>>(x, xq, in_dim, m, bpr, store_raw_sum ? 1 : 0);
    else
        quantize_q81_kernel<false><<<(unsigned)blocks, 32 * kQ81Warps, 0, s>>>(x, xq, in_dim, m, bpr, store_raw_sum ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t gemv_q81_launch(int fmt, const uint8_t *w, size_t rb, const uint8_t *xq, float *y, int out_dim, int in_dim,
                            cudaStream_t s) {
    const int bpr = (in_dim + 31) / 32;
    const unsigned grid = (unsigned)((out_dim + kQ81Warps - 1) / kQ81Warps);
    switch (fmt) {
    case kQ4_K: gemv_q81_kernel<kQ4_K><<<grid, 32 * kQ81Warps, 0, s>>>(w, rb, xq, y, out_dim, bpr); break;
    case kQ6_K: gemv_q81_kernel<kQ6_K><<<grid, 32 * kQ81Warps, 0, s>>>(w, rb, xq, y, out_dim, bpr); break;
    case kQ5_0: gemv_q81_kernel<kQ5_0><<<grid, 32 * kQ81Warps, 0, s>>>(w, rb, xq, y, out_dim, bpr); break;
    case kQ8_0: gemv_q81_kernel<kQ8_0><<<grid, 32 * kQ81Warps, 0, s>>>(w, rb, xq, y, out_dim, bpr); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ql
