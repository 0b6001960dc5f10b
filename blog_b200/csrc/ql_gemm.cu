// ql_gemm.cu -- tcgen05 prefill GEMM over GGUF Q4_K weights (see ql_gemm.cuh).
#include "ql_gemm.cuh"

namespace ql {
namespace {

// ---------------------------------------------------------------------------
// PTX wrappers: TMA 2-D load, TMEM allocation, tcgen05 MMA / commit / load.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrive (once) on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns of TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row
// atoms of 1024 B (stride byte offset), leading byte offset unused (1).
__device__ __forceinline__ uint64_t sw128_desc(const void *p) {
    const uint64_t a = smem_u32(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, M x N.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kGemmBN >> 3) << 17) | ((uint32_t)(kGemmBM >> 4) << 24);

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// (1024 + n) from a nibble pair placed at bits 0-3 / 16-19 -> n * D - M, in f16.
__device__ __forceinline__ uint32_t deq2(uint32_t nib, __half2 D, __half2 negM) {
    const __half2 h = bits_h2(nib | 0x64006400u);
    return h2_bits(__hfma2(__hsub2(h, __float2half2_rn(1024.f)), D, negM));
}

// ---------------------------------------------------------------------------
// Activation preparation (one CTA per row).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemm_xprep_kernel(const float *__restrict__ x, int64_t x_stride,
                                                         const float *__restrict__ gamma, float eps,
                                                         __half *__restrict__ xh, float *__restrict__ rinv, int K) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int m = blockIdx.x;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)m * x_stride);
    const float4 *gr = reinterpret_cast<const float4 *>(gamma);
    float mx = 0.f, ss = 0.f;
    bool nan = false;
    for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        float4 v = xr[i];
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        if (gamma) {
            const float4 g = gr[i];
            v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
        }
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        nan = nan || v.x != v.x || v.y != v.y || v.z != v.z || v.w != v.w;
    }
    if (nan) mx = __int_as_float(0x7f800000);
    __shared__ float red[2][8];
    for (int o = 16; o > 0; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = mx;
        red[1][threadIdx.x >> 5] = ss;
    }
    __syncthreads();
    mx = red[0][0];
    ss = red[1][0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
        mx = fmaxf(mx, red[0][w]);
        ss += red[1][w];
    }
    // s = 2^k with max|x| * s in [2^13, 2^14); s = 1 for an all-zero or non-finite row.
    int k = 0;
    if (mx > 0.f && mx < __int_as_float(0x7f800000)) {
        int ex;
        frexpf(mx, &ex);  // mx = f * 2^ex, f in [0.5, 1)
        k = 14 - ex;
        k = k > 126 ? 126 : k;
    }
    const float s = __int_as_float((127 + k) << 23), si = __int_as_float((127 - k) << 23);
    if (threadIdx.x == 0) rinv[m] = gamma ? si * rsqrtf(ss / (float)K + eps) : si;
    uint4 *out = reinterpret_cast<uint4 *>(xh + (size_t)m * K);
    for (int g = threadIdx.x; g < K / 8; g += blockDim.x) {
        float4 a = xr[2 * g], b = xr[2 * g + 1];
        if (gamma) {
            const float4 ga = gr[2 * g], gb = gr[2 * g + 1];
            a.x *= ga.x; a.y *= ga.y; a.z *= ga.z; a.w *= ga.w;
            b.x *= gb.x; b.y *= gb.y; b.z *= gb.z; b.w *= gb.w;
        }
        uint4 o;  // positions 0..7 <- elements 0,2,1,3,4,6,5,7
        o.x = h2_bits(__floats2half2_rn(a.x * s, a.z * s));
        o.y = h2_bits(__floats2half2_rn(a.y * s, a.w * s));
        o.z = h2_bits(__floats2half2_rn(b.x * s, b.z * s));
        o.w = h2_bits(__floats2half2_rn(b.y * s, b.w * s));
        out[g] = o;
    }
}

// Distributed shared memory: this CTA's shared address `addr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Q4_0 chunk p (inputs 64p .. 64p + 63 of the 256-input step = blocks 2p, 2p + 1 of the row's
// 8-block run at `row`, 18 B each: f16 d, then qs[16] with element i < 16 in the low nibble of
// qs[i] and element i + 16 in the high nibble) -> 8 groups of 8 f16 in the order the activation
// prep uses (0, 2, 1, 3, 4, 6, 5, 7), value d * (q - 8) rounded once.  A block at an even index
// starts 4-byte aligned (qs then 2 bytes off), at an odd index 2 bytes off (qs aligned).
__device__ __forceinline__ void dequant_q40_chunk(const uint8_t *row, int p, uint8_t *brow, int r) {
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
        const int b = 2 * p + bb;
        const uint8_t *base = row + 18 * b;
        uint32_t q[4], dbits;
        if ((b & 1) == 0) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base);
            const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
            dbits = w0 & 0xFFFFu;
            q[0] = __byte_perm(w0, w1, 0x5432);
            q[1] = __byte_perm(w1, w2, 0x5432);
            q[2] = __byte_perm(w2, w3, 0x5432);
            q[3] = __byte_perm(w3, w4, 0x5432);
        } else {
            dbits = *reinterpret_cast<const uint16_t *>(base);
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base + 2);
            q[0] = w[0]; q[1] = w[1]; q[2] = w[2]; q[3] = w[3];
        }
        const float d = half_bits_to_float(dbits);
        const __half2 D = __float2half2_rn(d), M = __float2half2_rn(-8.0f * d);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {  // elements 8jj .. 8jj + 7 of the block
            const int sh = jj < 2 ? 0 : 4;  // low nibbles for elements < 16, high nibbles above
            const uint32_t w0 = q[2 * (jj & 1)] >> sh, w1 = q[2 * (jj & 1) + 1] >> sh;
            uint4 o;
            o.x = deq2(w0 & 0x000F000Fu, D, M);
            o.y = deq2((w0 >> 8) & 0x000F000Fu, D, M);
            o.z = deq2(w1 & 0x000F000Fu, D, M);
            o.w = deq2((w1 >> 8) & 0x000F000Fu, D, M);
            *reinterpret_cast<uint4 *>(brow + (((4 * bb + jj) ^ (r & 7)) << 4)) = o;
        }
    }
}

// ---------------------------------------------------------------------------
// The GEMM.  EPI = kGemmPlain: 256 output columns per tile from one of up to
// three stacked sources.  EPI = kGemmSwiglu: 128 output columns per tile, the
// accumulator's columns 0-127 from the gate rows and 128-255 from the up rows.
// ---------------------------------------------------------------------------
template <int EPI, int FMT>  // FMT: kQ4_K or kQ4_0 (both 144 B of each row per 256 inputs)
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_q4k_kernel(const __grid_constant__ GemmArgs a) {
    constexpr int BNO = EPI == kGemmSwiglu ? kGemmBN / 2 : kGemmBN;  // output columns per tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = sA + kGemmNA * kGemmABytes;
    uint8_t *sR = sB + kGemmNB * kGemmBBytes;
    uint8_t *sRed = smem;  // epilogue fp32 tile [128][kGemmRedPitch], over the (then idle) rings
    uint64_t *bars = reinterpret_cast<uint64_t *>(sR + kGemmNR * kGemmRBytes);
    uint64_t *a_full = bars, *a_empty = a_full + kGemmNA;
    uint64_t *b_full = a_empty + kGemmNA, *b_empty = b_full + kGemmNB;
    uint64_t *r_full = b_empty + kGemmNB, *r_empty = r_full + kGemmNR;
    uint64_t *acc_full = r_empty + kGemmNR;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * BNO;
    const int s0 = (int)((int64_t)blockIdx.z * a.nsb / a.ksplit);
    const int s1 = (int)((int64_t)(blockIdx.z + 1) * a.nsb / a.ksplit);
    const int nsbl = s1 - s0, nch = 4 * nsbl;
    const int rows_valid = a.M - m0 < kGemmBM ? a.M - m0 : kGemmBM;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGemmNA; ++i) { mbar_init(&a_full[i], 1); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < kGemmNB; ++i) { mbar_init(&b_full[i], 8); mbar_init(&b_empty[i], 1); }
        for (int i = 0; i < kGemmNR; ++i) { mbar_init(&r_full[i], 1); mbar_init(&r_empty[i], kGemmDqWarps); }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, kGemmBN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Programmatic dependent launch: the weights do not depend on the previous kernel, so the
    // producer starts the raw-weight ring before it waits; every thread that reads the previous
    // kernel's output (activations, row scales, residual) waits first.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            // weight source of this tile (plain: stacked sources end on 256-row boundaries)
            int src = 0, row0 = n0;
            if (EPI == kGemmPlain) {
                while (src < 2 && n0 >= a.src_end[src]) ++src;
                row0 = n0 - (src > 0 ? a.src_end[src - 1] : 0);
            }
            int issued_r = 0, issued_a = 0;
            auto load_raw = [&](int sl) {
                const int rs = sl % kGemmNR;
                mbar_arrive_expect_tx(&r_full[rs], kGemmRBytes);
                if (FMT == kQ4_0) {  // 2-D byte view {row_bytes, rows}: 144 B = 8 blocks per step
                    if (EPI == kGemmSwiglu) {
                        tma_load_2d(sR + rs * kGemmRBytes, &a.tm_w[0], (s0 + sl) * 144, n0, &r_full[rs]);
                        tma_load_2d(sR + rs * kGemmRBytes + BNO * 144, &a.tm_w[1], (s0 + sl) * 144, n0, &r_full[rs]);
                    } else {
                        tma_load_2d(sR + rs * kGemmRBytes, &a.tm_w[src], (s0 + sl) * 144, row0, &r_full[rs]);
                    }
                } else if (EPI == kGemmSwiglu) {
                    tma_load_3d(sR + rs * kGemmRBytes, &a.tm_w[0], 0, s0 + sl, n0, &r_full[rs]);
                    tma_load_3d(sR + rs * kGemmRBytes + BNO * 144, &a.tm_w[1], 0, s0 + sl, n0, &r_full[rs]);
                } else {
                    tma_load_3d(sR + rs * kGemmRBytes, &a.tm_w[src], 0, s0 + sl, row0, &r_full[rs]);
                }
                issued_r = sl + 1;
            };
            const int early = nsbl < kGemmNR ? nsbl : kGemmNR;
            for (int sl = 0; sl < early; ++sl) load_raw(sl);  // before the dependency wait
            asm volatile("griddepcontrol.wait;" ::: "memory");  // activations come from the previous kernel
            for (int sl = 0; sl < nsbl && !*abort_flag; ++sl) {
                const int rs = sl % kGemmNR;
                if (sl >= kGemmNR) {
                    if (!mbar_wait(&r_empty[rs], (uint32_t)(sl / kGemmNR - 1) & 1u, a.err, kErrWaitEmpty)) {
                        *abort_flag = 1;
                        break;
                    }
                    load_raw(sl);
                }
                for (int p = 0; p < 4; ++p) {
                    const int c = 4 * sl + p, as = c % kGemmNA;
                    if (c >= kGemmNA &&
                        !mbar_wait(&a_empty[as], (uint32_t)(c / kGemmNA - 1) & 1u, a.err, kErrWaitEmpty)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&a_full[as], kGemmABytes);
                    tma_load_2d(sA + as * kGemmABytes, &a.tm_x, (4 * (s0 + sl) + p) * kGemmBK, m0, &a_full[as]);
                    issued_a = c + 1;
                }
            }
            // Never leave with copies in flight: wait (bounded) for the last fill of every slot.
            for (int j = issued_r > kGemmNR ? issued_r - kGemmNR : 0; j < issued_r; ++j)
                mbar_wait(&r_full[j % kGemmNR], (uint32_t)(j / kGemmNR) & 1u, nullptr, 0);
            for (int j = issued_a > kGemmNA ? issued_a - kGemmNA : 0; j < issued_a; ++j)
                mbar_wait(&a_full[j % kGemmNA], (uint32_t)(j / kGemmNA) & 1u, nullptr, 0);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            for (int c = 0; c < nch; ++c) {
                const int as = c % kGemmNA, bs = c % kGemmNB;
                if (*abort_flag || !mbar_wait(&a_full[as], (uint32_t)(c / kGemmNA) & 1u, a.err, kErrWaitFull) ||
                    !mbar_wait(&b_full[bs], (uint32_t)(c / kGemmNB) & 1u, a.err, kErrWaitFull)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kGemmBK / 16; ++kk)
                    mma_f16(tmem, sw128_desc(sA + as * kGemmABytes + 32 * kk), sw128_desc(sB + bs * kGemmBBytes + 32 * kk),
                            kIdesc, (c | kk) != 0);
                mma_commit(&a_empty[as]);
                mma_commit(&b_empty[bs]);
            }
            mma_commit(acc_full);
            // All MMAs complete before the CTA may reuse the rings or free TMEM.
            mbar_wait(acc_full, 0u, a.err, kErrWaitFull);
        }
        __syncwarp();
    } else {
        // ------------------ dequantizers, then the TMEM -> smem drain ------------------
        // row of the 256-row weight tile; with 16 dequantizer warps, two threads share a row and take
        // alternate 64-element chunks, so that both ring slots fill at once (b_full still counts 8 warps)
        const int r = (threadIdx.x - 64) & 255, pbeg = kGemmDqWarps == 16 ? ((threadIdx.x - 64) >> 8) : 0;
        constexpr int pstep = kGemmDqWarps == 16 ? 2 : 1;
        for (int sl = 0; sl < nsbl; ++sl) {
            const int rs = sl % kGemmNR;
            // every wait's outcome is made warp-uniform: the warp-synchronous code below needs all lanes
            if (!__all_sync(0xffffffffu,
                            !*abort_flag && mbar_wait(&r_full[rs], (uint32_t)(sl / kGemmNR) & 1u, a.err, kErrWaitFull))) {
                *abort_flag = 1;
                break;
            }
            const uint8_t *blk = sR + rs * kGemmRBytes + r * 144;
            const uint4 h = FMT == kQ4_K ? *reinterpret_cast<const uint4 *>(blk) : make_uint4(0u, 0u, 0u, 0u);
            const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
            // q4k_scale_min (reference kernel.cu:913-921), all eight sub-blocks as packed bytes
            const uint32_t sc03 = h.y & 0x3F3F3F3Fu, m03 = h.z & 0x3F3F3F3Fu;
            const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
            bool ok = true;
#pragma unroll
            for (int pp = 0; pp < 4 * 8 / kGemmDqWarps; ++pp) {
                const int p = pbeg + pstep * pp;
                const int c = 4 * sl + p, bs = c % kGemmNB;
                if (c >= kGemmNB &&
                    !__all_sync(0xffffffffu, !*abort_flag && mbar_wait(&b_empty[bs], (uint32_t)(c / kGemmNB - 1) & 1u,
                                                                       a.err, kErrWaitEmpty))) {
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                uint8_t *brow = sB + bs * kGemmBBytes + r * 128;
                if (FMT == kQ4_0) {
                    dequant_q40_chunk(blk, p, brow, r);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&b_full[bs]);
                    continue;
                }
                const uint32_t scw = p < 2 ? sc03 : sc47, mw = p < 2 ? m03 : m47;
                const int sh0 = 16 * (p & 1), sh1 = sh0 + 8;
                const __half2 D0 = __float2half2_rn(d * (float)((scw >> sh0) & 0xFFu));
                const __half2 M0 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh0) & 0xFFu)));
                const __half2 D1 = __float2half2_rn(d * (float)((scw >> sh1) & 0xFFu));
                const __half2 M1 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh1) & 0xFFu)));
                const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
                const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
                const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t w0 = W[2 * j], w1 = W[2 * j + 1];
                    uint4 lo, hi;  // sub-block 2p (low nibbles) and 2p+1 (high nibbles), elements 8j..8j+7
                    lo.x = deq2(w0 & 0x000F000Fu, D0, M0);
                    lo.y = deq2((w0 >> 8) & 0x000F000Fu, D0, M0);
                    lo.z = deq2(w1 & 0x000F000Fu, D0, M0);
                    lo.w = deq2((w1 >> 8) & 0x000F000Fu, D0, M0);
                    hi.x = deq2((w0 >> 4) & 0x000F000Fu, D1, M1);
                    hi.y = deq2((w0 >> 12) & 0x000F000Fu, D1, M1);
                    hi.z = deq2((w1 >> 4) & 0x000F000Fu, D1, M1);
                    hi.w = deq2((w1 >> 12) & 0x000F000Fu, D1, M1);
                    *reinterpret_cast<uint4 *>(brow + ((j ^ (r & 7)) << 4)) = lo;
                    *reinterpret_cast<uint4 *>(brow + (((4 + j) ^ (r & 7)) << 4)) = hi;
                }
                fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core's async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[bs]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&r_empty[rs]);
            if (!ok) break;
        }

        // Drain TMEM into the shared fp32 tile (row = accumulator lane).  The MMA
        // thread's completed acc_full also means every ring slot is idle.
        const bool ok = warp < 10 && __all_sync(0xffffffffu, !*abort_flag && mbar_wait(acc_full, 0u, a.err, kErrWaitFull));
        tc_fence_after();
        const int q = warp & 3, hcol = (warp - 2) >> 2;  // TMEM lane quadrant, column half (warps 2-9 drain)
        const int row = 32 * q + lane;
        if (ok) {
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t v[32];
                const int col = hcol * 128 + cc * 32;
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col, v);
                if (row < rows_valid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(sRed + (size_t)row * kGemmRedPitch + col * 4);
#pragma unroll
                    for (int i = 0; i < 8; ++i) dst[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kGemmBN);
    }

    // ---- epilogue: sum the cluster's partial tiles (fixed order), scale, store ----
    asm volatile("griddepcontrol.wait;" ::: "memory");  // row scales, bias and residual of earlier kernels
    const int ks = a.ksplit;
    if (ks > 1) cluster_sync_all();
    const int z = ks > 1 ? (int)cluster_rank() : 0;
    const int r_lo = z * rows_valid / ks, r_hi = (z + 1) * rows_valid / ks;
    constexpr int C4 = BNO / 4;  // float4 items per output row
    const uint32_t red_base = smem_u32(sRed);
    const bool good = !*abort_flag;
    static_assert(C4 % 32 == 0 && kGemmThreads % C4 == 0, "a warp's epilogue items must share one output row");
    // the warp-collective argmax reduction below needs whole warps in every iteration
    const int items = (r_hi - r_lo) * C4;
    for (int it = threadIdx.x; good && it - (threadIdx.x & 31) < items; it += kGemmThreads) {
        if (it >= items) {  // idle lanes of a partial warp still join the shuffles
            if (EPI == kGemmPlain && a.amax.amax != nullptr) warp_max_u64(0ull);
            continue;
        }
        const int rr = r_lo + it / C4, c4 = it % C4;
        const uint32_t off = red_base + (uint32_t)(rr * kGemmRedPitch + c4 * 16);
        float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0;
        for (int i = 0; i < ks; ++i) {  // cluster CTA order: a fixed summation order
            const uint32_t pa = ks > 1 ? mapa_shared(off, (uint32_t)i) : off;
            acc0 = f4_add(acc0, ld_cluster_v4(pa));
            if (EPI == kGemmSwiglu) acc1 = f4_add(acc1, ld_cluster_v4(pa + BNO * 4));
        }
        const int gm = m0 + rr, gn = n0 + 4 * c4;
        const float sc = a.rinv[gm];
        float o[4] = {acc0.x * sc, acc0.y * sc, acc0.z * sc, acc0.w * sc};
        if (EPI == kGemmSwiglu) {
            const float u[4] = {acc1.x * sc, acc1.y * sc, acc1.z * sc, acc1.w * sc};
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] = silu_mul(o[e], u[e]);
        }
        float *yp = a.y + (size_t)gm * a.y_stride + gn;
        if (a.vec && gn + 4 <= a.N) {
            float4 v4 = make_float4(o[0], o[1], o[2], o[3]);
            if (EPI == kGemmPlain && a.bias) v4 = f4_add(v4, *reinterpret_cast<const float4 *>(a.bias + gn));
            if (EPI == kGemmPlain && a.accumulate) v4 = f4_add(v4, *reinterpret_cast<const float4 *>(yp));
            if (a.y) *reinterpret_cast<float4 *>(yp) = v4;
            o[0] = v4.x; o[1] = v4.y; o[2] = v4.z; o[3] = v4.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (gn + e < a.N) {
                    float v = o[e];
                    if (EPI == kGemmPlain && a.bias) v += a.bias[gn + e];
                    if (EPI == kGemmPlain && a.accumulate) v += yp[e];
                    if (a.y) yp[e] = v;
                    o[e] = v;
                }
        }
        if (EPI == kGemmPlain && a.amax.amax != nullptr) {
            // a warp's items lie in one output row (C4 and the thread count are multiples of 32 items)
            unsigned long long k = 0ull;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const unsigned long long ke = gn + e < a.N ? amax_key(o[e], (uint32_t)(gn + e + a.amax.offset)) : 0ull;
                k = ke > k ? ke : k;
            }
            k = warp_max_u64(k);
            if ((threadIdx.x & 31) == 0 && k != 0ull) atomicMax(&a.amax.amax[gm], k);
        }
    }
    if (EPI == kGemmPlain && a.amax.amax != nullptr) {
        __syncthreads();
        if (threadIdx.x == 0) amax_cta_done(a.amax, a.M);
    }
    if (ks > 1) cluster_sync_all();  // peers may still be reading this CTA's tile
}


// ---------------------------------------------------------------------------
// Prefill GEMM with the weights as the MMA's M side (gemm_ta): one CTA per 128 weight rows
// (SwiGLU: 64 gate + 64 up) x NTOK tokens.  The dequantizers write the weights straight into
// tensor memory (tcgen05.st; the MMA reads A from TMEM), so each weight is dequantized once per
// NTOK tokens and never passes through shared memory; the activations (xprep's f16 rows) are the
// B operand, loaded by TMA in the canonical K-major 128-byte-swizzled layout.  Warp 0: TMA; warp 1:
// TMEM owner and MMA issuer (M 128, N NTOK, K 16; fp32 accumulator in TMEM columns [0, NTOK));
// warps 2-9: thread = weight row (TMEM lane) x half block, then the epilogue (TMEM -> registers ->
// global, one token column per register).
// ---------------------------------------------------------------------------
constexpr int kTaThreads = 320;
constexpr int kTaNR = 4;         // raw weight ring slots (barrier arrays; Q8_0 uses 2 of them)
constexpr int kTaNX = 4;         // activation ring: NTOK tokens x 64 inputs
constexpr int kTaNA = 2;         // dequantized blocks in TMEM (128 columns each)
constexpr uint32_t kTaTmemA = 256;
// Bytes of one weight row per 256 inputs: Q4_K one super-block, Q4_0 8 x 18, Q8_0 8 x 34.
__host__ __device__ constexpr int ta_row_bytes(int fmt) { return fmt == kQ8_0 ? 272 : 144; }
// Raw weight ring depth: 4 stages of 128 x 144 B, or 2 of 128 x 272 B (Q8_0), within 227 KB.
__host__ __device__ constexpr int ta_ring(int fmt) { return fmt == kQ8_0 ? 2 : kTaNR; }
__host__ __device__ constexpr int ta_smem(int ntok, int fmt) {
    return 1024 + kTaNX * ntok * 128 + ta_ring(fmt) * 128 * ta_row_bytes(fmt) + 256;
}
static_assert(ta_smem(256, kQ8_0) <= 232448 && ta_smem(256, kQ4_K) <= 232448, "gemm_ta shared memory");

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}

// Q4_K: the 64 f16 values of chunk p (sub-blocks 2p, 2p+1) of a row's block, as 32 TMEM columns
// (column 4jj + i: elements of sub-block 2p, group jj; 16 + 4jj + i: sub-block 2p + 1).
__device__ __forceinline__ void q4k_chunk_cols(const uint8_t *blk, const uint4 &hd, int p, uint32_t (&v)[32]) {
    const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
    const uint32_t scw = p < 2 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
    const uint32_t mw = p < 2 ? (hd.z & 0x3F3F3F3Fu) : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
    const int sh0 = 16 * (p & 1), sh1 = sh0 + 8;
    const __half2 D0 = __float2half2_rn(d * (float)((scw >> sh0) & 0xFFu));
    const __half2 M0 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh0) & 0xFFu)));
    const __half2 D1 = __float2half2_rn(d * (float)((scw >> sh1) & 0xFFu));
    const __half2 M1 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh1) & 0xFFu)));
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
    const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const uint32_t w0 = W[2 * jj], w1 = W[2 * jj + 1];
        v[4 * jj + 0] = deq2(w0 & 0x000F000Fu, D0, M0);
        v[4 * jj + 1] = deq2((w0 >> 8) & 0x000F000Fu, D0, M0);
        v[4 * jj + 2] = deq2(w1 & 0x000F000Fu, D0, M0);
        v[4 * jj + 3] = deq2((w1 >> 8) & 0x000F000Fu, D0, M0);
        v[16 + 4 * jj + 0] = deq2((w0 >> 4) & 0x000F000Fu, D1, M1);
        v[16 + 4 * jj + 1] = deq2((w0 >> 12) & 0x000F000Fu, D1, M1);
        v[16 + 4 * jj + 2] = deq2((w1 >> 4) & 0x000F000Fu, D1, M1);
        v[16 + 4 * jj + 3] = deq2((w1 >> 12) & 0x000F000Fu, D1, M1);
    }
}
// Q4_0: chunk p (blocks 2p, 2p + 1 of the row's 8-block run) as 32 TMEM columns in the same
// element order (columns 16 bb + 4 jj + i: block 2p + bb, elements 8 jj ..).
__device__ __forceinline__ void q40_chunk_cols(const uint8_t *row, int p, uint32_t (&v)[32]) {
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
        const int b = 2 * p + bb;
        const uint8_t *base = row + 18 * b;
        uint32_t q[4], dbits;
        if ((b & 1) == 0) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base);
            const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
            dbits = w0 & 0xFFFFu;
            q[0] = __byte_perm(w0, w1, 0x5432);
            q[1] = __byte_perm(w1, w2, 0x5432);
            q[2] = __byte_perm(w2, w3, 0x5432);
            q[3] = __byte_perm(w3, w4, 0x5432);
        } else {
            dbits = *reinterpret_cast<const uint16_t *>(base);
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base + 2);
            q[0] = w[0]; q[1] = w[1]; q[2] = w[2]; q[3] = w[3];
        }
        const float d = half_bits_to_float(dbits);
        const __half2 D = __float2half2_rn(d), M = __float2half2_rn(-8.0f * d);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int sh = jj < 2 ? 0 : 4;
            const uint32_t w0 = q[2 * (jj & 1)] >> sh, w1 = q[2 * (jj & 1) + 1] >> sh;
            v[16 * bb + 4 * jj + 0] = deq2(w0 & 0x000F000Fu, D, M);
            v[16 * bb + 4 * jj + 1] = deq2((w0 >> 8) & 0x000F000Fu, D, M);
            v[16 * bb + 4 * jj + 2] = deq2(w1 & 0x000F000Fu, D, M);
            v[16 * bb + 4 * jj + 3] = deq2((w1 >> 8) & 0x000F000Fu, D, M);
        }
    }
}

// Q8_0: chunk p (blocks 2p, 2p + 1 of the row's 8-block run, 34 B each) as 32 TMEM columns in the
// same element order (column 16 bb + 4 jj + i: block 2p + bb, elements 8 jj + {0, 2}, {1, 3}, {4, 6},
// {5, 7}).  Each quant is biased to an unsigned byte (q + 128) for the f16 magic-number conversion;
// d * (u - 128) is one f16 fma, so every weight is f16(d * q), rounded once.
__device__ __forceinline__ void q80_chunk_cols(const uint8_t *row, int p, uint32_t (&v)[32]) {
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
        const uint8_t *base = row + 34 * (2 * p + bb);
        uint32_t q[8], dbits;
        if (bb == 0) {  // the block starts on 4 bytes (row pitch 272 B, 68 B per chunk)
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base);
            uint32_t w9[9];
#pragma unroll
            for (int i = 0; i < 9; ++i) w9[i] = w[i];
            dbits = w9[0] & 0xFFFFu;
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = __byte_perm(w9[i], w9[i + 1], 0x5432);
        } else {  // 2 bytes past a 4-byte boundary: its quants start on 4 bytes
            dbits = *reinterpret_cast<const uint16_t *>(base);
            const uint32_t *w = reinterpret_cast<const uint32_t *>(base + 2);
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = w[i];
        }
        const float d = half_bits_to_float(dbits);
        const __half2 D = __float2half2_rn(d), M = __float2half2_rn(-128.0f * d);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const uint32_t w0 = q[2 * jj] ^ 0x80808080u, w1 = q[2 * jj + 1] ^ 0x80808080u;
            v[16 * bb + 4 * jj + 0] = deq2(w0 & 0x00FF00FFu, D, M);
            v[16 * bb + 4 * jj + 1] = deq2((w0 >> 8) & 0x00FF00FFu, D, M);
            v[16 * bb + 4 * jj + 2] = deq2(w1 & 0x00FF00FFu, D, M);
            v[16 * bb + 4 * jj + 3] = deq2((w1 >> 8) & 0x00FF00FFu, D, M);
        }
    }
}

template <int EPI, int FMT, int NTOK>
__global__ void __launch_bounds__(kTaThreads, 1) gemm_ta_kernel(const __grid_constant__ GemmArgs a) {
    constexpr int RO = EPI == kGemmSwiglu ? 64 : 128;  // output columns (weight rows) per tile
    constexpr int WRB = ta_row_bytes(FMT);              // bytes of one weight row per stage
    constexpr int NR = ta_ring(FMT);                    // raw weight ring depth
    constexpr int RBYTES = 128 * WRB;                   // one raw weight stage
    constexpr int XB = NTOK * 128;                     // bytes of one activation chunk slot
    constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(NTOK >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sX = smem;
    uint8_t *sR = sX + kTaNX * XB;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sR + NR * RBYTES);
    uint64_t *rfull = bars, *rempty = rfull + kTaNR, *xfull = rempty + kTaNR, *xempty = xfull + kTaNX;
    uint64_t *afull = xempty + kTaNX, *aempty = afull + kTaNA, *accfull = aempty + kTaNA;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accfull + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * NTOK, n0 = blockIdx.y * RO;
    const int nsb = a.nsb;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NR; ++i) { mbar_init(&rfull[i], 1); mbar_init(&rempty[i], 8); }
        for (int i = 0; i < kTaNX; ++i) { mbar_init(&xfull[i], 1); mbar_init(&xempty[i], 1); }
        for (int i = 0; i < kTaNA; ++i) { mbar_init(&afull[i], 8); mbar_init(&aempty[i], 1); }
        mbar_init(accfull, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane != 0) return;
        int src = 0, row0 = n0;
        if (EPI == kGemmPlain) {
            while (src < 2 && n0 >= a.src_end[src]) ++src;
            row0 = n0 - (src > 0 ? a.src_end[src - 1] : 0);
        }
        auto load_raw = [&](int b) {
            const int rs = b % NR;
            uint8_t *dst = sR + rs * RBYTES;
            mbar_arrive_expect_tx(&rfull[rs], RBYTES);
            if (FMT == kQ8_0) {  // 2-D view of 2-byte elements: 136 of them = 8 blocks = 256 inputs
                if (EPI == kGemmSwiglu) {
                    tma_load_2d(dst, &a.tm_w[0], b * 136, n0, &rfull[rs]);
                    tma_load_2d(dst + 64 * WRB, &a.tm_w[1], b * 136, n0, &rfull[rs]);
                } else {
                    tma_load_2d(dst, &a.tm_w[src], b * 136, row0, &rfull[rs]);
                }
            } else if (FMT == kQ4_0) {
                if (EPI == kGemmSwiglu) {
                    tma_load_2d(dst, &a.tm_w[0], b * 144, n0, &rfull[rs]);
                    tma_load_2d(dst + 64 * 144, &a.tm_w[1], b * 144, n0, &rfull[rs]);
                } else {
                    tma_load_2d(dst, &a.tm_w[src], b * 144, row0, &rfull[rs]);
                }
            } else if (EPI == kGemmSwiglu) {
                tma_load_3d(dst, &a.tm_w[0], 0, b, n0, &rfull[rs]);
                tma_load_3d(dst + 64 * 144, &a.tm_w[1], 0, b, n0, &rfull[rs]);
            } else {
                tma_load_3d(dst, &a.tm_w[src], 0, b, row0, &rfull[rs]);
            }
        };
        const int early = nsb < NR ? nsb : NR;
        for (int b = 0; b < early; ++b) load_raw(b);  // weights do not depend on the previous kernel
        asm volatile("griddepcontrol.wait;" ::: "memory");  // activations: xprep's output
        int issued_r = early, issued_x = 0;
        for (int b = 0; b < nsb && !*abort_flag; ++b) {
            if (b >= NR) {
                if (!mbar_wait(&rempty[b % NR], (uint32_t)(b / NR - 1) & 1u, a.err, kErrWaitEmpty)) {
                    *abort_flag = 1;
                    break;
                }
                load_raw(b);
                issued_r = b + 1;
            }
            for (int c = 0; c < 4; ++c) {
                const int qx = 4 * b + c, xs = qx % kTaNX;
                if (qx >= kTaNX &&
                    !mbar_wait(&xempty[xs], (uint32_t)(qx / kTaNX - 1) & 1u, a.err, kErrWaitEmpty)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&xfull[xs], XB);
                tma_load_2d(sX + xs * XB, &a.tm_x, 256 * b + 64 * c, m0, &xfull[xs]);
                issued_x = qx + 1;
            }
        }
        // never leave with copies in flight
        for (int j = issued_r > NR ? issued_r - NR : 0; j < issued_r; ++j)
            mbar_wait(&rfull[j % NR], (uint32_t)(j / NR) & 1u, nullptr, 0);
        for (int j = issued_x > kTaNX ? issued_x - kTaNX : 0; j < issued_x; ++j)
            mbar_wait(&xfull[j % kTaNX], (uint32_t)(j / kTaNX) & 1u, nullptr, 0);
        return;
    }
    if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            for (int b = 0; b < nsb; ++b) {
                const int as = b % kTaNA;
                if (*abort_flag || !mbar_wait(&afull[as], (uint32_t)(b / kTaNA) & 1u, a.err, kErrWaitFull)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                bool ok = true;
                for (int c = 0; c < 4; ++c) {
                    const int qx = 4 * b + c, xs = qx % kTaNX;
                    if (!mbar_wait(&xfull[xs], (uint32_t)(qx / kTaNX) & 1u, a.err, kErrWaitFull)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_f16_ta(tmem, tmem + kTaTmemA + 128u * (uint32_t)as + 32u * (uint32_t)c + 8u * (uint32_t)kk,
                                   sw128_desc(sX + xs * XB + 32 * kk), IDESC, (b | c | kk) != 0);
                    mma_commit(&xempty[xs]);
                }
                mma_commit(&aempty[as]);
                if (!ok) break;
            }
            mma_commit(accfull);
            // every MMA has completed before TMEM may be freed
            mbar_wait(accfull, 0u, a.err, kErrWaitFull);
        }
        __syncwarp();
    } else {
        // ------------------- dequantizers, then the epilogue -------------------
        const int q = warp & 3, hf = (warp - 2) >> 2;
        const int r = 32 * q + lane;  // TMEM lane = the MMA's output row
        // staged weight row this thread decodes: plain = its TMEM lane; SwiGLU = gate row 16q + l (lanes
        // 0-15) or up row 16q + l - 16 (lanes 16-31), so one warp holds both halves of 16 output columns
        const int srow = EPI == kGemmSwiglu ? (lane < 16 ? 16 * q + lane : 64 + 16 * q + lane - 16) : r;
        bool ok = true;
        for (int b = 0; b < nsb; ++b) {
            const int rs = b % NR, as = b % kTaNA;
            if (!__all_sync(0xffffffffu,
                            !*abort_flag && mbar_wait(&rfull[rs], (uint32_t)(b / NR) & 1u, a.err, kErrWaitFull))) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            if (b >= kTaNA &&
                !__all_sync(0xffffffffu, !*abort_flag && mbar_wait(&aempty[as], (uint32_t)(b / kTaNA - 1) & 1u, a.err,
                                                                    kErrWaitEmpty))) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            const uint8_t *rowp = sR + rs * RBYTES + srow * WRB;
            const uint4 hd = FMT == kQ4_K ? *reinterpret_cast<const uint4 *>(rowp) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const int pch = 2 * hf + cc;
                uint32_t v[32];
                if (FMT == kQ8_0) q80_chunk_cols(rowp, pch, v);
                else if (FMT == kQ4_0) q40_chunk_cols(rowp, pch, v);
                else q4k_chunk_cols(rowp, hd, pch, v);
                tmem_st32(tmem + ((uint32_t)(32 * q) << 16) + kTaTmemA + 128u * (uint32_t)as + 32u * (uint32_t)pch, v);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&afull[as]);
                mbar_arrive(&rempty[rs]);
            }
        }
        ok = __all_sync(0xffffffffu, ok && !*abort_flag && mbar_wait(accfull, 0u, a.err, kErrWaitFull));
        tc_fence_after();
        asm volatile("griddepcontrol.wait;" ::: "memory");  // row scales, bias and residual of earlier kernels
        // token columns [hf * NTOK / 2, (hf + 1) * NTOK / 2) of the accumulator, 32 at a time
        for (int cb = 0; cb < NTOK / 64; ++cb) {
            const int col0 = hf * (NTOK / 2) + 32 * cb;
            uint32_t v[32];
            tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)col0, v);
            if (EPI == kGemmSwiglu) {
                // lanes l and l ^ 16 hold the gate and up sums of output column n0 + 16q + (l & 15):
                // one exchange, then lanes 0-15 finish tokens col0 .. +15 and lanes 16-31 the rest
                const int n = n0 + 16 * q + (lane & 15);
                const bool up = lane >= 16;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float mine = __uint_as_float(v[i]);
                    const float other = __shfl_xor_sync(0xffffffffu, mine, 16);
                    const int t = m0 + col0 + i;
                    if (ok && (i >= 16) == up && t < a.M && n < a.N) {
                        const float sc = a.rinv[t];
                        a.y[(size_t)t * a.y_stride + n] = silu_mul((up ? other : mine) * sc, (up ? mine : other) * sc);
                    }
                }
            } else if (ok) {
                const int n = n0 + r;
                if (n < a.N) {
                    const float bv = a.bias != nullptr ? a.bias[n] : 0.f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int t = m0 + col0 + i;
                        if (t < a.M) {
                            float *yp = a.y + (size_t)t * a.y_stride + n;
                            float o = __uint_as_float(v[i]) * a.rinv[t] + bv;
                            if (a.accumulate) o += *yp;
                            *yp = o;
                        }
                    }
                }
            }
        }
    }
    // warps 1..9 meet before TMEM is freed (warp 0 has returned)
    tc_fence_before();
    named_bar_sync(2, kTaThreads - 32);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}
}  // namespace

cudaError_t gemm_xprep_launch(const float *x, int64_t x_stride, const float *gamma, float eps, __half *xh,
                              float *rinv, int M, int K, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = gemv_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_xprep_kernel, x, x_stride, gamma, eps, xh, rinv, K);
}

template <int EPI, int FMT>
cudaError_t gemm_launch_t(const GemmArgs &a, cudaStream_t s) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e =
            cudaFuncSetAttribute(gemm_q4k_kernel<EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    constexpr int BNO = EPI == kGemmSwiglu ? kGemmBN / 2 : kGemmBN;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((a.M + kGemmBM - 1) / kGemmBM, (a.N + BNO - 1) / BNO, a.ksplit);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = kGemmSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (gemv_pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (a.ksplit > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = (unsigned)a.ksplit;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, gemm_q4k_kernel<EPI, FMT>, a);
}


template <int EPI, int FMT, int NTOK>
cudaError_t gemm_ta_launch_t(const GemmArgs &a, cudaStream_t s) {
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemm_ta_kernel<EPI, FMT, NTOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             ta_smem(NTOK, FMT));
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    constexpr int RO = EPI == kGemmSwiglu ? 64 : 128;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((a.M + NTOK - 1) / NTOK, (a.N + RO - 1) / RO, 1);
    cfg.blockDim = dim3(kTaThreads);
    cfg.dynamicSmemBytes = ta_smem(NTOK, FMT);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = gemv_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_ta_kernel<EPI, FMT, NTOK>, a);
}

// 256-token tiles dequantize each weight half as often as 128-token tiles, but only when they still
// give every SM a tile; otherwise the smaller tiles fill more SMs.
int gemm_ta_tokens(int M, int row_tiles, int sms) {
    return (M >= 256 && (int64_t)((M + 255) / 256) * row_tiles >= sms) ? 256 : 128;
}

cudaError_t gemm_ta_launch(const GemmArgs &a, int epi, int ntok, cudaStream_t s) {
    if (ntok == 256) {
        if (a.fmt == kQ8_0)
            return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ8_0, 256>(a, s)
                                      : gemm_ta_launch_t<kGemmPlain, kQ8_0, 256>(a, s);
        if (a.fmt == kQ4_0)
            return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ4_0, 256>(a, s)
                                      : gemm_ta_launch_t<kGemmPlain, kQ4_0, 256>(a, s);
        return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ4_K, 256>(a, s)
                                  : gemm_ta_launch_t<kGemmPlain, kQ4_K, 256>(a, s);
    }
    if (a.fmt == kQ8_0)
        return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ8_0, 128>(a, s)
                                  : gemm_ta_launch_t<kGemmPlain, kQ8_0, 128>(a, s);
    if (a.fmt == kQ4_0)
        return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ4_0, 128>(a, s)
                                  : gemm_ta_launch_t<kGemmPlain, kQ4_0, 128>(a, s);
    return epi == kGemmSwiglu ? gemm_ta_launch_t<kGemmSwiglu, kQ4_K, 128>(a, s)
                              : gemm_ta_launch_t<kGemmPlain, kQ4_K, 128>(a, s);
}

cudaError_t gemm_q4k_launch(const GemmArgs &a, int epi, cudaStream_t s) {
    if (a.fmt == kQ4_0)
        return epi == kGemmSwiglu ? gemm_launch_t<kGemmSwiglu, kQ4_0>(a, s) : gemm_launch_t<kGemmPlain, kQ4_0>(a, s);
    return epi == kGemmSwiglu ? gemm_launch_t<kGemmSwiglu, kQ4_K>(a, s) : gemm_launch_t<kGemmPlain, kQ4_K>(a, s);
}

}  // namespace ql
