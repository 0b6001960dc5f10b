// ql_bchain.cu -- batched decode: a decode step's Q4_K projections for up to 32 tokens in one
// persistent launch on the tensor cores.
//
// The reference runs batched decode and prefill as one warp per (token, output row) on the
// CUDA cores (quant_matmul_kernel, AI/codes/local-llm/src/backend/cuda/ops/kernel.cu:1253-1279,
// via launch_quant_matmul, launch.cu:101-119), or as dequantize-to-f16 plus cuBLAS
// (TensorTool.cpp:127-144).  At 8..32 tokens the step is still bound by the weight stream (each
// weight is used by every token once), so the design goal is to decode every weight exactly once
// per step, with few instructions, straight into tensor-core operands:
//
//   * One cooperative launch of one CTA per SM runs the whole op list (same semantics as
//     ql_gemv_chain: stacked q/k/v with RMSNorm and bias, o + residual, gate/up SwiGLU, down +
//     residual, ..., LM head + greedy argmax) for M tokens.  Ops are separated by a grid barrier
//     (monotonic arrival counters, so a CUDA graph can replay the launch without resets).
//   * Work unit = a tile of 128 output rows (SwiGLU: 64 gate + 64 up rows) x one Q4_K block (256
//     inputs).  Units are split over the CTAs in equal contiguous ranges (stream-K); a tile shared
//     by several CTAs is finished by the last to arrive, which sums the parts in CTA order
//     (deterministic).
//   * Warp 0 streams the raw Q4_K bytes of every unit (TMA box {144 B, 1 block, 128 rows}) into a
//     4-slot ring as far ahead as the ring allows, across op boundaries (weights do not depend on
//     activations).  Warp 1 waits for the op's grid barrier and then streams the unit's activations,
//     fp32 [tokens][256], as a 128-byte-swizzled TMA box into a 2-slot ring.
//   * Warps 2..9 (2 row sets of 64 rows x 4 k-chunks of 64 inputs; two consumer warps per
//     scheduler partition hide each other's latency) decode their weights in registers into f16
//     mma.sync A fragments: one 32-bit word of Q4_K nibbles gives four f16x2
//     operands through (w & 0x000F000F) | 0x6400 (= 1024 + n, exact), an exact f16 subtraction of
//     1024 and one f16 FMA with the sub-block's (d*sc, -dmin*m) -- the reference's value formula
//     d*sc*q - dmin*m (kernel.cu:913-921,1090-1119) rounded once to f16.  Activations are read from
//     the swizzled tile, multiplied by the RMSNorm weight and converted to f16 B fragments in
//     registers.  mma.sync.m16n8k16 accumulates in fp32 (64 rows x 32 tokens per warp).
//     The k order inside a 16-element step is permuted identically on both operands (element
//     4t + {0, 2, 1, 3} of a step goes to logical position 2t, 2t+1, 2t+8, 2t+9), which lets one
//     AND extract two operands from bytes 0 and 2 (or 1 and 3) of a word.
//   * At the end of a tile the four k-chunk partials meet in shared memory and the epilogue runs
//     (RMSNorm factor, bias, residual add, SwiGLU, greedy-argmax keys).  The RMSNorm factor of an op
//     needs the sum of squares of its whole input row per token: the op that produced that input
//     (an ADD or STORE of the chain) accumulates it in its epilogue in 64-bit fixed point (exact,
//     order-free, so deterministic); an input written outside the chain is summed by each CTA.
//
// Numerics: weights and activations (x * gamma) rounded to f16, fp32 accumulation; |x * gamma|
// must stay below 65504.  Every wait is bounded (about 2 s): on expiry the kernel records an error
// in the device error word, stops waiting and exits (ql_check_device reports QL_EDEVICE).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <string>
#include <vector>

#include "../../include/qlinear_b200.h"
#include "ql_common.cuh"

namespace ql {
int set_last_error(int code, const char *msg);
void set_launch_count(int n);
bool q4k_tensor_map_public(CUtensorMap *out, const uint8_t *base, int blocks, uint64_t rows, size_t row_bytes,
                           int box_blocks, int box_rows);
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder_public();
int chain_workspace(float **part, unsigned **counters, int **err, int *sms);

namespace {

constexpr int kBMaxTok = 32;
constexpr int kBRows = 128;                        // output rows per tile
constexpr int kBCw = 8;                            // consumer warps: 2 row sets (64 rows) x 4 k-chunks
constexpr int kBThreads = (2 + kBCw) * 32;         // weight producer, activation producer, consumers
constexpr int kBWSlots = 4;
constexpr int kBXSlots = 2;
constexpr int kBWBytes = kBRows * 144;             // 18,432 B: one block column of a tile
constexpr int kBXBytes = kBMaxTok * 256 * 4;       // 32 KB: one block of up to 32 tokens, fp32
constexpr int kBRedPitch = kBRows + 4;             // floats per (k-chunk, token) row of the reduction tile
constexpr int kBRedBytes = 4 * kBMaxTok * kBRedPitch * 4;
constexpr int kBHdr = 1024;
constexpr int kBOffW = kBHdr;
constexpr int kBOffX = kBOffW + kBWSlots * kBWBytes;     // 1024-byte aligned (128-byte swizzle)
constexpr int kBOffRed = kBOffX + kBXSlots * kBXBytes;
constexpr int kBOffMisc = kBOffRed + kBRedBytes;         // per-warp token reductions
constexpr int kBOffGamma = kBOffMisc + 2 * kBCw * kBMaxTok * 8;  // the op's RMSNorm weight
constexpr int kBGammaMax = 4096;                         // inputs whose RMSNorm weight is staged
constexpr int kBOffPslot = kBOffGamma + kBGammaMax * 4;  // stream-K part slots of the tile being finished
constexpr int kBSmem = kBOffPslot + 256 * 4;
static_assert(kBOffX % 1024 == 0, "activation ring must be 1024-byte aligned");
static_assert(kBSmem <= 227 * 1024, "shared memory");
constexpr int kErrBarrier = 5;
constexpr double kSsFix = 16777216.0;  // 2^24: fixed-point sums of squares

enum BKind : int { kBStore = 0, kBAdd = 1, kBSwiglu = 2 };

struct __align__(128) BOp {
    CUtensorMap wmap[3];  // Q4_K sources {144, blocks, rows}, box {144, 1, 128} (SwiGLU: 64 rows each)
    CUtensorMap xmap;     // activations {32, tokens, K/32} fp32, box {32, 8*NT, 8}, 128-byte swizzle
    int kind, nmat, rows, K, U, tiles;
    int split0, split1;   // stacked sources: first rows of sources 1 and 2 (multiples of 128)
    int64_t T;            // units = tiles * U
    const float *x;
    int64_t xs;
    const float *gamma;
    float eps;
    const float *bias;
    float *y;
    int64_t ys;
    int ss_in;            // slot holding the sums of squares of this op's input rows; -1: sum x here
    int ss_out;           // slot this op's epilogue sums its output's squares into; -1: none
    AmaxOut amax;
    const int *rope_pos;  // RoPE on rows [0, rope_rows): positions per token
    float rope_theta;
    int rope_rows, head_dim;
    __device__ float bias_at(int row) const { return bias != nullptr ? bias[row] : 0.f; }
};

struct BArgs {
    const BOp *ops;
    int nops;
    int M, NT;
    unsigned *done;       // [nops] arrival counters (monotonic)
    unsigned *epoch;      // completed launches
    float *part;          // [C][2][32][128] stream-K partial tiles
    unsigned *counters;   // per-tile arrival counters (zero between ops)
    int *err;
    long long *ss;        // [2][nslots][32] fixed-point sums of squares, by launch parity
    int nslots;
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tmap_acquire(const void *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tma_load_3d_plain(void *dst, const void *tmap, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// Two Q4_K nibbles (bits 0-3 and 16-19 of w) -> f16x2 of n * A + B with (A, B) = ab (f16 lo, hi).
__device__ __forceinline__ uint32_t dq2(uint32_t w, uint32_t aa, uint32_t bb) {
    uint32_t v, n, r;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(v) : "r"(w));  // (w & m) | c
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(n) : "r"(v), "r"(0x64006400u));     // n, exact
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(n), "r"(aa), "r"(bb));
    return r;
}
__device__ __forceinline__ void hmma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (d*sc, -dmin*m) of sub-block j of a Q4_K block header h (bytes 0..15) as f16 (lo: A, hi: B).
__device__ __forceinline__ uint32_t q4k_ab(const uint4 &h, int j) {
    const uint32_t s03 = h.y, s47 = h.z, s811 = h.w;  // scales bytes 0-3, 4-7, 8-11
    uint32_t sc, m;
    if (j < 4) {
        sc = (s03 >> (8 * j)) & 63u;
        m = (s47 >> (8 * j)) & 63u;
    } else {
        const int i = j - 4;
        const uint32_t b8 = (s811 >> (8 * i)) & 0xFFu;
        sc = (b8 & 0x0Fu) | (((s03 >> (8 * i)) >> 6 & 3u) << 4);
        m = (b8 >> 4) | (((s47 >> (8 * i)) >> 6 & 3u) << 4);
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    return pack_h2(d * (float)sc, -dmin * (float)m);
}
// Token of column g of an 8-token MMA tile: 0, 4, 1, 5, 2, 6, 3, 7 (see the B-fragment loads).
__device__ __forceinline__ int tperm(int g) { return (g >> 1) | ((g & 1) << 2); }
__device__ __forceinline__ long long ss_to_fixed(float v) { return __float2ll_rn(v * (float)kSsFix); }
// Stream-K split of an op's T units over min(C, T) CTAs (every participating CTA gets at least
// one unit, so every CTA whose range touches a tile arrives on that tile's counter).
__device__ __forceinline__ int op_ctas(int64_t T, int C) { return T < C ? (int)T : C; }
__device__ __forceinline__ int64_t op_start(int64_t T, int Cp, int c) { return c >= Cp ? T : (int64_t)c * T / Cp; }

template <int NT>  // 8-token MMA tiles per launch (tokens <= 8 * NT)
__global__ void __launch_bounds__(kBThreads, 1) bchain_kernel(const __grid_constant__ BArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *wfull = reinterpret_cast<uint64_t *>(smem);
    uint64_t *wempty = wfull + kBWSlots;
    uint64_t *xfull = wempty + kBWSlots;
    uint64_t *xempty = xfull + kBXSlots;
    int *abort_flag = reinterpret_cast<int *>(xempty + kBXSlots);
    unsigned *epoch_s = reinterpret_cast<unsigned *>(abort_flag + 1);
    int *bcast = reinterpret_cast<int *>(epoch_s + 1);
    float *inv_rms = reinterpret_cast<float *>(smem + 256);           // [32]
    float *red = reinterpret_cast<float *>(smem + kBOffRed);          // [4 chunks][32 tokens][132]
    unsigned long long *wkey = reinterpret_cast<unsigned long long *>(smem + kBOffMisc);  // [warp][32]
    float *wss = reinterpret_cast<float *>(smem + kBOffMisc + kBCw * kBMaxTok * 8);        // [warp][32]
    float *gsm = reinterpret_cast<float *>(smem + kBOffGamma);        // [K] RMSNorm weight of the op
    int *pslot = reinterpret_cast<int *>(smem + kBOffPslot);          // [parts of a shared tile]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, cta = blockIdx.x;
    const int M = a.M;
    if (tid == 0) {
        for (int s = 0; s < kBWSlots; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kBCw);
        }
        for (int s = 0; s < kBXSlots; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], kBCw);
        }
        *abort_flag = 0;
        *epoch_s = *reinterpret_cast<volatile unsigned *>(a.epoch);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned epoch = *epoch_s;
    const unsigned target = (epoch + 1u) * (unsigned)C;
    long long *ss_cur = a.ss + (size_t)(epoch & 1u) * a.nslots * kBMaxTok;
    if (cta == 0)  // the other parity is next launch's: zero it now
        for (int i = tid; i < a.nslots * kBMaxTok; i += blockDim.x)
            a.ss[(size_t)((epoch + 1u) & 1u) * a.nslots * kBMaxTok + i] = 0;
    auto aborted = [&]() { return *reinterpret_cast<volatile int *>(abort_flag) != 0; };

    if (warp == 0) {
        // ---------------------------- weight producer ----------------------------
        if (lane != 0) return;
        int it = 0;
        const uint64_t pol = l2_evict_first_policy();
        for (int p = 0; p < a.nops; ++p) {
            const BOp &o = a.ops[p];
            const int U = o.U, nmat = o.nmat, split0 = o.split0, split1 = o.split1;
            const int64_t T = o.T;
            for (int i = 0; i < 3; ++i) tmap_acquire(&o.wmap[i]);
            const int Cp = op_ctas(T, C);
            const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
            for (int64_t u = u0; u < u1; ++u, ++it) {
                const int slot = it % kBWSlots;
                if (it >= kBWSlots && !aborted() &&
                    !mbar_wait(&wempty[slot], ((uint32_t)(it / kBWSlots) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
                const bool live = !aborted();
                const int tile = (int)(u / U), blk = (int)(u % U);
                uint8_t *dst = smem + kBOffW + slot * kBWBytes;
                mbar_arrive_expect_tx(&wfull[slot], live ? (uint32_t)kBWBytes : 0u);
                if (!live) continue;
                if (nmat == 2) {
                    tma_load_3d_hint(dst, &o.wmap[0], 0, blk, tile * 64, &wfull[slot], pol);
                    tma_load_3d_hint(dst + 64 * 144, &o.wmap[1], 0, blk, tile * 64, &wfull[slot], pol);
                } else {
                    const int row0 = tile * kBRows;
                    const int src = (row0 >= split0) + (row0 >= split1);
                    const int lrow = row0 - (src == 0 ? 0 : (src == 1 ? split0 : split1));
                    tma_load_3d_hint(dst, &o.wmap[src], 0, blk, lrow, &wfull[slot], pol);
                }
            }
        }
        for (int j = (it > kBWSlots ? it - kBWSlots : 0); j < it; ++j)
            mbar_wait(&wfull[j % kBWSlots], (uint32_t)(j / kBWSlots) & 1u, nullptr, 0);
        return;
    }
    if (warp == 1) {
        // -------------------------- activation producer --------------------------
        if (lane != 0) return;
        int it = 0;
        const uint32_t xbytes = (uint32_t)(NT * 8 * 256 * 4);
        for (int p = 0; p < a.nops; ++p) {
            const BOp &o = a.ops[p];
            const int U = o.U;
            const int64_t T = o.T;
            if (p > 0 && !aborted()) {  // grid barrier: op p reads what earlier ops wrote
                const unsigned *d = a.done + (p - 1);
                if (ld_acquire(d) < target) {
                    const uint64_t t0 = global_timer_ns();
                    while (ld_acquire(d) < target) {
                        if (global_timer_ns() - t0 > 2000000000ull) {
                            atomicExch(a.err, kErrBarrier);
                            *abort_flag = 1;
                            break;
                        }
                    }
                }
            }
            // the activations were written by generic-proxy stores; the tensor copies read them
            asm volatile("fence.proxy.async.global;" ::: "memory");
            tmap_acquire(&o.xmap);
            const int Cp = op_ctas(T, C);
            const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
            for (int64_t u = u0; u < u1; ++u, ++it) {
                const int slot = it % kBXSlots;
                if (it >= kBXSlots && !aborted() &&
                    !mbar_wait(&xempty[slot], ((uint32_t)(it / kBXSlots) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
                const bool live = !aborted();
                mbar_arrive_expect_tx(&xfull[slot], live ? xbytes : 0u);
                if (live)
                    tma_load_3d_plain(smem + kBOffX + slot * kBXBytes, &o.xmap, 0, 0, (int)(u % U) * 8, &xfull[slot]);
            }
        }
        for (int j = (it > kBXSlots ? it - kBXSlots : 0); j < it; ++j)
            mbar_wait(&xfull[j % kBXSlots], (uint32_t)(j / kBXSlots) & 1u, nullptr, 0);
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int cw = warp - 2, ctid = tid - 64;
    const int rs = cw >> 2, kc = cw & 3;  // row set (rows 64rs ..), k-chunk (inputs 64kc .. 64kc + 63)
    const int g = lane >> 2, t = lane & 3;
    int itw = 0, itx = 0;
    for (int p = 0; p < a.nops; ++p) {
        const BOp &o = a.ops[p];
        const int kind = o.kind, U = o.U, rows = o.rows, K = o.K;
        const int64_t T = o.T;
        const float *gamma = o.gamma;
        const int Cp = op_ctas(T, C);
            const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
        bool norm_ready = false;
        // the RMSNorm weight (a weight: it does not depend on earlier ops) into shared memory once
        // per op, so the k-steps read it at shared-memory latency
        const bool gstaged = gamma != nullptr && K <= kBGammaMax;
        if (gstaged && u0 < u1) {
            for (int i = ctid; i < K / 4; i += kBCw * 32)
                reinterpret_cast<float4 *>(gsm)[i] = __ldg(reinterpret_cast<const float4 *>(gamma) + i);
        }
        named_bar_sync(1, kBCw * 32);
        const float *gk = gstaged ? gsm : gamma;
        const bool track = o.amax.amax != nullptr || o.ss_out >= 0;
        // per-warp running results over the tiles this CTA finishes (greedy keys, sums of squares),
        // each slot written by one lane only: deterministic
        wkey[cw * kBMaxTok + lane] = 0ull;
        wss[cw * kBMaxTok + lane] = 0.f;
        float acc[4][4][4];  // rows 64rs + 16m + g (+8), tokens of n-tile n
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;

        for (int64_t u = u0; u < u1; ++u, ++itw, ++itx) {
            const int tile = (int)(u / U), blk = (int)(u % U);
            const int ws = itw % kBWSlots, xsl = itx % kBXSlots;
            if (!aborted() && !mbar_wait(&wfull[ws], (uint32_t)(itw / kBWSlots) & 1u, a.err, kErrWaitFull))
                *abort_flag = 1;
            if (!aborted() && !mbar_wait(&xfull[xsl], (uint32_t)(itx / kBXSlots) & 1u, a.err, kErrWaitFull))
                *abort_flag = 1;
            if (!__any_sync(0xffffffffu, aborted())) {
                const uint8_t *wb = smem + kBOffW + ws * kBWBytes + rs * 64 * 144;
                const uint8_t *xb = smem + kBOffX + xsl * kBXBytes;
                // This lane's rows are 16m + g and 16m + g + 8 of the row set (m = 0..3), its inputs
                // 4t .. 4t + 3 of each 16-input step.  Lane (g, t) decodes the sub-block scales of rows
                // 16t + g (+8); the four lanes of a quad then share them.  Few values stay live across
                // the k-steps: scales per sub-block, weight words per m-tile.
                uint32_t mine[2][2];  // [row 16t + g or 16t + g + 8][sub-block 2kc or 2kc + 1]
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 hd = *reinterpret_cast<const uint4 *>(wb + (16 * t + g + 8 * h) * 144);
                    mine[h][0] = q4k_ab(hd, 2 * kc);
                    mine[h][1] = q4k_ab(hd, 2 * kc + 1);
                }
                const uint8_t *wq = wb + g * 144 + 16 + 32 * kc + 4 * t;  // this lane's word of row g, j = 0
#pragma unroll 1
                for (int sh = 0; sh < 2; ++sh) {  // sub-block 2kc (low nibbles), 2kc + 1 (high nibbles)
                    const int sb = 2 * kc + sh;
                    uint32_t ab[4][2];
#pragma unroll
                    for (int m = 0; m < 4; ++m)
#pragma unroll
                        for (int h = 0; h < 2; ++h)
                            ab[m][h] = __shfl_sync(0xffffffffu, sh ? mine[h][1] : mine[h][0], (g << 2) | m);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {  // 16-input step
                        // B fragments: column g of n-tile n is token 8n + tperm(g) (tperm puts the two
                        // rows a quarter-warp reads 4 apart, so their swizzled chunks never collide);
                        // inputs 16j + 4t .. +3 of sub-block sb
                        float2 g01 = make_float2(1.f, 1.f), g23 = make_float2(1.f, 1.f);
                        if (gamma != nullptr) {
                            const float4 gm = *reinterpret_cast<const float4 *>(gk + 256 * blk + 32 * sb + 16 * j + 4 * t);
                            g01 = make_float2(gm.x, gm.z);
                            g23 = make_float2(gm.y, gm.w);
                        }
                        uint32_t bf[4][2];
#pragma unroll
                        for (int n = 0; n < 4; ++n) {
                            if (n < NT) {
                                const int tok = 8 * n + tperm(g);
                                const float4 v = *reinterpret_cast<const float4 *>(
                                    xb + ((size_t)sb * (NT * 8) + tok) * 128 + (((4 * j + t) ^ (tok & 7)) << 4));
                                const float2 p0 = fmul2(make_float2(v.x, v.z), g01);
                                const float2 p1 = fmul2(make_float2(v.y, v.w), g23);
                                bf[n][0] = pack_h2(p0.x, p0.y);
                                bf[n][1] = pack_h2(p1.x, p1.y);
                            } else {
                                bf[n][0] = bf[n][1] = 0u;
                            }
                        }
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const uint32_t a0 = ab[m][0], a1 = ab[m][1];
                            const uint32_t aa0 = __byte_perm(a0, 0, 0x1010), bb0 = __byte_perm(a0, 0, 0x3232);
                            const uint32_t aa1 = __byte_perm(a1, 0, 0x1010), bb1 = __byte_perm(a1, 0, 0x3232);
                            const uint32_t w0 = *reinterpret_cast<const uint32_t *>(wq + (16 * m) * 144 + 16 * j) >> (4 * sh);
                            const uint32_t w1 = *reinterpret_cast<const uint32_t *>(wq + (16 * m + 8) * 144 + 16 * j) >> (4 * sh);
                            uint32_t af[4];
                            af[0] = dq2(w0, aa0, bb0);        // row g,     inputs 4t, 4t+2
                            af[1] = dq2(w1, aa1, bb1);        // row g + 8, inputs 4t, 4t+2
                            af[2] = dq2(w0 >> 8, aa0, bb0);   // row g,     inputs 4t+1, 4t+3
                            af[3] = dq2(w1 >> 8, aa1, bb1);   // row g + 8, inputs 4t+1, 4t+3
#pragma unroll
                            for (int n = 0; n < 4; ++n)
                                if (n < NT) hmma(acc[m][n], af, bf[n][0], bf[n][1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&wempty[ws]);
                mbar_arrive(&xempty[xsl]);
            }
            const bool tile_end = (blk == U - 1) || (u + 1 == u1);
            if (!tile_end) continue;

            // ---------------- end of this CTA's part of a tile ----------------
            if (!norm_ready && gamma != nullptr) {
                // RMSNorm factors of the op's input rows (the op's activations are complete: this
                // CTA consumed at least one of their tiles)
                if (o.ss_in >= 0) {
                    if (ctid < M) {
                        const double s = (double)__ldcg(ss_cur + (size_t)o.ss_in * kBMaxTok + ctid) / kSsFix;
                        inv_rms[ctid] = rsqrtf((float)(s / K) + o.eps);
                    }
                } else {
                    for (int tok = cw; tok < M; tok += kBCw) {
                        const float *xr = o.x + (size_t)tok * o.xs;
                        float s = 0.f;
                        for (int k = 4 * lane; k < K; k += 128) {
                            const float4 v = __ldcg(reinterpret_cast<const float4 *>(xr + k));
                            s = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, s))));
                        }
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                        if (lane == 0) inv_rms[tok] = rsqrtf(s / (float)K + o.eps);
                    }
                }
                norm_ready = true;
            }
            // k-chunk partials -> red[kc][token][row]
            float *rw = red + (size_t)kc * kBMaxTok * kBRedPitch;
#pragma unroll
            for (int m = 0; m < 4; ++m)
#pragma unroll
                for (int n = 0; n < 4; ++n) {
                    if (n < NT) {
                        const int r = 64 * rs + 16 * m + g;
                        const int tk0 = 8 * n + tperm(2 * t), tk1 = 8 * n + tperm(2 * t + 1);
                        rw[tk0 * kBRedPitch + r] = acc[m][n][0];
                        rw[tk1 * kBRedPitch + r] = acc[m][n][1];
                        rw[tk0 * kBRedPitch + r + 8] = acc[m][n][2];
                        rw[tk1 * kBRedPitch + r + 8] = acc[m][n][3];
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;
                }
            named_bar_sync(1, kBCw * 32);
            // The tile's sums over the four k-chunks (from red), or, when the tile is shared with
            // other CTAs, over the parts those CTAs parked (in CTA order): computed per (token, row)
            // where needed, so that few values are live at once.
            const int64_t ts = (int64_t)tile * U, te = ts + U;
            // every decision that leads to a named barrier is uniform over the consumer threads
            // (never the abort flag, which another warp may set at any time)
            const bool partial = ts < u0 || te > u1;
            bool finish = true;
            int nparts = 0;
            auto red_sum = [&](int tk, int row) {
                return red[(0 * kBMaxTok + tk) * kBRedPitch + row] + red[(1 * kBMaxTok + tk) * kBRedPitch + row] +
                       red[(2 * kBMaxTok + tk) * kBRedPitch + row] + red[(3 * kBMaxTok + tk) * kBRedPitch + row];
            };
            if (partial) {
                // stream-K: park this part; the last CTA of the tile sums the parts in CTA order
                const int si = (tile == (int)(u0 / U)) ? 0 : 1;
                float *pp = a.part + ((size_t)cta * 2 + si) * (kBMaxTok * kBRows);
                const int r = ctid & (kBRows - 1), th = ctid >> 7;  // thread = (row, 16 tokens)
#pragma unroll 4
                for (int i = 0; i < 16; ++i) __stcg(pp + (16 * th + i) * kBRows + r, red_sum(16 * th + i, r));
                __threadfence();
                named_bar_sync(1, kBCw * 32);
                const int cf = (int)(((ts + 1) * (int64_t)Cp - 1) / T), cl = (int)((te * (int64_t)Cp - 1) / T);
                nparts = cl - cf + 1;
                if (ctid == 0) *bcast = (int)atomicAdd(&a.counters[tile], 1u) == cl - cf;
                // slot of each part: (CTA, first or last tile of its range)
                for (int i = ctid; i < nparts; i += kBCw * 32) {
                    const int c = cf + i;
                    pslot[i] = 2 * c + ((tile == (int)(op_start(T, Cp, c) / U)) ? 0 : 1);
                }
                named_bar_sync(1, kBCw * 32);
                finish = *bcast != 0;
                if (finish) {
                    __threadfence();
                    if (ctid == 0) a.counters[tile] = 0u;
                }
            }
            auto tile_sum = [&](int tk, int row) {
                if (!partial) return red_sum(tk, row);
                float sacc = 0.f;
                for (int i = 0; i < nparts; ++i)
                    sacc += __ldcg(a.part + (size_t)pslot[i] * (kBMaxTok * kBRows) + tk * kBRows + row);
                return sacc;
            };
            if (finish) {
                if (kind == kBSwiglu) {
                    // thread = (gate row r < 64, 8 tokens); its up row is r + 64
                    const int r = ctid & 63, tq = ctid >> 6;
                    const int row = tile * 64 + r;
                    if (row < rows) {
#pragma unroll 2
                        for (int i = 0; i < 8; ++i) {
                            const int tk = 8 * tq + i;
                            if (tk < M) {
                                const float nrm = gamma != nullptr ? inv_rms[tk] : 1.f;
                                const float gv = tile_sum(tk, r) * nrm, uv = tile_sum(tk, r + 64) * nrm;
                                o.y[(size_t)tk * o.ys + row] = gv / (1.0f + expf(-gv)) * uv;
                            }
                        }
                    }
                } else {
                    // thread = (row r, 16 tokens); warp cw holds rows 32(cw & 3) .., tokens 16(cw >> 2) ..
                    const int r = ctid & (kBRows - 1), th = ctid >> 7;
                    const int row = tile * kBRows + r;
                    const bool live = row < rows;
                    const float bias = (live && o.bias != nullptr) ? o.bias[row] : 0.f;
#pragma unroll 2
                    for (int i = 0; i < 16; ++i) {
                        const int tk = 16 * th + i;
                        float out = 0.f;
                        unsigned long long key = 0ull;
                        if (live && tk < M) {
                            const float nrm = gamma != nullptr ? inv_rms[tk] : 1.f;
                            out = tile_sum(tk, r) * nrm;
                            float *yp = o.y != nullptr ? o.y + (size_t)tk * o.ys + row : nullptr;
                            if (kind == kBAdd) {
                                out += __ldcg(yp);
                                __stcg(yp, out);
                            } else {
                                out += bias;
                                if (row < o.rope_rows) {
                                    // RoPE: rows i and i + half of a head pair up (the reference's
                                    // rotation, kernel.cu:186-260); both lie in this tile
                                    const int hd = o.head_dim, half = hd >> 1, pi = row % hd;
                                    const int i = pi % half, rp = r + (pi < half ? half : -half);
                                    const float xp = tile_sum(tk, rp) * nrm + o.bias_at(tile * kBRows + rp);
                                    const float inv_freq = 1.0f / powf(o.rope_theta, (float)(2 * i) / (float)hd);
                                    const float ang = (float)__ldg(o.rope_pos + tk) * inv_freq;
                                    const float c = cosf(ang), sn = sinf(ang);
                                    out = pi < half ? out * c - xp * sn : out * c + xp * sn;
                                }
                                if (yp) *yp = out;
                            }
                            if (o.amax.amax != nullptr) key = amax_key(out, (uint32_t)(row + o.amax.offset));
                        }
                        if (track) {  // warp-uniform: fold this tile into the warp's running slots
                            key = warp_max_u64(key);
                            float sq = out * out;
#pragma unroll
                            for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
                            if (lane == i) {
                                const unsigned long long kw = wkey[cw * kBMaxTok + tk];
                                wkey[cw * kBMaxTok + tk] = key > kw ? key : kw;
                                wss[cw * kBMaxTok + tk] += sq;
                            }
                        }
                    }
                }
            }
            named_bar_sync(1, kBCw * 32);  // red is free for the next tile
        }

        // ---------------- end of op p on this CTA ----------------
        named_bar_sync(1, kBCw * 32);
        if (track) {
            if (ctid < M) {
                // warps 4h .. 4h + 3 hold tokens 16h .. 16h + 15
                const int h = ctid >> 4;
                unsigned long long k = 0ull;
                float s = 0.f;
                for (int w = 4 * h; w < 4 * h + 4; ++w) {
                    const unsigned long long kw = wkey[w * kBMaxTok + ctid];
                    k = kw > k ? kw : k;
                    s += wss[w * kBMaxTok + ctid];
                }
                if (o.amax.amax != nullptr && k != 0ull) atomicMax(&o.amax.amax[ctid], k);
                if (o.ss_out >= 0)
                    atomicAdd(reinterpret_cast<unsigned long long *>(ss_cur + (size_t)o.ss_out * kBMaxTok + ctid),
                              (unsigned long long)ss_to_fixed(s));
            }
        }
        named_bar_sync(1, kBCw * 32);
        if (ctid == 0) {
            if (o.amax.amax != nullptr) amax_cta_done(o.amax, M);
            __threadfence();
            const unsigned prev = atomicAdd(&a.done[p], 1u);  // this CTA's part of op p is written
            if (p == a.nops - 1 && prev == target - 1u) atomicAdd(a.epoch, 1u);
        }
    }
}

using BKernel = void (*)(const BArgs);
BKernel bchain_kernel_for(int NT) {
    return NT == 1 ? bchain_kernel<1> : NT == 2 ? bchain_kernel<2> : NT == 3 ? bchain_kernel<3> : bchain_kernel<4>;
}

struct BChain {
    int magic = 0x42434821;  // "BCH!": told apart from the one-token chain by ql_gemv_chain_run
    BOp *ops_dev = nullptr;
    unsigned *done = nullptr;          // [nops] counters, [1] epoch, [nops] argmax counters
    unsigned long long *keys = nullptr;  // [nops][32]
    long long *ss = nullptr;
    float *part = nullptr;
    BArgs args{};
    int sms = 0;
};

bool f32_act_map(CUtensorMap *out, const float *x, int M, int64_t xs, int K, int NT) {
    auto enc = tensor_map_encoder_public();
    if (enc == nullptr) return false;
    const cuuint64_t dims[3] = {32, (cuuint64_t)M, (cuuint64_t)(K / 32)};
    const cuuint64_t strides[2] = {(cuuint64_t)xs * 4, 128};
    const cuuint32_t box[3] = {32, (cuuint32_t)(NT * 8), 8};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Batched chain creation (see include/qlinear_b200.h, ql_gemv_chain_create_batch).
int bchain_create(const ql_chain_op *ops, int nops, int tokens, void **chain) {
    if (!ops || nops <= 0 || !chain) return set_last_error(QL_EINVAL, "ql_gemv_chain_create_batch: need ops");
    if (tokens < 1 || tokens > kBMaxTok)
        return set_last_error(QL_EINVAL, "ql_gemv_chain_create_batch: tokens must be 1..32");
    float *wpart;
    unsigned *counters;
    int *err, sms;
    int st = chain_workspace(&wpart, &counters, &err, &sms);
    if (st) return st;
    const int NT = (tokens + 7) / 8;
    std::vector<BOp> h(nops);
    // rows each op writes (for the producer/consumer analysis of the RMSNorm sums)
    std::vector<int> out_w(nops, 0);
    std::vector<int64_t> out_s(nops, 0);
    int nslots = 0;
    for (int p = 0; p < nops; ++p) {
        const ql_chain_op &q = ops[p];
        BOp &o = h[p];
        memset(&o, 0, sizeof(o));
        const std::string what = "ql_gemv_chain_create_batch: op " + std::to_string(p);
        if (q.quant_type != QL_Q4_K) return set_last_error(QL_EINVAL, (what + ": only Q4_K").c_str());
        if (q.kind == QL_OP_ADD && !q.y) return set_last_error(QL_EINVAL, (what + ": ADD needs y").c_str());
        if (q.kind != QL_OP_STORE && q.kind != QL_OP_ADD && q.kind != QL_OP_SWIGLU)
            return set_last_error(QL_EINVAL, (what + ": STORE, ADD or SWIGLU (no fused MLP in batch mode)").c_str());
        if (q.reduce) return set_last_error(QL_EINVAL, (what + ": no tensor-parallel reduce in batch mode").c_str());
        const int nsrc = q.kind == QL_OP_SWIGLU ? 2 : q.nsrc;
        if (nsrc < 1 || nsrc > 3 || q.in_dim <= 0 || q.in_dim % 256 || !q.x || (!q.y && !q.argmax_idx))
            return set_last_error(QL_EINVAL, (what + ": sources, in_dim (a multiple of 256), x or y").c_str());
        const int64_t xs = q.x_stride ? q.x_stride : q.in_dim;
        if (reinterpret_cast<uintptr_t>(q.x) % 16 || xs % 4 || xs < q.in_dim ||
            reinterpret_cast<uintptr_t>(q.gamma) % 16)
            return set_last_error(QL_EINVAL, (what + ": x and gamma 16-byte aligned, x_stride a multiple of 4").c_str());
        const int blocks = q.in_dim / 256;
        int total = 0;
        for (int s = 0; s < nsrc; ++s) {
            if (!q.w[s] || reinterpret_cast<uintptr_t>(q.w[s]) % 16 || q.row_bytes[s] % 16 ||
                q.row_bytes[s] < (size_t)blocks * 144 || q.rows[s] <= 0)
                return set_last_error(QL_EINVAL, (what + ": weights (16-byte aligned rows)").c_str());
            if (q.kind != QL_OP_SWIGLU && s < nsrc - 1 && q.rows[s] % kBRows)
                return set_last_error(QL_EINVAL, (what + ": stacked sources but the last need multiples of 128 rows").c_str());
            const int box_rows = q.kind == QL_OP_SWIGLU ? 64 : kBRows;
            if (!q4k_tensor_map_public(&o.wmap[s], q.w[s], blocks, (uint64_t)q.rows[s], q.row_bytes[s], 1, box_rows))
                return set_last_error(QL_ECUDA, (what + ": tensor map").c_str());
            if (q.kind != QL_OP_SWIGLU) {
                total += q.rows[s];
                if (s == 0) o.split0 = o.split1 = total;
                if (s == 1) o.split1 = total;
            }
        }
        if (q.kind == QL_OP_SWIGLU) {
            if (q.rows[1] != q.rows[0]) return set_last_error(QL_EINVAL, (what + ": gate and up rows differ").c_str());
            total = q.rows[0];
        }
        if (nsrc == 1 && q.kind != QL_OP_SWIGLU) o.split0 = o.split1 = total;
        for (int s = nsrc; s < 3; ++s) o.wmap[s] = o.wmap[nsrc - 1];
        if (!f32_act_map(&o.xmap, q.x, tokens, xs, q.in_dim, NT))
            return set_last_error(QL_ECUDA, (what + ": activation tensor map").c_str());
        o.kind = q.kind == QL_OP_STORE ? kBStore : q.kind == QL_OP_ADD ? kBAdd : kBSwiglu;
        o.nmat = q.kind == QL_OP_SWIGLU ? 2 : 1;
        o.rows = total;
        o.K = q.in_dim;
        o.U = blocks;
        o.tiles = q.kind == QL_OP_SWIGLU ? (total + 63) / 64 : (total + kBRows - 1) / kBRows;
        o.T = (int64_t)o.tiles * blocks;
        if (o.tiles > (1 << 16)) return set_last_error(QL_EINVAL, (what + ": too many rows").c_str());
        o.x = q.x;
        o.xs = xs;
        o.gamma = q.gamma;
        o.eps = q.eps;
        o.bias = q.kind == QL_OP_SWIGLU ? nullptr : q.bias;
        o.y = q.y;
        o.ys = q.y_stride ? q.y_stride : total;
        if (q.y && o.ys < total) return set_last_error(QL_EINVAL, (what + ": y_stride below the output width").c_str());
        o.ss_in = o.ss_out = -1;
        if (q.rope_rows > 0) {
            const int hd = q.head_dim;
            const int limit = nsrc == 3 ? o.split1 : total;  // sources 0 and 1 only (q, k)
            if (q.kind != QL_OP_STORE || q.argmax_idx || !q.rope_pos || (hd != 32 && hd != 64 && hd != 128) ||
                q.rope_rows % hd || q.rope_rows > limit || (nsrc >= 2 && q.rope_rows > o.split0 && o.split0 % hd))
                return set_last_error(QL_EINVAL, (what + ": RoPE needs a STORE op without argmax, rope_pos, head_dim "
                                                         "32, 64 or 128 and rope_rows whole heads of sources 0 and 1").c_str());
            o.rope_pos = q.rope_pos;
            o.rope_theta = q.rope_theta;
            o.rope_rows = q.rope_rows;
            o.head_dim = hd;
        }
        if (q.argmax_idx) {
            if (q.kind != QL_OP_STORE) return set_last_error(QL_EINVAL, (what + ": argmax needs a store op").c_str());
            o.amax.idx = q.argmax_idx;
            o.amax.offset = q.argmax_offset;
        }
        out_w[p] = q.y ? total : 0;
        out_s[p] = o.ys;
    }
    // RMSNorm inputs produced inside the chain: the last earlier op that wrote them sums their
    // squares in its epilogue (same buffer, same row stride, covering all in_dim columns)
    for (int p = 0; p < nops; ++p) {
        if (h[p].gamma == nullptr) continue;
        const float *x0 = h[p].x, *x1 = x0 + (size_t)(tokens - 1) * h[p].xs + h[p].K;
        for (int q = p - 1; q >= 0; --q) {
            if (!h[q].y) continue;
            const float *y0 = h[q].y, *y1 = y0 + (size_t)(tokens - 1) * h[q].ys + out_w[q];
            if (!(y0 < x1 && x0 < y1)) continue;  // no overlap: keep looking
            if (y0 == x0 && h[q].ys == h[p].xs && out_w[q] == h[p].K && h[q].kind != kBSwiglu) {
                if (h[q].ss_out < 0) h[q].ss_out = nslots++;
                h[p].ss_in = h[q].ss_out;
            }
            break;  // the last writer decides; a partial writer leaves the sums to the consumer
        }
    }
    BChain *c = new BChain();
    c->sms = sms;
    cudaError_t e = cudaMalloc(&c->ops_dev, sizeof(BOp) * nops);
    if (e == cudaSuccess) e = cudaMalloc(&c->done, sizeof(unsigned) * (2 * nops + 1));
    if (e == cudaSuccess) e = cudaMalloc(&c->keys, sizeof(unsigned long long) * nops * kBMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&c->ss, sizeof(long long) * 2 * (nslots > 0 ? nslots : 1) * kBMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&c->part, sizeof(float) * (size_t)sms * 2 * kBMaxTok * kBRows);
    if (e == cudaSuccess) e = cudaMemset(c->done, 0, sizeof(unsigned) * (2 * nops + 1));
    if (e == cudaSuccess) e = cudaMemset(c->keys, 0, sizeof(unsigned long long) * nops * kBMaxTok);
    if (e == cudaSuccess) e = cudaMemset(c->ss, 0, sizeof(long long) * 2 * (nslots > 0 ? nslots : 1) * kBMaxTok);
    if (e == cudaSuccess) {
        for (int p = 0; p < nops; ++p)
            if (h[p].amax.idx) {
                h[p].amax.amax = c->keys + (size_t)p * kBMaxTok;
                h[p].amax.done = c->done + nops + 1 + p;
            }
        e = cudaMemcpy(c->ops_dev, h.data(), sizeof(BOp) * nops, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaFuncSetAttribute(bchain_kernel_for(NT), cudaFuncAttributeMaxDynamicSharedMemorySize, kBSmem);
    if (e != cudaSuccess) {
        if (c->ops_dev) cudaFree(c->ops_dev);
        if (c->done) cudaFree(c->done);
        if (c->keys) cudaFree(c->keys);
        if (c->ss) cudaFree(c->ss);
        if (c->part) cudaFree(c->part);
        delete c;
        return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create_batch: ") + cudaGetErrorString(e)).c_str());
    }
    c->args.ops = c->ops_dev;
    c->args.nops = nops;
    c->args.M = tokens;
    c->args.NT = NT;
    c->args.done = c->done;
    c->args.epoch = c->done + nops;
    c->args.part = c->part;
    c->args.counters = counters;
    c->args.err = err;
    c->args.ss = c->ss;
    c->args.nslots = nslots > 0 ? nslots : 1;
    *chain = c;
    return QL_OK;
}

bool bchain_is(void *chain) { return chain && static_cast<BChain *>(chain)->magic == 0x42434821; }

int bchain_run(void *chain, cudaStream_t s) {
    BChain *c = static_cast<BChain *>(chain);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(c->sms);
    cfg.blockDim = dim3(kBThreads);
    cfg.dynamicSmemBytes = kBSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers cannot deadlock
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, bchain_kernel_for(c->args.NT), c->args);
    set_launch_count(1);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

int bchain_destroy(void *chain) {
    BChain *c = static_cast<BChain *>(chain);
    cudaDeviceSynchronize();
    cudaFree(c->ops_dev);
    cudaFree(c->done);
    cudaFree(c->keys);
    cudaFree(c->ss);
    cudaFree(c->part);
    delete c;
    return QL_OK;
}

}  // namespace ql

extern "C" QL_API int ql_gemv_chain_create_batch(const ql_chain_op *ops, int nops, int tokens, void **chain) {
    return ql::bchain_create(ops, nops, tokens, chain);
}
