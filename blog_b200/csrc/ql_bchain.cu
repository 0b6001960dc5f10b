// ql_bchain.cu -- batched decode: a decode step's Q4_K projections for up to 32 tokens in one
// persistent launch on the 5th-generation tensor cores (tcgen05).
//
// The reference runs batched decode and prefill as one warp per (token, output row) on the
// CUDA cores (quant_matmul_kernel, AI/codes/local-llm/src/backend/cuda/ops/kernel.cu:1253-1279,
// via launch_quant_matmul, launch.cu:101-119), or as dequantize-to-f16 plus cuBLAS
// (TensorTool.cpp:127-144).  At 8..32 tokens the step is still bound by the weight stream (each
// weight is used by every token once), so the design goal is to decode every weight exactly once
// per step, with as few instructions as possible, straight into a tensor-core operand:
//
//   * One cooperative launch of one CTA per SM runs the whole op list (same semantics as
//     ql_gemv_chain: stacked q/k/v with RMSNorm and bias, o + residual, gate/up SwiGLU, down +
//     residual, ..., LM head + greedy argmax) for M tokens.  Ops are separated by a grid barrier
//     (monotonic arrival counters, so a CUDA graph can replay the launch without resets).
//   * Work unit = a tile of 128 output rows (SwiGLU: 64 gate + 64 up rows) x one Q4_K block (256
//     inputs).  Units are split over the CTAs in equal contiguous ranges (stream-K); a tile shared
//     by several CTAs is summed in a 64-bit fixed-point accumulator (integer reductions: exact, so
//     deterministic) and finished by the last CTA to arrive.
//   * The weights are the MMA's M side (128 rows), the tokens its N side (32 columns):
//     tcgen05.mma.kind::f16, M 128, N 32, K 16, fp32 accumulators in TMEM (two 32-column
//     buffers, so a tile's drain overlaps the next tile's MMAs).
//   * Warp 0 streams the raw Q4_K bytes of every unit (TMA box {144 B, 1 block, 128 rows}) into a
//     6-slot ring, across op boundaries (weights do not depend on activations).  Warp 1 waits for
//     the op's grid barrier and streams the unit's activations: f16, [32 tokens][256 inputs], four
//     TMA boxes {64, 32} with 128-byte swizzle, i.e. already the MMA's canonical K-major B layout.
//     Warp 2 owns TMEM and one of its threads issues the MMAs.
//   * Warps 3..10 (thread = weight row x half block) dequantize their 128 weights per unit straight
//     into tensor memory (tcgen05.st: the MMA reads A from TMEM, lane = weight row, so the weights
//     never pass through shared memory; a 3-unit TMEM ring): a 32-bit word of nibbles gives f16 pairs
//     through (w & 0x000F000F) | 0x6400 (= 1024 + n, exact), an exact f16 subtraction of 1024 and
//     one f16 FMA with the sub-block's (d*sc, -dmin*m) -- the reference's value formula
//     d*sc*q - dmin*m (kernel.cu:913-921,1090-1119) rounded once to f16.  Elements are emitted in
//     the order 0, 2, 1, 3, 4, 6, 5, 7 inside every group of 8 (two nibbles per AND); the
//     activations are stored in the same order.  At a tile end the same warps drain the
//     accumulator (tcgen05.ld) and run the epilogue.
//   * Activations: each op's input, times its RMSNorm weight, rounded to f16, lives in one of two
//     global buffers [32][K].  It is written by the epilogue of the op that produced the input (the
//     previous op: rows of its output are the next op's inputs), or, for an op whose input comes
//     from outside the chain, by all CTAs at the op's start followed by a second grid barrier.
//     The RMSNorm factor is one scalar per token applied in the epilogue: the op that produced the
//     input accumulates its sum of squares in 64-bit fixed point (exact, order-free, so
//     deterministic); an input written outside the chain is summed by each CTA.
//
// Numerics: weights and activations (x * gamma) rounded to f16, fp32 accumulation; |x * gamma|
// must stay below 65504.  Every wait is bounded (about 2 s): on expiry the kernel records an error
// in the device error word, stops waiting and exits (ql_check_device reports QL_EDEVICE).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
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

constexpr int kBMaxTok = 32;                       // MMA N
constexpr int kBRows = 128;                        // output rows per tile = MMA M
constexpr int kBCw = 8;                            // dequantizer / epilogue warps
constexpr int kBThreads = (3 + kBCw) * 32;         // weight TMA, activation TMA, MMA, consumers
constexpr int kBWSlots = 6;                        // raw weight ring
constexpr int kBXSlots = 4;                        // activation ring
constexpr int kBASlots = 3;                        // dequantized units in TMEM (128 columns each)
constexpr int kBWBytes = kBRows * 144;             // 18,432 B: one block column of a tile
constexpr int kBXBox = kBMaxTok * 64 * 2;          // 4 KB: 32 tokens x 64 inputs, f16
constexpr int kBXBytes = 4 * kBXBox;               // one block of activations
constexpr int kBRedPitch = kBRows + 4;             // floats per token row of the drained tile
constexpr int kBRedBytes = kBMaxTok * kBRedPitch * 4;
constexpr int kBHdr = 1024;
constexpr int kBOffW = kBHdr;
constexpr int kBOffX = kBOffW + kBWSlots * kBWBytes;
constexpr int kBOffRed = kBOffX + kBXSlots * kBXBytes;
constexpr int kBOffMisc = kBOffRed + kBRedBytes;   // per-warp token reductions
constexpr int kBSmem = kBOffMisc + 2 * kBCw * kBMaxTok * 8;
constexpr uint32_t kBTmemCols = 512;               // two 32-column accumulators, then the A ring
constexpr uint32_t kBTmemA = 64;                   // first column of the A ring
static_assert(kBTmemA + 128 * kBASlots <= kBTmemCols, "tensor memory");
static_assert(kBOffX % 1024 == 0, "swizzled ring must be 1024-byte aligned");
static_assert(kBSmem <= 227 * 1024, "shared memory");
constexpr int kErrBarrier = 5;
constexpr double kSsFix = 16777216.0;  // 2^24: fixed-point sums of squares
// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, M 128, N 32.
constexpr uint32_t kBIdesc = (1u << 4) | ((uint32_t)(kBMaxTok >> 3) << 17) | ((uint32_t)(kBRows >> 4) << 24);

enum BKind : int { kBStore = 0, kBAdd = 1, kBSwiglu = 2 };

struct __align__(128) BOp {
    CUtensorMap wmap[3];  // Q4_K sources {144, blocks, rows}, box {144, 1, 128} (SwiGLU: 64 rows each)
    CUtensorMap xmap;     // f16 input xh_in {K, 32}, box {64, 32}, 128-byte swizzle
    int kind, nmat, rows, K, U, tiles;
    int split0, split1;   // stacked sources: first rows of sources 1 and 2 (multiples of 128)
    int64_t T;            // units = tiles * U
    const float *x;       // fp32 input [M][xs]
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
    const float *rope_inv;  // [head_dim / 2] inverse frequencies 1 / theta^(2i / head_dim)
    int rope_rows, head_dim;
    __half *xh_in;        // this op's f16 input [32][K] (x * gamma, permuted inside groups of 8)
    int convert;          // 1: this op writes xh_in from x itself (its input comes from outside)
    int k_out;            // > 0: rows [0, k_out) of the output, times g_out, are the next op's input
    __half *xh_out;       // ... written here [32][k_out]
    const float *g_out;   // the next op's RMSNorm weight (or null)
    __device__ float bias_at(int row) const { return bias != nullptr ? bias[row] : 0.f; }
};

struct BArgs {
    const BOp *ops;
    int nops;
    int M;
    unsigned *done;       // [nops] arrival counters (monotonic)
    unsigned *cdone;      // [nops] input-conversion arrival counters (monotonic)
    unsigned *epoch;      // completed launches
    long long *fixacc;    // [tiles][32][128] stream-K tile accumulators in fixed point (zero between ops)
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
// Bounded wait until *p >= target (a grid barrier); false (and the error word set) on expiry.
__device__ __forceinline__ bool wait_counter(const unsigned *p, unsigned target, int *err) {
    if (ld_acquire(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire(p) < target) {
        if (global_timer_ns() - t0 > 2000000000ull) {
            atomicExch(err, kErrBarrier);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ void tmap_acquire(const void *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}
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
// D[tmem] (+)= A[tmem] * B[smem desc]^T, f16 inputs, f32 accumulate.
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes <- 32 registers per thread.
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
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Arrive (once) on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns of TMEM -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t a) {
    return ((uint64_t)(a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
// (1024 + n) from a nibble pair placed at bits 0-3 / 16-19 -> n * D - M, in f16.
__device__ __forceinline__ uint32_t deq2(uint32_t nib, __half2 D, __half2 negM) {
    const __half2 h = bits_h2(nib | 0x64006400u);
    return h2_bits(__hfma2(__hsub2(h, __float2half2_rn(1024.f)), D, negM));
}
// Position of input k inside its group of 8 in the f16 activation layout (elements 0, 2, 1, 3,
// 4, 6, 5, 7 at positions 0..7: the order in which the dequantizer emits nibbles).
__device__ __forceinline__ int xh_pos(int k) { return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1); }
__device__ __forceinline__ long long ss_to_fixed(float v) { return __float2ll_rn(v * (float)kSsFix); }
// Stream-K partial sums in fixed point: 32 fractional bits in an int64 (|v| < 2^31).
__device__ __forceinline__ long long to_fixed32(float v) { return __float2ll_rn(v * 4294967296.0f); }
__device__ __forceinline__ float from_fixed32(long long v) { return (float)((double)v * (1.0 / 4294967296.0)); }
// Warp reductions of 8 values per lane over the 32 lanes, in a fixed order (deterministic): three
// exchange-half steps (lane bits 4, 3, 2), then two butterfly steps (bits 1, 0).  Lane l ends with
// the result for value index reduce8_index(l).
__device__ __forceinline__ int reduce8_index(int lane) {
    return 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
}
__device__ __forceinline__ float reduce8_sum(const float (&v)[8], int lane) {
    float w[4], x[2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool hi = lane & 16;
        w[k] = (hi ? v[k + 4] : v[k]) + __shfl_xor_sync(0xffffffffu, hi ? v[k] : v[k + 4], 16);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const bool hi = lane & 8;
        x[k] = (hi ? w[k + 2] : w[k]) + __shfl_xor_sync(0xffffffffu, hi ? w[k] : w[k + 2], 8);
    }
    const bool hi = lane & 4;
    float y = (hi ? x[1] : x[0]) + __shfl_xor_sync(0xffffffffu, hi ? x[0] : x[1], 4);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    return y;
}
__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }
__device__ __forceinline__ unsigned long long reduce8_max(const unsigned long long (&v)[8], int lane) {
    unsigned long long w[4], x[2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool hi = lane & 16;
        w[k] = umax64(hi ? v[k + 4] : v[k], __shfl_xor_sync(0xffffffffu, hi ? v[k] : v[k + 4], 16));
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const bool hi = lane & 8;
        x[k] = umax64(hi ? w[k + 2] : w[k], __shfl_xor_sync(0xffffffffu, hi ? w[k] : w[k + 2], 8));
    }
    const bool hi = lane & 4;
    unsigned long long y = umax64(hi ? x[1] : x[0], __shfl_xor_sync(0xffffffffu, hi ? x[0] : x[1], 4));
    y = umax64(y, __shfl_xor_sync(0xffffffffu, y, 2));
    y = umax64(y, __shfl_xor_sync(0xffffffffu, y, 1));
    return y;
}

// Stream-K split of an op's T units over min(C, T) CTAs (every participating CTA gets at least
// one unit, so every CTA whose range touches a tile arrives on that tile's counter).
__device__ __forceinline__ int op_ctas(int64_t T, int C) { return T < C ? (int)T : C; }
__device__ __forceinline__ int64_t op_start(int64_t T, int Cp, int c) { return c >= Cp ? T : (int64_t)c * T / Cp; }

__global__ void __launch_bounds__(kBThreads, 1) bchain_kernel(const __grid_constant__ BArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *wfull = reinterpret_cast<uint64_t *>(smem);
    uint64_t *wempty = wfull + kBWSlots;
    uint64_t *xfull = wempty + kBWSlots;
    uint64_t *xempty = xfull + kBXSlots;
    uint64_t *afull = xempty + kBXSlots;       // [slot] of the TMEM A ring
    uint64_t *aempty = afull + kBASlots;
    uint64_t *accfull = aempty + kBASlots;     // [2] accumulator buffers
    uint64_t *accempty = accfull + 2;
    uint64_t *mma_done = accempty + 2;
    uint64_t *tmem_free = mma_done + 1;
    int *abort_flag = reinterpret_cast<int *>(tmem_free + 1);
    unsigned *epoch_s = reinterpret_cast<unsigned *>(abort_flag + 1);
    int *bcast = reinterpret_cast<int *>(epoch_s + 1);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bcast + 1);
    float *inv_rms = reinterpret_cast<float *>(smem + 384);           // [32]
    float *red = reinterpret_cast<float *>(smem + kBOffRed);          // [32 tokens][132]
    unsigned long long *wkey = reinterpret_cast<unsigned long long *>(smem + kBOffMisc);  // [warp][32]
    float *wss = reinterpret_cast<float *>(smem + kBOffMisc + kBCw * kBMaxTok * 8);        // [warp][32]
    const uint32_t sX = smem_u32(smem + kBOffX);

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
            mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < kBASlots; ++s) {
            mbar_init(&afull[s], kBCw);
            mbar_init(&aempty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&accfull[b], 1);
            mbar_init(&accempty[b], 1);
        }
        mbar_init(mma_done, 1);
        mbar_init(tmem_free, kBCw);
        *abort_flag = 0;
        *epoch_s = *reinterpret_cast<volatile unsigned *>(a.epoch);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) tmem_alloc(tmem_slot, kBTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
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
            int tile = (int)(u0 / U), blk = (int)(u0 % U);  // (tile, block) of unit u, stepped below
            for (int64_t u = u0; u < u1; ++u, ++it, blk = blk + 1 == U ? 0 : blk + 1, tile += blk == 0) {
                const int slot = it % kBWSlots;
                if (it >= kBWSlots && !aborted() &&
                    !mbar_wait(&wempty[slot], ((uint32_t)(it / kBWSlots) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
                const bool live = !aborted();
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
        for (int p = 0; p < a.nops; ++p) {
            const BOp &o = a.ops[p];
            const int U = o.U;
            const int64_t T = o.T;
            // grid barrier: the op's f16 input is complete (written by the previous op's epilogues,
            // or by every CTA's conversion step)
            if (!aborted()) {
                const unsigned *d = o.convert ? a.cdone + p : (p > 0 ? a.done + (p - 1) : nullptr);
                if (d != nullptr && !wait_counter(d, target, a.err)) *abort_flag = 1;
            }
            // the activations were written by generic-proxy stores; the tensor copies read them
            asm volatile("fence.proxy.async.global;" ::: "memory");
            tmap_acquire(&o.xmap);
            const int Cp = op_ctas(T, C);
            const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
            int blk = (int)(u0 % U);
            for (int64_t u = u0; u < u1; ++u, ++it, blk = blk + 1 == U ? 0 : blk + 1) {
                const int slot = it % kBXSlots;
                if (it >= kBXSlots && !aborted() &&
                    !mbar_wait(&xempty[slot], ((uint32_t)(it / kBXSlots) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
                const bool live = !aborted();
                mbar_arrive_expect_tx(&xfull[slot], live ? (uint32_t)kBXBytes : 0u);
                if (live) {
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tma_load_2d(smem + kBOffX + slot * kBXBytes + c * kBXBox, &o.xmap, 256 * blk + 64 * c, 0,
                                    &xfull[slot]);
                }
            }
        }
        for (int j = (it > kBXSlots ? it - kBXSlots : 0); j < it; ++j)
            mbar_wait(&xfull[j % kBXSlots], (uint32_t)(j / kBXSlots) & 1u, nullptr, 0);
        return;
    }
    if (warp == 2) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            int uc = 0, tc = 0;  // units and tiles of this CTA, over all ops
            for (int p = 0; p < a.nops; ++p) {
                const BOp &o = a.ops[p];
                const int U = o.U;
                const int64_t T = o.T;
                const int Cp = op_ctas(T, C);
                const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
                int blk = (int)(u0 % U);
                for (int64_t u = u0; u < u1; ++u, ++uc, blk = blk + 1 == U ? 0 : blk + 1) {
                    const bool first = (u == u0) || blk == 0, last = (blk == U - 1) || (u + 1 == u1);
                    const int b = tc & 1;
                    if (first && tc >= 2 && !aborted() &&
                        !mbar_wait(&accempty[b], (uint32_t)((tc >> 1) - 1) & 1u, a.err, kErrWaitEmpty))
                        *abort_flag = 1;
                    const int xs = uc % kBXSlots, as = uc % kBASlots;
                    if (!aborted() && !mbar_wait(&xfull[xs], (uint32_t)(uc / kBXSlots) & 1u, a.err, kErrWaitFull))
                        *abort_flag = 1;
                    if (!aborted() && !mbar_wait(&afull[as], (uint32_t)(uc / kBASlots) & 1u, a.err, kErrWaitFull))
                        *abort_flag = 1;
                    tc_fence_after();
                    if (!aborted()) {
#pragma unroll
                        for (int c = 0; c < 4; ++c)
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                mma_f16_ta(tmem + 32u * (uint32_t)b, tmem + kBTmemA + 128u * (uint32_t)as + 32u * c + 8u * kk,
                                           sw128_desc(sX + xs * kBXBytes + c * kBXBox + 32 * kk), kBIdesc,
                                           (first && c == 0 && kk == 0) ? 0u : 1u);
                    }
                    mma_commit(&aempty[as]);
                    mma_commit(&xempty[xs]);
                    if (last) {
                        mma_commit(&accfull[b]);
                        ++tc;
                    }
                }
            }
            // every MMA has completed before TMEM is freed
            mma_commit(mma_done);
            mbar_wait(mma_done, 0u, a.err, kErrWaitFull);
        }
        __syncwarp();
        // the consumers have read the last accumulator
        mbar_wait(tmem_free, 0u, a.err, kErrWaitFull);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kBTmemCols);
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int cw = warp - 3, ctid = tid - 96;
    // weight row = TMEM lane (a warp reaches lanes 32 (warp % 4) ..), half block (sub-blocks 4hf .. 4hf + 3)
    const int q = warp & 3, dh = cw >> 2;              // TMEM lane quadrant, token half of the drain
    const int r = 32 * q + lane, hf = cw >> 2;
    int itw = 0, uc = 0, tc = 0;
    for (int p = 0; p < a.nops; ++p) {
        const BOp &o = a.ops[p];
        const int kind = o.kind, U = o.U, rows = o.rows, K = o.K;
        const int64_t T = o.T;
        const float *gamma = o.gamma;
        const int Cp = op_ctas(T, C);
        const int64_t u0 = op_start(T, Cp, cta), u1 = op_start(T, Cp, cta + 1);
        if (o.convert) {
            // this op's input comes from outside the chain (or from an op other than the previous
            // one): every CTA converts a share of it to f16 x gamma, then a second grid barrier
            if (p > 0) {
                if (ctid == 0 && !aborted() && !wait_counter(a.done + (p - 1), target, a.err)) *abort_flag = 1;
                named_bar_sync(1, kBCw * 32);
            }
            const int g8 = K / 8, ng = M * g8;
            for (int i = cta * kBCw * 32 + ctid; i < ng; i += C * kBCw * 32) {
                const int t = i / g8, k = 8 * (i - t * g8);
                const float4 *xp = reinterpret_cast<const float4 *>(o.x + (size_t)t * o.xs + k);
                float4 v0 = xp[0], v1 = xp[1];
                if (gamma != nullptr) {
                    const float4 g0 = reinterpret_cast<const float4 *>(gamma + k)[0];
                    const float4 g1 = reinterpret_cast<const float4 *>(gamma + k)[1];
                    v0.x *= g0.x; v0.y *= g0.y; v0.z *= g0.z; v0.w *= g0.w;
                    v1.x *= g1.x; v1.y *= g1.y; v1.z *= g1.z; v1.w *= g1.w;
                }
                uint4 hv;  // positions 0..7 <- elements 0, 2, 1, 3, 4, 6, 5, 7
                hv.x = h2_bits(__floats2half2_rn(v0.x, v0.z));
                hv.y = h2_bits(__floats2half2_rn(v0.y, v0.w));
                hv.z = h2_bits(__floats2half2_rn(v1.x, v1.z));
                hv.w = h2_bits(__floats2half2_rn(v1.y, v1.w));
                *reinterpret_cast<uint4 *>(o.xh_in + (size_t)t * K + k) = hv;
            }
            __threadfence();
            named_bar_sync(1, kBCw * 32);
            if (ctid == 0) atomicAdd(a.cdone + p, 1u);
        }
        bool norm_ready = false;
        const bool track = o.amax.amax != nullptr || o.ss_out >= 0;
        // per-warp running results over the tiles this CTA finishes (greedy keys, sums of squares),
        // each slot written by one lane only: deterministic
        wkey[cw * kBMaxTok + lane] = 0ull;
        wss[cw * kBMaxTok + lane] = 0.f;

        int tile = (int)(u0 / U), blk = (int)(u0 % U);  // (tile, block) of unit u, stepped below
        for (int64_t u = u0; u < u1; ++u, ++itw, ++uc, blk = blk + 1 == U ? 0 : blk + 1, tile += blk == 0) {
            const int ws = itw % kBWSlots;
            if (!__all_sync(0xffffffffu, !aborted() && mbar_wait(&wfull[ws], (uint32_t)(itw / kBWSlots) & 1u,
                                                                  a.err, kErrWaitFull)))
                *abort_flag = 1;
            {
                // ---- dequantize this thread's row, inputs 128 hf .. 128 hf + 127 of the block ----
                const uint8_t *wrow = smem + kBOffW + ws * kBWBytes + r * 144;
                const uint4 hd = *reinterpret_cast<const uint4 *>(wrow);
                const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
                // q4k_scale_min (reference kernel.cu:913-921): sub-blocks 0-3 or 4-7 as packed bytes
                const uint32_t scw = hf == 0 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
                const uint32_t mw = hf == 0 ? (hd.z & 0x3F3F3F3Fu)
                                            : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
                const int as = uc % kBASlots;
                // the ring slot is free once the MMAs that read it three units ago have completed
                if (uc >= kBASlots &&
                    !__all_sync(0xffffffffu, !aborted() && mbar_wait(&aempty[as], (uint32_t)(uc / kBASlots - 1) & 1u,
                                                                      a.err, kErrWaitEmpty)))
                    *abort_flag = 1;
                tc_fence_after();
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int pch = 2 * hf + cc;  // 64-input chunk of the block: sub-blocks 2 pch, 2 pch + 1
                    const int sh0 = 16 * cc, sh1 = sh0 + 8;
                    const __half2 D0 = __float2half2_rn(d * (float)((scw >> sh0) & 0xFFu));
                    const __half2 M0 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh0) & 0xFFu)));
                    const __half2 D1 = __float2half2_rn(d * (float)((scw >> sh1) & 0xFFu));
                    const __half2 M1 = __hneg2(__float2half2_rn(dmin * (float)((mw >> sh1) & 0xFFu)));
                    const uint4 qa = *reinterpret_cast<const uint4 *>(wrow + 16 + 32 * pch);
                    const uint4 qb = *reinterpret_cast<const uint4 *>(wrow + 32 + 32 * pch);
                    const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    // columns 4 jj .. 4 jj + 3: elements 8 jj .. 8 jj + 7 of sub-block 2 pch (low nibbles);
                    // columns 16 + 4 jj ..: sub-block 2 pch + 1 (high nibbles); two f16 per column
                    uint32_t v[32];
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
                    tmem_st32(tmem + ((uint32_t)(32 * q) << 16) + kBTmemA + 128u * (uint32_t)as + 32u * (uint32_t)pch, v);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[as]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&wempty[ws]);
            const bool tile_end = (blk == U - 1) || (u + 1 == u1);
            if (!tile_end) continue;

            // ---------------- end of this CTA's part of a tile ----------------
            {
                const int b = tc & 1;
                if (!__all_sync(0xffffffffu, !aborted() && mbar_wait(&accfull[b], (uint32_t)(tc >> 1) & 1u, a.err,
                                                                      kErrWaitFull)))
                    *abort_flag = 1;
                tc_fence_after();
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + 32u * (uint32_t)b + 16u * (uint32_t)dh, v);
#pragma unroll
                for (int i = 0; i < 16; ++i) red[(16 * dh + i) * kBRedPitch + 32 * q + lane] = __uint_as_float(v[i]);
                tc_fence_before();
                named_bar_sync(1, kBCw * 32);
                if (ctid == 0) mbar_arrive(&accempty[b]);
                ++tc;
            }
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
                            const float4 xv = __ldcg(reinterpret_cast<const float4 *>(xr + k));
                            s = fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, fmaf(xv.z, xv.z, fmaf(xv.w, xv.w, s))));
                        }
#pragma unroll
                        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
                        if (lane == 0) inv_rms[tok] = rsqrtf(s / (float)K + o.eps);
                    }
                }
                norm_ready = true;
                named_bar_sync(1, kBCw * 32);
            }
            // The tile's sums (from red), or, when the tile is shared with other CTAs, over the parts
            // those CTAs parked (in CTA order): computed per (token, row) where needed.
            const int64_t ts = (int64_t)tile * U, te = ts + U;
            // every decision that leads to a named barrier is uniform over the consumer threads
            // (never the abort flag, which another warp may set at any time)
            const bool partial = ts < u0 || te > u1;
            bool finish = true;
            if (partial) {
                // stream-K: every CTA of the tile adds its part into the tile's fixed-point
                // accumulator (64-bit integer reductions: exact, so the sum does not depend on the
                // order of arrival); the last to arrive reads the total back and clears it
                long long *fa = a.fixacc + (size_t)tile * (kBMaxTok * kBRows);
                const int th = ctid >> 7;  // thread = (row r, 16 tokens)
#pragma unroll 4
                for (int i = 0; i < 16; ++i)
                    atomicAdd(reinterpret_cast<unsigned long long *>(fa + (16 * th + i) * kBRows + r),
                              (unsigned long long)to_fixed32(red[(16 * th + i) * kBRedPitch + r]));
                __threadfence();
                named_bar_sync(1, kBCw * 32);
                const int cf = (int)(((ts + 1) * (int64_t)Cp - 1) / T), cl = (int)((te * (int64_t)Cp - 1) / T);
                if (ctid == 0) *bcast = (int)atomicAdd(&a.counters[tile], 1u) == cl - cf;
                named_bar_sync(1, kBCw * 32);
                finish = *bcast != 0;
                if (finish) {
                    __threadfence();
                    long long v[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = __ldcg(fa + (16 * th + i) * kBRows + r);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        red[(16 * th + i) * kBRedPitch + r] = from_fixed32(v[i]);
                        __stcg(fa + (16 * th + i) * kBRows + r, 0ll);
                    }
                    if (ctid == 0) a.counters[tile] = 0u;
                    named_bar_sync(1, kBCw * 32);
                }
            }
            auto tile_sum = [&](int tk, int row) { return red[tk * kBRedPitch + row]; };
            // the next op's f16 input: rows < k_out of this output, times its RMSNorm weight
            auto put_next = [&](int tk, int row, float v) {
                if (row < o.k_out) {
                    const float g = o.g_out != nullptr ? __ldg(o.g_out + row) : 1.f;
                    o.xh_out[(size_t)tk * o.k_out + xh_pos(row)] = __float2half_rn(v * g);
                }
            };
            if (finish) {
                if (kind == kBSwiglu) {
                    // thread = (gate row rr < 64, 8 tokens); its up row is rr + 64
                    const int rr = ctid & 63, tq = ctid >> 6;
                    const int row = tile * 64 + rr;
                    if (row < rows) {
#pragma unroll 2
                        for (int i = 0; i < 8; ++i) {
                            const int tk = 8 * tq + i;
                            if (tk < M) {
                                const float nrm = gamma != nullptr ? inv_rms[tk] : 1.f;
                                const float gv = tile_sum(tk, rr) * nrm, uv = tile_sum(tk, rr + 64) * nrm;
                                const float out = gv / (1.0f + expf(-gv)) * uv;
                                if (o.y != nullptr) o.y[(size_t)tk * o.ys + row] = out;
                                put_next(tk, row, out);
                            }
                        }
                    }
                } else {
                    // thread = (row r, 16 tokens); warp cw holds rows 32 (warp % 4) .., tokens 16 (cw >> 2) ..
                    const int th = ctid >> 7;
                    const int row = tile * kBRows + r;
                    const bool live = row < rows;
                    const float bias = (live && o.bias != nullptr) ? o.bias[row] : 0.f;
#pragma unroll 1
                    for (int i0 = 0; i0 < 16; i0 += 8) {
                        float sqv[8];
                        unsigned long long keyv[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int tk = 16 * th + i0 + k;
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
                                        const int i2 = pi % half, rp = r + (pi < half ? half : -half);
                                        const float xp = tile_sum(tk, rp) * nrm + o.bias_at(tile * kBRows + rp);
                                        const float ang = (float)__ldg(o.rope_pos + tk) * __ldg(o.rope_inv + i2);
                                        float sn, c;
                                        sincosf(ang, &sn, &c);
                                        out = pi < half ? out * c - xp * sn : out * c + xp * sn;
                                    }
                                    if (yp) *yp = out;
                                }
                                put_next(tk, row, out);
                                if (o.amax.amax != nullptr) key = amax_key(out, (uint32_t)(row + o.amax.offset));
                            }
                            sqv[k] = out * out;
                            keyv[k] = key;
                        }
                        if (track) {  // warp-uniform: fold these 8 tokens into the warp's running slots
                            const float sq = reduce8_sum(sqv, lane);
                            const unsigned long long kmax = reduce8_max(keyv, lane);
                            if ((lane & 3) == 0) {  // lanes 4j hold token 16 th + i0 + reduce8_index(lane)
                                const int tk = 16 * th + i0 + reduce8_index(lane);
                                const unsigned long long kw = wkey[cw * kBMaxTok + tk];
                                wkey[cw * kBMaxTok + tk] = kmax > kw ? kmax : kw;
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
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_free);
}

struct BChain {
    int magic = 0x42434821;  // "BCH!": told apart from the one-token chain by ql_gemv_chain_run
    BOp *ops_dev = nullptr;
    unsigned *done = nullptr;          // [nops] counters, [1] epoch, [nops] argmax counters, [nops] conversions
    unsigned long long *keys = nullptr;  // [nops][32]
    long long *ss = nullptr;
    long long *fixacc = nullptr;
    __half *xh = nullptr;              // [2][32][kmax] f16 op inputs (by op parity)
    float *rope = nullptr;             // RoPE inverse-frequency tables
    BArgs args{};
    int sms = 0;
};

// f16 activations [32][K] viewed as {K, 32}; box {64, 32} with 128-byte swizzle.
bool f16_act_map(CUtensorMap *out, const __half *xh, int K) {
    auto enc = tensor_map_encoder_public();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)kBMaxTok};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kBMaxTok};
    const cuuint32_t estr[2] = {1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(xh), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void bchain_free(BChain *c) {
    if (c->ops_dev) cudaFree(c->ops_dev);
    if (c->done) cudaFree(c->done);
    if (c->keys) cudaFree(c->keys);
    if (c->ss) cudaFree(c->ss);
    if (c->fixacc) cudaFree(c->fixacc);
    if (c->xh) cudaFree(c->xh);
    if (c->rope) cudaFree(c->rope);
    delete c;
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
    std::vector<BOp> h(nops);
    // rows each op writes (for the producer/consumer analysis of the RMSNorm sums)
    std::vector<int> out_w(nops, 0);
    std::vector<std::pair<int, std::vector<float>>> rope_tables;  // (op, inverse frequencies)
    int nslots = 0, kmax = 0, tmax = 0;
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
            o.rope_rows = q.rope_rows;
            o.head_dim = hd;
            // the reference's inverse frequencies 1 / powf(theta, 2i / head_dim) (kernel.cu:186-260)
            std::vector<float> inv(hd / 2);
            for (int i = 0; i < hd / 2; ++i) inv[i] = 1.0f / powf(q.rope_theta, (float)(2 * i) / (float)hd);
            rope_tables.push_back({p, inv});
        }
        if (q.argmax_idx) {
            if (q.kind != QL_OP_STORE) return set_last_error(QL_EINVAL, (what + ": argmax needs a store op").c_str());
            o.amax.idx = q.argmax_idx;
            o.amax.offset = q.argmax_offset;
        }
        out_w[p] = q.y ? total : 0;
        kmax = q.in_dim > kmax ? q.in_dim : kmax;
        tmax = o.tiles > tmax ? o.tiles : tmax;
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
    const size_t xh_elems = (size_t)kBMaxTok * kmax;
    size_t nrope = 0;
    for (auto &rt : rope_tables) nrope += rt.second.size();
    cudaError_t e = cudaMalloc(&c->ops_dev, sizeof(BOp) * nops);
    if (e == cudaSuccess) e = cudaMalloc(&c->done, sizeof(unsigned) * (3 * nops + 1));
    if (e == cudaSuccess) e = cudaMalloc(&c->keys, sizeof(unsigned long long) * nops * kBMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&c->ss, sizeof(long long) * 2 * (nslots > 0 ? nslots : 1) * kBMaxTok);
    if (e == cudaSuccess) e = cudaMalloc(&c->fixacc, sizeof(long long) * (size_t)tmax * kBMaxTok * kBRows);
    if (e == cudaSuccess) e = cudaMemset(c->fixacc, 0, sizeof(long long) * (size_t)tmax * kBMaxTok * kBRows);
    if (e == cudaSuccess) e = cudaMalloc(&c->xh, sizeof(__half) * 2 * xh_elems);
    if (e == cudaSuccess && nrope) e = cudaMalloc(&c->rope, sizeof(float) * nrope);
    if (e == cudaSuccess) e = cudaMemset(c->done, 0, sizeof(unsigned) * (3 * nops + 1));
    if (e == cudaSuccess) e = cudaMemset(c->keys, 0, sizeof(unsigned long long) * nops * kBMaxTok);
    if (e == cudaSuccess) e = cudaMemset(c->ss, 0, sizeof(long long) * 2 * (nslots > 0 ? nslots : 1) * kBMaxTok);
    // token rows >= tokens stay zero: the MMA always runs 32 columns
    if (e == cudaSuccess) e = cudaMemset(c->xh, 0, sizeof(__half) * 2 * xh_elems);
    size_t at = 0;
    for (auto &rt : rope_tables) {
        if (e == cudaSuccess)
            e = cudaMemcpy(c->rope + at, rt.second.data(), rt.second.size() * sizeof(float), cudaMemcpyHostToDevice);
        h[rt.first].rope_inv = c->rope + at;
        at += rt.second.size();
    }
    if (e != cudaSuccess) {
        bchain_free(c);
        return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create_batch: ") + cudaGetErrorString(e)).c_str());
    }
    // f16 inputs: op p reads buffer p & 1.  Its input is written by op p - 1's epilogue when op p
    // reads op p - 1's output (same buffer and row stride, all in_dim columns written); otherwise op
    // p converts it at its start.
    for (int p = 0; p < nops; ++p) {
        BOp &o = h[p];
        o.xh_in = c->xh + (size_t)(p & 1) * xh_elems;
        const bool chained = p > 0 && h[p - 1].y == o.x && h[p - 1].ys == o.xs && out_w[p - 1] >= o.K;
        o.convert = chained ? 0 : 1;
        if (chained) {
            h[p - 1].k_out = o.K;
            h[p - 1].xh_out = o.xh_in;
            h[p - 1].g_out = o.gamma;
        }
        if (!f16_act_map(&o.xmap, o.xh_in, o.K)) {
            bchain_free(c);
            return set_last_error(QL_ECUDA, "ql_gemv_chain_create_batch: activation tensor map");
        }
    }
    for (int p = 0; p < nops; ++p)
        if (h[p].amax.idx) {
            h[p].amax.amax = c->keys + (size_t)p * kBMaxTok;
            h[p].amax.done = c->done + nops + 1 + p;
        }
    e = cudaMemcpy(c->ops_dev, h.data(), sizeof(BOp) * nops, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(bchain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBSmem);
    if (e != cudaSuccess) {
        bchain_free(c);
        return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create_batch: ") + cudaGetErrorString(e)).c_str());
    }
    c->args.ops = c->ops_dev;
    c->args.nops = nops;
    c->args.M = tokens;
    c->args.done = c->done;
    c->args.epoch = c->done + nops;
    c->args.cdone = c->done + 2 * nops + 1;
    c->args.fixacc = c->fixacc;
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, bchain_kernel, c->args);
    set_launch_count(1);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

int bchain_destroy(void *chain) {
    BChain *c = static_cast<BChain *>(chain);
    cudaDeviceSynchronize();
    bchain_free(c);
    return QL_OK;
}

}  // namespace ql

extern "C" QL_API int ql_gemv_chain_create_batch(const ql_chain_op *ops, int nops, int tokens, void **chain) {
    return ql::bchain_create(ops, nops, tokens, chain);
}
