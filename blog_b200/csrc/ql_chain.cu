// ql_chain.cu -- a decode step's chain of quantized GEMVs in one persistent kernel.
//
// The per-op entry points launch one kernel per projection; at batch 1 every
// launch pays a ramp (first weight stage, activation staging) and a tail (the
// last row groups, stream-K fix-ups) during which HBM idles, and the next
// launch cannot start its weight stream until an SM frees up.  ql_gemv_chain
// runs a whole list of ops (e.g. a decoder stack: q/k/v, o + residual, gate/up
// SwiGLU, down + residual, ..., LM head + argmax) in ONE cooperative launch of
// one CTA per SM:
//   * the TMA producer streams the weights of op p+1 as soon as a ring slot
//     frees up -- weights do not depend on activations -- so HBM stays busy
//     across op boundaries;
//   * an op's consumers wait at a grid barrier (a per-op arrival counter that
//     every CTA's finisher bumps after its last row group) before staging the
//     op's activations, which the previous op wrote;
//   * each op runs the streaming GEMV engine's stream-K plan over all CTAs with
//     the same decoders (Q4_K, one token) and epilogues (bias, residual add,
//     SwiGLU, fused RMSNorm, fused greedy argmax) as the per-op kernels.
// Arrival counters and the launch epoch are monotonic, so a CUDA graph can
// replay the launch without resets.  Every wait is bounded.
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qlinear_b200.h"
#include "ql_gemv_impl.cuh"

namespace ql {
int set_last_error(int code, const char *msg);

namespace {

constexpr int kChainSlots = 3;                       // most ring slots (two 32 x (<= 7)-block boxes each)
constexpr int kBox = kTmaSeg * 144 * kRowGroup;      // 32,256 B: the largest box
constexpr int kSlotBytes = 2 * kBox;
constexpr int kMaxWorld = 8;
constexpr int kErrChainPeer = 6;                     // a peer's partial sums never arrived
constexpr int kChainW = gemv_consumer_warps(true);   // 14 consumer warps
constexpr int kChainRed = kChainW * 2 * kRowGroup;   // floats per reduction buffer (up to 2 matrices)
constexpr int kChainThreads = (2 + kChainW) * 32;   // producer warp, finisher warp, consumers
constexpr int kErrChainBarrier = 5;
constexpr int kChainPreX = 1;                        // stages of an op issued before its activations are staged

enum ChainKind : int { kOpStore = 0, kOpAdd = 1, kOpSwiglu = 2, kOpMlp = 3 };
constexpr int kMlpBoxRows = kBox / 144;              // 224 rows of one block column per down-projection box
constexpr double kFix = 4294967296.0;                // fixed-point residual: 32 fractional bits in an int64
constexpr int kMlpSmem = 2048 + 128;                 // MLP chunk activations (fp32, limbs), sums and scale

struct __align__(128) ChainOp {
    CUtensorMap tmap[3];   // Q4_K sources {144, blocks, rows}, box {144, 7, 32}
    CUtensorMap tmap16[2]; // RoPE: sources 0 and 1 with 16-row boxes (a row group = two half boxes)
    int kind;              // ChainKind
    int nmat;              // 2 for SwiGLU (gate, up), else 1
    int split[2];          // stacked sources: first rows of sources 1 and 2
    int rows, K, U;
    Plan plan;
    const float *x;
    const float *gamma;
    float eps;
    const float *bias;
    float *y;
    AmaxOut amax;
    int bu;                // blocks per TMA box: min(7, U); a stage holds two boxes (one per matrix for SwiGLU)
    int reduce;            // tensor parallel: y += (sum over ranks of this rank's W.x) through peer memory
    int pre_y;             // ADD: y's last writer is at least two ops back, so y may be read early
    const long long *res_fixed;  // ADD two ops after a fused MLP on the same y: read the residual early
                                 // from the MLP's fixed-point copy (final when the MLP completes)
    int pair;              // one matrix, many stages per CTA: consumers take the two boxes' blocks in pairs
    long long xchg;        // first exchange cell of this op (reduce: [G][world][32]; argmax: [world][2])
    // fused MLP (kOpMlp): tmap[0..1] gate/up, tmap[2] the down projection (box {144, 1, 224});
    // split-K over 256-row chunks of the FFN, two CTAs per chunk (one per 128-row half)
    long long *y_fixed;     // MLP: the residual in fixed point (int64 atomics); ADD: also store y there
    const long long *x_fixed;  // the input in fixed point (the op right after an MLP reading its residual)
    const long long *mat_src;  // the op right after an MLP: copies its fixed-point residual ...
    float *mat_dst;            // ... back to fp32, a slice per CTA
    int mat_rows;
    int rows_d;             // MLP: rows of the down projection (= residual length)
    int half_rows;          // MLP: down rows [0, half_rows) go to the even CTA of a pair, the rest to the odd one
    int nunits;             // MLP: 2 x (FFN rows / 256)
    long long cells;        // MLP: first pair-exchange cell ([nunits][128])
    // RoPE on output rows [0, rope_rows): row group g of that range holds rows 16q .. 16q + 15 and
    // half + 16q .. half + 16q + 15 of head (32 g) / head_dim, q = ((32 g) % head_dim) / 32, so that
    // lanes l and l ^ 16 of the finisher hold the two rows a rotation pairs
    const int *rope_pos;
    const float *rope_inv;  // [head_dim / 2] inverse frequencies 1 / theta^(2i / head_dim)
    int rope_rows;
    int rope_half;          // head_dim / 2
};
static_assert(sizeof(ChainOp) % 128 == 0, "descriptor copies stay 128-byte aligned");
// Descriptor words copied to shared memory per op: everything after the tensor maps.  Reads of
// the global copy after a grid barrier miss L1 (the barrier's acquire invalidates it).
constexpr int kDescOff = offsetof(ChainOp, kind);
constexpr int kDescWords = (int)(sizeof(ChainOp) - kDescOff) / 4;

struct ChainArgs {
    const ChainOp *ops;
    int nops;
    int kmax;
    unsigned *done;     // [nops] arrival counters, monotonic
    unsigned *epoch;    // completed launches
    float *part;        // stream-K partial slots [C][2][2][32]
    unsigned *counters; // stream-K arrival counters (zero between ops)
    int *err;
    unsigned long long *xchg[kMaxWorld];  // every rank's exchange cells (index = rank), mapped here
    int rank, world;
    unsigned long long *mlp_cells;  // fused MLP pair exchange (tagged 64-bit cells)
    int nslots;                     // ring slots (2 or 3)
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Exchange cells: a 64-bit word (launch tag << 32 | payload), written and read whole
// (aligned 64-bit accesses are single-copy atomic), so no fence orders payload and flag.
__device__ __forceinline__ void st_cell(unsigned long long *p, unsigned tag, uint32_t payload) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)tag << 32) | payload)
                 : "memory");
}
__device__ __forceinline__ bool ld_cell(const unsigned long long *p, unsigned tag, uint32_t *payload, int *err) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    if ((unsigned)(v >> 32) != tag) {
        const uint64_t t0 = global_timer_ns();
        do {
            __nanosleep(64);
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            if (global_timer_ns() - t0 > 5000000000ull) {
                atomicExch(err, kErrChainPeer);
                return false;
            }
        } while ((unsigned)(v >> 32) != tag);
    }
    *payload = (uint32_t)v;
    return true;
}
// The same cells between CTAs of one GPU (the fused MLP's pair exchange): GPU scope, and a
// tight bounded spin -- the partner finishes its phase 1 at about the same time.
__device__ __forceinline__ void st_cell_gpu(unsigned long long *p, unsigned tag, uint32_t payload) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)tag << 32) | payload)
                 : "memory");
}
__device__ __forceinline__ bool ld_cell_gpu(const unsigned long long *p, unsigned tag, uint32_t *payload, int *err) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    if ((unsigned)(v >> 32) != tag) {
        const uint64_t t0 = global_timer_ns();
        do {
            asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
            if (global_timer_ns() - t0 > 2000000000ull) {
                atomicExch(err, kErrChainPeer);
                return false;
            }
        } while ((unsigned)(v >> 32) != tag);
    }
    *payload = (uint32_t)v;
    return true;
}
__device__ __forceinline__ void tensormap_acquire(const void *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

// ----------------------------------------------------------------------------
// Q4_K on the integer tensor cores (mma.sync m16n8k32, u8 weights x s8 activations, s32).
//
// Activations are staged per 256-element block b as fixed-point limbs: with 2^e_b > max|x'|
// over the block, V = rint(x' * 2^(20 - e_b)) (|V| <= 2^20) = l0 * 2^14 + l1 * 2^7 + l2 with
// l0 = V >> 14 (signed), l1 = (V >> 7) & 127, l2 = V & 127 -- three signed bytes, an exact
// split of V (21 bits; the staging error is below 2^-21 of the block's largest |x'|).
// Layout per block: [sub-block s 0..7][slot 0..3][32 bytes]; slot l < 3 holds limb l of the
// sub-block's 32 elements, slot 3 zeros.  B columns 0, 2, 4 carry limbs 0, 1, 2 and the odd
// columns zeros, so in the accumulator fragment thread (g, t) holds limb t of rows g, g+8.
//
// Weights go in raw: a 32-bit word of qs holds 4 low nibbles (sub-block 2q) and 4 high nibbles
// (2q+1) of consecutive elements; word & 0x0F0F0F0F gives n, word & 0xF0F0F0F0 gives 16 n, both
// valid u8 operands, so the decode is one AND per 4 elements.  Per (row, sub-block) the integer
// sums are scaled by the 6-bit sub-block scale (IMAD, exact: |16 T| < 2^29 per block); the
// block's d, the limb weight 2^(14 - 7t) and 2^(e_b - 24) apply once per block in fp32.  The
// min term dmin * sum_s m_s * X_s (X_s = fp32 sum of x' over sub-block s) is split over the
// four threads of a row (sub-blocks 2t, 2t+1).  The four threads' partial sums of a row are
// added at the end of the row group.  Same block math as q4k_dequant / vec_dot_q4_K
// (reference kernel.cu:913-921), with the activation rounding above in place of fp32 products.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One Q4_K block (256 elements) of the 32 rows of a TMA box (row r at box[mat] + r * pitch),
// against the staged limbs `xl` of that block (256 words), its sub-block sums `xs8` and its
// scale `xe` = 2^(e_b - 24).  acc[mat][j]: this thread's partial sum of row g + 8j.
// Matrix `mat` runs against activation block xl[mat]: the same block for gate/up, two blocks of one
// row range when a single matrix's blocks are processed in pairs.
template <int NM>
__device__ __forceinline__ void unit_q4k_imma(const uint8_t *const (&box)[NM], int pitch,
                                              const uint32_t *const (&xl)[NM], const float *const (&xs8)[NM],
                                              const float (&xe)[NM], int lane, float (&acc)[NM][4]) {
    const int g = lane >> 2, t = lane & 3;
    const int slot = (g < 6 && !(g & 1)) ? (g >> 1) : 3;
    const float lw = t == 0 ? 16384.f : t == 1 ? 128.f : t == 2 ? 1.f : 0.f;
    float dd[NM][4];
    uint32_t s03[NM][4], s47[NM][4];
#pragma unroll
    for (int mat = 0; mat < NM; ++mat)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 h = *reinterpret_cast<const uint4 *>(box[mat] + (g + 8 * j) * pitch);
            const float X0 = xs8[mat][2 * t], X1 = xs8[mat][2 * t + 1];
            dd[mat][j] = half_bits_to_float(h.x) * (xe[mat] * lw);
            s03[mat][j] = h.y & 0x3F3F3F3Fu;
            s47[mat][j] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t mw = t < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
            const float2 mf = byte_pair_f(mw, 2 * (t & 1));
            // the min term goes into the accumulator right away (fewer live registers)
            acc[mat][j] -= half_bits_to_float(h.x >> 16) * fmaf(mf.x, X0, mf.y * X1);
        }
    int te[NM][4], to[NM][4];
#pragma unroll
    for (int mat = 0; mat < NM; ++mat)
#pragma unroll
        for (int j = 0; j < 4; ++j) te[mat][j] = to[mat][j] = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int mat = 0; mat < NM; ++mat) {
            const uint32_t *xq = xl[mat] + (8 * q + slot) * 8 + t;  // sub-block 2q; 2q+1 is 32 words on
            const uint32_t b0e = xq[0], b1e = xq[4], b0o = xq[32], b1o = xq[36];
#pragma unroll
            for (int tile = 0; tile < 2; ++tile) {
                const uint8_t *ra = box[mat] + (g + 16 * tile) * pitch + 16 + 32 * q + 4 * t;
                const uint8_t *rb = ra + 8 * pitch;
                const uint32_t wa0 = *reinterpret_cast<const uint32_t *>(ra);
                const uint32_t wa1 = *reinterpret_cast<const uint32_t *>(ra + 16);
                const uint32_t wb0 = *reinterpret_cast<const uint32_t *>(rb);
                const uint32_t wb1 = *reinterpret_cast<const uint32_t *>(rb + 16);
                const uint32_t sa = q < 2 ? s03[mat][2 * tile] : s47[mat][2 * tile];
                const uint32_t sb = q < 2 ? s03[mat][2 * tile + 1] : s47[mat][2 * tile + 1];
                const uint32_t sel = 0x4440u + 2u * (q & 1);
                int c[4];
                imma_u8s8(c, wa0 & 0x0F0F0F0Fu, wb0 & 0x0F0F0F0Fu, wa1 & 0x0F0F0F0Fu, wb1 & 0x0F0F0F0Fu, b0e, b1e);
                te[mat][2 * tile] += (int)__byte_perm(sa, 0u, sel) * c[0];
                te[mat][2 * tile + 1] += (int)__byte_perm(sb, 0u, sel) * c[2];
                imma_u8s8(c, wa0 & 0xF0F0F0F0u, wb0 & 0xF0F0F0F0u, wa1 & 0xF0F0F0F0u, wb1 & 0xF0F0F0F0u, b0o, b1o);
                to[mat][2 * tile] += (int)__byte_perm(sa, 0u, sel + 1u) * c[0];
                to[mat][2 * tile + 1] += (int)__byte_perm(sb, 0u, sel + 1u) * c[2];
            }
        }
    }
#pragma unroll
    for (int mat = 0; mat < NM; ++mat)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            acc[mat][j] = fmaf(dd[mat][j], (float)(16 * te[mat][j] + to[mat][j]), acc[mat][j]);
}

// Packs byte 0 of each of four words.
__device__ __forceinline__ uint32_t pack_b0(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

// Stages one 256-element block for unit_q4k_imma from a warp: lane l holds x' elements
// 4l..4l+3 (xv[0]) and 128+4l..128+4l+3 (xv[1]).  Writes the block's limbs (256 words at xl),
// its eight sub-block sums (xsum) and its scale (*xe = 2^(e_b - 24), NaN when x' is not finite).
__device__ __forceinline__ void stage_block_limbs(const float4 (&xv)[2], uint32_t *xl, float *xsum, float *xe,
                                                  int lane) {
    float amax = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(xv[h].x), fabsf(xv[h].y)), fmaxf(fabsf(xv[h].z), fabsf(xv[h].w))));
        float bs = (xv[h].x + xv[h].y) + (xv[h].z + xv[h].w);
        bs += __shfl_xor_sync(0xffffffffu, bs, 1);
        bs += __shfl_xor_sync(0xffffffffu, bs, 2);
        bs += __shfl_xor_sync(0xffffffffu, bs, 4);
        if ((lane & 7) == 0) xsum[4 * h + (lane >> 3)] = bs;
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    // 2^e > amax with e = E - 126 (E: amax's biased exponent, at least 30 so that the factors
    // stay normal; smaller values are all but zero against 2^-96)
    int E = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
    const bool finite = E != 255;
    E = E < 30 ? 30 : E;
    const float f = __uint_as_float((uint32_t)(273 - E) << 23);  // 2^(20 - e)
    if (lane == 0) *xe = finite ? __uint_as_float((uint32_t)(E - 23) << 23) : __int_as_float(0x7fc00000);
    uint32_t *xb = xl + (lane & 7);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int V0 = __float2int_rn(xv[h].x * f), V1 = __float2int_rn(xv[h].y * f);
        const int V2 = __float2int_rn(xv[h].z * f), V3 = __float2int_rn(xv[h].w * f);
        uint32_t *xw = xb + (4 * h + (lane >> 3)) * 32;  // sub-block 4h + lane/8, slot 0
        xw[0] = pack_b0(V0 >> 14, V1 >> 14, V2 >> 14, V3 >> 14);
        xw[8] = pack_b0(V0 >> 7, V1 >> 7, V2 >> 7, V3 >> 7) & 0x7F7F7F7Fu;
        xw[16] = pack_b0(V0, V1, V2, V3) & 0x7F7F7F7Fu;
        xw[24] = 0u;
    }
}

__device__ __forceinline__ long long to_fixed(float v) { return __float2ll_rn(v * (float)kFix); }
__device__ __forceinline__ float from_fixed(long long v) { return __ll2float_rn(v) * (float)(1.0 / kFix); }

__global__ void __launch_bounds__(kChainThreads, 1) gemv_chain_kernel(const __grid_constant__ ChainArgs a) {
    constexpr int EW = 1, CW0 = 2, W = kChainW;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);   // [kChainSlots]
    uint64_t *empty = full + kChainSlots;                   // [kChainSlots]
    uint64_t *red_full = empty + kChainSlots;               // [2]
    uint64_t *red_empty = red_full + 2;                     // [2]
    int *abort_flag = reinterpret_cast<int *>(red_empty + 2);
    unsigned *epoch_s = reinterpret_cast<unsigned *>(abort_flag + 1);
    volatile unsigned *x_staged = reinterpret_cast<volatile unsigned *>(epoch_s + 1);  // ops whose x is staged
    float *inv_rms = reinterpret_cast<float *>(smem + 112);
    float *ss_part = reinterpret_cast<float *>(smem + 128);  // [W]
    uint64_t *a_ready = reinterpret_cast<uint64_t *>(smem + 192);  // MLP: the chunk's activations are staged
    uint64_t *p2_done = reinterpret_cast<uint64_t *>(smem + 200);  // MLP: the consumers finished a unit
    static_assert(128 + 4 * kChainW <= 192, "header layout");
    size_t off = kGemvHeaderBytes;
    uint32_t *xl = reinterpret_cast<uint32_t *>(smem + off);  // activation limbs, 1 KB per 256-element block
    off += ((size_t)a.kmax * 4 + 127) / 128 * 128;
    float *xsum = reinterpret_cast<float *>(smem + off);        // per 32-element sub-block
    off += ((size_t)(a.kmax / 32) * 4 + 127) / 128 * 128;
    float *xe = reinterpret_cast<float *>(smem + off);          // per block: 2^(e_b - 24)
    off += ((size_t)(a.kmax / 256) * 4 + 127) / 128 * 128;
    float *red = reinterpret_cast<float *>(smem + off);  // [2][W][2][32]
    off += ((size_t)2 * kChainRed * 4 + 127) / 128 * 128;
    uint8_t *desc = smem + off;  // [2] copies of the current op's descriptor (all but the tensor maps)
    off += 2 * sizeof(ChainOp);
    float *abuf = reinterpret_cast<float *>(smem + off);      // MLP: the chunk's 256 activations
    uint32_t *xa = reinterpret_cast<uint32_t *>(smem + off + 1024);  // ... as limbs
    float *xsa = reinterpret_cast<float *>(smem + off + 2048);        // ... sub-block sums, [8] then the scale
    off += kMlpSmem;
    off = (off + 1023) / 1024 * 1024;
    uint8_t *ring = smem + off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, cta = blockIdx.x;
    const int NS = a.nslots;  // ring slots in use (3 when shared memory allows)
    if (tid == 0) {
        for (int s = 0; s < a.nslots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&red_full[b], W);
            mbar_init(&red_empty[b], 1);
        }
        mbar_init(a_ready, 1);
        mbar_init(p2_done, W);
        *abort_flag = 0;
        *x_staged = 0u;
        *epoch_s = *reinterpret_cast<volatile unsigned *>(a.epoch);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned tag = *epoch_s + 1u;                     // exchange-cell tag of this launch
    const unsigned target = tag * (unsigned)C;             // every op's counter after this launch

    if (warp == 0) {
        // ---------------------------- producer (TMA) ----------------------------
        if (lane != 0) return;
        int it = 0;
        const uint64_t pol = l2_evict_first_policy();  // weights are read once per launch
        // waits for a free ring slot (and, past an op's first stage, for its activations)
        auto claim_slot = [&](int p, int sio) -> bool {
            if (sio == kChainPreX && *x_staged < (unsigned)(p + 1) && !*reinterpret_cast<volatile int *>(abort_flag)) {
                const uint64_t tw = global_timer_ns();
                while (*x_staged < (unsigned)(p + 1)) {
                    __nanosleep(64);
                    if (global_timer_ns() - tw > 2000000000ull) {
                        atomicExch(a.err, kErrWaitEmpty);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            const int slot = it % NS;
            if (it >= NS && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&empty[slot], ((uint32_t)(it / NS) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
            }
            return !*reinterpret_cast<volatile int *>(abort_flag);
        };
        for (int p = 0; p < a.nops; ++p) {
            // the descriptor's scalars in registers: reloads after the waits below would miss L1
            const ChainOp &o = a.ops[p];
            const int kind = o.kind, nmat = o.nmat, bu = o.bu, U = o.U, split0 = o.split[0], split1 = o.split[1];
            const int rope_rows = o.rope_rows, rope_half = o.rope_half;
            const int nunits = o.nunits, half_rows = o.half_rows, rows_d = o.rows_d;
            const Plan plan = o.plan;
            for (int i = 0; i < ((nmat == 2 && kind != kOpMlp) ? 2 : 3); ++i) tensormap_acquire(&o.tmap[i]);
            if (rope_rows > 0) {
                tensormap_acquire(&o.tmap16[0]);
                tensormap_acquire(&o.tmap16[1]);
            }
            if (kind == kOpMlp) {
                // per unit: the half chunk's gate/up rows (4 row groups x all blocks), then the
                // down projection's block column of the chunk over this half's rows
                const uint32_t kb = (uint32_t)bu * 144u * kRowGroup;
                const int Ce = C & ~1;
                int sio = 0;
                for (int u = cta; cta < Ce && u < nunits; u += Ce) {
                    const int ci = u >> 1, hh = u & 1;
                    for (int r = 0; r < 4; ++r)
                        for (int us = 0; us < U; us += bu) {
                            const bool live = claim_slot(p, sio++);
                            const int slot = it % NS;
                            uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                            const int row0 = 256 * ci + 128 * hh + 32 * r;
                            mbar_arrive_expect_tx(&full[slot], live ? 2u * kb : 0u);
                            if (live) {
                                tma_load_3d_hint(sb, &o.tmap[0], 0, us, row0, &full[slot], pol);
                                tma_load_3d_hint(sb + kb, &o.tmap[1], 0, us, row0, &full[slot], pol);
                            }
                            ++it;
                        }
                    const int r_beg = hh ? half_rows : 0, r_end = hh ? rows_d : half_rows;
                    for (int r = r_beg; r < r_end; r += 2 * kMlpBoxRows) {
                        const bool live = claim_slot(p, sio++);
                        const int slot = it % NS;
                        uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                        const int nbox = r + kMlpBoxRows < r_end ? 2 : 1;
                        mbar_arrive_expect_tx(&full[slot], live ? (uint32_t)(nbox * kBox) : 0u);
                        if (live) {
                            tma_load_3d_hint(sb, &o.tmap[2], 0, ci, r, &full[slot], pol);
                            if (nbox == 2) tma_load_3d_hint(sb + kBox, &o.tmap[2], 0, ci, r + kMlpBoxRows, &full[slot], pol);
                        }
                        ++it;
                    }
                }
                continue;
            }
            const int seg = 2 * bu / nmat;
            const uint32_t kb = (uint32_t)bu * 144u * kRowGroup;
            int64_t t = cta < plan.C ? plan_start(plan, cta) : 0;
            const int64_t t1 = cta < plan.C ? plan_start(plan, cta + 1) : 0;
            Stage st;
            int sio = 0;  // stage index within the op
            while (next_stage(t, t1, U, seg, 0, st)) {
                const int slot = it % NS;
                // Past the op's first stage, let the activation loads go first: TMA data queued
                // ahead of them on the SM's inbound path would add its transfer time to their latency.
                if (sio++ == kChainPreX && *x_staged < (unsigned)(p + 1) &&
                    !*reinterpret_cast<volatile int *>(abort_flag)) {
                    const uint64_t tw = global_timer_ns();
                    while (*x_staged < (unsigned)(p + 1)) {
                        __nanosleep(64);
                        if (global_timer_ns() - tw > 2000000000ull) {
                            atomicExch(a.err, kErrWaitEmpty);
                            *abort_flag = 1;
                            break;
                        }
                    }
                }
                if (it >= NS && !*reinterpret_cast<volatile int *>(abort_flag)) {
                    if (!mbar_wait(&empty[slot], ((uint32_t)(it / NS) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                        *abort_flag = 1;
                }
                const bool live = !*reinterpret_cast<volatile int *>(abort_flag);
                uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                const int row0 = st.g * kRowGroup;
                if (nmat == 2) {
                    mbar_arrive_expect_tx(&full[slot], live ? 2u * kb : 0u);
                    if (live) {
                        tma_load_3d_hint(sb, &o.tmap[0], 0, st.us, row0, &full[slot], pol);
                        tma_load_3d_hint(sb + kb, &o.tmap[1], 0, st.us, row0, &full[slot], pol);
                    }
                } else {
                    const int src = (row0 >= split0) + (row0 >= split1);
                    const int lrow = row0 - (src == 0 ? 0 : (src == 1 ? split0 : split1));
                    const int nbox = st.ue - st.us > bu ? 2 : 1;
                    mbar_arrive_expect_tx(&full[slot], live ? (uint32_t)nbox * kb : 0u);
                    if (live && row0 < rope_rows) {
                        // RoPE group: rows 16q.. and half + 16q.. of the head, as two 16-row half boxes
                        // that land where one 32-row box would (rows are contiguous in the slot)
                        const int hd = 2 * rope_half, hb = lrow / hd * hd, q16 = 16 * ((lrow % hd) / 32);
                        const int ra = hb + q16, rbw = hb + rope_half + q16;
                        const uint32_t hoff = 16u * (uint32_t)bu * 144u;
                        for (int b2 = 0; b2 < nbox; ++b2) {
                            tma_load_3d_hint(sb + b2 * kb, &o.tmap16[src], 0, st.us + b2 * bu, ra, &full[slot], pol);
                            tma_load_3d_hint(sb + b2 * kb + hoff, &o.tmap16[src], 0, st.us + b2 * bu, rbw, &full[slot], pol);
                        }
                    } else if (live) {
                        tma_load_3d_hint(sb, &o.tmap[src], 0, st.us, lrow, &full[slot], pol);
                        if (nbox == 2) tma_load_3d_hint(sb + kb, &o.tmap[src], 0, st.us + bu, lrow, &full[slot], pol);
                    }
                }
                ++it;
            }
        }
        for (int j = (it > NS ? it - NS : 0); j < it; ++j)
            mbar_wait(&full[j % NS], (uint32_t)(j / NS) & 1u, nullptr, 0);
        return;
    }

    if (warp == EW) {
        // ------------------------------ finisher ------------------------------
        int gi = 0;
        int mu = 0, p2_waited = 0;  // MLP units of this CTA so far; their p2_done phases consumed
        auto wait_p2 = [&](int upto) {
            for (; p2_waited < upto; ++p2_waited)
                if (!*reinterpret_cast<volatile int *>(abort_flag) &&
                    !mbar_wait(p2_done, (uint32_t)p2_waited & 1u, a.err, kErrWaitFull))
                    *abort_flag = 1;
        };
        for (int p = 0; p < a.nops; ++p) {
            // the consumers copied op p's descriptor to shared memory before staging its activations
            if (*x_staged < (unsigned)(p + 1) && !*reinterpret_cast<volatile int *>(abort_flag)) {
                const uint64_t tw = global_timer_ns();
                while (*x_staged < (unsigned)(p + 1)) {
                    __nanosleep(32);
                    if (global_timer_ns() - tw > 2000000000ull) {
                        atomicExch(a.err, kErrWaitFull);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            __threadfence_block();
            __syncwarp();
            const ChainOp &o = *reinterpret_cast<const ChainOp *>(desc + (p & 1) * sizeof(ChainOp));
            // the op right after a fused MLP: the MLP's fixed-point residual back to fp32, a slice per
            // CTA (the consumers of this op read the fixed-point copy; later ops read the fp32 one;
            // the fence before this CTA's arrival on done[p] publishes it)
            if (o.mat_src != nullptr) {
                const int n0 = (int)((int64_t)o.mat_rows * cta / C), n1 = (int)((int64_t)o.mat_rows * (cta + 1) / C);
                for (int n = n0 + lane; n < n1; n += 32) __stcg(o.mat_dst + n, from_fixed(__ldcg(o.mat_src + n)));
            }
            if (o.kind == kOpMlp) {
                const int Ce = C & ~1;
                for (int u = cta; cta < Ce && u < o.nunits; u += Ce, ++mu) {
                    const int hh = u & 1;
                    // phase 1: SwiGLU of the half chunk's four row groups -> smem and the pair's cells
                    bool okc = true;
                    for (int r = 0; r < 4; ++r, ++gi) {
                        const int bsel = gi & 1;
                        if (!*reinterpret_cast<volatile int *>(abort_flag) &&
                            !mbar_wait(&red_full[bsel], (uint32_t)(gi >> 1) & 1u, a.err, kErrWaitFull))
                            *abort_flag = 1;
                        const float nrm = o.gamma != nullptr ? inv_rms[0] : 1.0f;  // written before any group
                        const float *rb = red + bsel * kChainRed;
                        float gs = 0.f, us = 0.f;
                        for (int w = 0; w < W; ++w) {
                            gs += rb[(w * 2 + 0) * kRowGroup + lane];
                            us += rb[(w * 2 + 1) * kRowGroup + lane];
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&red_empty[bsel]);
                        const float gv = gs * nrm, uv = us * nrm;
                        const float act = gv / (1.0f + expf(-gv)) * uv;
                        abuf[128 * hh + 32 * r + lane] = act;
                        st_cell_gpu(a.mlp_cells + o.cells + (size_t)u * 128 + 32 * r + lane, tag, __float_as_uint(act));
                        // the pair CTA's previous row group (it runs about in step): only its last group's
                        // exchange latency remains after phase 1
                        if (r > 0 && okc) {
                            uint32_t bits = 0;
                            okc = ld_cell_gpu(a.mlp_cells + o.cells + (size_t)(u ^ 1) * 128 + 32 * (r - 1) + lane, tag,
                                              &bits, a.err);
                            abuf[128 * (hh ^ 1) + 32 * (r - 1) + lane] = __uint_as_float(bits);
                        }
                    }
                    if (okc) {
                        uint32_t bits = 0;
                        okc = ld_cell_gpu(a.mlp_cells + o.cells + (size_t)(u ^ 1) * 128 + 96 + lane, tag, &bits, a.err);
                        abuf[128 * (hh ^ 1) + 96 + lane] = __uint_as_float(bits);
                    }
                    if (!__all_sync(0xffffffffu, okc)) *abort_flag = 1;
                    // the previous unit's consumers are done with the staged activations
                    wait_p2(mu);
                    __syncwarp();
                    float4 av[2];
                    av[0] = reinterpret_cast<const float4 *>(abuf)[lane];
                    av[1] = reinterpret_cast<const float4 *>(abuf)[32 + lane];
                    stage_block_limbs(av, xa, xsa, xsa + 8, lane);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a_ready);
                }
                wait_p2(mu);
                if (lane == 0) {
                    __threadfence();
                    const unsigned prev = atomicAdd(&a.done[p], 1u);
                    if (p == a.nops - 1 && prev == target - 1u) atomicAdd(a.epoch, 1u);
                }
                __syncwarp();
                continue;
            }
            const int NM = o.nmat, U = o.U;
            const int64_t t0 = cta < o.plan.C ? plan_start(o.plan, cta) : 0;
            const int64_t t1 = cta < o.plan.C ? plan_start(o.plan, cta + 1) : 0;
            for (int64_t gg = t0 / U; gg * U < t1; ++gg, ++gi) {
                const int g = (int)gg;
                const int bsel = gi & 1;
                // loads the epilogue needs, issued before waiting for the consumers: the bias, and the
                // residual when its last writer finished before op p-1 started (o.pre_y)
                // output row of this lane (RoPE groups hold two 16-row halves of a head)
                int vv = g * kRowGroup + lane;
                float rope_c = 1.f, rope_s = 0.f;
                if (vv < o.rope_rows) {
                    const int hd = 2 * o.rope_half, hb = vv / hd * hd, q16 = 16 * ((vv % hd) / 32);
                    vv = hb + q16 + (lane & 15) + ((lane & 16) ? o.rope_half : 0);
                    // the rotation angle depends only on the position: computed while the consumers work
                    const float ang = (float)__ldg(o.rope_pos) * __ldg(o.rope_inv + (q16 + (lane & 15)));
                    sincosf(ang, &rope_s, &rope_c);
                }
                if (o.pre_y && p >= 2 && lane == 0 && !*reinterpret_cast<volatile int *>(abort_flag)) {
                    // a CTA with no row group in op p-1 gets here without having waited for op p-2
                    const unsigned *d2 = a.done + (p - 2);
                    const uint64_t tw = global_timer_ns();
                    while (ld_acquire_gpu(d2) < target) {
                        if (global_timer_ns() - tw > 2000000000ull) {
                            atomicExch(a.err, kErrChainBarrier);
                            *abort_flag = 1;
                            break;
                        }
                    }
                }
                __syncwarp();
                const float bias_v = (o.bias != nullptr && vv < o.rows) ? o.bias[vv] : 0.f;
                const float res_v = (o.kind == kOpAdd && o.pre_y && vv < o.rows)
                                        ? (o.res_fixed != nullptr ? from_fixed(__ldcg(o.res_fixed + vv)) : __ldcg(o.y + vv))
                                        : 0.f;
                bool ok = !*reinterpret_cast<volatile int *>(abort_flag);
                if (ok && !mbar_wait(&red_full[bsel], (uint32_t)(gi >> 1) & 1u, a.err, kErrWaitFull)) {
                    *abort_flag = 1;
                    ok = false;
                }
                float val[2];
                const float *rb = red + bsel * kChainRed;
                for (int mat = 0; mat < 2; ++mat) {
                    float sum = 0.f;
                    if (mat < NM)
                        for (int w = 0; w < W; ++w) sum += rb[(w * 2 + mat) * kRowGroup + lane];
                    val[mat] = sum;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_empty[bsel]);
                const int64_t gs = (int64_t)g * U, ge = gs + U;
                bool finish = ok;
                if (ok && (gs < t0 || ge > t1)) {
                    const int si = (g == (int)(t0 / U)) ? 0 : 1;
                    float *pp = a.part + ((size_t)cta * 2 + si) * (2 * kRowGroup);
                    pp[lane] = val[0];
                    pp[kRowGroup + lane] = val[1];
                    __threadfence();
                    __syncwarp();
                    const int cf = plan_cta_of(o.plan, gs), cl = plan_cta_of(o.plan, ge - 1);
                    unsigned prev = 0;
                    if (lane == 0) prev = atomicAdd(&a.counters[g], 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    finish = (prev == (unsigned)(cl - cf));
                    if (finish) {
                        __threadfence();
                        val[0] = val[1] = 0.f;
                        for (int c = cf; c <= cl; ++c) {
                            const int sj = (g == (int)(plan_start(o.plan, c) / U)) ? 0 : 1;
                            const float *qp = a.part + ((size_t)c * 2 + sj) * (2 * kRowGroup);
                            val[0] += __ldcg(qp + lane);
                            val[1] += __ldcg(qp + kRowGroup + lane);
                        }
                        if (lane == 0) a.counters[g] = 0u;
                    }
                }
                const int v = vv;
                if (finish) {
                    const float nrm = o.gamma != nullptr ? inv_rms[0] : 1.0f;
                    float out = 0.f;
                    // RoPE group (warp-uniform): rotate the pair x1 = row i, x2 = row i + half held by
                    // lanes l and l ^ 16 (the reference's rotation, kernel.cu:186-260)
                    const bool rope = g * kRowGroup < o.rope_rows;
                    float rot = 0.f;
                    if (rope) {
                        const float x = val[0] * nrm + bias_v;
                        const float xp = __shfl_xor_sync(0xffffffffu, x, 16);
                        rot = (lane & 16) ? x * rope_c + xp * rope_s : x * rope_c - xp * rope_s;
                    }
                    if (v < o.rows) {
                        float *yp = o.y + v;
                        if (o.kind == kOpSwiglu) {
                            const float gv = val[0] * nrm, uv = val[1] * nrm;
                            out = gv / (1.0f + expf(-gv)) * uv;
                            *yp = out;
                        } else {
                            out = val[0] * nrm;
                            if (o.bias != nullptr) out += bias_v;
                            if (rope) out = rot;
                            if (o.kind == kOpAdd && !o.reduce) {  // residual written by other SMs: L2, not L1
                                const float yn = (o.pre_y ? res_v : __ldcg(yp)) + out;
                                __stcg(yp, yn);
                                if (o.y_fixed != nullptr) __stcg(o.y_fixed + v, to_fixed(yn));
                            }
                            else if (o.kind != kOpAdd && o.y != nullptr) *yp = out;
                        }
                    }
                    if (o.reduce) {
                        // tensor parallel: this rank's partial of the row group to every rank, then the
                        // sum over ranks in rank order (bit-identical on every rank) onto the residual
                        const size_t cell = (size_t)o.xchg + ((size_t)g * a.world + a.rank) * kRowGroup + lane;
                        const uint32_t bits = __float_as_uint(v < o.rows ? out : 0.f);
                        for (int d = 0; d < a.world; ++d) st_cell(a.xchg[d] + cell, tag, bits);
                        float sum = 0.f;
                        bool okp = true;
                        for (int r = 0; r < a.world && okp; ++r) {
                            uint32_t pb = 0;
                            okp = ld_cell(a.xchg[a.rank] + (size_t)o.xchg + ((size_t)g * a.world + r) * kRowGroup + lane,
                                          tag, &pb, a.err);
                            sum += __uint_as_float(pb);
                        }
                        if (!__all_sync(0xffffffffu, okp)) *abort_flag = 1;
                        else if (v < o.rows) __stcg(o.y + v, (o.pre_y ? res_v : __ldcg(o.y + v)) + sum);
                    }
                    if (o.kind == kOpStore && o.amax.amax != nullptr) {
                        unsigned long long k = v < o.rows ? amax_key(out, (uint32_t)(v + o.amax.offset)) : 0ull;
                        k = warp_max_u64(k);
                        if (lane == 0 && k != 0ull) atomicMax(&o.amax.amax[0], k);
                    }
                }
            }
            if (lane == 0) {
                if (o.kind == kOpStore && o.amax.amax != nullptr) {
                    if (a.world == 1) {
                        amax_cta_done(o.amax, 1);
                    } else {
                        // last CTA of this rank: local key -> every rank; the largest key over ranks wins
                        __threadfence();
                        const unsigned prev = atomicAdd(o.amax.done, 1u);
                        if (prev == (unsigned)C - 1u) {
                            __threadfence();
                            const unsigned long long k = atomicExch(o.amax.amax, 0ull);
                            atomicExch(o.amax.done, 0u);
                            for (int d = 0; d < a.world; ++d) {
                                st_cell(a.xchg[d] + o.xchg + 2 * a.rank, tag, (uint32_t)(k >> 32));
                                st_cell(a.xchg[d] + o.xchg + 2 * a.rank + 1, tag, (uint32_t)k);
                            }
                            unsigned long long best = 0ull;
                            // after an abort (e.g. a peer that never arrived) no further peer waits
                            for (int r = 0; r < a.world && !*reinterpret_cast<volatile int *>(abort_flag); ++r) {
                                uint32_t hi = 0, lo = 0;
                                if (!ld_cell(a.xchg[a.rank] + o.xchg + 2 * r, tag, &hi, a.err) ||
                                    !ld_cell(a.xchg[a.rank] + o.xchg + 2 * r + 1, tag, &lo, a.err)) {
                                    *abort_flag = 1;
                                    break;
                                }
                                const unsigned long long kr = ((unsigned long long)hi << 32) | lo;
                                best = kr > best ? kr : best;
                            }
                            if (o.amax.idx) o.amax.idx[0] = amax_index(best);
                        }
                    }
                }
                __threadfence();
                const unsigned prev = atomicAdd(&a.done[p], 1u);  // this CTA's part of op p is written
                if (p == a.nops - 1 && prev == target - 1u) atomicAdd(a.epoch, 1u);
            }
            __syncwarp();
        }
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int cw = warp - CW0;
    const int nthr = W * 32;
    const int ctid = tid - 32 * CW0;
    int it = 0, gi = 0, ucount = 0, mu = 0;
    for (int p = 0; p < a.nops; ++p) {
        {
            // this op's descriptor into shared memory (loads issued before the barrier wait), and
            // the RMSNorm weight, which does not depend on earlier ops, into L2
            const ChainOp &og = a.ops[p];
            const uint32_t *src = reinterpret_cast<const uint32_t *>(reinterpret_cast<const uint8_t *>(&og) + kDescOff);
            uint32_t *dst = reinterpret_cast<uint32_t *>(desc + (p & 1) * sizeof(ChainOp) + kDescOff);
            for (int i = ctid; i < kDescWords; i += nthr) dst[i] = __ldg(src + i);
            const float *gm = og.gamma;
            const int Kg = og.K;
            if (gm != nullptr)
                for (int i = ctid * 32; i < Kg; i += nthr * 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(gm + i));
        }
        // grid barrier: op p reads what op p-1 wrote
        if (p > 0) {
            if (ctid == 0 && !*reinterpret_cast<volatile int *>(abort_flag)) {
                const unsigned *d = a.done + (p - 1);
                if (ld_acquire_gpu(d) < target) {
                    const uint64_t tw = global_timer_ns();
                    while (ld_acquire_gpu(d) < target) {
                        if (global_timer_ns() - tw > 2000000000ull) {
                            atomicExch(a.err, kErrChainBarrier);
                            *abort_flag = 1;
                            break;
                        }
                    }
                }
            }
        }
        named_bar_sync(1, nthr);
        const ChainOp &o = *reinterpret_cast<const ChainOp *>(desc + (p & 1) * sizeof(ChainOp));
        const int K = o.K, U = o.U, NM = o.nmat;
        // prologue: x' = x * g staged as limbs per 256-element block (see unit_q4k_imma), with the
        // sub-block sums of x' and the block scales; sum x^2 for a fused RMSNorm.  Warp cw stages
        // blocks cw, cw + W, ...: lane l holds elements 4l..4l+3 and 128+4l..128+4l+3 of a block.
        float ss = 0.f;
        {
            const int nb = K / 256;
            constexpr int B = 2;  // blocks per warp per pass (one pass for in_dim <= 7168)
            for (int b0 = cw; b0 < nb; b0 += B * W) {
                float4 vv[B][2], gg[B][2];
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int b = b0 + u * W;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int j = b * 64 + 32 * h + lane;
                        // L2 only: another SM wrote x during the previous op, after this SM may have cached it
                        if (b >= nb) {
                            vv[u][h] = make_float4(0.f, 0.f, 0.f, 0.f);
                        } else if (o.x_fixed != nullptr) {
                            const longlong2 lo = __ldcg(reinterpret_cast<const longlong2 *>(o.x_fixed) + 2 * j);
                            const longlong2 hi = __ldcg(reinterpret_cast<const longlong2 *>(o.x_fixed) + 2 * j + 1);
                            vv[u][h] = make_float4(from_fixed(lo.x), from_fixed(lo.y), from_fixed(hi.x), from_fixed(hi.y));
                        } else {
                            vv[u][h] = __ldcg(reinterpret_cast<const float4 *>(o.x) + j);
                        }
                        gg[u][h] = (b < nb && o.gamma != nullptr) ? reinterpret_cast<const float4 *>(o.gamma)[j]
                                                                  : make_float4(1.f, 1.f, 1.f, 1.f);
                    }
                }
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int b = b0 + u * W;
                    if (b >= nb) break;  // warp-uniform
                    float4 xv[2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        xv[h] = vv[u][h];
                        if (o.gamma != nullptr) {
                            ss += fmaf(xv[h].x, xv[h].x, fmaf(xv[h].y, xv[h].y, fmaf(xv[h].z, xv[h].z, xv[h].w * xv[h].w)));
                            const float4 gm = gg[u][h];
                            xv[h].x *= gm.x; xv[h].y *= gm.y; xv[h].z *= gm.z; xv[h].w *= gm.w;
                        }
                    }
                    stage_block_limbs(xv, xl + b * 256, xsum + b * 8, xe + b, lane);
                }
            }
        }
        if (o.gamma != nullptr) {
            const float wsum = warp_sum(ss);
            if (lane == 0) ss_part[cw] = wsum;
        }
        named_bar_sync(1, nthr);
        if (ctid == 0) {  // the producer may issue the op's remaining stages; the finisher may read the descriptor
            __threadfence_block();
            *x_staged = (unsigned)(p + 1);
        }
        if (o.gamma != nullptr && cw == 0) {
            const float tsum = warp_sum(lane < W ? ss_part[lane] : 0.f);
            if (lane == 0) inv_rms[0] = rsqrtf(tsum / (float)K + o.eps);
        }

        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};  // rows lane/4 + 8j, this thread's share
        // end of a row group: the four threads of a row hold its limb / min-term shares; sum
        // them, then thread t of group g stores row g + 8t for the finisher
        auto flush_group = [&]() {
            const int bsel = gi & 1;
            if (gi >= 2 && !*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&red_empty[bsel], ((uint32_t)(gi >> 1) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                    *abort_flag = 1;
            }
            float *rb = red + bsel * kChainRed;
#pragma unroll
            for (int mat = 0; mat < 2; ++mat) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[mat][j] += __shfl_xor_sync(0xffffffffu, acc[mat][j], 1);
                    acc[mat][j] += __shfl_xor_sync(0xffffffffu, acc[mat][j], 2);
                }
                const int tq = lane & 3;
                const float mine = tq == 0 ? acc[mat][0] : tq == 1 ? acc[mat][1] : tq == 2 ? acc[mat][2] : acc[mat][3];
                rb[(cw * 2 + mat) * kRowGroup + (lane >> 2) + 8 * tq] = mine;
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[mat][j] = 0.f;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_full[bsel]);
            ++gi;
        };
        if (o.kind == kOpMlp) {
            const int bu = o.bu, kb = bu * 144 * kRowGroup, pitch = bu * 144;
            const int Ce = C & ~1;
            auto wait_full = [&](int slot) {
                if (!*reinterpret_cast<volatile int *>(abort_flag) &&
                    !mbar_wait(&full[slot], (uint32_t)(it / NS) & 1u, a.err, kErrWaitFull))
                    *abort_flag = 1;
                return !__any_sync(0xffffffffu, *reinterpret_cast<volatile int *>(abort_flag) != 0);
            };
            for (int u = cta; cta < Ce && u < o.nunits; u += Ce, ++mu) {
                const int hh = u & 1;
                // phase 1: gate/up of the half chunk (four row groups)
                for (int r = 0; r < 4; ++r) {
                    for (int us = 0; us < U; us += bu) {
                        const int slot = it % NS;
                        const int n = U - us < bu ? U - us : bu;
                        if (wait_full(slot)) {
                            const uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                            for (int lu = ((cw - ucount) % W + W) % W; lu < n; lu += W) {
                                const int b = us + lu;
                                const uint8_t *bp[2] = {sb + lu * 144, sb + kb + lu * 144};
                                const uint32_t *xp[2] = {xl + b * 256, xl + b * 256};
                                const float *sp[2] = {xsum + b * 8, xsum + b * 8};
                                const float ep[2] = {xe[b], xe[b]};
                                unit_q4k_imma<2>(bp, pitch, xp, sp, ep, lane, acc);
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty[slot]);
                        ucount += n;
                        ++it;
                    }
                    flush_group();
                }
                // phase 2: this half's rows of the down projection against the chunk's 256
                // activations (staged by the finisher); per-row partials into the fixed-point residual
                if (!*reinterpret_cast<volatile int *>(abort_flag) &&
                    !mbar_wait(a_ready, (uint32_t)mu & 1u, a.err, kErrWaitFull))
                    *abort_flag = 1;
                const int r_beg = hh ? o.half_rows : 0, r_end = hh ? o.rows_d : o.half_rows;
                for (int r = r_beg; r < r_end; r += 2 * kMlpBoxRows) {
                    const int slot = it % NS;
                    const int span = r_end - r < 2 * kMlpBoxRows ? r_end - r : 2 * kMlpBoxRows;
                    const int n = (span + kRowGroup - 1) / kRowGroup;
                    if (wait_full(slot)) {
                        const uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                        for (int lu = ((cw - ucount) % W + W) % W; lu < n; lu += W) {
                            const uint8_t *bp[1] = {sb + (lu / kTmaSeg) * kBox + (lu % kTmaSeg) * kRowGroup * 144};
                            float pa[1][4] = {{0.f, 0.f, 0.f, 0.f}};
                            const uint32_t *xp[1] = {xa};
                            const float *sp[1] = {xsa};
                            const float ep[1] = {xsa[8]};
                            unit_q4k_imma<1>(bp, 144, xp, sp, ep, lane, pa);
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                pa[0][j] += __shfl_xor_sync(0xffffffffu, pa[0][j], 1);
                                pa[0][j] += __shfl_xor_sync(0xffffffffu, pa[0][j], 2);
                            }
                            const int tq = lane & 3;
                            const float mine = tq == 0 ? pa[0][0] : tq == 1 ? pa[0][1] : tq == 2 ? pa[0][2] : pa[0][3];
                            const int row = r + lu * kRowGroup + (lane >> 2) + 8 * tq;
                            if (row < r_end)
                                atomicAdd(reinterpret_cast<unsigned long long *>(o.y_fixed + row),
                                          (unsigned long long)to_fixed(mine));
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                    ucount += n;
                    ++it;
                }
                __threadfence();  // the residual's atomics, before the finisher reports the op done
                __syncwarp();
                if (lane == 0) mbar_arrive(p2_done);
            }
            continue;
        }
        const int bu = o.bu, seg = 2 * bu / NM;
        const int kb = bu * 144 * kRowGroup, pitch = bu * 144;
        int64_t t = cta < o.plan.C ? plan_start(o.plan, cta) : 0;
        const int64_t t1 = cta < o.plan.C ? plan_start(o.plan, cta + 1) : 0;
        Stage st;
        while (next_stage(t, t1, U, seg, 0, st)) {
            const int slot = it % NS;
            const uint32_t ph = (uint32_t)(it / NS) & 1u;
            if (!*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&full[slot], ph, a.err, kErrWaitFull)) *abort_flag = 1;
            }
            const int n = st.ue - st.us;
            // units: gate/up block pairs (NM = 2); for one matrix either single blocks, or (long ops,
            // o.pair) the block pairs (j, j + bu) of the stage's two boxes -- same rows, two
            // activation blocks, twice the independent work per warp
            const bool pr = NM == 1 && o.pair;
            const int nu = (pr && n > bu) ? bu : n;
            // warp-uniform (the tensor-core decoder is warp-collective); rows past the op's end
            // are zero-filled by the tensor map and never stored
            const bool aborted = __any_sync(0xffffffffu, *reinterpret_cast<volatile int *>(abort_flag) != 0);
            if (!aborted) {
                const uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                const int first = ((cw - ucount) % W + W) % W;
                for (int lu = first; lu < nu; lu += W) {
                    const int b = st.us + lu;
                    if (NM == 2) {
                        const uint8_t *bp[2] = {sb + lu * 144, sb + kb + lu * 144};
                        const uint32_t *xp[2] = {xl + b * 256, xl + b * 256};
                        const float *sp[2] = {xsum + b * 8, xsum + b * 8};
                        const float ep[2] = {xe[b], xe[b]};
                        unit_q4k_imma<2>(bp, pitch, xp, sp, ep, lane, acc);
                    } else if (pr && lu + bu < n) {
                        const int b2 = b + bu;  // same rows, the second box's block
                        const uint8_t *bp[2] = {sb + lu * 144, sb + kb + lu * 144};
                        const uint32_t *xp[2] = {xl + b * 256, xl + b2 * 256};
                        const float *sp[2] = {xsum + b * 8, xsum + b2 * 8};
                        const float ep[2] = {xe[b], xe[b2]};
                        float acc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                        unit_q4k_imma<2>(bp, pitch, xp, sp, ep, lane, acc2);
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[0][j] += acc2[0][j] + acc2[1][j];
                    } else {
                        const uint8_t *bp[1] = {sb + (lu / bu) * kb + (lu % bu) * 144};
                        const uint32_t *xp[1] = {xl + b * 256};
                        const float *sp[1] = {xsum + b * 8};
                        const float ep[1] = {xe[b]};
                        float acc1[1][4] = {{acc[0][0], acc[0][1], acc[0][2], acc[0][3]}};
                        unit_q4k_imma<1>(bp, pitch, xp, sp, ep, lane, acc1);
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[0][j] = acc1[0][j];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ucount += nu;
            ++it;
            if (st.last_in_group) flush_group();
        }
    }
}

}  // namespace
}  // namespace ql

using namespace ql;

namespace ql {
bool q4k_tensor_map_public(CUtensorMap *out, const uint8_t *base, int blocks, uint64_t rows, size_t row_bytes,
                           int box_blocks, int box_rows);
int chain_workspace(float **part, unsigned **counters, int **err, int *sms);
bool bchain_is(void *chain);
int bchain_run(void *chain, cudaStream_t s);
int bchain_destroy(void *chain);
}

namespace {
// Reductions of at most this many blocks run one row group per CTA.  80 includes the
// down projection (74 blocks), measured faster than stream-K there.
constexpr int kChainMaxUnitsOneGroup = 80;

// The reference's RoPE inverse frequencies 1 / powf(theta, 2i / head_dim), i < head_dim / 2
// (kernel.cu:186-260), computed once on the host.
std::vector<float> rope_inverse_frequencies(float theta, int head_dim) {
    std::vector<float> t(head_dim / 2);
    for (int i = 0; i < head_dim / 2; ++i) t[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
    return t;
}

struct Chain {
    int magic = 0x43484e31;  // the batched chain (ql_bchain.cu) starts with a different magic word
    ChainOp *ops_dev = nullptr;
    void *mlp_mem = nullptr;             // fused MLP: fixed-point residuals, then pair-exchange cells
    float *rope_mem = nullptr;           // RoPE inverse-frequency tables
    unsigned long long *keys = nullptr;  // [nops] fused-argmax keys
    unsigned *done = nullptr;   // [nops] arrival counters, [nops] epoch, [nops+1 ..] argmax arrival counters
    unsigned *epoch = nullptr;
    ChainArgs args{};
    int smem = 0;
    int sms = 0;
};
}  // namespace

extern "C" {

// Exchange cells a tensor-parallel chain needs per rank (64-bit words).
long long chain_cells(const ql_chain_op *ops, int nops, int world) {
    long long n = 0;
    for (int p = 0; p < nops; ++p) {
        const ql_chain_op &q = ops[p];
        if (q.kind == QL_OP_ADD && q.reduce) n += (long long)((q.rows[0] + kRowGroup - 1) / kRowGroup) * world * kRowGroup;
        if (q.argmax_idx) n += 2LL * world;
    }
    return n;
}

int chain_create(const ql_chain_op *ops, int nops, int rank, int world, void *const *exchange, void **chain) {
    if (!ops || nops <= 0 || !chain) return set_last_error(QL_EINVAL, "ql_gemv_chain_create: need ops and nops > 0");
    if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || (world > 1 && !exchange))
        return set_last_error(QL_EINVAL, "ql_gemv_chain_create: bad rank/world or missing exchange buffers");
    float *part;
    unsigned *counters;
    int *err, sms;
    int st = chain_workspace(&part, &counters, &err, &sms);
    if (st) return st;
    std::vector<ChainOp> h(nops);
    std::vector<std::pair<int, std::vector<float>>> rope_tables;  // (op, inverse frequencies)
    int kmax = 0;
    for (int p = 0; p < nops; ++p) {
        const ql_chain_op &q = ops[p];
        ChainOp &o = h[p];
        memset(&o, 0, sizeof(o));
        const std::string what = "ql_gemv_chain_create: op " + std::to_string(p);
        if (q.quant_type != QL_Q4_K) return set_last_error(QL_EINVAL, (what + ": only Q4_K").c_str());
        if (q.kind < QL_OP_STORE || q.kind > QL_OP_MLP) return set_last_error(QL_EINVAL, (what + ": kind").c_str());
        if (q.kind == QL_OP_MLP) {
            // y += down(SiLU(gate . x^) * (up . x^)), x^ = RMSNorm(x) when gamma is set
            const int F = q.rows[0], blocks = q.in_dim > 0 ? q.in_dim / 256 : 0;
            if (world != 1) return set_last_error(QL_EINVAL, (what + ": MLP ops run on one GPU (use SWIGLU + ADD)").c_str());
            if (q.in_dim <= 0 || q.in_dim % 256 || !q.x || !q.y || q.bias || q.argmax_idx || q.reduce)
                return set_last_error(QL_EINVAL, (what + ": MLP needs in_dim % 256 == 0, x and y, no bias/argmax").c_str());
            if (F <= 0 || F % 256 || q.rows[1] != F || q.rows[2] < kRowGroup)
                return set_last_error(QL_EINVAL, (what + ": MLP rows: gate = up = a multiple of 256, down >= 32").c_str());
            if (reinterpret_cast<uintptr_t>(q.x) % 16 || reinterpret_cast<uintptr_t>(q.gamma) % 16)
                return set_last_error(QL_EINVAL, (what + ": x and gamma must be 16-byte aligned").c_str());
            for (int s = 0; s < 3; ++s) {
                const int kb = s < 2 ? blocks : F / 256;
                if (!q.w[s] || reinterpret_cast<uintptr_t>(q.w[s]) % 16 || q.row_bytes[s] % 16 ||
                    q.row_bytes[s] < (size_t)kb * 144)
                    return set_last_error(QL_EINVAL, (what + ": weights (16-byte aligned rows)").c_str());
            }
            o.bu = blocks < kTmaSeg ? blocks : kTmaSeg;
            for (int s = 0; s < 2; ++s)
                if (!q4k_tensor_map_public(&o.tmap[s], q.w[s], blocks, (uint64_t)F, q.row_bytes[s], o.bu, kRowGroup))
                    return set_last_error(QL_ECUDA, (what + ": tensor map").c_str());
            if (!q4k_tensor_map_public(&o.tmap[2], q.w[2], F / 256, (uint64_t)q.rows[2], q.row_bytes[2], 1, kMlpBoxRows))
                return set_last_error(QL_ECUDA, (what + ": tensor map").c_str());
            o.kind = kOpMlp;
            o.nmat = 2;
            o.rows = F;
            o.K = q.in_dim;
            o.U = blocks;
            o.x = q.x;
            o.gamma = q.gamma;
            o.eps = q.eps;
            o.y = q.y;
            o.rows_d = q.rows[2];
            o.half_rows = (q.rows[2] + 2 * kRowGroup - 1) / (2 * kRowGroup) * kRowGroup;
            o.nunits = 2 * (F / 256);
            if (q.in_dim > kmax) kmax = q.in_dim;
            continue;
        }
        const int nsrc = q.kind == QL_OP_SWIGLU ? 2 : q.nsrc;
        if (nsrc < 1 || nsrc > 3 || q.in_dim <= 0 || q.in_dim % 256 || !q.x || (!q.y && !q.argmax_idx))
            return set_last_error(QL_EINVAL, (what + ": sources, in_dim (a multiple of 256), x or y").c_str());
        if (reinterpret_cast<uintptr_t>(q.x) % 16 || reinterpret_cast<uintptr_t>(q.gamma) % 16)
            return set_last_error(QL_EINVAL, (what + ": x and gamma must be 16-byte aligned").c_str());
        const int blocks = q.in_dim / 256;
        o.bu = blocks < kTmaSeg ? blocks : kTmaSeg;
        if (q.reduce && (q.kind != QL_OP_ADD || world < 2 || q.bias))
            return set_last_error(QL_EINVAL, (what + ": reduce needs an ADD op without bias and world > 1").c_str());
        o.reduce = q.reduce ? 1 : 0;
        int total = 0;
        for (int s = 0; s < nsrc; ++s) {
            if (!q.w[s] || reinterpret_cast<uintptr_t>(q.w[s]) % 16 || q.row_bytes[s] % 16 ||
                q.row_bytes[s] < (size_t)blocks * 144 || q.rows[s] < kRowGroup)
                return set_last_error(QL_EINVAL, (what + ": weights (16-byte aligned, >= 32 rows)").c_str());
            if (q.kind != QL_OP_SWIGLU && s < nsrc - 1 && q.rows[s] % kRowGroup)
                return set_last_error(QL_EINVAL, (what + ": stacked sources but the last need multiples of 32 rows").c_str());
            if (!q4k_tensor_map_public(&o.tmap[s], q.w[s], blocks, (uint64_t)q.rows[s], q.row_bytes[s], o.bu, kRowGroup))
                return set_last_error(QL_ECUDA, (what + ": tensor map").c_str());
            if (q.kind != QL_OP_SWIGLU) {
                total += q.rows[s];
                if (s < 2) o.split[s] = total;
            }
        }
        if (q.kind == QL_OP_SWIGLU) {
            if (q.rows[1] != q.rows[0]) return set_last_error(QL_EINVAL, (what + ": gate and up rows differ").c_str());
            total = q.rows[0];
            o.split[0] = o.split[1] = total;
        }
        for (int s = nsrc; s < 3; ++s) {
            o.tmap[s] = o.tmap[nsrc - 1];
            if (s < 2 && q.kind != QL_OP_SWIGLU) o.split[s] = total;
        }
        if (q.rope_rows > 0) {
            const int hd = q.head_dim;
            const int limit = nsrc == 3 ? o.split[1] : total;  // sources 0 and 1 only (q, k)
            if (q.kind != QL_OP_STORE || q.argmax_idx || !q.rope_pos || hd <= 0 || hd % 32 || q.rope_rows % hd ||
                q.rope_rows > limit || (nsrc >= 2 && q.rope_rows > o.split[0] && o.split[0] % hd))
                return set_last_error(QL_EINVAL, (what + ": RoPE needs a STORE op without argmax, rope_pos, head_dim a "
                                                         "multiple of 32 and rope_rows whole heads of sources 0 and 1").c_str());
            for (int s = 0; s < (nsrc < 2 ? nsrc : 2); ++s)
                if (!q4k_tensor_map_public(&o.tmap16[s], q.w[s], blocks, (uint64_t)q.rows[s], q.row_bytes[s], o.bu, 16))
                    return set_last_error(QL_ECUDA, (what + ": tensor map").c_str());
            if (nsrc < 2) o.tmap16[1] = o.tmap16[0];
            o.rope_pos = q.rope_pos;
            o.rope_rows = q.rope_rows;
            o.rope_half = hd / 2;
            rope_tables.push_back({p, rope_inverse_frequencies(q.rope_theta, hd)});
        }
        o.kind = q.kind == QL_OP_STORE ? kOpStore : q.kind == QL_OP_ADD ? kOpAdd : kOpSwiglu;
        o.nmat = q.kind == QL_OP_SWIGLU ? 2 : 1;
        o.rows = total;
        o.K = q.in_dim;
        o.U = blocks;
        const int G = (total + kRowGroup - 1) / kRowGroup;
        // like the per-op launcher: short reductions with at most one wave of row groups take one
        // group per CTA (no stream-K fix-ups, whose latency would sit on the chain's critical path)
        const int copt = (G <= sms && blocks <= kChainMaxUnitsOneGroup) ? G : sms;
        o.plan = Plan{(int64_t)G * blocks, G, blocks, copt};
        // stream-K ops (several row groups per CTA, e.g. the LM head) are throughput-bound: pair the
        // blocks; one-group-per-CTA ops are latency-bound and keep one block per warp
        o.pair = (copt == sms && G > sms) ? 1 : 0;
        o.x = q.x;
        o.gamma = q.gamma;
        o.eps = q.eps;
        o.bias = q.kind == QL_OP_SWIGLU ? nullptr : q.bias;
        o.y = q.y;
        if (q.argmax_idx) {
            if (q.kind != QL_OP_STORE) return set_last_error(QL_EINVAL, (what + ": argmax needs a store op").c_str());
            o.amax.idx = q.argmax_idx;
            o.amax.offset = q.argmax_offset;
        }
        if (q.in_dim > kmax) kmax = q.in_dim;
    }
    // fused MLP ops: the residual y in fixed point (int64, written by the last ADD into y before
    // the MLP, accumulated by the MLP's atomics), read back by the next op, which also restores y
    auto overlaps = [](const float *a0, int na, const float *b0, int nb) {
        return a0 && b0 && a0 < b0 + nb && b0 < a0 + na;
    };
    std::vector<size_t> fixed_off(nops, 0), cell_off(nops, 0);
    std::vector<int> seed(nops, -1);
    size_t fixed_total = 0, cell_total = 0;
    for (int p = 0; p < nops; ++p) {
        ChainOp &o = h[p];
        if (o.kind != kOpMlp) continue;
        const std::string what = "ql_gemv_chain_create: MLP op " + std::to_string(p);
        int q = p - 1;
        while (q >= 0 && !(h[q].kind != kOpMlp && overlaps(h[q].y, h[q].rows, o.y, o.rows_d)) &&
               !(h[q].kind == kOpMlp && overlaps(h[q].y, h[q].rows_d, o.y, o.rows_d)))
            --q;
        if (q < 0 || h[q].kind != kOpAdd || h[q].y != o.y || h[q].rows != o.rows_d || h[q].y_fixed)
            return set_last_error(QL_EINVAL, (what + ": its residual y must be last written by an ADD op of the chain "
                                                      "with the same y and rows").c_str());
        if (p + 1 >= nops || h[p + 1].kind == kOpMlp ||
            (h[p + 1].kind == kOpAdd && overlaps(h[p + 1].y, h[p + 1].rows, o.y, o.rows_d)))
            return set_last_error(QL_EINVAL, (what + ": must be followed by a STORE or SWIGLU op, or an ADD into "
                                                      "another buffer").c_str());
        seed[p] = q;
        fixed_off[p] = fixed_total;
        fixed_total += (size_t)o.rows_d;
        cell_off[p] = cell_total;
        cell_total += (size_t)o.nunits * 128;
    }
    // ADD ops may read their residual before op p-1 completes when no op since p-2 wrote it
    for (int p = 0; p < nops; ++p) {
        ChainOp &o = h[p];
        o.pre_y = 0;
        if (o.kind != kOpAdd) continue;
        const bool prev_writes = p > 0 && (overlaps(h[p - 1].y, h[p - 1].rows, o.y, o.rows) ||
                                           (h[p - 1].kind == kOpMlp && overlaps(h[p - 1].y, h[p - 1].rows_d, o.y, o.rows)) ||
                                           (p >= 2 && h[p - 2].kind == kOpMlp &&
                                            overlaps(h[p - 2].y, h[p - 2].rows_d, o.y, o.rows)));
        o.pre_y = prev_writes ? 0 : 1;
    }
    // exchange cells (tensor parallel): reduce ops [G][world][32], argmax ops [world][2]
    {
        long long cell = 0;
        for (int p = 0; p < nops; ++p) {
            h[p].xchg = cell;
            if (h[p].reduce) cell += (long long)h[p].plan.G * world * kRowGroup;
            if (ops[p].argmax_idx && world > 1) cell += 2LL * world;
        }
    }
    Chain *c = new Chain();
    c->sms = sms;
    cudaError_t e = cudaSuccess;
    if (fixed_total + cell_total) {
        e = cudaMalloc(&c->mlp_mem, (fixed_total + cell_total) * 8);
        if (e == cudaSuccess) e = cudaMemset(c->mlp_mem, 0, (fixed_total + cell_total) * 8);
        if (e != cudaSuccess) {
            delete c;
            return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create: ") + cudaGetErrorString(e)).c_str());
        }
        long long *fixed = static_cast<long long *>(c->mlp_mem);
        for (int p = 0; p < nops; ++p) {
            if (h[p].kind != kOpMlp) continue;
            long long *yf = fixed + fixed_off[p];
            h[p].y_fixed = yf;
            h[p].cells = (long long)cell_off[p];
            h[seed[p]].y_fixed = yf;
            ChainOp &nx = h[p + 1];
            nx.mat_src = yf;
            nx.mat_dst = h[p].y;
            nx.mat_rows = h[p].rows_d;
            if (nx.x == h[p].y && nx.K <= h[p].rows_d) nx.x_fixed = yf;
        }
        // an ADD two ops after an MLP on the same residual (o_proj after q/k/v) reads that residual from
        // the MLP's fixed-point copy before its partial sums are ready: op p-1 only restores the fp32
        // copy, with the same values
        for (int p = 2; p < nops; ++p) {
            ChainOp &o = h[p];
            const ChainOp &m = h[p - 2], &mid = h[p - 1];
            if (o.kind != kOpAdd || o.reduce || m.kind != kOpMlp || m.y != o.y || m.rows_d != o.rows) continue;
            if (mid.kind == kOpMlp || overlaps(mid.y, mid.rows, o.y, o.rows)) continue;
            o.res_fixed = m.y_fixed;
            o.pre_y = 1;
        }
        c->args.mlp_cells = reinterpret_cast<unsigned long long *>(fixed + fixed_total);
    }
    if (!rope_tables.empty()) {
        size_t nf = 0;
        for (auto &rt : rope_tables) nf += rt.second.size();
        e = cudaMalloc(&c->rope_mem, nf * sizeof(float));
        size_t at = 0;
        for (auto &rt : rope_tables) {
            if (e == cudaSuccess)
                e = cudaMemcpy(c->rope_mem + at, rt.second.data(), rt.second.size() * sizeof(float), cudaMemcpyHostToDevice);
            h[rt.first].rope_inv = c->rope_mem + at;
            at += rt.second.size();
        }
        if (e != cudaSuccess) {
            if (c->mlp_mem) cudaFree(c->mlp_mem);
            if (c->rope_mem) cudaFree(c->rope_mem);
            delete c;
            return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create: ") + cudaGetErrorString(e)).c_str());
        }
    }
    e = cudaMalloc(&c->ops_dev, sizeof(ChainOp) * nops);
    // per-op argmax keys and arrival counter: one slot per op at the end of the counter block
    unsigned long long *keys = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&c->done, sizeof(unsigned) * (nops + 1) * 2);
    if (e == cudaSuccess) e = cudaMalloc(&keys, sizeof(unsigned long long) * nops);
    if (e == cudaSuccess) e = cudaMemset(c->done, 0, sizeof(unsigned) * (nops + 1) * 2);
    if (e == cudaSuccess) e = cudaMemset(keys, 0, sizeof(unsigned long long) * nops);
    if (e == cudaSuccess) {
        for (int p = 0; p < nops; ++p)
            if (h[p].amax.idx) {
                h[p].amax.amax = keys + p;
                h[p].amax.done = c->done + nops + 1 + p;
            }
        c->epoch = c->done + nops;
        c->keys = keys;
        e = cudaMemcpy(c->ops_dev, h.data(), sizeof(ChainOp) * nops, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        if (c->ops_dev) cudaFree(c->ops_dev);
        if (c->done) cudaFree(c->done);
        if (keys) cudaFree(keys);
        if (c->mlp_mem) cudaFree(c->mlp_mem);
        if (c->rope_mem) cudaFree(c->rope_mem);
        delete c;
        return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create: ") + cudaGetErrorString(e)).c_str());
    }
    size_t off = kGemvHeaderBytes;
    off += ((size_t)kmax * 4 + 127) / 128 * 128;
    off += ((size_t)(kmax / 32) * 4 + 127) / 128 * 128;
    off += ((size_t)(kmax / 256) * 4 + 127) / 128 * 128;
    off += ((size_t)2 * kChainRed * 4 + 127) / 128 * 128;
    off += 2 * sizeof(ChainOp);
    off += kMlpSmem;
    off = (off + 1023) / 1024 * 1024;
    int nslots = kChainSlots;
    while (nslots > 2 && off + (size_t)nslots * kSlotBytes > 227 * 1024) --nslots;
    off += (size_t)nslots * kSlotBytes;
    if (off > 227 * 1024) {
        ql_gemv_chain_destroy(c);
        return set_last_error(QL_EINVAL, "ql_gemv_chain_create: in_dim too large for the shared-memory stage");
    }
    c->smem = (int)off;
    c->args.ops = c->ops_dev;
    c->args.nops = nops;
    c->args.kmax = kmax;
    c->args.done = c->done;
    c->args.epoch = c->epoch;
    c->args.part = part;
    c->args.counters = counters;
    c->args.err = err;
    c->args.rank = rank;
    c->args.world = world;
    c->args.nslots = nslots;
    for (int r = 0; r < world; ++r)
        c->args.xchg[r] = world > 1 ? static_cast<unsigned long long *>(exchange[r]) : nullptr;
    *chain = c;
    return QL_OK;
}

int ql_gemv_chain_create(const ql_chain_op *ops, int nops, void **chain) {
    return chain_create(ops, nops, 0, 1, nullptr, chain);
}

size_t ql_gemv_chain_exchange_bytes(const ql_chain_op *ops, int nops, int world) {
    if (!ops || nops <= 0 || world < 1 || world > kMaxWorld) return 0;
    return (size_t)chain_cells(ops, nops, world) * sizeof(unsigned long long);
}

int ql_gemv_chain_create_tp(const ql_chain_op *ops, int nops, int rank, int world, void *const *exchange,
                            void **chain) {
    return chain_create(ops, nops, rank, world, exchange, chain);
}

int ql_gemv_chain_run(void *chain) {
    Chain *c = static_cast<Chain *>(chain);
    if (!c) return set_last_error(QL_EINVAL, "ql_gemv_chain_run: null chain");
    if (bchain_is(chain)) return bchain_run(chain, static_cast<cudaStream_t>(ql_get_stream()));
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
        attr_set = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(c->sms);
    cfg.blockDim = dim3(kChainThreads);
    cfg.dynamicSmemBytes = c->smem;
    cfg.stream = static_cast<cudaStream_t>(ql_get_stream());
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barriers cannot deadlock
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_chain_kernel, c->args);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

int ql_gemv_chain_destroy(void *chain) {
    Chain *c = static_cast<Chain *>(chain);
    if (!c) return QL_OK;
    if (bchain_is(chain)) return bchain_destroy(chain);
    cudaDeviceSynchronize();
    if (c->ops_dev) cudaFree(c->ops_dev);
    if (c->done) cudaFree(c->done);
    if (c->keys) cudaFree(c->keys);
    if (c->mlp_mem) cudaFree(c->mlp_mem);
    if (c->rope_mem) cudaFree(c->rope_mem);
    delete c;
    return QL_OK;
}

}  // extern "C"
