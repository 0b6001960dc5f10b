// ql_gemv.cuh -- the streaming block-quantized GEMV engine (decode path, M <= 4).
//
// Replaces the reference's warp-per-row kernels quant_gemv_kernel,
// quant_gemv_add_kernel, quant_matmul_kernel, quant_swiglu_kernel,
// quant_swiglu_indexed_kernel and quant_down_f32_indexed_accum_ordered_kernel
// (AI/codes/local-llm/src/backend/cuda/ops/kernel.cu:1191-1385,2252-2287).
//
// Design (B200, sm_100a):
//  * One producer warp streams the raw GGUF bytes of 32 output rows x SEG
//    blocks per stage into a shared-memory ring with 1-D TMA bulk copies
//    (cp.async.bulk + mbarrier complete_tx, L2 evict-first).  Unaligned row
//    starts (34/18/22-byte blocks) are handled by copying the 16-byte-aligned
//    interior in bulk and the ragged head/tail bytes with plain loads, so no
//    byte outside the requested range is ever read.
//  * Consumer warps: lane = output row.  Warp w takes every W-th block of the
//    stream.  The activation is staged once per CTA in shared memory,
//    pre-multiplied by 2^(96-p), p being the bit position its weight nibble or
//    byte occupies after one AND: the masked integer reinterpreted as a float
//    is the exact denormal q * 2^(p-149), so one LOP3 and one FMA per weight
//    give q * x * 2^-53 in fp32.  Scales and mins are applied once per 32-
//    element sub-block: dot = D * 2^53 * S - M * X, X the block sum of the
//    activation (precomputed).  Accumulation is fp32 throughout.
//  * Row groups are split over CTAs in equal tile counts (stream-K); a group
//    shared by several CTAs is finished by the last one to arrive, which sums
//    the parts in K order, so results are deterministic.
//  * Fused RMSNorm prologue (f32 gamma) and store / add / SwiGLU / bias
//    epilogues.
#pragma once

#include <cuda.h>  // CUtensorMap (types only; the encoder is resolved at run time)

#include "ql_common.cuh"

namespace ql {

// kSrcStacked: up to 3 matrices sharing the activation, stacked by rows (fused
// q/k/v): rows [0, split0) come from w[0], [split0, split1) from w[1], the rest
// from w[2]; every split is a multiple of 32 so a row group has one source.
enum SrcKind : int { kSrcPlain = 0, kSrcIndexedRows = 1, kSrcIndexedK = 2, kSrcStacked = 3 };
constexpr int kMaxStacked = 3;
enum EpiKind : int { kEpiStore = 0, kEpiAdd = 1, kEpiSwiglu = 2 };

// 16 warps per CTA (4 per scheduler, 128 registers each): producers, one
// row-group finisher, consumers.  TMA staging needs one producer warp; cp.async
// staging uses 4 (bytes in flight scale with the number of issuing warps).
constexpr int kGemvThreads = 512;
__host__ __device__ constexpr int gemv_producer_warps(bool tma) { return tma ? 1 : 4; }
__host__ __device__ constexpr int gemv_consumer_warps(bool tma) { return 16 - gemv_producer_warps(tma) - 1; }
// Programmatic dependent launch (always on).
bool gemv_pdl_enabled();
constexpr int kGemvStages = 4;  // most stages (the host may pick fewer to fit shared memory)
constexpr int kGemvMaxTokens = 4;

// Blocks per stage for each format (about 1 KB of each row per stage, so that
// half the consumer warps get one block each).
__host__ __device__ constexpr int gemv_seg(int t) {
    return t == kQ4_K ? 8 : t == kQ6_K ? 4 : t == kQ8_0 ? 32 : t == kQ4_0 ? 64 : t == kQ5_0 ? 48 : 0;
}
// Shared-memory pitch of one row slot: data + 16 bytes of alignment slack +
// 16 bytes of over-read slack, rounded so that pitch % 128 == 16 (lanes reading
// the same offset of consecutive rows hit distinct bank groups).
__host__ __device__ constexpr int gemv_pitch(int t) {
    return ((gemv_seg(t) * block_bytes(t) + 32 + 127) / 128) * 128 + 16;
}

// Tensor-map (TMA) staging.  Q4_K: one 3-D box {144 B, 7 blocks, 32 rows} per matrix per
// stage, landing as [32 rows][7 blocks][144 B], a row pitch of 1008 B (= 112 mod 128), so lanes
// reading consecutive rows at the same offset fall in distinct 16-byte bank groups.  The
// 32-element formats (rows a multiple of 16 bytes long): a 2-D view {row_bytes / 8, rows} of
// 8-byte elements, one box {pitch / 8, 32 rows} per stage starting at the 16-byte boundary at or
// before the stage's first block (blocks are 18/22/34 bytes, so a stage may start mid-chunk);
// the pitch covers the stage's blocks plus that 0..15-byte lead and is 16 mod 128.
constexpr int kTmaSeg = 7;
__host__ __device__ constexpr int tma_seg(int t) {
    return t == kQ4_K ? kTmaSeg : t == kQ4_0 ? 56 : t == kQ8_0 ? 32 : t == kQ5_0 ? 48 : 0;
}
__host__ __device__ constexpr int tma_pitch(int t) {
    return t == kQ4_K ? kTmaSeg * 144 : ((tma_seg(t) * block_bytes(t) + 15 - 16 + 127) / 128) * 128 + 16;
}
__host__ __device__ constexpr bool tma_format(int t) { return tma_seg(t) > 0; }
__host__ __device__ constexpr int stage_seg(int t, bool tma) { return tma ? tma_seg(t) : gemv_seg(t); }
__host__ __device__ constexpr int stage_pitch(int t, bool tma) { return tma ? tma_pitch(t) : gemv_pitch(t); }
static_assert(tma_pitch(kQ4_0) == 1040 && tma_pitch(kQ8_0) == 1168 && tma_pitch(kQ5_0) == 1168, "TMA pitches");

// Shared-memory header of the GEMV kernel: mbarriers, abort flag, RMSNorm
// factors [4] and per-warp partial sums of squares [14][4].
constexpr int kGemvHeaderBytes = 512;

struct GemvArgs {
    const uint8_t *w[kMaxStacked];   // weight buffers (raw GGUF blocks): SwiGLU gate/up, or stacked sources
    size_t row_bytes[kMaxStacked];   // bytes per output row
    size_t expert_bytes[2];          // bytes per expert (indexed kinds)
    int split[2];                    // stacked sources: first row of w[1] and of w[2]
    int rows;                 // output rows of the launch (virtual rows for indexed-rows)
    int K;                    // reduction length in elements (virtual length for indexed-K)
    int U;                    // blocks per row = K / block_elems
    int units_per_route;      // indexed-K: blocks per route
    int rows_per_route;       // indexed-rows: output rows per route
    int M;                    // tokens in this launch (<= MT)
    const float *x;           // activations [M][x_stride] (indexed-K: [k][F] route-major)
    int64_t x_stride;
    const float *gamma;       // optional fused RMSNorm weight (f32, length K); null = none
    float eps;
    const int *ids;           // expert id per route (indexed kinds)
    const float *route_w;     // route weights (indexed-K)
    const float *bias;        // optional per-row bias (kEpiStore / kEpiAdd)
    float *y;                 // output [M][y_stride]
    int64_t y_stride;
    int nst;                  // stages in the shared-memory ring (2..kGemvStages)
    int pre_x;                // stages the producer may issue before the activations are staged
    int tma_pair;             // 32-element formats with rows a multiple of 8 (not 16) bytes long: the tensor
                              // maps view row pairs as 16-byte-aligned super-rows; a stage is two 16-row boxes
                              // (even rows, then odd rows of the group)
    CUtensorMap tmap[kMaxStacked];   // tensor maps (TMA kernels only): Q4_K {144 B, blocks, rows},
                                     // 32-element formats {row_bytes / 8, rows} of 8-byte elements
    Plan plan;
    float *part;              // stream-K partial slots [C][2][MT][NMAT][32]
    unsigned *counters;       // stream-K arrival counters [G], zero between launches
    int *err;                 // device error word
    AmaxOut amax;             // fused greedy argmax over the rows (kEpiStore; amax.amax null = off)
};

// One stage of a CTA's stream: row group g, blocks [us, ue) of the group's
// rows.  A stage never straddles a route boundary of an indexed-K source.
struct Stage {
    int g, us, ue;
    bool last_in_group;
};

// Advances a CTA's stage cursor.  `t` is the next tile (g * U + u) to cover,
// `t1` the end of the CTA's range.  Returns false when the range is exhausted.
__host__ __device__ inline bool next_stage(int64_t &t, int64_t t1, int U, int seg, int upr, Stage &s) {
    if (t >= t1) return false;
    const int g = (int)(t / U);
    const int u = (int)(t - (int64_t)g * U);
    const int64_t gend = ((int64_t)g + 1) * U < t1 ? ((int64_t)g + 1) * U : t1;
    const int uend = u + (int)(gend - t);
    int ue = u + seg < uend ? u + seg : uend;
    if (upr > 0) {
        const int rb = (u / upr + 1) * upr;
        if (rb < ue) ue = rb;
    }
    s.g = g;
    s.us = u;
    s.ue = ue;
    s.last_in_group = (ue == uend);
    t += ue - u;
    return true;
}

// Address of block `u` of output row `v` of matrix `mat`, or nullptr when the
// row's expert id is negative (the route is skipped).  `ids` may be a host or
// device pointer; it is read only for indexed sources.
// Stacked sources: which matrix holds virtual row v, and its local row.
__host__ __device__ inline int stacked_source(const GemvArgs &a, int v, int *local) {
    const int s = (v >= a.split[0]) + (v >= a.split[1]);
    *local = v - (s == 0 ? 0 : a.split[s - 1]);
    return s;
}

template <int SRC, int FMT>
__host__ __device__ inline const uint8_t *gemv_block_ptr(const GemvArgs &a, const int *ids, int mat, int v, int u) {
    constexpr int BB = block_bytes(FMT);
    if (SRC == kSrcPlain) return a.w[mat] + (size_t)v * a.row_bytes[mat] + (size_t)u * BB;
    if (SRC == kSrcStacked) {
        int local;
        const int s = stacked_source(a, v, &local);
        return a.w[s] + (size_t)local * a.row_bytes[s] + (size_t)u * BB;
    }
    if (SRC == kSrcIndexedRows) {
        const int r = v / a.rows_per_route, row = v - r * a.rows_per_route;
        const int e = ids[r];
        if (e < 0) return nullptr;
        return a.w[mat] + (size_t)e * a.expert_bytes[mat] + (size_t)row * a.row_bytes[mat] + (size_t)u * BB;
    }
    const int r = u / a.units_per_route, lu = u - r * a.units_per_route;
    const int e = ids[r];
    if (e < 0) return nullptr;
    return a.w[mat] + (size_t)e * a.expert_bytes[mat] + (size_t)v * a.row_bytes[mat] + (size_t)lu * BB;
}

// Host-side description of a launch (grid, shared memory) for one format.
struct GemvShape {
    int seg, pitch, stage_bytes, xs_floats, xsum_floats, red_floats, nst, smem_bytes;
};
__host__ inline GemvShape gemv_shape(int fmt, int MT, int NMAT, int K, int nst, bool tma) {
    GemvShape s;
    s.seg = stage_seg(fmt, tma);
    s.pitch = stage_pitch(fmt, tma);
    s.stage_bytes = NMAT * kRowGroup * s.pitch;
    s.xs_floats = MT * K;
    s.xsum_floats = MT * (K / 32);
    s.red_floats = 2 * gemv_consumer_warps(tma) * MT * NMAT * kRowGroup;
    s.nst = nst;
    int off = kGemvHeaderBytes;  // mbarriers, abort flag, RMSNorm factors and partial sums
    off += ((s.xs_floats * 4 + 127) / 128) * 128;
    off += ((s.xsum_floats * 4 + 127) / 128) * 128;
    off += ((s.red_floats * 4 + 127) / 128) * 128;
    off += nst * s.stage_bytes;
    s.smem_bytes = off;
    return s;
}

}  // namespace ql
