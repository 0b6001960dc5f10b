// Causal decode attention with an output gate over a KV cache (the reference's
// full_attention_attend{,_batch}, kernel.cu:355-490 / launch.cu:676-709):
//   out_h = softmax_j((q_h . k_j) / sqrt(head_dim)) . v_j * sigmoid(gate_h),  j = 0..pos,
// cache layout [max_seq_len][kv_heads][head_dim], f32 or bf16.
//
// The reference runs one CTA per query head over all keys, so the 7 query heads of a GQA group
// (Qwen2-7B: 28 / 4) each read the group's keys and values, and one CTA per head leaves most SMs
// idle.  Here a CTA takes one KV head and one split of the keys (flash-decoding): it loads each
// 64-key tile of K and V into shared memory once for all the group's query heads, keeps a running
// max / sum / weighted value per head, and writes them as a partial; a second launch (programmatic
// dependent: placed while the first runs, waiting on it in hardware) merges the splits (max-rescaled
// sums) and applies the gate.  The split count follows the cache length (so
// the grid is fixed for a CUDA graph) and each CTA sizes its range from the device-side position.
#include <cuda_bf16.h>

#include <type_traits>

#include "ql_attn.cuh"
#include "ql_common.cuh"

namespace ql {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kAttnTile = 64;        // keys per shared-memory tile
constexpr int kAttnMaxGroup = 16;    // query heads per KV head on the head_dim-specialised kernels
constexpr int kAttnMaxSplits = 512;  // key splits per (token, KV head)
// CTAs per SM of the head_dim-specialised split kernel (its launch bound; the host sizes the split
// count by it): with head_dim <= 128 tiles are staged by cp.async and three fit.
constexpr int attn_hd_ctas_per_sm(int hd) { return hd <= 128 ? 3 : 1; }

template <typename KvT>
__device__ __forceinline__ float kv_f32(KvT v);
template <>
__device__ __forceinline__ float kv_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float kv_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// Key range of one split: equal ranges rounded to whole tiles.
__device__ __forceinline__ void split_range(const AttnArgs &a, int split, int tok, int &j0, int &j1) {
    const int pos = (a.pos_dev != nullptr ? *a.pos_dev : a.start_pos) + tok;
    const int n_keys = min(pos + 1, a.max_seq_len);
    const int per = ((n_keys + a.splits - 1) / a.splits + kAttnTile - 1) / kAttnTile * kAttnTile;
    j0 = min(split * per, n_keys);
    j1 = min(j0 + per, n_keys);
}

// Online softmax over one tile's scores p[G][kAttnTile] (a warp per head): p <- exp(s - m_new),
// running max m, running sum l, and the rescale factor of the earlier terms in corr.
__device__ __forceinline__ void tile_softmax(float *p_s, float *m_s, float *l_s, float *c_s, int G, int nt, int warp,
                                             int lane) {
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float *pg = p_s + g * kAttnTile;
        float tmax = -INFINITY;
        for (int jj = lane; jj < kAttnTile; jj += 32) tmax = fmaxf(tmax, pg[jj]);
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float m_old = m_s[g], m_new = fmaxf(m_old, tmax);
        float tsum = 0.f;
        for (int jj = lane; jj < kAttnTile; jj += 32) {
            const float pv = jj < nt ? expf(pg[jj] - m_new) : 0.f;
            pg[jj] = pv;
            tsum += pv;
        }
        for (int o = 16; o > 0; o >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
        if (lane == 0) {
            const float corr = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
            c_s[g] = corr;
            l_s[g] = l_s[g] * corr + tsum;
            m_s[g] = m_new;
        }
    }
}

// Any head_dim (<= 256).  Shared memory: q[G][hd] | acc[G][hd] | K[kAttnTile][hd + 1] |
// V[kAttnTile][hd] | p[G][kAttnTile] | m, l, corr[G].
template <typename KvT>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the merge waits for this grid
    const int hd = a.head_dim, G = a.n_heads / a.kv_heads;
    float *q_s = sm, *acc_s = q_s + G * hd, *k_s = acc_s + G * hd, *v_s = k_s + kAttnTile * (hd + 1);
    float *p_s = v_s + kAttnTile * hd, *m_s = p_s + G * kAttnTile, *l_s = m_s + G, *c_s = l_s + G;
    const int split = blockIdx.x, kh = blockIdx.y, tok = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int j0, j1;
    split_range(a, split, tok, j0, j1);
    const float scale = rsqrtf((float)hd);
    const KvT *kc = static_cast<const KvT *>(a.key_cache), *vc = static_cast<const KvT *>(a.value_cache);

    const size_t q_base = ((size_t)tok * a.n_heads + (size_t)kh * G) * hd;  // the group's heads are adjacent
    for (int i = tid; i < G * hd; i += kAttnThreads) {
        q_s[i] = a.q[q_base + i];
        acc_s[i] = 0.f;
    }
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    __syncthreads();
    for (int t0 = j0; t0 < j1; t0 += kAttnTile) {
        const int nt = min(kAttnTile, j1 - t0);
        // K and V rows of this tile (each key's head_dim values are contiguous)
        for (int i = tid; i < nt * hd; i += kAttnThreads) {
            const int jj = i / hd, d = i - jj * hd;
            const size_t src = ((size_t)(t0 + jj) * a.kv_heads + kh) * hd + d;
            k_s[jj * (hd + 1) + d] = kv_f32<KvT>(kc[src]);
            v_s[jj * hd + d] = kv_f32<KvT>(vc[src]);
        }
        __syncthreads();
        // scores: lane = key (padded K rows: 32 keys in 32 banks), q broadcast
        for (int i = tid; i < G * kAttnTile; i += kAttnThreads) {
            const int g = i / kAttnTile, jj = i - g * kAttnTile;
            float s = -INFINITY;
            if (jj < nt) {
                const float *qg = q_s + g * hd, *kr = k_s + jj * (hd + 1);
                float dot = 0.f;
                for (int d = 0; d < hd; ++d) dot = fmaf(qg[d], kr[d], dot);
                s = dot * scale;
            }
            p_s[i] = s;
        }
        __syncthreads();
        tile_softmax(p_s, m_s, l_s, c_s, G, nt, warp, lane);
        __syncthreads();
        // weighted values: thread = (head, dim), consecutive dims in a warp
        for (int i = tid; i < G * hd; i += kAttnThreads) {
            const int g = i / hd, d = i - g * hd;
            const float *pg = p_s + g * kAttnTile;
            float acc = acc_s[i] * c_s[g];
            for (int jj = 0; jj < nt; ++jj) acc = fmaf(pg[jj], v_s[jj * hd + d], acc);
            acc_s[i] = acc;
        }
        __syncthreads();
    }
    // partial of this split: per head (m, l, acc[hd])
    const size_t pbase = (((size_t)tok * a.n_heads + (size_t)kh * G) * a.splits + split);
    for (int i = tid; i < G * hd; i += kAttnThreads) {
        const int g = i / hd, d = i - g * hd;
        a.part_acc[(pbase + (size_t)g * a.splits) * hd + d] = acc_s[i];
    }
    if (tid < G) {
        a.part_ml[(pbase + (size_t)tid * a.splits) * 2] = m_s[tid];
        a.part_ml[(pbase + (size_t)tid * a.splits) * 2 + 1] = l_s[tid];
    }
}

// 16-byte global -> shared copy that bypasses the registers (completion by commit / wait groups).
__device__ __forceinline__ void attn_cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Shared-memory K/V tiles, read in 4-element pieces as float4.  f32 rows padded by 4 floats (the 8
// lanes of a 16-byte load phase, reading 8 rows, hit distinct banks); bf16 rows (cp.async-staged, raw)
// padded by 8 elements, widened on read.
template <typename TileT, int HD>
struct AttnTile;
template <int HD>
struct AttnTile<float, HD> {
    static constexpr int kPitch = HD + 4;
    static __device__ __forceinline__ float4 get4(const float *t, int i) {
        return *reinterpret_cast<const float4 *>(t + i);
    }
};
template <int HD>
struct AttnTile<__nv_bfloat16, HD> {
    static constexpr int kPitch = HD + 8;
    static __device__ __forceinline__ float4 get4(const __nv_bfloat16 *t, int i) {
        const uint2 p = *reinterpret_cast<const uint2 *>(t + i);  // bf16: the top 16 bits of an f32
        return make_float4(__uint_as_float(p.x << 16), __uint_as_float(p.x & 0xFFFF0000u), __uint_as_float(p.y << 16),
                           __uint_as_float(p.y & 0xFFFF0000u));
    }
};

// Scores of one key row for the heads g0, g0 + 4, ... (NH of them): the key row is read from shared
// memory once for all of them; per head two accumulators (x, z and y, w lanes of each float4).
template <int NH, int HD, typename TileT>
__device__ __forceinline__ void score_heads(const float *q_s, const TileT *k_t, float *p_s, int jj, int g0, int nt,
                                            float scale) {
    constexpr int Q4 = HD / 4, KP = AttnTile<TileT, HD>::kPitch;
    const TileT *kr = k_t + jj * KP;
    float d0[NH], d1[NH];
#pragma unroll
    for (int h = 0; h < NH; ++h) d0[h] = d1[h] = 0.f;
#pragma unroll 4
    for (int c4 = 0; c4 < Q4; ++c4) {
        const float4 kk = AttnTile<TileT, HD>::get4(kr, 4 * c4);
#pragma unroll
        for (int h = 0; h < NH; ++h) {
            const float4 qq = reinterpret_cast<const float4 *>(q_s + (g0 + 4 * h) * HD)[c4];
            d0[h] = fmaf(qq.x, kk.x, d0[h]);
            d1[h] = fmaf(qq.y, kk.y, d1[h]);
            d0[h] = fmaf(qq.z, kk.z, d0[h]);
            d1[h] = fmaf(qq.w, kk.w, d1[h]);
        }
    }
#pragma unroll
    for (int h = 0; h < NH; ++h) p_s[(g0 + 4 * h) * kAttnTile + jj] = jj < nt ? (d0[h] + d1[h]) * scale : -INFINITY;
}

// Tile element type of the head_dim-specialised kernel: the cache's own type where tiles are staged
// by cp.async (head_dim <= 128), f32 (widened through registers) for head_dim 256.
template <typename KvT, int HD>
using AttnTileT = typename std::conditional<(HD <= 128), KvT, float>::type;

// The same for a head_dim known at compile time (64, 128, 256) and groups of <= MG heads (8 or 16).
// Scores: thread = key (64 per tile) x head phase g0 (0..3), every head g0 + 4i of the group from one
// read of the key row.  Weighted values: thread = (key parity, head pair, 4 dims): each V piece read
// once for two heads, the even and odd keys of a tile summed by different threads (running sums in
// registers, rescaled per tile) and added at the end.  Shared memory: q[G][HD] f32 | K[kAttnTile][pitch] |
// V[kAttnTile][HD] (tile type) | p[G][kAttnTile] | m, l, corr[G].
template <typename KvT, int HD, int MG>
__global__ void __launch_bounds__(kAttnThreads, attn_hd_ctas_per_sm(HD))
    attn_split_hd_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    using TileT = AttnTileT<KvT, HD>;
    using Tile = AttnTile<TileT, HD>;
    constexpr int Q4 = HD / 4, KP = Tile::kPitch;
    constexpr int QV = (MG * Q4 + kAttnThreads - 1) / kAttnThreads;  // float4 pieces of q per thread
    constexpr int GPR = kAttnThreads / 2 / Q4;                       // head pairs per value round
    constexpr int VR = (MG / 2 + GPR - 1) / GPR;                     // value rounds
    // the merge kernel may be scheduled now; it waits for this grid before reading the partials
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int G = a.n_heads / a.kv_heads;
    float *q_s = sm;
    TileT *k_t = reinterpret_cast<TileT *>(q_s + G * HD), *v_t = k_t + kAttnTile * KP;
    float *p_s = reinterpret_cast<float *>(v_t + kAttnTile * HD);
    float *m_s = p_s + G * kAttnTile, *l_s = m_s + G, *c_s = l_s + G;
    const int split = blockIdx.x, kh = blockIdx.y, tok = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float scale = rsqrtf((float)HD);
    // the group's queries (adjacent heads) are loaded before the position is read
    const size_t q_base = ((size_t)tok * a.n_heads + (size_t)kh * G) * HD;
    float4 qv[QV];
#pragma unroll
    for (int u = 0; u < QV; ++u) {
        const int i = tid + u * kAttnThreads;
        if (i < G * Q4) qv[u] = reinterpret_cast<const float4 *>(a.q + q_base)[i];
    }
    int j0, j1;
    split_range(a, split, tok, j0, j1);
#pragma unroll
    for (int u = 0; u < QV; ++u) {
        const int i = tid + u * kAttnThreads;
        if (i < G * Q4) reinterpret_cast<float4 *>(q_s)[i] = qv[u];
    }
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    // value-phase ownership: key parity vh, head pair vgp + GPR r, dims 4 vc4 .. 4 vc4 + 3
    const int vh = tid / (kAttnThreads / 2), vgp = (tid % (kAttnThreads / 2)) / Q4, vc4 = tid % Q4;
    float4 acc[VR][2];
#pragma unroll
    for (int r = 0; r < VR; ++r) acc[r][0] = acc[r][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();
    // Tile loads.  head_dim <= 128 (kAsync): 16-byte cp.async chunks straight into the tiles in the
    // cache's type, K and V in separate groups, each tile's next contents issued as soon as its last
    // reader is done (K after the scores, V after the values), so no registers hold pieces and three CTAs
    // share an SM.  head_dim 256: NL 4-element pieces of K and of V per thread loaded into registers
    // before any is stored (widened to f32), the next tile's in flight while the current one computes.
    constexpr bool kAsync = HD <= 128;
    constexpr int NL = kAttnTile * Q4 / kAttnThreads;
    constexpr int CE = 16 / sizeof(TileT), QC = HD / CE, NC = kAttnTile * QC / kAttnThreads;  // chunks
    using Piece = typename std::conditional<sizeof(KvT) == 4, float4, uint2>::type;
    Piece kp[kAsync ? 1 : NL], vp[kAsync ? 1 : NL];
    auto copy_rows = [&](TileT *dst, int pitch, const void *cache, int t0) {
        const int nt = min(kAttnTile, j1 - t0);
#pragma unroll
        for (int u = 0; u < NC; ++u) {
            const int i = tid + u * kAttnThreads, jj = i / QC, c = i - jj * QC;
            if (jj < nt)
                attn_cp_async16(dst + jj * pitch + CE * c,
                                static_cast<const TileT *>(cache) + ((size_t)(t0 + jj) * a.kv_heads + kh) * HD + CE * c);
        }
    };
    auto issue = [&](int t0) {
        const int nt = min(kAttnTile, j1 - t0);
#pragma unroll
        for (int u = 0; u < NL; ++u) {
            const int i = tid + u * kAttnThreads, jj = i / Q4, c4 = i - jj * Q4;
            if (jj < nt) {
                const size_t src = ((size_t)(t0 + jj) * a.kv_heads + kh) * HD + 4 * c4;
                kp[u] = *reinterpret_cast<const Piece *>(static_cast<const KvT *>(a.key_cache) + src);
                vp[u] = *reinterpret_cast<const Piece *>(static_cast<const KvT *>(a.value_cache) + src);
            }
        }
    };
    auto widen = [](const Piece &p) -> float4 {
        if constexpr (sizeof(KvT) == 4) {
            return p;
        } else {  // bf16: the top 16 bits of an f32
            return make_float4(__uint_as_float(p.x << 16), __uint_as_float(p.x & 0xFFFF0000u),
                               __uint_as_float(p.y << 16), __uint_as_float(p.y & 0xFFFF0000u));
        }
    };
    if constexpr (kAsync) {
        if (j0 < j1) copy_rows(k_t, KP, a.key_cache, j0);
        asm volatile("cp.async.commit_group;" ::: "memory");
        if (j0 < j1) copy_rows(v_t, HD, a.value_cache, j0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
        if (j0 < j1) issue(j0);
    }
    for (int t0 = j0; t0 < j1; t0 += kAttnTile) {
        const int nt = min(kAttnTile, j1 - t0);
        if constexpr (kAsync) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");  // this tile's K (its V may be in flight)
        } else {
#pragma unroll
            for (int u = 0; u < NL; ++u) {
                const int i = tid + u * kAttnThreads, jj = i / Q4, c4 = i - jj * Q4;
                if (jj < nt) {
                    if constexpr (!kAsync) {  // f32 tiles
                        *reinterpret_cast<float4 *>(k_t + jj * KP + 4 * c4) = widen(kp[u]);
                        *reinterpret_cast<float4 *>(v_t + jj * HD + 4 * c4) = widen(vp[u]);
                    }
                }
            }
        }
        __syncthreads();
        if constexpr (!kAsync) {
            if (t0 + kAttnTile < j1) issue(t0 + kAttnTile);  // in flight while this tile computes
        }
        {
            const int jj = tid & (kAttnTile - 1), g0 = tid / kAttnTile;
            switch (G > g0 ? (G - g0 + 3) / 4 : 0) {
                case 1: score_heads<1, HD>(q_s, k_t, p_s, jj, g0, nt, scale); break;
                case 2: score_heads<2, HD>(q_s, k_t, p_s, jj, g0, nt, scale); break;
                case 3:
                    if constexpr (MG > 8) score_heads<3, HD>(q_s, k_t, p_s, jj, g0, nt, scale);
                    break;
                case 4:
                    if constexpr (MG > 8) score_heads<4, HD>(q_s, k_t, p_s, jj, g0, nt, scale);
                    break;
                default: break;
            }
        }
        __syncthreads();
        if constexpr (kAsync) {  // the K tile is free: the next tile's keys land during softmax and values
            if (t0 + kAttnTile < j1) copy_rows(k_t, KP, a.key_cache, t0 + kAttnTile);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        tile_softmax(p_s, m_s, l_s, c_s, G, nt, warp, lane);
        if constexpr (kAsync) asm volatile("cp.async.wait_group 1;" ::: "memory");  // this tile's V
        __syncthreads();
#pragma unroll
        for (int r = 0; r < VR; ++r) {
            const int g = 2 * (vgp + GPR * r);
            if (g < G) {
                const int g1 = g + 1 < G ? g + 1 : g;  // an odd group's last pair repeats its head
                const float *p0 = p_s + g * kAttnTile, *p1 = p_s + g1 * kAttnTile;
                const float c0 = c_s[g], c1 = c_s[g1];
                float4 r0 = make_float4(acc[r][0].x * c0, acc[r][0].y * c0, acc[r][0].z * c0, acc[r][0].w * c0);
                float4 r1 = make_float4(acc[r][1].x * c1, acc[r][1].y * c1, acc[r][1].z * c1, acc[r][1].w * c1);
#pragma unroll 4
                for (int jj = vh; jj < nt; jj += 2) {
                    const float4 vv = Tile::get4(v_t, jj * HD + 4 * vc4);
                    const float pa = p0[jj], pb = p1[jj];
                    r0.x = fmaf(pa, vv.x, r0.x);
                    r0.y = fmaf(pa, vv.y, r0.y);
                    r0.z = fmaf(pa, vv.z, r0.z);
                    r0.w = fmaf(pa, vv.w, r0.w);
                    r1.x = fmaf(pb, vv.x, r1.x);
                    r1.y = fmaf(pb, vv.y, r1.y);
                    r1.z = fmaf(pb, vv.z, r1.z);
                    r1.w = fmaf(pb, vv.w, r1.w);
                }
                acc[r][0] = r0;
                acc[r][1] = r1;
            }
        }
        __syncthreads();
        if constexpr (kAsync) {  // the V tile is free: the next tile's values land during its scores
            if (t0 + kAttnTile < j1) copy_rows(v_t, HD, a.value_cache, t0 + kAttnTile);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
    }
    if constexpr (kAsync) asm volatile("cp.async.wait_group 0;" ::: "memory");  // (only empty groups remain)
    // the odd-key sums pass through shared memory (the V tile is free) to the even-key threads
    float4 *odd = reinterpret_cast<float4 *>(v_t);  // [G][Q4] (G HD floats fit in the V tile)
    if (vh == 1) {
#pragma unroll
        for (int r = 0; r < VR; ++r) {
            const int g = 2 * (vgp + GPR * r);
            if (g < G) odd[g * Q4 + vc4] = acc[r][0];
            if (g + 1 < G) odd[(g + 1) * Q4 + vc4] = acc[r][1];
        }
    }
    __syncthreads();
    const size_t pbase = (((size_t)tok * a.n_heads + (size_t)kh * G) * a.splits + split);
    if (vh == 0) {
#pragma unroll
        for (int r = 0; r < VR; ++r) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int g = 2 * (vgp + GPR * r) + e;
                if (g < G) {
                    const float4 o = odd[g * Q4 + vc4];
                    const float4 t = make_float4(acc[r][e].x + o.x, acc[r][e].y + o.y, acc[r][e].z + o.z,
                                                 acc[r][e].w + o.w);
                    *reinterpret_cast<float4 *>(a.part_acc + (pbase + (size_t)g * a.splits) * HD + 4 * vc4) = t;
                }
            }
        }
    }
    if (tid < G) {
        a.part_ml[(pbase + (size_t)tid * a.splits) * 2] = m_s[tid];
        a.part_ml[(pbase + (size_t)tid * a.splits) * 2 + 1] = l_s[tid];
    }
}

// out[tok][h] = (sum_s w_s acc_s) / (sum_s w_s l_s) * sigmoid(gate), w_s = exp(m_s - max_s m_s) for
// the splits that saw keys; the weights are computed once per head into shared memory.
__global__ void attn_combine_kernel(const __grid_constant__ AttnArgs a) {
    __shared__ float w_s[kAttnMaxSplits];
    __shared__ float inv_l;
    const int h = blockIdx.x, tok = blockIdx.y, hd = a.head_dim;
    const size_t pbase = ((size_t)tok * a.n_heads + h) * a.splits;
    const size_t o = ((size_t)tok * a.n_heads + h) * hd;
    const bool vec = hd % 4 == 0 && hd <= 4 * kAttnThreads;
    // The gate does not come from the split kernel: its sigmoid is taken before waiting for that
    // kernel (this launch may start while the split kernel runs; the wait covers its stores).
    float sg[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec && threadIdx.x < hd / 4)
        for (int e = 0; e < 4; ++e) sg[e] = 1.0f / (1.0f + expf(-a.gate[o + 4 * threadIdx.x + e]));
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // vector path: thread = (4 dims, split group); eight partials' loads per batch, the first batch in
    // flight while warp 0 computes the split weights
    constexpr int kBatch = 8;
    const int q4 = vec ? hd / 4 : 1, ng = kAttnThreads / q4;
    const int c4 = threadIdx.x % q4, grp = threadIdx.x / q4;
    float4 v[kBatch];
    auto load_batch = [&](int s0) {
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int s = s0 + u * ng;
            v[u] = s < a.splits ? *reinterpret_cast<const float4 *>(a.part_acc + (pbase + s) * hd + 4 * c4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    if (vec && grp < ng) load_batch(grp);
    if (threadIdx.x < 32) {
        // each lane's (max, sum) pairs loaded once, all in flight
        constexpr int kPer = kAttnMaxSplits / 32;
        const int lane = threadIdx.x;
        float2 ml[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int s = lane + 32 * u;
            ml[u] = s < a.splits ? reinterpret_cast<const float2 *>(a.part_ml)[pbase + s] : make_float2(-INFINITY, 0.f);
        }
        float m = -INFINITY;
#pragma unroll
        for (int u = 0; u < kPer; ++u)
            if (ml[u].y > 0.f) m = fmaxf(m, ml[u].x);
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.f;
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int s = lane + 32 * u;
            if (s < a.splits) {
                const float w = ml[u].y > 0.f ? expf(ml[u].x - m) : 0.f;
                w_s[s] = w;
                l += w * ml[u].y;
            }
        }
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) inv_l = 1.0f / l;
    }
    __syncthreads();
    if (vec) {
        // split groups summed through shared memory in a fixed order
        __shared__ float4 red[kAttnThreads];
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (grp < ng)
            for (int s0 = grp; s0 < a.splits; s0 += kBatch * ng) {
                if (s0 != grp) load_batch(s0);
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    const int s = s0 + u * ng;
                    if (s < a.splits) {
                        const float w = w_s[s];
                        acc.x = fmaf(v[u].x, w, acc.x);
                        acc.y = fmaf(v[u].y, w, acc.y);
                        acc.z = fmaf(v[u].z, w, acc.z);
                        acc.w = fmaf(v[u].w, w, acc.w);
                    }
                }
            }
        red[threadIdx.x] = acc;
        __syncthreads();
        if (threadIdx.x < q4) {
            float4 t = red[threadIdx.x];
            for (int g2 = 1; g2 < ng; ++g2) {
                const float4 u = red[g2 * q4 + threadIdx.x];
                t.x += u.x;
                t.y += u.y;
                t.z += u.z;
                t.w += u.w;
            }
            const float r[4] = {t.x, t.y, t.z, t.w};
            for (int e = 0; e < 4; ++e) a.attn[o + 4 * threadIdx.x + e] = r[e] * inv_l * sg[e];
        }
        return;
    }
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.f;
        for (int s = 0; s < a.splits; ++s) acc = fmaf(a.part_acc[(pbase + s) * hd + d], w_s[s], acc);
        const float g = a.gate[o + d];
        a.attn[o + d] = acc * inv_l * (1.0f / (1.0f + expf(-g)));
    }
}

template <typename KvT, int HD, int MG>
cudaError_t attn_hd_launch_g(const AttnArgs &a, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(attn_split_hd_kernel<KvT, HD, MG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attn_split_hd_kernel<KvT, HD, MG><<<dim3(a.splits, a.kv_heads, a.tokens), kAttnThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <typename KvT, int HD>
cudaError_t attn_hd_launch(const AttnArgs &a, cudaStream_t s) {
    const int G = a.n_heads / a.kv_heads;
    using TileT = AttnTileT<KvT, HD>;
    const size_t smem = sizeof(float) * ((size_t)G * HD + (size_t)G * kAttnTile + 3 * (size_t)G) +
                        sizeof(TileT) * ((size_t)kAttnTile * AttnTile<TileT, HD>::kPitch + (size_t)kAttnTile * HD);
    return G <= 8 ? attn_hd_launch_g<KvT, HD, 8>(a, smem, s) : attn_hd_launch_g<KvT, HD, kAttnMaxGroup>(a, smem, s);
}

template <typename KvT>
cudaError_t attn_launch_t(const AttnArgs &a, cudaStream_t s) {
    cudaError_t e;
    const bool vec = reinterpret_cast<uintptr_t>(a.key_cache) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(a.value_cache) % 16 == 0 && reinterpret_cast<uintptr_t>(a.q) % 16 == 0 &&
                     a.n_heads / a.kv_heads <= kAttnMaxGroup;
    if (vec && a.head_dim == 128) {
        e = attn_hd_launch<KvT, 128>(a, s);
    } else if (vec && a.head_dim == 64) {
        e = attn_hd_launch<KvT, 64>(a, s);
    } else if (vec && a.head_dim == 256) {
        e = attn_hd_launch<KvT, 256>(a, s);
    } else {
        const size_t smem = attn_smem_bytes(a.n_heads / a.kv_heads, a.head_dim);
        e = cudaFuncSetAttribute(attn_split_kernel<KvT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attn_split_kernel<KvT><<<dim3(a.splits, a.kv_heads, a.tokens), kAttnThreads, smem, s>>>(a);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
    // the merge is a programmatic dependent launch: its CTAs are placed while the split kernel runs
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.n_heads, a.tokens);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_combine_kernel, a);
}
}  // namespace

// Shared memory of the general kernel (the larger of the two layouts).
size_t attn_smem_bytes(int group, int head_dim) {
    return sizeof(float) * ((size_t)2 * group * head_dim + (size_t)kAttnTile * (head_dim + 4) +
                            (size_t)kAttnTile * head_dim + (size_t)group * kAttnTile + 3 * (size_t)group);
}
int attn_tile() { return kAttnTile; }
int attn_ctas_per_sm(int head_dim) {
    return head_dim == 64 || head_dim == 128 || head_dim == 256 ? attn_hd_ctas_per_sm(head_dim) : 2;
}
int attn_max_splits() { return kAttnMaxSplits; }

cudaError_t attn_launch(const AttnArgs &a, bool kv_bf16, cudaStream_t s) {
    return kv_bf16 ? attn_launch_t<__nv_bfloat16>(a, s) : attn_launch_t<float>(a, s);
}

}  // namespace ql
