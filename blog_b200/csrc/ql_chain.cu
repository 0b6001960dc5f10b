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
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/qlinear_b200.h"
#include "ql_gemv_impl.cuh"

namespace ql {
int set_last_error(int code, const char *msg);

namespace {

constexpr int kChainSlots = 2;                       // ring slots of two 32 x 7-block boxes each
constexpr int kBox = kTmaSeg * 144 * kRowGroup;      // 32,256 B
constexpr int kSlotBytes = 2 * kBox;
constexpr int kChainW = gemv_consumer_warps(true);   // 14 consumer warps
constexpr int kChainRed = kChainW * 2 * kRowGroup;   // floats per reduction buffer (up to 2 matrices)
constexpr int kErrChainBarrier = 5;

enum ChainKind : int { kOpStore = 0, kOpAdd = 1, kOpSwiglu = 2 };

struct __align__(128) ChainOp {
    CUtensorMap tmap[3];   // Q4_K sources {144, blocks, rows}, box {144, 7, 32}
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
};

struct ChainArgs {
    const ChainOp *ops;
    int nops;
    int kmax;
    unsigned *done;     // [nops] arrival counters, monotonic
    unsigned *epoch;    // completed launches
    float *part;        // stream-K partial slots [C][2][2][32]
    unsigned *counters; // stream-K arrival counters (zero between ops)
    int *err;
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tensormap_acquire(const void *map) {
    asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(map) : "memory");
}

__global__ void __launch_bounds__(kGemvThreads, 1) gemv_chain_kernel(const __grid_constant__ ChainArgs a) {
    constexpr int EW = 1, CW0 = 2, W = kChainW;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);   // [kChainSlots]
    uint64_t *empty = full + kChainSlots;                   // [kChainSlots]
    uint64_t *red_full = empty + kChainSlots;               // [2]
    uint64_t *red_empty = red_full + 2;                     // [2]
    int *abort_flag = reinterpret_cast<int *>(red_empty + 2);
    unsigned *epoch_s = reinterpret_cast<unsigned *>(abort_flag + 1);
    float *inv_rms = reinterpret_cast<float *>(smem + 112);
    float *ss_part = reinterpret_cast<float *>(smem + 128);  // [W]
    size_t off = kGemvHeaderBytes;
    float *xs = reinterpret_cast<float *>(smem + off);
    off += ((size_t)a.kmax * 4 + 127) / 128 * 128;
    float *xsum = reinterpret_cast<float *>(smem + off);
    off += ((size_t)(a.kmax / 32) * 4 + 127) / 128 * 128;
    float *red = reinterpret_cast<float *>(smem + off);  // [2][W][2][32]
    off += ((size_t)2 * kChainRed * 4 + 127) / 128 * 128;
    off = (off + 1023) / 1024 * 1024;
    uint8_t *ring = smem + off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = gridDim.x, cta = blockIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kChainSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&red_full[b], W);
            mbar_init(&red_empty[b], 1);
        }
        *abort_flag = 0;
        *epoch_s = *reinterpret_cast<volatile unsigned *>(a.epoch);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const unsigned target = (*epoch_s + 1u) * (unsigned)C;  // every op's counter after this launch

    if (warp == 0) {
        // ---------------------------- producer (TMA) ----------------------------
        if (lane != 0) return;
        int it = 0;
        for (int p = 0; p < a.nops; ++p) {
            const ChainOp &o = a.ops[p];
            for (int i = 0; i < (o.nmat == 2 ? 2 : 3); ++i) tensormap_acquire(&o.tmap[i]);
            const int seg = 2 * kTmaSeg / o.nmat;
            int64_t t = cta < o.plan.C ? plan_start(o.plan, cta) : 0;
            const int64_t t1 = cta < o.plan.C ? plan_start(o.plan, cta + 1) : 0;
            Stage st;
            while (next_stage(t, t1, o.U, seg, 0, st)) {
                const int slot = it % kChainSlots;
                if (it >= kChainSlots && !*reinterpret_cast<volatile int *>(abort_flag)) {
                    if (!mbar_wait(&empty[slot], ((uint32_t)(it / kChainSlots) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                        *abort_flag = 1;
                }
                const bool live = !*reinterpret_cast<volatile int *>(abort_flag);
                uint8_t *sb = ring + (size_t)slot * kSlotBytes;
                const int row0 = st.g * kRowGroup;
                if (o.nmat == 2) {
                    mbar_arrive_expect_tx(&full[slot], live ? 2u * kBox : 0u);
                    if (live) {
                        tma_load_3d(sb, &o.tmap[0], 0, st.us, row0, &full[slot]);
                        tma_load_3d(sb + kBox, &o.tmap[1], 0, st.us, row0, &full[slot]);
                    }
                } else {
                    const int src = (row0 >= o.split[0]) + (row0 >= o.split[1]);
                    const int lrow = row0 - (src == 0 ? 0 : o.split[src - 1]);
                    const int nbox = st.ue - st.us > kTmaSeg ? 2 : 1;
                    mbar_arrive_expect_tx(&full[slot], live ? (uint32_t)(nbox * kBox) : 0u);
                    if (live) {
                        tma_load_3d(sb, &o.tmap[src], 0, st.us, lrow, &full[slot]);
                        if (nbox == 2) tma_load_3d(sb + kBox, &o.tmap[src], 0, st.us + kTmaSeg, lrow, &full[slot]);
                    }
                }
                ++it;
            }
        }
        for (int j = (it > kChainSlots ? it - kChainSlots : 0); j < it; ++j)
            mbar_wait(&full[j % kChainSlots], (uint32_t)(j / kChainSlots) & 1u, nullptr, 0);
        return;
    }

    if (warp == EW) {
        // ------------------------------ finisher ------------------------------
        int gi = 0;
        for (int p = 0; p < a.nops; ++p) {
            const ChainOp &o = a.ops[p];
            const int NM = o.nmat, U = o.U;
            const int64_t t0 = cta < o.plan.C ? plan_start(o.plan, cta) : 0;
            const int64_t t1 = cta < o.plan.C ? plan_start(o.plan, cta + 1) : 0;
            for (int64_t gg = t0 / U; gg * U < t1; ++gg, ++gi) {
                const int g = (int)gg;
                const int bsel = gi & 1;
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
                const int v = g * kRowGroup + lane;
                if (finish) {
                    const float nrm = o.gamma != nullptr ? inv_rms[0] : 1.0f;
                    float out = 0.f;
                    if (v < o.rows) {
                        float *yp = o.y + v;
                        if (o.kind == kOpSwiglu) {
                            const float gv = val[0] * nrm, uv = val[1] * nrm;
                            out = gv / (1.0f + expf(-gv)) * uv;
                            *yp = out;
                        } else {
                            out = val[0] * nrm;
                            if (o.bias != nullptr) out += o.bias[v];
                            if (o.kind == kOpAdd) __stcg(yp, __ldcg(yp) + out);  // residual written by other SMs
                            else if (o.y != nullptr) *yp = out;
                        }
                    }
                    if (o.kind == kOpStore && o.amax.amax != nullptr) {
                        unsigned long long k = v < o.rows ? amax_key(out, (uint32_t)(v + o.amax.offset)) : 0ull;
                        k = warp_max_u64(k);
                        if (lane == 0 && k != 0ull) atomicMax(&o.amax.amax[0], k);
                    }
                }
            }
            if (lane == 0) {
                if (o.kind == kOpStore && o.amax.amax != nullptr) amax_cta_done(o.amax, 1);
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
    int it = 0, gi = 0, ucount = 0;
    for (int p = 0; p < a.nops; ++p) {
        const ChainOp &o = a.ops[p];
        const int K = o.K, nblk = K / 32, U = o.U, NM = o.nmat;
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
            named_bar_sync(1, nthr);
        }
        // prologue: stage x * g * 2^(96-p) and the block sums of x * g; sum x^2 for a fused RMSNorm
        float ss = 0.f;
        {
            const int nch = K / 4;
            constexpr int B = 12;
            for (int j0 = ctid; j0 - lane < nch; j0 += B * nthr) {
                float4 vv[B], gg[B];
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int j = j0 + u * nthr;
                    // L2 only: another SM wrote x during the previous op, after this SM may have cached it
                    vv[u] = j < nch ? __ldcg(reinterpret_cast<const float4 *>(o.x) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                    gg[u] = (j < nch && o.gamma != nullptr) ? reinterpret_cast<const float4 *>(o.gamma)[j]
                                                            : make_float4(1.f, 1.f, 1.f, 1.f);
                }
#pragma unroll
                for (int u = 0; u < B; ++u) {
                    const int j = j0 + u * nthr;
                    const bool ok = j < nch;
                    const int k = ok ? 4 * j : 0;
                    float4 xv = vv[u];
                    if (ok && o.gamma != nullptr) {
                        ss += fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, fmaf(xv.z, xv.z, xv.w * xv.w)));
                        const float4 g = gg[u];
                        xv.x *= g.x; xv.y *= g.y; xv.z *= g.z; xv.w *= g.w;
                    }
                    float bs = (xv.x + xv.y) + (xv.z + xv.w);
                    bs += __shfl_xor_sync(0xffffffffu, bs, 1);
                    bs += __shfl_xor_sync(0xffffffffu, bs, 2);
                    bs += __shfl_xor_sync(0xffffffffu, bs, 4);
                    if (ok) {
                        float4 q;
                        q.x = xv.x * pow2_dev(96 - weight_bitpos<kQ4_K>(k + 0));
                        q.y = xv.y * pow2_dev(96 - weight_bitpos<kQ4_K>(k + 1));
                        q.z = xv.z * pow2_dev(96 - weight_bitpos<kQ4_K>(k + 2));
                        q.w = xv.w * pow2_dev(96 - weight_bitpos<kQ4_K>(k + 3));
                        *reinterpret_cast<float4 *>(xs + k) = q;
                        if ((k & 31) == 0) xsum[k >> 5] = bs;
                    }
                }
            }
        }
        if (o.gamma != nullptr) {
            const float wsum = warp_sum(ss);
            if (lane == 0) ss_part[cw] = wsum;
        }
        named_bar_sync(1, nthr);
        if (o.gamma != nullptr && cw == 0) {
            const float tsum = warp_sum(lane < W ? ss_part[lane] : 0.f);
            if (lane == 0) inv_rms[0] = rsqrtf(tsum / (float)K + o.eps);
        }

        float acc[2][1] = {{0.f}, {0.f}};
        const int seg = 2 * kTmaSeg / NM;
        int64_t t = cta < o.plan.C ? plan_start(o.plan, cta) : 0;
        const int64_t t1 = cta < o.plan.C ? plan_start(o.plan, cta + 1) : 0;
        Stage st;
        while (next_stage(t, t1, U, seg, 0, st)) {
            const int slot = it % kChainSlots;
            const uint32_t ph = (uint32_t)(it / kChainSlots) & 1u;
            if (!*reinterpret_cast<volatile int *>(abort_flag)) {
                if (!mbar_wait(&full[slot], ph, a.err, kErrWaitFull)) *abort_flag = 1;
            }
            const int n = st.ue - st.us;
            const int v = st.g * kRowGroup + lane;
            const bool aborted = *reinterpret_cast<volatile int *>(abort_flag) != 0;
            if (!aborted && v < o.rows) {
                const uint8_t *sb = ring + (size_t)slot * kSlotBytes + (size_t)lane * (kTmaSeg * 144);
                const int first = ((cw - ucount) % W + W) % W;
                for (int lu = first; lu < n; lu += W) {
                    const int k0 = (st.us + lu) * 256;
                    if (NM == 2) {
                        const uint8_t *bp[2] = {sb + lu * 144, sb + kBox + lu * 144};
                        float acc2[2][1] = {{acc[0][0]}, {acc[1][0]}};
                        unit_q4k<1, 2>(bp, xs, K, xsum, nblk, k0, acc2);
                        acc[0][0] = acc2[0][0];
                        acc[1][0] = acc2[1][0];
                    } else {
                        const uint8_t *bp[1] = {sb + (lu / kTmaSeg) * kBox + (lu % kTmaSeg) * 144};
                        float acc1[1][1] = {{acc[0][0]}};
                        unit_q4k<1, 1>(bp, xs, K, xsum, nblk, k0, acc1);
                        acc[0][0] = acc1[0][0];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ucount += n;
            ++it;
            if (st.last_in_group) {
                const int bsel = gi & 1;
                if (gi >= 2 && !*reinterpret_cast<volatile int *>(abort_flag)) {
                    if (!mbar_wait(&red_empty[bsel], ((uint32_t)(gi >> 1) & 1u) ^ 1u, a.err, kErrWaitEmpty))
                        *abort_flag = 1;
                }
                float *rb = red + bsel * kChainRed;
                rb[(cw * 2 + 0) * kRowGroup + lane] = acc[0][0];
                rb[(cw * 2 + 1) * kRowGroup + lane] = acc[1][0];
                acc[0][0] = acc[1][0] = 0.f;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_full[bsel]);
                ++gi;
            }
        }
    }
}

}  // namespace
}  // namespace ql

using namespace ql;

namespace ql {
bool q4k_tensor_map_public(CUtensorMap *out, const uint8_t *base, int blocks, uint64_t rows, size_t row_bytes);
int chain_workspace(float **part, unsigned **counters, int **err, int *sms);
}

namespace {
// Reductions of at most this many blocks run one row group per CTA (QL_CHAIN_ONEGROUP overrides, for tuning).
int chain_max_units_one_group() {
    static const int v = [] {
        const char *e = getenv("QL_CHAIN_ONEGROUP");
        return e ? atoi(e) : 80;  // includes the down projection (74 blocks): measured faster than stream-K there
    }();
    return v;
}

struct Chain {
    ChainOp *ops_dev = nullptr;
    unsigned long long *keys = nullptr;  // [nops] fused-argmax keys
    unsigned *done = nullptr;   // [nops] arrival counters, [nops] epoch, [nops+1 ..] argmax arrival counters
    unsigned *epoch = nullptr;
    ChainArgs args{};
    int smem = 0;
    int sms = 0;
};
}  // namespace

extern "C" {

int ql_gemv_chain_create(const ql_chain_op *ops, int nops, void **chain) {
    if (!ops || nops <= 0 || !chain) return set_last_error(QL_EINVAL, "ql_gemv_chain_create: need ops and nops > 0");
    float *part;
    unsigned *counters;
    int *err, sms;
    int st = chain_workspace(&part, &counters, &err, &sms);
    if (st) return st;
    std::vector<ChainOp> h(nops);
    int kmax = 0;
    for (int p = 0; p < nops; ++p) {
        const ql_chain_op &q = ops[p];
        ChainOp &o = h[p];
        memset(&o, 0, sizeof(o));
        const std::string what = "ql_gemv_chain_create: op " + std::to_string(p);
        if (q.quant_type != QL_Q4_K) return set_last_error(QL_EINVAL, (what + ": only Q4_K").c_str());
        if (q.kind < QL_OP_STORE || q.kind > QL_OP_SWIGLU) return set_last_error(QL_EINVAL, (what + ": kind").c_str());
        const int nsrc = q.kind == QL_OP_SWIGLU ? 2 : q.nsrc;
        if (nsrc < 1 || nsrc > 3 || q.in_dim <= 0 || q.in_dim % 256 || !q.x || (!q.y && !q.argmax_idx))
            return set_last_error(QL_EINVAL, (what + ": sources, in_dim (a multiple of 256), x or y").c_str());
        if (reinterpret_cast<uintptr_t>(q.x) % 16 || reinterpret_cast<uintptr_t>(q.gamma) % 16)
            return set_last_error(QL_EINVAL, (what + ": x and gamma must be 16-byte aligned").c_str());
        const int blocks = q.in_dim / 256;
        if (blocks < kTmaSeg) return set_last_error(QL_EINVAL, (what + ": in_dim must be >= 1792").c_str());
        int total = 0;
        for (int s = 0; s < nsrc; ++s) {
            if (!q.w[s] || reinterpret_cast<uintptr_t>(q.w[s]) % 16 || q.row_bytes[s] % 16 ||
                q.row_bytes[s] < (size_t)blocks * 144 || q.rows[s] < kRowGroup)
                return set_last_error(QL_EINVAL, (what + ": weights (16-byte aligned, >= 32 rows)").c_str());
            if (q.kind != QL_OP_SWIGLU && s < nsrc - 1 && q.rows[s] % kRowGroup)
                return set_last_error(QL_EINVAL, (what + ": stacked sources but the last need multiples of 32 rows").c_str());
            if (!q4k_tensor_map_public(&o.tmap[s], q.w[s], blocks, (uint64_t)q.rows[s], q.row_bytes[s]))
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
        o.kind = q.kind == QL_OP_STORE ? kOpStore : q.kind == QL_OP_ADD ? kOpAdd : kOpSwiglu;
        o.nmat = q.kind == QL_OP_SWIGLU ? 2 : 1;
        o.rows = total;
        o.K = q.in_dim;
        o.U = blocks;
        const int G = (total + kRowGroup - 1) / kRowGroup;
        // like the per-op launcher: short reductions with at most one wave of row groups take one
        // group per CTA (no stream-K fix-ups, whose latency would sit on the chain's critical path)
        const int copt = (G <= sms && blocks <= chain_max_units_one_group()) ? G : sms;
        o.plan = Plan{(int64_t)G * blocks, G, blocks, copt};
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
    Chain *c = new Chain();
    c->sms = sms;
    cudaError_t e = cudaMalloc(&c->ops_dev, sizeof(ChainOp) * nops);
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
        delete c;
        return set_last_error(QL_ECUDA, (std::string("ql_gemv_chain_create: ") + cudaGetErrorString(e)).c_str());
    }
    size_t off = kGemvHeaderBytes;
    off += ((size_t)kmax * 4 + 127) / 128 * 128;
    off += ((size_t)(kmax / 32) * 4 + 127) / 128 * 128;
    off += ((size_t)2 * kChainRed * 4 + 127) / 128 * 128;
    off = (off + 1023) / 1024 * 1024;
    off += (size_t)kChainSlots * kSlotBytes;
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
    *chain = c;
    return QL_OK;
}

int ql_gemv_chain_run(void *chain) {
    Chain *c = static_cast<Chain *>(chain);
    if (!c) return set_last_error(QL_EINVAL, "ql_gemv_chain_run: null chain");
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
        attr_set = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(c->sms);
    cfg.blockDim = dim3(kGemvThreads);
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
    cudaDeviceSynchronize();
    if (c->ops_dev) cudaFree(c->ops_dev);
    if (c->done) cudaFree(c->done);
    if (c->keys) cudaFree(c->keys);
    delete c;
    return QL_OK;
}

}  // extern "C"
