// ql_capi.cu -- the C ABI of libqlinear_b200.so (declared in include/qlinear_b200.h).
//
// Host-side mirror of the reference's launch layer (src/backend/cuda/ops/launch.cu):
// dtype dispatch, grid sizing and the process-global current stream, plus what
// the reference lacks: argument validation with status codes, a per-device
// workspace allocated once (never inside a launch, so launches can be captured
// into CUDA graphs), and a device error word for bounded waits that expired.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "../../include/qlinear_b200.h"
#include "ql_common.cuh"
#include "ql_gemm.cuh"
#include "ql_gemv.cuh"
#include "ql_moe.cuh"
#include "ql_attn.cuh"
#include "ql_q81.cuh"

namespace ql {
cudaError_t gemv_launch(int fmt, int kind, const GemvArgs &a, int MT, bool tma, int smem, cudaStream_t s);
cudaError_t dequant_f16_launch(int t, const uint8_t *src, uint16_t *out, int64_t n, cudaStream_t s);
cudaError_t embedding_launch(int t, const int *ids, float *out, const uint8_t *table, size_t rb, int hidden, int n,
                             cudaStream_t s);
cudaError_t argmax_launch(const float *x, int n, int *out, float *pv, int *pi, int max_parts, cudaStream_t s);
cudaError_t router_launch(const float *logits, int *idx, float *w, int tokens, int E, int k, float scale,
                          cudaStream_t s);
cudaError_t rmsnorm_launch(const float *x, float *y, const float *gamma, int rows, int H, float eps,
                           cudaStream_t s);
cudaError_t synth_launch(int t, uint64_t seed, int64_t rows, int K, float std, uint8_t *dst, cudaStream_t s);

// Programmatic dependent launch for the GEMV / GEMM kernels: a launch may start
// streaming its weights while the previous kernel drains (always on).
bool gemv_pdl_enabled() { return true; }

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxGroups = 1 << 16;   // row groups per launch: out_dim <= 2,097,152
constexpr int kArgmaxParts = 1024;
constexpr int kMaxArgmaxRows = 4096;  // tokens per fused LM-head argmax launch

struct Workspace {
    bool ready = false;
    int sms = 0;
    int max_ctas = 0;
    float *part = nullptr;       // [max_ctas][2][kGemvMaxTokens][2][32]
    unsigned *counters = nullptr;
    int *err = nullptr;
    float *am_v = nullptr;
    int *am_i = nullptr;
    unsigned long long *amax = nullptr;  // [kMaxArgmaxRows] fused-argmax keys, zero between launches
    unsigned *amax_done = nullptr;       // fused-argmax CTA arrival counter
    // tensor-core prefill scratch, grown on demand (ql_reserve_prefill)
    __half *xh = nullptr;
    size_t xh_cap = 0;
    float *rinv = nullptr;
    size_t rinv_cap = 0;
    // grouped routed experts: per-(token, route) down rows and local expert ids, grown on demand
    float *moe_y = nullptr;
    size_t moe_y_cap = 0;
    int *moe_ids = nullptr;
    size_t moe_ids_cap = 0;
    float *moe_bsum = nullptr;
    size_t moe_bsum_cap = 0;
    int *moe_off = nullptr;  // expert buckets of the (token, route) pairs
    size_t moe_off_cap = 0;
    int *moe_list = nullptr;
    size_t moe_list_cap = 0;
    float *attn_part = nullptr;  // decode attention: per-split partials
    size_t attn_part_cap = 0;
};

std::mutex g_mu;
Workspace g_ws[kMaxDevices];
cudaStream_t g_stream = nullptr;
thread_local std::string t_err;
thread_local int t_launches = 0;

int fail(int code, const std::string &msg) {
    t_err = msg;
    return code;
}
int cuda_fail(cudaError_t e, const char *what) {
    return fail(QL_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int init_device(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return fail(QL_EINVAL, "device index out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    Workspace &w = g_ws[dev];
    if (w.ready) return QL_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    w.sms = sms;
    w.max_ctas = 4 * sms;
    const size_t part_floats = (size_t)w.max_ctas * 2 * kGemvMaxTokens * 2 * kRowGroup;
    if ((e = cudaMalloc(&w.part, part_floats * sizeof(float))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.counters, kMaxGroups * sizeof(unsigned))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.err, sizeof(int))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.am_v, kArgmaxParts * sizeof(float))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.am_i, kArgmaxParts * sizeof(int))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.amax, kMaxArgmaxRows * sizeof(unsigned long long))) != cudaSuccess)
        return cuda_fail(e, "workspace");
    if ((e = cudaMalloc(&w.amax_done, sizeof(unsigned))) != cudaSuccess) return cuda_fail(e, "workspace");
    if ((e = cudaMemset(w.amax, 0, kMaxArgmaxRows * sizeof(unsigned long long))) != cudaSuccess)
        return cuda_fail(e, "memset");
    if ((e = cudaMemset(w.amax_done, 0, sizeof(unsigned))) != cudaSuccess) return cuda_fail(e, "memset");
    if ((e = cudaMemset(w.counters, 0, kMaxGroups * sizeof(unsigned))) != cudaSuccess) return cuda_fail(e, "memset");
    if ((e = cudaMemset(w.err, 0, sizeof(int))) != cudaSuccess) return cuda_fail(e, "memset");
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "init sync");
    w.ready = true;
    cudaSetDevice(prev);
    return QL_OK;
}

Workspace *workspace(int *status) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *status = cuda_fail(e, "cudaGetDevice");
        return nullptr;
    }
    if (!g_ws[dev].ready) {
        *status = init_device(dev);
        if (*status != QL_OK) return nullptr;
        cudaSetDevice(dev);
    }
    *status = QL_OK;
    return &g_ws[dev];
}

bool quant_ok(int t) { return t == kQ4_0 || t == kQ5_0 || t == kQ8_0 || t == kQ4_K || t == kQ6_K; }

// Validates a weight operand: dtype, block multiple, row size, alignment the
// decoders rely on (Q4_K reads whole 16-byte lines; the others 2-byte words).
int check_weight(int t, const void *w, size_t row_bytes, size_t expert_bytes, int in_dim, const char *what) {
    if (!quant_ok(t)) return fail(QL_EINVAL, std::string(what) + ": unsupported quant_type " + std::to_string(t));
    const int be = block_elems(t), bb = block_bytes(t);
    if (in_dim <= 0 || in_dim % be != 0)
        return fail(QL_EINVAL, std::string(what) + ": in_dim " + std::to_string(in_dim) +
                                   " is not a positive multiple of the block size " + std::to_string(be));
    if (row_bytes < (size_t)(in_dim / be) * bb)
        return fail(QL_EINVAL, std::string(what) + ": row_bytes smaller than in_dim/block*block_bytes");
    if (w == nullptr) return fail(QL_EINVAL, std::string(what) + ": null weight");
    const size_t align = (t == kQ4_K) ? 16 : 2;
    if (reinterpret_cast<uintptr_t>(w) % align || row_bytes % align || expert_bytes % align)
        return fail(QL_EINVAL, std::string(what) + ": weight, row_bytes and expert_bytes must be multiples of " +
                                   std::to_string(align) + " bytes for this quant_type");
    return QL_OK;
}

// ---- Q4_K tensor maps ----------------------------------------------------------
// A Q4_K matrix is viewed as a 3-D uint8 tensor {144 B of a block, block index,
// row} with strides {144, row_bytes}; the engine loads {144, 7, 32} boxes.  Maps
// are encoded on the host (no device work, so this is safe during stream
// capture) and cached by (base, blocks, rows, row_bytes).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

std::mutex g_map_mu;
std::map<std::tuple<uintptr_t, int, uint64_t, size_t, int>, CUtensorMap> g_maps;

// box_rows = 32 with box_blocks = 7 (GEMV ring) or 256 with 1 (tensor-core GEMM).
bool q4k_tensor_map(CUtensorMap *out, const uint8_t *base, int blocks, uint64_t rows, size_t row_bytes,
                    int box_blocks = kTmaSeg, int box_rows = kRowGroup) {
    const auto key =
        std::make_tuple(reinterpret_cast<uintptr_t>(base), blocks, rows, row_bytes, box_blocks * 1024 + box_rows);
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    CUtensorMap m;
    const cuuint64_t dims[3] = {144, (cuuint64_t)blocks, rows};
    const cuuint64_t strides[2] = {144, (cuuint64_t)row_bytes};
    const cuuint32_t box[3] = {144, (cuuint32_t)box_blocks, (cuuint32_t)box_rows};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

// A 32-element-block matrix (Q4_0 / Q5_0 / Q8_0) as a 2-D tensor {row_bytes / 8, rows} of 8-byte
// elements with boxes {pitch / 8, 32 rows} (the GEMV engine's TMA stage); rows must start on 16 bytes.
// pair: rows a multiple of 8 bytes long, an even row count: each pair of rows is one 16-byte-aligned
// super-row {2 row_bytes / 8, rows / 2} read in boxes of 16 super-rows.
bool small_tensor_map(CUtensorMap *out, const uint8_t *base, uint64_t rows, size_t row_bytes, int fmt, bool pair) {
    if (reinterpret_cast<uintptr_t>(base) % 16 || row_bytes % (pair ? 8 : 16) || (pair && rows % 2)) return false;
    const int bw = tma_pitch(fmt) / 8;
    const auto key = std::make_tuple(reinterpret_cast<uintptr_t>(base), -fmt, rows, row_bytes, bw + (pair ? 1 << 20 : 0));
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return true;
    }
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    CUtensorMap m;
    const uint64_t f = pair ? 2 : 1;
    const cuuint64_t dims[2] = {(cuuint64_t)(f * row_bytes / 8), rows / f};
    const cuuint64_t strides[1] = {(cuuint64_t)(f * row_bytes)};
    const cuuint32_t box[2] = {(cuuint32_t)bw, (cuuint32_t)(kRowGroup / f)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t *>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

// Whether a launch can stage through tensor maps (Q4_K; Q4_0 / Q5_0 / Q8_0 with rows that start on
// 16 bytes), and the maps if so.
// Indexed sources view the packed expert tensor as one tall matrix whose row
// count is not known here, so a generous extent is declared; only rows of
// valid experts are ever requested.
bool prepare_tma(int fmt, int kind, GemvArgs &a) {
    if (!tma_format(fmt)) return false;
    const int NMAT = (kind == 2 || kind == 3) ? 2 : 1;
    // 32-element formats: rows that all start on 16 bytes, or all on 8 bytes (row pairs)
    bool all16 = true;
    for (int m = 0; m < (kind == 5 ? kMaxStacked : NMAT); ++m)
        if (a.w[m] != nullptr && a.row_bytes[m] % 16) all16 = false;
    a.tma_pair = (fmt != kQ4_K && !all16) ? 1 : 0;
    // a stage box no wider than the (super-)row: rows shorter than one stage only as row pairs
    if (a.U < tma_seg(fmt) && !(a.tma_pair && 2 * (size_t)a.U * block_bytes(fmt) >= (size_t)tma_pitch(fmt)))
        return false;
    auto make_map = [&](CUtensorMap *out, const uint8_t *base, int blocks, uint64_t nrows, size_t rb) {
        return fmt == kQ4_K ? q4k_tensor_map(out, base, blocks, nrows, rb)
                            : small_tensor_map(out, base, nrows, rb, fmt, a.tma_pair != 0);
    };
    uint64_t rows = (uint64_t)a.rows;
    if (kind <= 2 || kind == 5) {
        if (a.rows < kRowGroup) return false;
    } else if (kind == 3) {
        if (a.rows_per_route % kRowGroup) return false;
        for (int m = 0; m < NMAT; ++m)
            if (a.expert_bytes[m] != (size_t)a.rows_per_route * a.row_bytes[m]) return false;
        rows = 1ull << 24;
    } else {
        if (a.rows % kRowGroup || a.units_per_route < tma_seg(fmt)) return false;
        if (a.expert_bytes[0] != (size_t)a.rows * a.row_bytes[0]) return false;
        rows = 1ull << 24;
    }
    const int blocks = (kind == 4) ? a.units_per_route : a.U;
    if (kind == 5) {  // stacked sources: one map per source, each with its own row count
        const int starts[3] = {0, a.split[0], a.split[1]};
        const int ends[3] = {a.split[0], a.split[1], a.rows};
        for (int m = 0; m < kMaxStacked; ++m) {
            if (ends[m] <= starts[m]) continue;
            if (ends[m] - starts[m] < kRowGroup) return false;
            if (!make_map(&a.tmap[m], a.w[m], blocks, (uint64_t)(ends[m] - starts[m]), a.row_bytes[m])) return false;
        }
        return true;
    }
    for (int m = 0; m < NMAT; ++m)
        if (!make_map(&a.tmap[m], a.w[m], blocks, rows, a.row_bytes[m])) return false;
    return true;
}

// The engine stages activations (and the fused-norm weight) with 16-byte loads.
int check_act(const float *x, int64_t x_stride, const float *gamma, const char *what) {
    if (reinterpret_cast<uintptr_t>(x) % 16 || x_stride % 4 || reinterpret_cast<uintptr_t>(gamma) % 16)
        return fail(QL_EINVAL, std::string(what) + ": activations (and norm weight) must be 16-byte aligned with a "
                                                   "row stride that is a multiple of 4 floats");
    return QL_OK;
}

// Weight stages a GEMV CTA issues before its activations are staged (the rest
// wait, so the activation loads are not queued behind the weight stream).
int gemv_pre_x() { return 1; }

// Most ring stages a GEMV CTA keeps in flight (2..4).  More stages than needed
// to cover memory latency only lengthen the memory queues every other load waits in.
int gemv_max_stages() { return kGemvStages; }

// Plans and launches the streaming GEMV engine over M tokens (chunks of <= 4).
int run_gemv(int fmt, int kind, GemvArgs base, int M, const char *what) {
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    const int NMAT = (kind == 2 || kind == 3) ? 2 : 1;
    const int BE = block_elems(fmt);
    base.U = base.K / BE;
    base.part = ws->part;
    base.counters = ws->counters;
    base.err = ws->err;
    const int G = (base.rows + kRowGroup - 1) / kRowGroup;
    if (G > kMaxGroups) return fail(QL_EINVAL, std::string(what) + ": out_dim too large");
    if (G == 0 || M == 0) return QL_OK;
    const int64_t T = (int64_t)G * base.U;
    const bool tma = prepare_tma(fmt, kind, base);
    if (!tma) base.tma_pair = 0;
    int done = 0;
    while (done < M) {
        // most tokens per launch (<= 4), then most stages (<= 4, >= 2), that fit 227 KB
        const int mt_cap = NMAT == 2 ? 2 : kGemvMaxTokens;  // two-matrix launches: at most 2 tokens
        int MT = M - done < mt_cap ? M - done : mt_cap;
        GemvShape sh{};
        bool fits = false;
        for (; MT > 0 && !fits; MT -= fits ? 0 : 1)
            for (int nst = gemv_max_stages(); nst >= 2 && !fits; --nst) {
                sh = gemv_shape(fmt, MT, NMAT, base.K, nst, tma);
                fits = sh.smem_bytes <= 227 * 1024;
            }
        if (!fits) return fail(QL_EINVAL, std::string(what) + ": in_dim too large for the shared-memory stage");
        GemvArgs a = base;
        a.M = MT;
        a.nst = sh.nst;
        a.pre_x = gemv_pre_x();
        a.x = base.x + (size_t)done * base.x_stride;
        a.y = base.y ? base.y + (size_t)done * base.y_stride : nullptr;
        if (a.amax.amax != nullptr) {
            a.amax.amax = ws->amax + done;
            a.amax.done = ws->amax_done;
            if (a.amax.idx) a.amax.idx = base.amax.idx + done;
            if (a.amax.key) a.amax.key = base.amax.key + done;
        }
        // Small reductions with at most one wave of row groups: one group per CTA
        // (no stream-K fixups); otherwise equal tile ranges over all SMs.
        int64_t C = (G <= ws->sms && base.U <= 32) ? G : (T < ws->sms ? T : ws->sms);
        if (C > ws->max_ctas) C = ws->max_ctas;
        a.plan = Plan{T, G, base.U, (int)C};
        cudaError_t e = gemv_launch(fmt, kind, a, MT, tma, sh.smem_bytes, g_stream);
        ++t_launches;
        if (e != cudaSuccess) return cuda_fail(e, what);
        done += MT;
    }
    return QL_OK;
}

// ---- tensor-core prefill GEMM ---------------------------------------------------
// Grows the prefill scratch to hold `tokens` x `k` f16 activations and `tokens` row scales.
int ensure_prefill(Workspace *ws, size_t tokens, size_t k) {
    cudaError_t e;
    if (tokens * k > ws->xh_cap) {
        if (ws->xh) cudaFree(ws->xh);
        ws->xh = nullptr;
        ws->xh_cap = 0;
        if ((e = cudaMalloc(&ws->xh, tokens * k * sizeof(__half))) != cudaSuccess) return cuda_fail(e, "prefill scratch");
        ws->xh_cap = tokens * k;
    }
    if (tokens > ws->rinv_cap) {
        if (ws->rinv) cudaFree(ws->rinv);
        ws->rinv = nullptr;
        ws->rinv_cap = 0;
        if ((e = cudaMalloc(&ws->rinv, tokens * sizeof(float))) != cudaSuccess) return cuda_fail(e, "prefill scratch");
        ws->rinv_cap = tokens;
    }
    return QL_OK;
}

// Fewest tokens routed to the tensor-core GEMM by the automatic path selection; below it the
// streaming GEMV engine (<= 4 tokens per weight pass) is faster.  Q8_0 runs only the weights-as-M
// kernel (tiles of 128 tokens, no split-K), which pays off from 32 tokens.
int tc_min_tokens(int t) { return t == kQ8_0 ? 32 : 8; }

// One tensor-core GEMM launch pair: plain (1..3 stacked sources) or SwiGLU (gate, up).
struct TcJob {
    int epi = kGemmPlain;
    int nsrc = 1;
    const uint8_t *w[3] = {nullptr, nullptr, nullptr};
    size_t rb[3] = {0, 0, 0};
    int rows[3] = {0, 0, 0};
    const float *x = nullptr;
    int64_t xs = 0;
    float *y = nullptr;
    int64_t ys = 0;
    int K = 0, M = 0;
    const float *gamma = nullptr;
    float eps = 0.f;
    const float *bias = nullptr;
    int accumulate = 0;
    AmaxOut amax{};  // fused argmax (plain only; amax.amax non-null = on, filled by run_gemm_tc)
};

// Whether the tensor-core GEMM can run the job: Q4_K, Q4_0 or Q8_0 (not with the fused argmax,
// which only the tokens-as-M kernel has), K % 256, row strides that are TMA-legal, and (stacked)
// sources that end on 256-row tile boundaries.
bool tc_eligible(int t, const TcJob &j) {
    if ((t != kQ4_K && t != kQ4_0 && t != kQ8_0) || j.K % 256 != 0) return false;
    if (t == kQ8_0 && j.amax.amax != nullptr) return false;
    for (int i = 0; i < j.nsrc; ++i) {
        if (j.rb[i] % 16 != 0) return false;
        if (j.epi == kGemmPlain && i < j.nsrc - 1 && j.rows[i] % kGemmBN != 0) return false;
    }
    return true;
}

// A Q4_0 matrix as a 2-D byte tensor {row_bytes, rows} with boxes of 144 B (8 blocks = 256
// inputs) x box_rows rows (row_bytes a multiple of 16: in_dim a multiple of 256).
bool q40_tensor_map(CUtensorMap *out, const uint8_t *base, uint64_t rows, size_t row_bytes, int box_rows) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {144, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A Q8_0 matrix as a 2-D tensor of 2-byte elements {row_bytes / 2, rows} with boxes of 136
// elements (272 B = 8 blocks = 256 inputs) x box_rows rows (row_bytes = 272 * in_dim / 256).
bool q80_tensor_map(CUtensorMap *out, const uint8_t *base, uint64_t rows, size_t row_bytes, int box_rows) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 2), rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {136, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int run_gemm_tc(int t, const TcJob &j, const char *what) {
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    const bool swiglu = j.epi == kGemmSwiglu;
    const int BNO = swiglu ? kGemmBN / 2 : kGemmBN;
    int N = 0;
    for (int i = 0; i < (swiglu ? 1 : j.nsrc); ++i) N += j.rows[i];
    if (N == 0 || j.M == 0) return QL_OK;
    const int nsb = j.K / 256;
    const int64_t mt = (j.M + kGemmBM - 1) / kGemmBM, nt = (N + BNO - 1) / BNO, tiles = mt * nt;
    if (mt > 65535 || nt > 65535) return fail(QL_EINVAL, std::string(what) + ": shape too large for the tensor-core grid");
    // Prefill-sized token counts run the weights-as-M kernel (weights dequantized into tensor memory
    // once per 128 or 256 tokens); small batches and the fused argmax keep the tokens-as-M kernel.
    const bool ta = (j.M >= 128 || t == kQ8_0) && j.amax.amax == nullptr;
    const int ntok = ta ? gemm_ta_tokens(j.M, (N + (swiglu ? 63 : 127)) / (swiglu ? 64 : 128), ws->sms) : 0;
    const int box_rows = ta ? (swiglu ? 64 : 128) : BNO;
    // K split over a cluster when the tiles alone would leave SMs idle
    int ks = 1;
    if (!ta && tiles < ws->sms) {
        ks = (int)(ws->sms / tiles);
        if (ks > kGemmMaxSplit) ks = kGemmMaxSplit;
        if (ks > nsb) ks = nsb;
        if (ks < 1) ks = 1;
    }
    if ((st = ensure_prefill(ws, (size_t)j.M, (size_t)j.K))) return st;
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return fail(QL_ECUDA, std::string(what) + ": cuTensorMapEncodeTiled unavailable");
    GemmArgs a;
    memset(&a, 0, sizeof(a));
    int end = 0;
    for (int i = 0; i < 3; ++i) {
        if (i < j.nsrc) {
            const bool okm =
                t == kQ8_0   ? q80_tensor_map(&a.tm_w[i], j.w[i], (uint64_t)j.rows[i], j.rb[i], box_rows)
                : t == kQ4_0 ? q40_tensor_map(&a.tm_w[i], j.w[i], (uint64_t)j.rows[i], j.rb[i], box_rows)
                             : q4k_tensor_map(&a.tm_w[i], j.w[i], nsb, (uint64_t)j.rows[i], j.rb[i], 1, box_rows);
            if (!okm) return fail(QL_ECUDA, std::string(what) + ": weight tensor map");
            end += j.rows[i];
        } else {
            a.tm_w[i] = a.tm_w[j.nsrc - 1];
        }
        a.src_end[i] = swiglu ? N : end;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)j.K, (cuuint64_t)j.M};
        const cuuint64_t strides[1] = {(cuuint64_t)j.K * sizeof(__half)};
        const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)(ta ? ntok : kGemmBM)};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(&a.tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ws->xh, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(QL_ECUDA, std::string(what) + ": activation tensor map");
    }
    a.rinv = ws->rinv;
    a.bias = swiglu ? nullptr : j.bias;
    a.y = j.y;
    a.y_stride = j.ys;
    a.accumulate = swiglu ? 0 : j.accumulate;
    a.vec = (reinterpret_cast<uintptr_t>(j.y) % 16 == 0) && (j.ys % 4 == 0) &&
            (reinterpret_cast<uintptr_t>(a.bias) % 16 == 0);
    a.M = j.M;
    a.N = N;
    a.K = j.K;
    a.nsb = nsb;
    a.fmt = t;
    a.ksplit = ks;
    a.err = ws->err;
    if (!swiglu && j.amax.amax != nullptr) {
        a.amax = j.amax;
        a.amax.amax = ws->amax;
        a.amax.done = ws->amax_done;
    }
    cudaError_t e = gemm_xprep_launch(j.x, j.xs, j.gamma, j.eps, ws->xh, ws->rinv, j.M, j.K, g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    e = ta ? gemm_ta_launch(a, j.epi, ntok, g_stream) : gemm_q4k_launch(a, j.epi, g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    return QL_OK;
}

TcJob plain_job(const uint8_t *w, size_t rb, const float *x, int64_t xs, float *y, int64_t ys, int N, int K, int M,
                const float *gamma, float eps, const float *bias, int accumulate) {
    TcJob j;
    j.w[0] = w;
    j.rb[0] = rb;
    j.rows[0] = N;
    j.x = x;
    j.xs = xs;
    j.y = y;
    j.ys = ys;
    j.K = K;
    j.M = M;
    j.gamma = gamma;
    j.eps = eps;
    j.bias = bias;
    j.accumulate = accumulate;
    return j;
}

GemvArgs blank() {
    GemvArgs a;
    memset(&a, 0, sizeof(a));
    return a;
}

}  // namespace

// Records `msg` as this thread's last error (for entry points in other files).
int set_last_error(int code, const char *msg) { return fail(code, msg); }
// Entry points defined in other files report their kernel launches here (ql_last_launch_count).
void set_launch_count(int n) { t_launches = n; }

// Q4_K tensor map with the GEMV ring's {144, 7, 32} box, for the chain kernel.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder_public() { return tensor_map_encoder(); }

bool q4k_tensor_map_public(CUtensorMap *out, const uint8_t *base, int blocks, uint64_t rows, size_t row_bytes,
                           int box_blocks, int box_rows) {
    return q4k_tensor_map(out, base, blocks, rows, row_bytes, box_blocks, box_rows);
}

// Stream-K scratch, error word and SM count of the current device, for the chain kernel.
int chain_workspace(float **part, unsigned **counters, int **err, int *sms) {
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    *part = ws->part;
    *counters = ws->counters;
    *err = ws->err;
    *sms = ws->sms;
    return QL_OK;
}

// The current device's error word (initialising the workspace if needed), or null.
int *device_error_word() {
    int st;
    Workspace *ws = workspace(&st);
    return ws ? ws->err : nullptr;
}
}  // namespace ql

using namespace ql;

extern "C" {

int ql_set_stream(void *stream) {
    g_stream = static_cast<cudaStream_t>(stream);
    return QL_OK;
}
void *ql_get_stream(void) { return g_stream; }
int ql_init(int device) { return init_device(device); }
const char *ql_last_error(void) { return t_err.c_str(); }
int ql_last_launch_count(void) { return t_launches; }

int ql_check_device(void) {
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    cudaError_t e = cudaStreamSynchronize(g_stream);
    if (e != cudaSuccess) return cuda_fail(e, "stream sync");
    int h = 0;
    if ((e = cudaMemcpy(&h, ws->err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "read error word");
    if (h != 0) {
        cudaMemset(ws->err, 0, sizeof(int));
        cudaMemset(ws->counters, 0, kMaxGroups * sizeof(unsigned));
        cudaMemset(ws->amax, 0, kMaxArgmaxRows * sizeof(unsigned long long));
        cudaMemset(ws->amax_done, 0, sizeof(unsigned));
        cudaDeviceSynchronize();
        return fail(QL_EDEVICE, "a kernel gave up a bounded wait (device error code " + std::to_string(h) + ")");
    }
    return QL_OK;
}

size_t ql_row_bytes(int32_t t, int in_dim) {
    if (!quant_ok(t) || in_dim <= 0 || in_dim % block_elems(t)) return 0;
    return (size_t)(in_dim / block_elems(t)) * block_bytes(t);
}

int ql_quant_gemv_ex(int32_t t, const uint8_t *w, size_t rb, const float *x, int64_t xs, float *y, int64_t ys,
                     int out_dim, int in_dim, int m, const float *gamma, float eps, const float *bias,
                     int accumulate) {
    t_launches = 0;
    if (out_dim < 0 || m < 0) return fail(QL_EINVAL, "ql_quant_gemv: negative size");
    if (out_dim == 0 || m == 0) return QL_OK;
    int st = check_weight(t, w, rb, 0, in_dim, "ql_quant_gemv");
    if (st) return st;
    if (!x || !y) return fail(QL_EINVAL, "ql_quant_gemv: null x or y");
    if ((st = check_act(x, xs, gamma, "ql_quant_gemv"))) return st;
    {
        const TcJob j = plain_job(w, rb, x, xs, y, ys, out_dim, in_dim, m, gamma, eps, bias, accumulate);
        if (m >= tc_min_tokens(t) && tc_eligible(t, j)) return run_gemm_tc(t, j, "ql_quant_gemv");
    }
    GemvArgs a = blank();
    a.w[0] = w;
    a.row_bytes[0] = rb;
    a.rows = out_dim;
    a.K = in_dim;
    a.x = x;
    a.x_stride = xs;
    a.y = y;
    a.y_stride = ys;
    a.gamma = gamma;
    a.eps = eps;
    a.bias = bias;
    return run_gemv(t, accumulate ? 1 : 0, a, m, "ql_quant_gemv");
}

int ql_quant_gemv_argmax_ex(int32_t t, const uint8_t *w, size_t rb, const float *x, int64_t xs, float *logits,
                            int64_t ls, int out_dim, int in_dim, int m, const float *gamma, float eps, int index_offset,
                            int *out_idx, uint64_t *out_key) {
    t_launches = 0;
    if (out_dim <= 0 || m <= 0 || m > kMaxArgmaxRows)
        return fail(QL_EINVAL, "ql_quant_gemv_argmax_ex: need out_dim > 0 and 0 < m <= 4096");
    if (!out_idx && !out_key) return fail(QL_EINVAL, "ql_quant_gemv_argmax_ex: null out_idx and out_key");
    int st = check_weight(t, w, rb, 0, in_dim, "ql_quant_gemv_argmax_ex");
    if (st) return st;
    if (!x) return fail(QL_EINVAL, "ql_quant_gemv_argmax_ex: null x");
    if ((st = check_act(x, xs, gamma, "ql_quant_gemv_argmax_ex"))) return st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    AmaxOut am{};
    am.amax = ws->amax;
    am.done = ws->amax_done;
    am.idx = out_idx;
    am.key = reinterpret_cast<unsigned long long *>(out_key);
    am.offset = index_offset;
    {
        TcJob j = plain_job(w, rb, x, xs, logits, ls, out_dim, in_dim, m, gamma, eps, nullptr, 0);
        j.amax = am;
        if (m >= tc_min_tokens(t) && tc_eligible(t, j)) return run_gemm_tc(t, j, "ql_quant_gemv_argmax_ex");
    }
    GemvArgs a = blank();
    a.w[0] = w;
    a.row_bytes[0] = rb;
    a.rows = out_dim;
    a.K = in_dim;
    a.x = x;
    a.x_stride = xs;
    a.y = logits;
    a.y_stride = ls;
    a.gamma = gamma;
    a.eps = eps;
    a.amax = am;
    return run_gemv(t, 0, a, m, "ql_quant_gemv_argmax_ex");
}

int ql_quant_matmul_ex(int32_t t, const uint8_t *w, size_t rb, const float *x, int64_t xs, float *y, int64_t ys,
                       int out_dim, int in_dim, int m, const float *gamma, float eps, const float *bias, int accumulate,
                       int path) {
    t_launches = 0;
    if (path < QL_PATH_AUTO || path > QL_PATH_TENSOR) return fail(QL_EINVAL, "ql_quant_matmul_ex: unknown path");
    if (out_dim < 0 || m < 0) return fail(QL_EINVAL, "ql_quant_matmul_ex: negative size");
    if (out_dim == 0 || m == 0) return QL_OK;
    int st = check_weight(t, w, rb, 0, in_dim, "ql_quant_matmul_ex");
    if (st) return st;
    if (!x || !y) return fail(QL_EINVAL, "ql_quant_matmul_ex: null x or y");
    if ((st = check_act(x, xs, gamma, "ql_quant_matmul_ex"))) return st;
    const TcJob j = plain_job(w, rb, x, xs, y, ys, out_dim, in_dim, m, gamma, eps, bias, accumulate);
    const bool tc = tc_eligible(t, j);
    if (path == QL_PATH_TENSOR && !tc)
        return fail(QL_EINVAL, "ql_quant_matmul_ex: the tensor-core path needs Q4_K, Q4_0 or Q8_0, in_dim % 256 == 0 "
                               "and row_bytes % 16 == 0");
    if (path == QL_PATH_TENSOR || (path == QL_PATH_AUTO && tc && m >= tc_min_tokens(t)))
        return run_gemm_tc(t, j, "ql_quant_matmul_ex");
    GemvArgs a = blank();
    a.w[0] = w;
    a.row_bytes[0] = rb;
    a.rows = out_dim;
    a.K = in_dim;
    a.x = x;
    a.x_stride = xs;
    a.y = y;
    a.y_stride = ys;
    a.gamma = gamma;
    a.eps = eps;
    a.bias = bias;
    return run_gemv(t, accumulate ? 1 : 0, a, m, "ql_quant_matmul_ex");
}

int ql_reserve_prefill(int max_tokens, int max_in_dim) {
    if (max_tokens < 0 || max_in_dim < 0) return fail(QL_EINVAL, "ql_reserve_prefill: negative size");
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    return ensure_prefill(ws, (size_t)max_tokens, (size_t)max_in_dim);
}

int ql_quant_gemv_stacked_ex(int32_t t, int nsrc, const uint8_t *const *w, const size_t *rb, const int *rows,
                             const float *x, int64_t xs, float *y, int64_t ys, int in_dim, int m, const float *gamma,
                             float eps, const float *bias) {
    t_launches = 0;
    if (nsrc < 1 || nsrc > kMaxStacked || !w || !rb || !rows)
        return fail(QL_EINVAL, "ql_quant_gemv_stacked_ex: need 1..3 sources");
    if (m < 0) return fail(QL_EINVAL, "ql_quant_gemv_stacked_ex: negative size");
    GemvArgs a = blank();
    int total = 0;
    for (int i = 0; i < nsrc; ++i) {
        int st = check_weight(t, w[i], rb[i], 0, in_dim, "ql_quant_gemv_stacked_ex");
        if (st) return st;
        if (rows[i] < 0 || (i < nsrc - 1 && rows[i] % kRowGroup))
            return fail(QL_EINVAL, "ql_quant_gemv_stacked_ex: every source but the last needs a multiple of 32 rows");
        a.w[i] = w[i];
        a.row_bytes[i] = rb[i];
        total += rows[i];
        if (i < 2) a.split[i] = total;
    }
    for (int i = nsrc; i < kMaxStacked; ++i) {
        a.w[i] = w[nsrc - 1];
        a.row_bytes[i] = rb[nsrc - 1];
        if (i < 2 && i >= nsrc) a.split[i] = total;
    }
    if (total == 0 || m == 0) return QL_OK;
    if (!x || !y) return fail(QL_EINVAL, "ql_quant_gemv_stacked_ex: null x or y");
    int st = check_act(x, xs, gamma, "ql_quant_gemv_stacked_ex");
    if (st) return st;
    if (m >= tc_min_tokens(t)) {
        TcJob j = plain_job(w[0], rb[0], x, xs, y, ys, rows[0], in_dim, m, gamma, eps, bias, 0);
        j.nsrc = nsrc;
        for (int i = 1; i < nsrc; ++i) {
            j.w[i] = w[i];
            j.rb[i] = rb[i];
            j.rows[i] = rows[i];
        }
        if (tc_eligible(t, j)) return run_gemm_tc(t, j, "ql_quant_gemv_stacked_ex");
    }
    a.rows = total;
    a.K = in_dim;
    a.x = x;
    a.x_stride = xs;
    a.y = y;
    a.y_stride = ys;
    a.gamma = gamma;
    a.eps = eps;
    a.bias = bias;
    return run_gemv(t, 5, a, m, "ql_quant_gemv_stacked_ex");
}

int ql_quant_gemv(int32_t t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim,
                  int m) {
    return ql_quant_gemv_ex(t, w, rb, x, in_dim, y, out_dim, out_dim, in_dim, m, nullptr, 0.f, nullptr, 0);
}

int ql_quant_gemv_add(int32_t t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim) {
    return ql_quant_gemv_ex(t, w, rb, x, in_dim, y, out_dim, out_dim, in_dim, 1, nullptr, 0.f, nullptr, 1);
}

int ql_quant_matmul(int32_t t, const uint8_t *w, size_t rb, const float *x, float *y, int out_dim, int in_dim,
                    int m) {
    return ql_quant_gemv_ex(t, w, rb, x, in_dim, y, out_dim, out_dim, in_dim, m, nullptr, 0.f, nullptr, 0);
}

int ql_quant_swiglu_ex(int32_t t, const uint8_t *g, const uint8_t *u, size_t grb, size_t urb, const float *x,
                       int64_t xs, float *act, int64_t as, int ffn_dim, int in_dim, int m, const float *gamma,
                       float eps) {
    t_launches = 0;
    if (ffn_dim < 0 || m < 0) return fail(QL_EINVAL, "ql_quant_swiglu: negative size");
    if (ffn_dim == 0 || m == 0) return QL_OK;
    int st = check_weight(t, g, grb, 0, in_dim, "ql_quant_swiglu(gate)");
    if (st) return st;
    if ((st = check_weight(t, u, urb, 0, in_dim, "ql_quant_swiglu(up)"))) return st;
    if (!x || !act) return fail(QL_EINVAL, "ql_quant_swiglu: null x or act");
    if ((st = check_act(x, xs, gamma, "ql_quant_swiglu"))) return st;
    if (m >= tc_min_tokens(t)) {
        TcJob j = plain_job(g, grb, x, xs, act, as, ffn_dim, in_dim, m, gamma, eps, nullptr, 0);
        j.epi = kGemmSwiglu;
        j.nsrc = 2;
        j.w[1] = u;
        j.rb[1] = urb;
        j.rows[1] = ffn_dim;
        if (tc_eligible(t, j)) return run_gemm_tc(t, j, "ql_quant_swiglu");
    }
    GemvArgs a = blank();
    a.w[0] = g;
    a.w[1] = u;
    a.row_bytes[0] = grb;
    a.row_bytes[1] = urb;
    a.rows = ffn_dim;
    a.K = in_dim;
    a.x = x;
    a.x_stride = xs;
    a.y = act;
    a.y_stride = as;
    a.gamma = gamma;
    a.eps = eps;
    return run_gemv(t, 2, a, m, "ql_quant_swiglu");
}

int ql_quant_swiglu(int32_t t, const uint8_t *g, const uint8_t *u, size_t grb, size_t urb, const float *x,
                    float *act, int ffn_dim, int in_dim) {
    return ql_quant_swiglu_ex(t, g, u, grb, urb, x, in_dim, act, ffn_dim, ffn_dim, in_dim, 1, nullptr, 0.f);
}

int ql_quant_swiglu_indexed(int32_t t, const uint8_t *g, const uint8_t *u, size_t geb, size_t ueb, size_t grb,
                            size_t urb, const float *x, const int *ids, float *act, int k, int ffn_dim,
                            int in_dim) {
    t_launches = 0;
    if (k < 0 || ffn_dim < 0) return fail(QL_EINVAL, "ql_quant_swiglu_indexed: negative size");
    if (k == 0 || ffn_dim == 0) return QL_OK;
    int st = check_weight(t, g, grb, geb, in_dim, "ql_quant_swiglu_indexed(gate)");
    if (st) return st;
    if ((st = check_weight(t, u, urb, ueb, in_dim, "ql_quant_swiglu_indexed(up)"))) return st;
    if (!x || !ids || !act) return fail(QL_EINVAL, "ql_quant_swiglu_indexed: null pointer");
    if ((st = check_act(x, in_dim, nullptr, "ql_quant_swiglu_indexed"))) return st;
    GemvArgs a = blank();
    a.w[0] = g;
    a.w[1] = u;
    a.row_bytes[0] = grb;
    a.row_bytes[1] = urb;
    a.expert_bytes[0] = geb;
    a.expert_bytes[1] = ueb;
    a.rows = k * ffn_dim;
    a.rows_per_route = ffn_dim;
    a.K = in_dim;
    a.x = x;
    a.x_stride = in_dim;
    a.ids = ids;
    a.y = act;
    a.y_stride = (int64_t)k * ffn_dim;
    return run_gemv(t, 3, a, 1, "ql_quant_swiglu_indexed");
}

int ql_quant_down_f32_indexed_accum_ordered(int32_t t, const uint8_t *d, size_t deb, size_t drb, const float *act,
                                            const int *ids, const float *rw, float *out, int k, int hidden,
                                            int ffn_dim) {
    t_launches = 0;
    if (k < 0 || hidden < 0) return fail(QL_EINVAL, "ql_quant_down_f32_indexed_accum_ordered: negative size");
    if (k == 0 || hidden == 0) return QL_OK;
    int st = check_weight(t, d, drb, deb, ffn_dim, "ql_quant_down_f32_indexed_accum_ordered");
    if (st) return st;
    if (!act || !ids || !rw || !out) return fail(QL_EINVAL, "ql_quant_down_f32_indexed_accum_ordered: null pointer");
    if ((st = check_act(act, ffn_dim, nullptr, "ql_quant_down_f32_indexed_accum_ordered"))) return st;
    GemvArgs a = blank();
    a.w[0] = d;
    a.row_bytes[0] = drb;
    a.expert_bytes[0] = deb;
    a.rows = hidden;
    a.K = k * ffn_dim;
    a.units_per_route = ffn_dim / block_elems(t);
    a.x = act;
    a.x_stride = ffn_dim;
    a.ids = ids;
    a.route_w = rw;
    a.y = out;
    a.y_stride = hidden;
    return run_gemv(t, 4, a, 1, "ql_quant_down_f32_indexed_accum_ordered");
}

int ql_moe_router_topk(const float *logits, int *idx, float *w, int tokens, int E, int k, float scale) {
    t_launches = 0;
    if (tokens < 0 || E <= 0 || E > 64 || k <= 0 || k > E)
        return fail(QL_EINVAL, "ql_moe_router_topk: need 0 < k <= n_experts <= 64");
    if (tokens == 0) return QL_OK;
    if (!logits || !idx || !w) return fail(QL_EINVAL, "ql_moe_router_topk: null pointer");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = router_launch(logits, idx, w, tokens, E, k, scale, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_moe_router_topk");
}

// ---- grouped routed experts ------------------------------------------------------
namespace {
// Grows a scratch buffer to hold n elements of elem bytes.
int grow(void **buf, size_t *cap, size_t n, size_t elem, const char *what) {
    if (n <= *cap) return QL_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(buf, n * elem);
    if (e != cudaSuccess) return cuda_fail(e, what);
    *cap = n;
    return QL_OK;
}
// Whether the grouped kernel can stage a matrix: 64 rows in shared memory, and a 16-byte-aligned
// base (each row's bulk copy starts at the 16-byte boundary at or before the row).
bool moe_stageable(const uint8_t *w, size_t rb) {
    return reinterpret_cast<uintptr_t>(w) % 16 == 0 && moe_row_pitch(rb) <= moe_max_row_pitch();
}
// Buckets the call's (token, route) pairs by expert (one launch) into the workspace.
int moe_buckets(Workspace *ws, const int *ids, int npairs, int e_begin, int n_experts, MoeArgs &a, const char *what) {
    int st;
    if ((st = grow(reinterpret_cast<void **>(&ws->moe_off), &ws->moe_off_cap, (size_t)n_experts + 2, sizeof(int),
                   what)))
        return st;
    if ((st = grow(reinterpret_cast<void **>(&ws->moe_list), &ws->moe_list_cap, (size_t)npairs, sizeof(int), what)))
        return st;
    cudaError_t e = moe_bucket_launch(ids, npairs, e_begin, n_experts, ws->moe_off, ws->moe_list, g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    a.bucket_off = ws->moe_off;
    a.bucket = ws->moe_list;
    return QL_OK;
}
int moe_check(int t, int tokens, int k, int e_begin, int n_experts, const char *what) {
    if (tokens < 0 || k <= 0 || n_experts <= 0 || e_begin < 0)
        return fail(QL_EINVAL, std::string(what) + ": need tokens >= 0, k > 0, n_experts > 0, expert_begin >= 0");
    if (t != kQ4_0 && t != kQ5_0 && t != kQ8_0 && t != kQ4_K)
        return fail(QL_EINVAL, std::string(what) + ": quant_type must be Q4_0, Q5_0, Q8_0 or Q4_K");
    if ((int64_t)tokens * k > (1 << 30)) return fail(QL_EINVAL, std::string(what) + ": too many routes");
    return QL_OK;
}
}  // namespace

int ql_moe_swiglu_grouped(int32_t t, const uint8_t *g, const uint8_t *u, size_t geb, size_t ueb, size_t grb,
                          size_t urb, const float *x, int64_t xs, const int *ids, int e_begin, int n_experts,
                          float *act, int tokens, int k, int ffn_dim, int in_dim) {
    const char *what = "ql_moe_swiglu_grouped";
    t_launches = 0;
    int st = moe_check(t, tokens, k, e_begin, n_experts, what);
    if (st) return st;
    if (ffn_dim < 0) return fail(QL_EINVAL, std::string(what) + ": negative ffn_dim");
    if (tokens == 0 || ffn_dim == 0) return QL_OK;
    if ((st = check_weight(t, g, grb, geb, in_dim, "ql_moe_swiglu_grouped(gate)"))) return st;
    if ((st = check_weight(t, u, urb, ueb, in_dim, "ql_moe_swiglu_grouped(up)"))) return st;
    if (!x || !ids || !act) return fail(QL_EINVAL, std::string(what) + ": null pointer");
    if ((st = check_act(x, xs, nullptr, what))) return st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    const int npairs = tokens * k;
    if (!moe_stageable(g, grb) || !moe_stageable(u, urb) || n_experts > moe_max_experts()) {
        // rows too long for the grouped kernel's slabs: the per-token indexed launches
        if ((st = grow(reinterpret_cast<void **>(&ws->moe_ids), &ws->moe_ids_cap, (size_t)npairs, sizeof(int), what))) return st;
        cudaError_t e = moe_local_ids_launch(ids, e_begin, n_experts, ws->moe_ids, npairs, g_stream);
        ++t_launches;
        if (e != cudaSuccess) return cuda_fail(e, what);
        for (int tok = 0; tok < tokens; ++tok) {
            GemvArgs a = blank();
            a.w[0] = g;
            a.w[1] = u;
            a.row_bytes[0] = grb;
            a.row_bytes[1] = urb;
            a.expert_bytes[0] = geb;
            a.expert_bytes[1] = ueb;
            a.rows = k * ffn_dim;
            a.rows_per_route = ffn_dim;
            a.K = in_dim;
            a.x = x + (size_t)tok * xs;
            a.x_stride = in_dim;
            a.ids = ws->moe_ids + (size_t)tok * k;
            a.y = act + (size_t)tok * k * ffn_dim;
            a.y_stride = (int64_t)k * ffn_dim;
            if ((st = run_gemv(t, 3, a, 1, what))) return st;  // counts its launches
        }
        return QL_OK;
    }
    if ((st = ensure_prefill(ws, (size_t)tokens, 2 * (size_t)in_dim))) return st;  // two f16 limbs per input
    if ((st = grow(reinterpret_cast<void **>(&ws->moe_bsum), &ws->moe_bsum_cap, (size_t)tokens * (in_dim / 32),
                   sizeof(float), what)))
        return st;
    cudaError_t e = moe_xprep_launch(x, xs, reinterpret_cast<uint4 *>(ws->xh), ws->rinv, ws->moe_bsum, tokens, in_dim,
                                     g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    MoeArgs a{};
    a.w[0] = g;
    a.w[1] = u;
    a.eb[0] = geb;
    a.eb[1] = ueb;
    a.rb[0] = grb;
    a.rb[1] = urb;
    a.row_pitch = moe_row_pitch(grb > urb ? grb : urb);
    a.rows = ffn_dim;
    a.K = in_dim;
    a.xq = reinterpret_cast<const uint4 *>(ws->xh);
    a.rinv = ws->rinv;
    a.bsum = ws->moe_bsum;
    a.ids = ids;
    a.e_begin = e_begin;
    a.n_experts = n_experts;
    a.npairs = npairs;
    a.k = k;
    a.y = act;
    a.y_stride = ffn_dim;
    a.err = ws->err;
    if ((st = moe_buckets(ws, ids, npairs, e_begin, n_experts, a, what))) return st;
    e = moe_grouped_launch(a, t, true, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, what);
}

int ql_moe_down_grouped_accum_ordered(int32_t t, const uint8_t *d, size_t deb, size_t drb, const float *act,
                                      const int *ids, int e_begin, int n_experts, const float *rw, float *out,
                                      int64_t out_stride, int tokens, int k, int hidden, int ffn_dim) {
    const char *what = "ql_moe_down_grouped_accum_ordered";
    t_launches = 0;
    int st = moe_check(t, tokens, k, e_begin, n_experts, what);
    if (st) return st;
    if (hidden < 0) return fail(QL_EINVAL, std::string(what) + ": negative hidden");
    if (tokens == 0 || hidden == 0) return QL_OK;
    if ((st = check_weight(t, d, drb, deb, ffn_dim, what))) return st;
    if (!act || !ids || !rw || !out) return fail(QL_EINVAL, std::string(what) + ": null pointer");
    if ((st = check_act(act, ffn_dim, nullptr, what))) return st;
    if (out_stride < hidden) return fail(QL_EINVAL, std::string(what) + ": out_stride < hidden");
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    const int npairs = tokens * k;
    if (!moe_stageable(d, drb) || n_experts > moe_max_experts()) {
        if ((st = grow(reinterpret_cast<void **>(&ws->moe_ids), &ws->moe_ids_cap, (size_t)npairs, sizeof(int), what))) return st;
        cudaError_t e = moe_local_ids_launch(ids, e_begin, n_experts, ws->moe_ids, npairs, g_stream);
        ++t_launches;
        if (e != cudaSuccess) return cuda_fail(e, what);
        for (int tok = 0; tok < tokens; ++tok) {
            GemvArgs a = blank();
            a.w[0] = d;
            a.row_bytes[0] = drb;
            a.expert_bytes[0] = deb;
            a.rows = hidden;
            a.K = k * ffn_dim;
            a.units_per_route = ffn_dim / block_elems(t);
            a.x = act + (size_t)tok * k * ffn_dim;
            a.x_stride = ffn_dim;
            a.ids = ws->moe_ids + (size_t)tok * k;
            a.route_w = rw + (size_t)tok * k;
            a.y = out + (size_t)tok * out_stride;
            a.y_stride = hidden;
            if ((st = run_gemv(t, 4, a, 1, what))) return st;  // counts its launches
        }
        return QL_OK;
    }
    if ((st = ensure_prefill(ws, (size_t)npairs, 2 * (size_t)ffn_dim))) return st;
    if ((st = grow(reinterpret_cast<void **>(&ws->moe_y), &ws->moe_y_cap, (size_t)npairs * hidden, sizeof(float), what)))
        return st;
    if ((st = grow(reinterpret_cast<void **>(&ws->moe_bsum), &ws->moe_bsum_cap, (size_t)npairs * (ffn_dim / 32),
                   sizeof(float), what)))
        return st;
    cudaError_t e = moe_xprep_launch(act, ffn_dim, reinterpret_cast<uint4 *>(ws->xh), ws->rinv, ws->moe_bsum, npairs,
                                     ffn_dim, g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    MoeArgs a{};
    a.w[0] = a.w[1] = d;
    a.eb[0] = a.eb[1] = deb;
    a.rb[0] = a.rb[1] = drb;
    a.row_pitch = moe_row_pitch(drb);
    a.rows = hidden;
    a.K = ffn_dim;
    a.xq = reinterpret_cast<const uint4 *>(ws->xh);
    a.rinv = ws->rinv;
    a.bsum = ws->moe_bsum;
    a.ids = ids;
    a.e_begin = e_begin;
    a.n_experts = n_experts;
    a.npairs = npairs;
    a.k = k;
    a.y = ws->moe_y;
    a.y_stride = hidden;
    a.err = ws->err;
    if ((st = moe_buckets(ws, ids, npairs, e_begin, n_experts, a, what))) return st;
    e = moe_grouped_launch(a, t, false, g_stream);
    ++t_launches;
    if (e != cudaSuccess) return cuda_fail(e, what);
    e = moe_combine_launch(ws->moe_y, ids, e_begin, n_experts, rw, out, out_stride, tokens, k, hidden, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, what);
}

// ---- causal gated decode attention --------------------------------------------
namespace {
int attention(const float *q, const float *gate, const void *kc, const void *vc, int kv_bf16, float *attn, int tokens,
              int n_heads, int kv_heads, int head_dim, int max_seq_len, const int *pos_dev, int start_pos,
              const char *what) {
    t_launches = 0;
    if (tokens < 0 || n_heads <= 0 || kv_heads <= 0 || n_heads % kv_heads || head_dim <= 0 || head_dim > 256 ||
        max_seq_len <= 0 || start_pos < 0)
        return fail(QL_EINVAL, std::string(what) + ": need n_heads a multiple of kv_heads > 0, 0 < head_dim <= 256, "
                                                   "max_seq_len > 0, start_pos >= 0");
    if (tokens == 0) return QL_OK;
    if (!q || !gate || !kc || !vc || !attn) return fail(QL_EINVAL, std::string(what) + ": null pointer");
    const int group = n_heads / kv_heads;
    if (attn_smem_bytes(group, head_dim) > 232448)
        return fail(QL_EINVAL, std::string(what) + ": n_heads / kv_heads x head_dim too large for shared memory");
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    // splits: enough CTAs to fill every SM's resident slots over the cache length (the grid does not
    // depend on the position, so a captured launch replays for any position)
    const int keys = pos_dev != nullptr ? max_seq_len : std::min(max_seq_len, start_pos + tokens);
    const int by_len = (keys + attn_tile() - 1) / attn_tile();
    const int by_sms = std::max(1, attn_ctas_per_sm(head_dim) * ws->sms / (kv_heads * tokens));
    const int splits = std::max(1, std::min(std::min(by_len, by_sms), attn_max_splits()));
    const size_t per = (size_t)tokens * n_heads * splits;
    const size_t acc_off = (per * 2 + 3) & ~size_t(3);  // the accumulators start on 16 bytes (float4 stores)
    if ((st = grow(reinterpret_cast<void **>(&ws->attn_part), &ws->attn_part_cap, acc_off + per * head_dim,
                   sizeof(float), what)))
        return st;
    AttnArgs a{};
    a.q = q;
    a.gate = gate;
    a.key_cache = kc;
    a.value_cache = vc;
    a.attn = attn;
    a.pos_dev = pos_dev;
    a.start_pos = start_pos;
    a.tokens = tokens;
    a.n_heads = n_heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.max_seq_len = max_seq_len;
    a.splits = splits;
    a.part_ml = ws->attn_part;
    a.part_acc = ws->attn_part + acc_off;
    cudaError_t e = attn_launch(a, kv_bf16 != 0, g_stream);
    t_launches += 2;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, what);
}
}  // namespace

int ql_full_attention_attend(const float *q, const float *gate, const void *key_cache, const void *value_cache,
                             int kv_bf16, float *attn, int n_heads, int kv_heads, int head_dim, int max_seq_len,
                             const int *pos_dev) {
    if (!pos_dev) return fail(QL_EINVAL, "ql_full_attention_attend: null pos_dev");
    return attention(q, gate, key_cache, value_cache, kv_bf16, attn, 1, n_heads, kv_heads, head_dim, max_seq_len,
                     pos_dev, 0, "ql_full_attention_attend");
}

int ql_full_attention_attend_batch(const float *q, const float *gate, const void *key_cache, const void *value_cache,
                                   int kv_bf16, float *attn, int tokens, int n_heads, int kv_heads, int head_dim,
                                   int max_seq_len, int start_pos) {
    if (start_pos + (int64_t)tokens > max_seq_len)
        return fail(QL_EINVAL, "ql_full_attention_attend_batch: start_pos + tokens > max_seq_len");
    return attention(q, gate, key_cache, value_cache, kv_bf16, attn, tokens, n_heads, kv_heads, head_dim, max_seq_len,
                     nullptr, start_pos, "ql_full_attention_attend_batch");
}

// ---- opt-in Q8_1 activation path ----------------------------------------------------
size_t ql_q8_1_row_bytes(int in_dim) { return in_dim > 0 ? q81_row_bytes(in_dim) : 0; }

int ql_quantize_q8_1(const float *x, uint8_t *x_q8_1, int in_dim, int m, int store_raw_sum) {
    t_launches = 0;
    if (in_dim <= 0 || m < 0) return fail(QL_EINVAL, "ql_quantize_q8_1: need in_dim > 0 and m >= 0");
    if (m == 0) return QL_OK;
    if (!x || !x_q8_1) return fail(QL_EINVAL, "ql_quantize_q8_1: null pointer");
    if (reinterpret_cast<uintptr_t>(x_q8_1) % 4)
        return fail(QL_EINVAL, "ql_quantize_q8_1: x_q8_1 must be 4-byte aligned");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = quantize_q81_launch(x, x_q8_1, in_dim, m, store_raw_sum != 0, false, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_quantize_q8_1");
}

size_t ql_q8_1_mmq_row_bytes(int in_dim) { return in_dim > 0 ? q81_mmq_row_bytes(in_dim) : 0; }

int ql_quantize_q8_1_mmq(const float *x, uint8_t *x_mmq, int in_dim, int m, int store_raw_sum) {
    t_launches = 0;
    if (in_dim <= 0 || m < 0) return fail(QL_EINVAL, "ql_quantize_q8_1_mmq: need in_dim > 0 and m >= 0");
    if (m == 0) return QL_OK;
    if (!x || !x_mmq) return fail(QL_EINVAL, "ql_quantize_q8_1_mmq: null pointer");
    if (reinterpret_cast<uintptr_t>(x_mmq) % 4)
        return fail(QL_EINVAL, "ql_quantize_q8_1_mmq: x_q8_1 must be 4-byte aligned");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = quantize_q81_launch(x, x_mmq, in_dim, m, store_raw_sum != 0, true, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_quantize_q8_1_mmq");
}

int ql_quant_gemv_q8_1(int32_t t, const uint8_t *w, size_t rb, const uint8_t *x_q8_1, float *y, int out_dim,
                       int in_dim) {
    t_launches = 0;
    if (t != kQ4_K && t != kQ6_K && t != kQ5_0 && t != kQ8_0)
        return fail(QL_EINVAL, "ql_quant_gemv_q8_1: quant_type must be Q4_K, Q6_K, Q5_0 or Q8_0");
    if (out_dim < 0) return fail(QL_EINVAL, "ql_quant_gemv_q8_1: negative out_dim");
    if (out_dim == 0) return QL_OK;
    int st = check_weight(t, w, rb, 0, in_dim, "ql_quant_gemv_q8_1");
    if (st) return st;
    if (!x_q8_1 || !y) return fail(QL_EINVAL, "ql_quant_gemv_q8_1: null pointer");
    if (reinterpret_cast<uintptr_t>(x_q8_1) % 4)
        return fail(QL_EINVAL, "ql_quant_gemv_q8_1: x_q8_1 must be 4-byte aligned");
    if (!workspace(&st)) return st;
    cudaError_t e = gemv_q81_launch(t, w, rb, x_q8_1, y, out_dim, in_dim, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_quant_gemv_q8_1");
}

namespace {
int matmul_q81(int32_t t, const uint8_t *w, size_t rb, const uint8_t *x_q8_1, float *y, int out_dim, int in_dim,
               int m, bool mmq) {
    t_launches = 0;
    if (t != kQ4_K && t != kQ6_K && t != kQ5_0 && t != kQ8_0)
        return fail(QL_EINVAL, "ql_quant_matmul_q8_1: quant_type must be Q4_K, Q6_K, Q5_0 or Q8_0");
    if (out_dim < 0 || m < 0) return fail(QL_EINVAL, "ql_quant_matmul_q8_1: negative size");
    if (out_dim == 0 || m == 0) return QL_OK;
    int st = check_weight(t, w, rb, 0, in_dim, "ql_quant_matmul_q8_1");
    if (st) return st;
    if (!x_q8_1 || !y) return fail(QL_EINVAL, "ql_quant_matmul_q8_1: null pointer");
    if (reinterpret_cast<uintptr_t>(x_q8_1) % 4)
        return fail(QL_EINVAL, "ql_quant_matmul_q8_1: x_q8_1 must be 4-byte aligned");
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    const int pitch = q81_mm_row_pitch(rb);
    if (mmq && (reinterpret_cast<uintptr_t>(w) % 16 || (size_t)64 * pitch > 232448 - 1024))
        return fail(QL_EINVAL, "ql_quant_matmul_q8_1_mmq: weight rows must be 16-byte aligned and short enough to "
                               "stage 64 of them (about 3.5 KB)");
    if (reinterpret_cast<uintptr_t>(w) % 16 || (size_t)64 * pitch > 232448 - 1024) {
        // rows too long to stage 64 of them (or an unaligned base): the GEMV per token row
        for (int r = 0; r < m; ++r) {
            cudaError_t e = gemv_q81_launch(t, w, rb, x_q8_1 + (size_t)r * q81_row_bytes(in_dim), y + (size_t)r * out_dim,
                                            out_dim, in_dim, g_stream);
            ++t_launches;
            if (e != cudaSuccess) return cuda_fail(e, "ql_quant_matmul_q8_1");
        }
        return QL_OK;
    }
    Q81MmArgs a{};
    a.w = w;
    a.rb = rb;
    a.xq = x_q8_1;
    a.y = y;
    a.out_dim = out_dim;
    a.in_dim = in_dim;
    a.m = m;
    a.row_pitch = pitch;
    a.err = ws->err;
    cudaError_t e = matmul_q81_launch(t, a, mmq, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_quant_matmul_q8_1");
}
}  // namespace

int ql_quant_matmul_q8_1(int32_t t, const uint8_t *w, size_t rb, const uint8_t *x_q8_1, float *y, int out_dim,
                         int in_dim, int m) {
    return matmul_q81(t, w, rb, x_q8_1, y, out_dim, in_dim, m, false);
}

int ql_quant_matmul_q8_1_mmq(int32_t t, const uint8_t *w, size_t rb, const uint8_t *x_mmq, float *y, int out_dim,
                             int in_dim, int m) {
    if (t != kQ4_K && t != kQ6_K) return fail(QL_EINVAL, "ql_quant_matmul_q8_1_mmq: quant_type must be Q4_K or Q6_K");
    return matmul_q81(t, w, rb, x_mmq, y, out_dim, in_dim, m, true);
}

int ql_quant_embedding(int32_t t, const int *ids, float *out, const uint8_t *table, size_t rb, int hidden, int n) {
    t_launches = 0;
    if (n < 0) return fail(QL_EINVAL, "ql_quant_embedding: negative size");
    if (n == 0) return QL_OK;
    if (!quant_ok(t) || hidden <= 0 || hidden % block_elems(t))
        return fail(QL_EINVAL, "ql_quant_embedding: bad quant_type or hidden_size");
    if (!ids || !out || !table) return fail(QL_EINVAL, "ql_quant_embedding: null pointer");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = embedding_launch(t, ids, out, table, rb, hidden, n, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_quant_embedding");
}

int ql_dequantize_to_f16(int32_t t, const uint8_t *src, uint16_t *out, int64_t n) {
    t_launches = 0;
    if (!quant_ok(t) || n < 0 || n % block_elems(t))
        return fail(QL_EINVAL, "ql_dequantize_to_f16: bad quant_type or element count");
    if (n == 0) return QL_OK;
    if (!src || !out) return fail(QL_EINVAL, "ql_dequantize_to_f16: null pointer");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = dequant_f16_launch(t, src, out, n, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_dequantize_to_f16");
}
int ql_dequantize_q4k_to_f16(const uint8_t *s, uint16_t *o, int64_t n) { return ql_dequantize_to_f16(kQ4_K, s, o, n); }
int ql_dequantize_q80_to_f16(const uint8_t *s, uint16_t *o, int64_t n) { return ql_dequantize_to_f16(kQ8_0, s, o, n); }
int ql_dequantize_q50_to_f16(const uint8_t *s, uint16_t *o, int64_t n) { return ql_dequantize_to_f16(kQ5_0, s, o, n); }
int ql_dequantize_q6k_to_f16(const uint8_t *s, uint16_t *o, int64_t n) { return ql_dequantize_to_f16(kQ6_K, s, o, n); }
int ql_dequantize_q40_to_f16(const uint8_t *s, uint16_t *o, int64_t n) { return ql_dequantize_to_f16(kQ4_0, s, o, n); }

int ql_argmax(const float *logits, int n, int *out_idx) {
    t_launches = 0;
    if (n <= 0 || !logits || !out_idx) return fail(QL_EINVAL, "ql_argmax: need n > 0 and non-null pointers");
    int st;
    Workspace *ws = workspace(&st);
    if (!ws) return st;
    cudaError_t e = argmax_launch(logits, n, out_idx, ws->am_v, ws->am_i, kArgmaxParts, g_stream);
    t_launches += 2;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_argmax");
}

int ql_rms_norm_f32(const float *x, float *y, const float *gamma, int rows, int hidden, float eps) {
    t_launches = 0;
    if (rows < 0 || hidden <= 0 || !x || !y) return fail(QL_EINVAL, "ql_rms_norm_f32: bad arguments");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = rmsnorm_launch(x, y, gamma, rows, hidden, eps, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_rms_norm_f32");
}

int ql_synth_quantized(int32_t t, uint64_t seed, int64_t rows, int in_dim, float std, uint8_t *dst) {
    t_launches = 0;
    if ((t != kQ4_K && t != kQ8_0 && t != kQ4_0 && t != kQ5_0) || rows < 0 || in_dim <= 0 ||
        in_dim % block_elems(t) || !dst)
        return fail(QL_EINVAL, "ql_synth_quantized: bad arguments");
    int st;
    if (!workspace(&st)) return st;
    cudaError_t e = synth_launch(t, seed, rows, in_dim, std, dst, g_stream);
    ++t_launches;
    return e == cudaSuccess ? QL_OK : cuda_fail(e, "ql_synth_quantized");
}

}  // extern "C"
