// ql_common.cuh -- shared definitions for the B200 block-quantized linear library.
//
// GGUF block formats as consumed by the reference engine
// (AI/codes/local-llm/src/backend/cuda/ops/kernel.cu:911-1185) plus Q4_0.
// All kernels read the weights in the raw GGUF byte layout that the reference
// uploads unchanged (CudaWeightPool.cpp:148-175), so a weight pointer plus
// row_bytes / expert_bytes means exactly what it means in the reference.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace ql {

// GGML type codes == reference DType values (src/tensor/TensorCommon.h:15-33).
enum QType : int32_t { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ5_0 = 6, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14 };

// Elements / bytes per GGUF block (reference GgufFile.cpp:35-55).
__host__ __device__ constexpr int block_elems(int t) {
    return (t == kQ4_K || t == kQ6_K) ? 256 : (t == kQ4_0 || t == kQ5_0 || t == kQ8_0) ? 32 : 0;
}
__host__ __device__ constexpr int block_bytes(int t) {
    return t == kQ4_0 ? 18 : t == kQ5_0 ? 22 : t == kQ8_0 ? 34 : t == kQ4_K ? 144 : t == kQ6_K ? 210 : 0;
}
inline bool is_quant(int t) { return block_elems(t) > 0; }

// ---------------------------------------------------------------------------
// Work plan of the streaming GEMV engine, shared by host and device so the
// host can enumerate and bounds-check every bulk copy before a launch.
//
// The output rows of one launch are cut into row groups of 32 (one output row
// per lane of a consumer warp).  The reduction dimension is cut into units
// (one GGUF block: 256 elements for K-quants, 32 for the 32-element formats).
// The T = G * U (group, unit) tiles are split into C contiguous, balanced
// ranges, one per CTA ("stream-K"): a row group that straddles CTA ranges is
// finished by whichever of its CTAs arrives last, summing the parts in K order.
// ---------------------------------------------------------------------------
struct Plan {
    int64_t T;  // total tiles = G * U
    int G;      // row groups
    int U;      // units per row group (whole reduction dimension)
    int C;      // CTAs
};

__host__ __device__ inline int64_t plan_start(const Plan &p, int c) { return (int64_t)c * p.T / p.C; }
// CTA whose range holds tile t: the largest c with start(c) <= t.
__host__ __device__ inline int plan_cta_of(const Plan &p, int64_t t) {
    return (int)(((t + 1) * (int64_t)p.C - 1) / p.T);
}

constexpr int kRowGroup = 32;
constexpr int kMaxParts = 64;  // most CTAs that may share one row group

// Error codes written to the device error word (read back by the host).
enum DevErr : int { kErrNone = 0, kErrWaitFull = 1, kErrWaitEmpty = 2, kErrBadExpert = 3 };

// ---------------------------------------------------------------------------
// PTX helpers (sm_100a).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Potentially blocking test: the hardware may suspend the thread until the phase completes
// or a system-dependent time limit passes (measured marginally faster than a 0.1 ms hint).
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~2 s, records `code` in *err and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > 2000000000ull) {
            if (err) atomicExch(err, code);
            return false;
        }
    }
    return true;
}
// One-dimensional bulk copy global -> shared (TMA engine), completion counted
// on `bar` in bytes.  dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// 3-D tiled tensor copy global -> shared through a tensor map (TMA), completion
// counted on `bar` in bytes (the full box, including zero-filled out-of-range
// elements).  The map must live in kernel-parameter (grid constant) memory.
__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int c0, int c1, int c2, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor copy global -> shared (TMA), completion counted on `bar` in bytes.
__device__ __forceinline__ void tma_box2d(void *dst, const void *tmap, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// tma_load_3d with an L2 eviction-priority policy (e.g. evict-first for streamed weights, so
// that they do not push the kernel's code, descriptors and activations out of L2).
__device__ __forceinline__ void tma_load_3d_hint(void *dst, const void *tmap, int c0, int c1, int c2, uint64_t *bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte asynchronous copy global -> shared (LDGSTS), L2-only, with an L2
// eviction-priority policy.  Addresses must be 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "l"(policy)
                 : "memory");
}
// Arrive on `bar` once every cp.async this thread has issued so far has landed
// (the arrival is not pre-counted: the barrier's expected count includes it).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Named barrier among `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Packed fp32x2 fused multiply-add (sm_100): acc.{x,y} = a.{x,y} * b.{x,y} + acc.{x,y}.
__device__ __forceinline__ void ffma2(float2 &acc, float2 a, float2 b) {
    unsigned long long c = *reinterpret_cast<unsigned long long *>(&acc);
    const unsigned long long x = *reinterpret_cast<unsigned long long *>(&a);
    const unsigned long long y = *reinterpret_cast<unsigned long long *>(&b);
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c) : "l"(x), "l"(y));
    acc = *reinterpret_cast<float2 *>(&c);
}

// Packed fp32x2 add (sm_100).
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long c;
    const unsigned long long x = *reinterpret_cast<unsigned long long *>(&a);
    const unsigned long long y = *reinterpret_cast<unsigned long long *>(&b);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(x), "l"(y));
    return *reinterpret_cast<float2 *>(&c);
}

// Greedy-argmax key, order-preserving in one 64-bit word: a larger key is a larger
// logit, then a lower index (reference argmax, kernel.cu:3531-3592: strict '>' in
// ascending order keeps the lowest index; NaN never wins; nothing selected -> 0).
// -0 and +0 compare equal; NaN and -inf get key 0 and never win.
__device__ __forceinline__ unsigned long long amax_key(float v, uint32_t idx) {
    if (!(v > -INFINITY)) return 0ull;
    const uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ int amax_index(unsigned long long k) { return k ? (int)(0xFFFFFFFFu - (uint32_t)k) : 0; }
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, k, o);
        k = t > k ? t : k;
    }
    return k;
}
// Fused greedy argmax of a launch: CTAs atomically max keys into amax[m]; the last
// CTA to finish (arrival counter) turns them into indices / keys and resets both.
struct AmaxOut {
    unsigned long long *amax;  // [M] running keys (zero between launches)
    unsigned *done;            // CTA arrival counter (zero between launches)
    int *idx;                  // [M] argmax index, or null
    unsigned long long *key;   // [M] final key (for combining vocabulary shards), or null
    int offset;                // added to every index (vocabulary shard offset)
};
__device__ __forceinline__ void amax_cta_done(const AmaxOut &o, int M) {
    __threadfence();
    const unsigned prev = atomicAdd(o.done, 1u);
    const unsigned total = gridDim.x * gridDim.y * gridDim.z;
    if (prev == total - 1) {
        __threadfence();
        for (int m = 0; m < M; ++m) {
            const unsigned long long k = atomicExch(&o.amax[m], 0ull);
            if (o.idx) o.idx[m] = amax_index(k);
            if (o.key) o.key[m] = k;
        }
        atomicExch(o.done, 0u);
    }
}

// Packed fp32x2 multiply (sm_100).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long c;
    const unsigned long long x = *reinterpret_cast<unsigned long long *>(&a);
    const unsigned long long y = *reinterpret_cast<unsigned long long *>(&b);
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(c) : "l"(x), "l"(y));
    return *reinterpret_cast<float2 *>(&c);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

// 2^e as a float, exact, for e in [-126, 127].
__host__ __device__ constexpr float pow2f(int e) {
    return e >= 0 ? (e == 0 ? 1.0f : 2.0f * pow2f(e - 1)) : 0.5f * pow2f(e + 1);
}

}  // namespace ql
