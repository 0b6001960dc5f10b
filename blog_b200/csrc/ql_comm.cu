// ql_comm.cu -- tensor-parallel exchange over NVLink peer memory.
//
// The decode step's row-parallel projections (o_proj and down, split by input
// blocks across ranks) leave each rank with a partial of the hidden vector that
// must be summed over ranks: the "one all-reduce per block" of the tensor-parallel
// layout.  At decode sizes (hidden 3584 floats per token) a library collective is
// latency-bound, so this file implements a one-shot all-reduce on peer memory:
//
//   * every rank owns one exchange buffer (cudaMalloc, exported through CUDA IPC,
//     mapped by every peer): a step counter, arrival flags and an inbox;
//   * ql_allreduce_f32 runs `nslices` CTAs; CTA j stores slice j of the local
//     vector into every rank's inbox (plain stores over NVLink), fences at
//     system scope and sets one flag per destination, then waits (bounded) for
//     slice j's flags from all ranks in its own memory and sums slice j over
//     ranks in rank order -- so every rank ends with bit-identical sums;
//   * flags carry step + 1 and the inbox is double-buffered by step parity, so a
//     rank that runs ahead into the next step never overwrites data a peer has
//     not read yet (it cannot pass the next step's first exchange without that
//     peer's flags).
//
// Every wait is bounded (~5 s); a wait that expires records an error in the
// library's device error word (read by ql_check_device) and skips the sum.
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qlinear_b200.h"
#include "ql_common.cuh"

namespace ql {
int set_last_error(int code, const char *msg);
int *device_error_word();

namespace {

constexpr int kMaxWorld = 8;
constexpr int kSlices = 8;          // CTAs per all-reduce; each owns one slice of the vector
constexpr int kHeaderBytes = 256;   // step counter
constexpr int kErrCommWait = 16;    // device error code: a peer's flag never arrived

struct CommDev {
    float *inbox[kMaxWorld];        // every rank's inbox base (index = rank), mapped into this process
    unsigned *flags[kMaxWorld];     // every rank's flag array
    const unsigned *step;           // this rank's step counter
    int rank, world, max_floats, slots;
    int *err;
};

struct Comm {
    CommDev d;
    void *own = nullptr;                 // this rank's exchange buffer
    void *mapped[kMaxWorld] = {};        // peers' buffers mapped through IPC
    int device = 0;
};

size_t flags_bytes(int world, int slots) {
    return ((size_t)slots * kSlices * world * sizeof(unsigned) + 255) / 256 * 256;
}
size_t comm_bytes(int world, int max_floats, int slots) {
    return kHeaderBytes + flags_bytes(world, slots) + (size_t)slots * 2 * world * max_floats * sizeof(float);
}
void layout(void *base, int world, int slots, unsigned **step, unsigned **flags, float **inbox) {
    uint8_t *b = static_cast<uint8_t *>(base);
    *step = reinterpret_cast<unsigned *>(b);
    *flags = reinterpret_cast<unsigned *>(b + kHeaderBytes);
    *inbox = reinterpret_cast<float *>(b + kHeaderBytes + flags_bytes(world, slots));
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) allreduce_kernel(const CommDev c, float *buf, int n, int slot) {
    __shared__ int ok;
    const unsigned target = *c.step + 1u;
    const int par = (int)(target & 1u);
    const int j = blockIdx.x;
    const int lo = (int)((int64_t)j * n / kSlices), hi = (int)((int64_t)(j + 1) * n / kSlices);
    const size_t box = ((size_t)(slot * 2 + par) * c.world) * c.max_floats;  // [slot][parity] block of the inbox
    // 1. this rank's slice j -> inbox[slot][parity][rank] of every rank
    for (int d = 0; d < c.world; ++d) {
        float *dst = c.inbox[d] + box + (size_t)c.rank * c.max_floats;
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = buf[i];
    }
    __syncthreads();
    // 2. one flag per destination, after a system-scope fence (orders the CTA's stores, seen through bar.sync)
    if (threadIdx.x < c.world) {
        __threadfence_system();
        st_release_sys(c.flags[threadIdx.x] + ((size_t)slot * kSlices + j) * c.world + c.rank, target);
    }
    // 3. wait for slice j from every rank (flags live in this rank's memory)
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < c.world) {
        const unsigned *f = c.flags[c.rank] + ((size_t)slot * kSlices + j) * c.world + threadIdx.x;
        if (ld_acquire_sys(f) < target) {
            const uint64_t t0 = global_timer_ns();
            while (ld_acquire_sys(f) < target) {
                if (global_timer_ns() - t0 > 5000000000ull) {
                    atomicExch(c.err, kErrCommWait);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    // 4. sum slice j over ranks in rank order (identical on every rank)
    const float *in = c.inbox[c.rank] + box;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float s = 0.f;
        for (int r = 0; r < c.world; ++r) s += in[(size_t)r * c.max_floats + i];
        buf[i] = s;
    }
}

__global__ void step_kernel(unsigned *step) { *step += 1u; }

std::mutex g_comm_mu;

}  // namespace
}  // namespace ql

using namespace ql;

extern "C" {

int ql_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle) {
    if (!ptr || !handle || bytes == 0) return set_last_error(QL_EINVAL, "ql_ipc_alloc: need bytes > 0 and outputs");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return set_last_error(QL_ECUDA, (std::string("ql_ipc_alloc: ") + cudaGetErrorString(e)).c_str());
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return QL_OK;
}

int ql_ipc_free(void *ptr) {
    if (ptr) cudaFree(ptr);
    return QL_OK;
}

int ql_ipc_open(const uint8_t *handle, void **ptr) {
    if (!handle || !ptr) return set_last_error(QL_EINVAL, "ql_ipc_open: null handle or output");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, (std::string("ql_ipc_open: ") + cudaGetErrorString(e)).c_str());
    return QL_OK;
}

int ql_ipc_close(void *ptr) {
    if (ptr) cudaIpcCloseMemHandle(ptr);
    return QL_OK;
}

size_t ql_comm_bytes(int world, int max_floats, int slots) {
    if (world < 1 || world > kMaxWorld || max_floats < 1 || slots < 1) return 0;
    return comm_bytes(world, max_floats, slots);
}

int ql_comm_alloc(int world, int max_floats, int slots, void **exch, uint8_t *handle) {
    if (!exch || !handle || world < 1 || world > kMaxWorld || max_floats < 1 || slots < 1)
        return set_last_error(QL_EINVAL, "ql_comm_alloc: need 1 <= world <= 8, max_floats >= 1, slots >= 1");
    const size_t bytes = comm_bytes(world, max_floats, slots);
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return set_last_error(QL_ECUDA, (std::string("ql_comm_alloc: ") + cudaGetErrorString(e)).c_str());
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == QL_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *exch = p;
    return QL_OK;
}

int ql_comm_create(int rank, int world, int max_floats, int slots, void *own, const uint8_t *handles, void **comm) {
    if (!comm || !own || !handles || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || max_floats < 1 ||
        slots < 1)
        return set_last_error(QL_EINVAL, "ql_comm_create: bad rank/world/sizes or null pointer");
    Comm *c = new Comm();
    memset(&c->d, 0, sizeof(c->d));
    cudaGetDevice(&c->device);
    c->own = own;
    for (int r = 0; r < world; ++r) {
        void *base = own;
        if (r != rank) {
            cudaIpcMemHandle_t h;
            memcpy(&h, handles + (size_t)r * QL_IPC_HANDLE_BYTES, sizeof(h));
            cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                for (int q = 0; q < r; ++q)
                    if (c->mapped[q]) cudaIpcCloseMemHandle(c->mapped[q]);
                delete c;
                return set_last_error(QL_ECUDA, (std::string("ql_comm_create: ") + cudaGetErrorString(e)).c_str());
            }
            c->mapped[r] = base;
        }
        unsigned *step, *flags;
        float *inbox;
        layout(base, world, slots, &step, &flags, &inbox);
        c->d.flags[r] = flags;
        c->d.inbox[r] = inbox;
        if (r == rank) c->d.step = step;
    }
    c->d.rank = rank;
    c->d.world = world;
    c->d.max_floats = max_floats;
    c->d.slots = slots;
    c->d.err = device_error_word();
    if (!c->d.err) {
        ql_comm_destroy(c);
        return set_last_error(QL_ECUDA, "ql_comm_create: no device workspace");
    }
    *comm = c;
    return QL_OK;
}

int ql_comm_destroy(void *comm) {
    if (!comm) return QL_OK;
    Comm *c = static_cast<Comm *>(comm);
    for (int r = 0; r < kMaxWorld; ++r)
        if (c->mapped[r]) cudaIpcCloseMemHandle(c->mapped[r]);
    if (c->own) cudaFree(c->own);
    delete c;
    return QL_OK;
}

int ql_allreduce_f32(void *comm, float *buf, int n, int slot) {
    Comm *c = static_cast<Comm *>(comm);
    if (!c || !buf || n < 0 || n > c->d.max_floats || slot < 0 || slot >= c->d.slots)
        return set_last_error(QL_EINVAL, "ql_allreduce_f32: null comm/buffer, n > max_floats or slot out of range");
    if (n == 0) return QL_OK;
    allreduce_kernel<<<kSlices, 256, 0, static_cast<cudaStream_t>(ql_get_stream())>>>(c->d, buf, n, slot);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

int ql_comm_step(void *comm) {
    Comm *c = static_cast<Comm *>(comm);
    if (!c) return set_last_error(QL_EINVAL, "ql_comm_step: null comm");
    step_kernel<<<1, 1, 0, static_cast<cudaStream_t>(ql_get_stream())>>>(const_cast<unsigned *>(c->d.step));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}

}  // extern "C"
