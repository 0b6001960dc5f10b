// ql_noalloc.cu -- ql_argmax_noalloc: the greedy argmax for callers that must
// not allocate device memory.
//
// Who needs it: ql_argmax keeps its block partials in the library workspace,
// which the first call on a device allocates with cudaMalloc.  Some callers
// cannot let a library allocate: a runtime whose device memory is all owned by
// its own pool or budgeted up front (an inference server that sizes HBM for
// weights and KV cache at start-up and treats any later cudaMalloc as a
// fault), or code running under a memory-allocation ban after start-up.
// This entry point keeps the same two-stage partials in a fixed 8 KB array in
// the library's own device image instead, and never calls cudaMalloc, cudaFree
// or an allocating library routine.
//
// Contract:
//  * n must not exceed kNoAllocArgmaxMaxN (16,777,216); larger n is rejected
//    with QL_EINVAL.  The array holds kNoAllocParts (1024) partial results.
//  * The array is shared by every call in the process on a device and keeps the
//    last call's contents.  Every call overwrites all partials it reads, so
//    nothing needs clearing; but calls that overlap on the GPU (e.g. on two
//    streams) race on it and must be serialized by the caller.
//  * The first call on a device does a one-time set-up for that device (it
//    resolves the array's device address with cudaGetSymbolAddress); make that
//    first call before any stream capture.  Each device that loads the library
//    holds the 8 KB until the process exits.
//  * The resolved address is kept for the life of the process.  After
//    cudaDeviceReset (or any teardown of the device's primary context) the
//    library's device image is loaded again and the array may move: do not call
//    this entry point on a device after resetting it.
#include <mutex>

#include "../../include/qlinear_b200.h"
#include "ql_common.cuh"

namespace ql {
cudaError_t argmax_launch(const float *x, int n, int *out, float *pv, int *pi, int max_parts, cudaStream_t s);
int set_last_error(int code, const char *msg);
void set_launch_count(int n);

namespace {
constexpr int kNoAllocParts = 1024;
constexpr int kNoAllocArgmaxMaxN = 1 << 24;
constexpr int kMaxDevices = 64;

// [0, kNoAllocParts): partial values (float bits); [kNoAllocParts, 2x): partial indices.
static __device__ __align__(256) uint32_t g_argmax_scratch[2 * kNoAllocParts];

std::mutex g_mu;
uint32_t *g_scratch_addr[kMaxDevices] = {};
}  // namespace
}  // namespace ql

using namespace ql;

extern "C" QL_API int ql_argmax_noalloc(const float *logits, int n, int *out_idx) {
    set_launch_count(0);
    if (n <= 0 || !logits || !out_idx) return set_last_error(QL_EINVAL, "ql_argmax_noalloc: need n > 0 and non-null pointers");
    if (n > kNoAllocArgmaxMaxN)
        return set_last_error(QL_EINVAL, "ql_argmax_noalloc: n exceeds the no-allocation maximum of 16777216");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return set_last_error(QL_EINVAL, "ql_argmax_noalloc: device index out of range");
    uint32_t *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_scratch_addr[dev] == nullptr) {
            // One-time set-up on this device (it is current): the host-side name of a
            // __device__ array is not a device address; ask the runtime for it.
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_argmax_scratch);
            if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
            g_scratch_addr[dev] = static_cast<uint32_t *>(p);
        }
        scratch = g_scratch_addr[dev];
    }
    float *pv = reinterpret_cast<float *>(scratch);
    int *pi = reinterpret_cast<int *>(scratch + kNoAllocParts);
    e = argmax_launch(logits, n, out_idx, pv, pi, kNoAllocParts, static_cast<cudaStream_t>(ql_get_stream()));
    set_launch_count(2);
    if (e != cudaSuccess) return set_last_error(QL_ECUDA, cudaGetErrorString(e));
    return QL_OK;
}
