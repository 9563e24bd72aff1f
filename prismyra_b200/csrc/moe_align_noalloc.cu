// Expert alignment for callers that must not allocate device memory.
//
// pm_moe_align needs a small caller-provided scratch table (per-chunk expert counts).  Some callers cannot
// provide one on demand: hosts that hand every byte of device memory to their own pool and do not let a library
// call cudaMalloc behind their back, and latency-critical loops that cannot risk the implicit device
// synchronisation a cudaMalloc or cudaFree may trigger.  pm_moe_align_noalloc serves them: the count table lives
// in a file-scope device array of fixed size that is part of the library image, so the call allocates nothing.
//
// Costs and limits, stated for the user:
//   * every GPU that loads the library holds the array (kNoallocCountBytes = 256 KiB) until the process exits;
//   * it accepts at most kNoallocMaxFlat = 2^20 routed (token, slot) pairs (T * k) and at most 256 experts, and
//     rejects anything larger with PM_ERR_TOO_LARGE;
//   * all calls share the one array and it keeps the previous call's contents; every entry a call reads is first
//     written by that same call, so nothing needs clearing -- but two calls whose kernels overlap on the GPU (for
//     example on two streams) race on it and must be serialised by the caller;
//   * the first call on each device looks up the array's device address with cudaGetSymbolAddress (with that
//     device current) and caches it; make that first call before any stream capture begins.
#include <mutex>

#include "prismyra_moe.h"
#include "moe_internal.h"

namespace pm {
namespace {

constexpr long kNoallocMaxFlat = 1L << 20;
constexpr int kNoallocMaxExperts = 256;
constexpr int kNoallocChunks = kAlignMaxChunks;
constexpr size_t kNoallocCountBytes = sizeof(int32_t) * (size_t)kNoallocChunks * kNoallocMaxExperts;

static __device__ __align__(256) int32_t g_noalloc_counts[kNoallocChunks * kNoallocMaxExperts];

int32_t* g_noalloc_ptr[64] = {};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_counts on the current device (looked up once per device and kept: a cudaDeviceReset
// or a destroyed primary context invalidates it, and the entry point's documentation rules calls after either out).
int noalloc_counts(int32_t** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PM_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_counts) != cudaSuccess || p == nullptr) return PM_ERR_CUDA;
        g_noalloc_ptr[dev] = static_cast<int32_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return PM_OK;
}

static_assert(kNoallocCountBytes == 256 * 1024, "the documented size of the static count table");

}  // namespace
}  // namespace pm

using namespace pm;

extern "C" int pm_moe_align_noalloc(const int32_t* topk_ids, int T, int k, int E, int32_t* sorted_ids,
                                    int32_t* expert_ids, int32_t* num_post_pad, int32_t* expert_off,
                                    pm_stream_t stream) {
    if (T < 0 || k <= 0 || E <= 0) return PM_ERR_INVALID;
    if ((long)T * k > kNoallocMaxFlat || E > kNoallocMaxExperts) return PM_ERR_TOO_LARGE;
    if (!sorted_ids || !expert_ids || !num_post_pad || (T > 0 && !topk_ids)) return PM_ERR_INVALID;
    int major = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return PM_ERR_CUDA;
    if (major != 10) return PM_ERR_DEVICE;
    int32_t* counts = nullptr;
    const int st = noalloc_counts(&counts);
    if (st != PM_OK) return st;
    const cudaError_t e = launch_align(topk_ids, T * k, E, counts, sorted_ids, expert_ids, num_post_pad, expert_off,
                                       nullptr, (cudaStream_t)stream);
    return e == cudaSuccess ? PM_OK : PM_ERR_CUDA;
}
