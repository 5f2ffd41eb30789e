// noalloc.cu -- the allocation-free variant of the token -> expert dispatch plan.
//
// glc_dispatch_plan_dev needs a scratch group table on the device and gets it
// with cudaMalloc/cudaFree on every call.  Some callers cannot allocate: a
// host driving a latency-critical decode loop (cudaMalloc and cudaFree may
// synchronise the whole device and stall every other stream), a host that
// budgets device memory up front and forbids the library from allocating
// behind its back, or code that enqueues work where the allocator must not be
// entered at all.  For them, glc_dispatch_plan_noalloc_dev keeps the scratch
// in a fixed device array that belongs to this library: it allocates nothing,
// frees nothing and does not synchronise the stream.
//
// The scratch is one file-scope __device__ array sized for at most
// kNoAllocMaxPairs (token, slot) pairs and kNoAllocMaxExperts experts
// (51 KB).  Every GPU that loads the library holds it until the process exits.
// Its device address is looked up once per device, by the first call made on
// that device (with that device current), so make that first call before any
// stream capture.  All calls on a device share the array and it keeps the last
// call's contents; the dispatch kernel rewrites every entry it reads, so
// nothing needs clearing, but calls that overlap on the GPU (different streams,
// or another thread) race on it and must be serialised by the caller.
#include <mutex>

#include "../../../../include/glacier_b200.h"
#include "kernels.h"

namespace {

constexpr int kNoAllocMaxPairs = 65536;
constexpr int kNoAllocMaxExperts = 64;
constexpr int kNoAllocMaxGroups = kNoAllocMaxExperts + kNoAllocMaxPairs / glc::kGroupTokens + 1;
constexpr int kNoAllocScratchInts = 6 * kNoAllocMaxGroups + kNoAllocMaxExperts + 2;

static __device__ __align__(256) int g_plan_scratch[kNoAllocScratchInts];

int* g_scratch_addr[glc::kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

}  // namespace

extern "C" int glc_dispatch_plan_noalloc_dev(const int32_t* ids, int32_t P, int32_t E, int32_t* counts,
                                             int32_t* offsets, int32_t* perm, int32_t* inv, void* stream) {
    if (!ids || !counts || !offsets || !perm || !inv)
        return glc::set_last_error(GLC_ERR_INVALID_ARG, "null pointer");
    if (P < 0 || P > kNoAllocMaxPairs)
        return glc::set_last_error(GLC_ERR_INVALID_ARG,
                                   "P out of range: the allocation-free dispatch plan handles at most 65536 pairs");
    if (E <= 0 || E > kNoAllocMaxExperts)
        return glc::set_last_error(GLC_ERR_INVALID_ARG,
                                   "E out of range: the allocation-free dispatch plan handles 1..64 experts");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= glc::kMaxDevices)
        return glc::set_last_error(GLC_ERR_CUDA, "cudaGetDevice failed");
    int* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            void* ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_plan_scratch) != cudaSuccess || !ptr)
                return glc::set_last_error(GLC_ERR_CUDA, "cudaGetSymbolAddress of the dispatch scratch failed");
            g_scratch_addr[dev] = static_cast<int*>(ptr);
        }
        scratch = g_scratch_addr[dev];
    }
    const int gmax = glc::plan_max_groups(P, E);
    glc::DispatchPlan plan{};
    plan.counts = counts;
    plan.offsets = offsets;
    plan.perm = perm;
    plan.inv = inv;
    plan.grp_e = scratch;
    plan.grp_ntok = scratch + gmax;
    plan.grp_N = scratch + 2 * gmax;
    plan.grp_pos0 = scratch + 3 * gmax;
    plan.grp_units = scratch + 4 * gmax;
    plan.grp_first = scratch + 5 * gmax;
    plan.meta = scratch + 5 * gmax + E;
    const cudaError_t e = glc::dispatch_plan_launch(ids, P, E, plan, (cudaStream_t)stream);
    if (e != cudaSuccess) return glc::set_last_error(GLC_ERR_CUDA, cudaGetErrorString(e));
    return GLC_OK;
}
