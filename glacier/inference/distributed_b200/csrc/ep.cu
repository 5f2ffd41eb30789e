// ep.cu -- expert-parallel dispatch helpers.
//
// The reference has no expert parallelism: a token's experts run one after
// another on one worker (DistributedPipelineCoordinator.cs:181-206).  With the
// experts of a layer split into contiguous shards, one per rank
// (expert e lives on rank e / (E / world)), a rank's (token, slot) pairs are
// grouped by destination rank -- a stable counting sort of the rank keys,
// done by dispatch_plan_kernel -- and the activation row of each pair is
// gathered into a send buffer in that order, with its global expert id.
#include "common.cuh"
#include "kernels.h"

namespace glc {

__global__ void __launch_bounds__(256) ep_rank_keys_kernel(const int* __restrict__ ids, int P, int epr, int world,
                                                           int* __restrict__ keys) {
    const int p = blockIdx.x * 256 + threadIdx.x;
    if (p >= P) return;
    int r = ids[p];
    r = r < 0 ? 0 : r / epr;
    keys[p] = r >= world ? world - 1 : r;
}

// One CTA per send position: rows[pos] = xin[perm[pos] / k], row_ids[pos] = ids[perm[pos]].
__global__ void __launch_bounds__(256) ep_gather_kernel(const float* __restrict__ xin, const int* __restrict__ ids,
                                                        int D, int k, const int* __restrict__ perm,
                                                        float* __restrict__ rows, int* __restrict__ row_ids) {
    const int pos = blockIdx.x;
    const int pair = perm[pos];
    const float* src = xin + (size_t)(pair / k) * D;
    float* dst = rows + (size_t)pos * D;
    if ((D & 3) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < D; i += 256) dst[i] = src[i];
    }
    if (threadIdx.x == 0) row_ids[pos] = ids[pair];
}

// Global expert ids -> indices into this rank's shard [begin, begin + count), clamped
// like GpuFirstExpertStageWorker.ProcessRoutedTopK clamps ids (GpuFirstExpertStageWorker.cs:452).
__global__ void __launch_bounds__(256) localize_ids_kernel(const int* __restrict__ ids, int n, int begin, int count,
                                                           int* __restrict__ out) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= n) return;
    const int e = ids[i] - begin;
    out[i] = e < 0 ? 0 : (e >= count ? count - 1 : e);
}

__global__ void __launch_bounds__(256) fill_kernel(float* __restrict__ p, int n, float v) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < n) p[i] = v;
}

cudaError_t ep_dispatch_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world,
                               int* keys, const DispatchPlan& plan, float* rows, int* row_ids, cudaStream_t st) {
    const int P = T * k;
    if (P <= 0) return cudaSuccess;
    if (world < 1 || world > 64 || num_experts % world) return cudaErrorInvalidValue;
    ep_rank_keys_kernel<<<(P + 255) / 256, 256, 0, st>>>(ids, P, num_experts / world, world, keys);
    cudaError_t e = dispatch_plan_launch(keys, P, world, plan, st);
    if (e != cudaSuccess) return e;
    ep_gather_kernel<<<P, 256, 0, st>>>(xin, ids, D, k, plan.perm, rows, row_ids);
    return cudaGetLastError();
}

cudaError_t localize_ids_launch(const int* ids, int n, int begin, int count, int* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    localize_ids_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, n, begin, count, out);
    return cudaGetLastError();
}

cudaError_t fill_launch(float* p, int n, float v, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(p, n, v);
    return cudaGetLastError();
}

}  // namespace glc
