// router.cu -- MoE router on sm_100a: optional RMSNorm ingress, gate GEMV
// (logits = xin . Wr), softmax, top-k with ties to the lower expert index,
// optional renormalisation, and the Qwen shared-expert sigmoid gate.
//
// The reference receives expert ids and weights as inputs
// (DistributedPipelineCoordinator.ExecuteStep, DistributedPipelineCoordinator.cs:72-78;
// GpuFirstExpertStageWorker.ProcessRoutedTopK, GpuFirstExpertStageWorker.cs:416-423);
// the router itself lives in the un-vendored model code.  Expert ids must be
// bit-exact against the CPU oracle, so every fp32 sum here uses one canonical
// order that the oracle replays: 256 strided fused partials (d = t, t+256, ...
// in increasing d), a xor butterfly inside each warp, and a fixed pairwise tree
// over the 8 warp sums.  Top-k is taken on the logits, so exp() differences
// cannot change the selection.  Loads are batched UNROLL deep per thread so a
// single CTA keeps enough requests in flight for the latency-bound T=1 case.
#include "common.cuh"
#include "kernels.h"

namespace glc {

constexpr int kRouterThreads = 256;

// EP: compile-time expert capacity (runtime E <= EP), TB: tokens per CTA.
template <int EP, int TB, int UNROLL>
__global__ void __launch_bounds__(kRouterThreads) router_kernel(const __grid_constant__ RouterParams p) {
    __shared__ float red[8][TB * EP];
    __shared__ float logits[TB * EP];
    __shared__ float rms_s[TB];
    __shared__ float gate_s[TB];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, D = p.D;
    const int t0 = blockIdx.x * TB;
    const int ntb = min(TB, p.T - t0);
    const float* __restrict__ X = p.x + (size_t)t0 * D;

    // ---- RMSNorm scale per token: canonical sum of squares
    if (p.rmsnorm) {
        float a[TB];
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) a[tb] = 0.f;
        for (int d0 = tid; d0 < D; d0 += UNROLL * kRouterThreads) {
            float v[UNROLL][TB];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                for (int tb = 0; tb < TB; ++tb) {
                    const int d = d0 + u * kRouterThreads;
                    v[u][tb] = (d < D && tb < ntb) ? __ldg(X + (size_t)tb * D + d) : 0.f;
                }
#pragma unroll
            for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                for (int tb = 0; tb < TB; ++tb)
                    if (d0 + u * kRouterThreads < D) a[tb] = fmaf(v[u][tb], v[u][tb], a[tb]);
        }
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) {
            const float s = warp_tree(a[tb]);
            if (lane == 0) red[warp][tb] = s;
        }
        __syncthreads();
        if (tid < ntb) {
            float s[8];
            for (int w = 0; w < 8; ++w) s[w] = red[w][tid];
            const float ss = tree8(s);
            rms_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
        }
        __syncthreads();
    }

    // ---- gate GEMV partials (+ shared-expert gate), xin written on the way
    float acc[TB][EP];
    float gacc[TB];
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) {
        gacc[tb] = 0.f;
#pragma unroll
        for (int e = 0; e < EP; ++e) acc[tb][e] = 0.f;
    }
    float rms[TB];
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) rms[tb] = p.rmsnorm ? rms_s[tb < ntb ? tb : 0] : 1.0f;
    for (int d0 = tid; d0 < D; d0 += UNROLL * kRouterThreads) {
        float xv[UNROLL][TB];
        float wv[UNROLL][EP];
        float gv[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int d = d0 + u * kRouterThreads;
            const bool in = d < D;
#pragma unroll
            for (int tb = 0; tb < TB; ++tb) {
                const float raw = (in && tb < ntb) ? __ldg(X + (size_t)tb * D + d) : 0.f;
                xv[u][tb] = p.rmsnorm ? __fmul_rn(raw, rms[tb]) : raw;
            }
#pragma unroll
            for (int e = 0; e < EP; ++e) wv[u][e] = (in && e < E) ? __ldg(p.Wr + (size_t)d * E + e) : 0.f;
            gv[u] = (in && p.gate_vec) ? __ldg(p.gate_vec + d) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int d = d0 + u * kRouterThreads;
            if (d < D) {
#pragma unroll
                for (int tb = 0; tb < TB; ++tb) {
#pragma unroll
                    for (int e = 0; e < EP; ++e) acc[tb][e] = fmaf(xv[u][tb], wv[u][e], acc[tb][e]);
                    gacc[tb] = fmaf(xv[u][tb], gv[u], gacc[tb]);
                    if (p.xin && tb < ntb) p.xin[(size_t)(t0 + tb) * D + d] = xv[u][tb];
                }
            }
        }
    }
#pragma unroll
    for (int tb = 0; tb < TB; ++tb)
#pragma unroll
        for (int e = 0; e < EP; ++e) {
            const float v = warp_tree(acc[tb][e]);
            if (lane == 0) red[warp][tb * EP + e] = v;
        }
    __syncthreads();
    for (int i = tid; i < ntb * EP; i += kRouterThreads) {
        float s[8];
        for (int w = 0; w < 8; ++w) s[w] = red[w][i];
        logits[i] = tree8(s);
    }
    __syncthreads();
    if (p.gate_vec) {
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) {
            const float v = warp_tree(gacc[tb]);
            if (lane == 0) red[warp][tb] = v;
        }
        __syncthreads();
        if (tid < ntb) {
            float s[8];
            for (int w = 0; w < 8; ++w) s[w] = red[w][tid];
            const float g = tree8(s);
            gate_s[tid] = 1.0f / (1.0f + expf(-g));
        }
        __syncthreads();
    }

    // ---- softmax / top-k, one thread per token
    if (tid < ntb) {
        const int t = t0 + tid;
        const float* l = logits + tid * EP;
        if (p.logits)
            for (int e = 0; e < E; ++e) p.logits[(size_t)t * E + e] = l[e];
        uint64_t taken = 0;
        int ids[16];
        for (int j = 0; j < p.k; ++j) {
            int best = -1;
            float bv = 0.f;
            for (int e = 0; e < E; ++e) {
                if ((taken >> e) & 1ull) continue;
                const float v = isnan(l[e]) ? -INFINITY : l[e];
                if (best < 0 || v > bv) { best = e; bv = v; }
            }
            taken |= 1ull << best;
            ids[j] = best;
        }
        const float mx = isnan(l[ids[0]]) ? -INFINITY : l[ids[0]];
        float den = 0.f;
        if (p.renorm) {
            for (int j = 0; j < p.k; ++j) den += expf(l[ids[j]] - mx);
        } else {
            for (int e = 0; e < E; ++e) den += expf(l[e] - mx);
        }
        for (int j = 0; j < p.k; ++j) {
            p.ids[(size_t)t * p.k + j] = ids[j];
            p.w[(size_t)t * p.k + j] = expf(l[ids[j]] - mx) / den;
        }
        if (p.gate_vec && p.gate_out) p.gate_out[t] = gate_s[tid];
    }
}

template <int EP, int TB, int UNROLL>
static cudaError_t launch_router(const RouterParams& p, cudaStream_t stream) {
    const int grid = (p.T + TB - 1) / TB;
    router_kernel<EP, TB, UNROLL><<<grid, kRouterThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t router_launch(const RouterParams& p, cudaStream_t stream) {
    if (p.T <= 0) return cudaSuccess;
    if (p.E <= 0 || p.E > 64 || p.k <= 0 || p.k > 16 || p.k > p.E || p.D <= 0)
        return cudaErrorInvalidValue;
    // Few tokens: one token per CTA for parallelism; many: amortise Wr loads.
    const bool many = p.T > 64;
    if (p.E <= 8) return many ? launch_router<8, 4, 4>(p, stream) : launch_router<8, 1, 4>(p, stream);
    if (p.E <= 16) return many ? launch_router<16, 2, 4>(p, stream) : launch_router<16, 1, 4>(p, stream);
    if (p.E <= 32) return launch_router<32, 1, 2>(p, stream);
    return launch_router<64, 1, 2>(p, stream);
}

}  // namespace glc
