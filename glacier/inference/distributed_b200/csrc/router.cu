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
#include <cooperative_groups.h>

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
            const float eps = p.norm_w ? p.norm_eps : 1e-5f;
            rms_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
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
            const float nw = (in && p.norm_w) ? __ldg(p.norm_w + d) : 1.0f;
#pragma unroll
            for (int tb = 0; tb < TB; ++tb) {
                const float raw = (in && tb < ntb) ? __ldg(X + (size_t)tb * D + d) : 0.f;
                xv[u][tb] = p.rmsnorm ? __fmul_rn(raw, rms[tb]) : raw;
                if (p.norm_w) xv[u][tb] = __fmul_rn(xv[u][tb], nw);
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

// Wide routers (E > 8, up to 64 experts: 917 KB of fp32 router at D = 3584):
// one thread-block cluster per TB tokens, CTA g of the cluster computing the
// logits of experts [8g, 8g + 8) -- 32 contiguous bytes of every router row,
// so a warp's loads are whole sectors -- in the same canonical order as
// router_kernel (256 strided fused partials, warp butterfly, pairwise tree
// over the 8 warps), and storing them straight into the leader CTA's shared
// memory (distributed shared memory).  After one cluster barrier the leader
// ranks the experts of each token with one warp (an expert's rank = experts
// ahead of it by logit, lower index first on ties, NaN as -inf: the order of
// router_kernel's repeated arg-max) and forms the softmax weights with the
// same expf arguments and the same sequential sums, so ids and weights are
// bit-identical to router_kernel's.  Rank 0 also writes xin and the shared-
// expert gate.
constexpr int kWideGroup = 8;     // experts per CTA

// Two CTAs per SM: the four-token instantiation is held to 128 registers
// (from 139, a few bytes spilled), which took the 256-token Qwen2-57B router
// from 52 to 34 us.
template <int TB, int UNROLL>
__global__ void __launch_bounds__(kRouterThreads, 2) router_wide_kernel(const __grid_constant__ RouterParams p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    __shared__ float red[8][TB * kWideGroup + TB];
    __shared__ float logits[TB * 64];  // the leader's copy receives every CTA's experts
    __shared__ float rms_s[TB];
    __shared__ float gate_s[TB];
    __shared__ float ex[TB][64];
    __shared__ int sid[TB][16];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, D = p.D;
    const int g = (int)cl.block_rank();
    const int e0 = g * kWideGroup;
    const int t0 = blockIdx.y * TB;
    const int ntb = min(TB, p.T - t0);
    const bool lead = g == 0;
    const bool gate = lead && p.gate_vec != nullptr;
    const float* __restrict__ X = p.x + (size_t)t0 * D;

    if (p.rmsnorm) {  // every CTA: the canonical sum of squares
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
    float rms[TB];
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) rms[tb] = p.rmsnorm ? rms_s[tb < ntb ? tb : 0] : 1.0f;

    float acc[TB][kWideGroup], gacc[TB];
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) {
        gacc[tb] = 0.f;
#pragma unroll
        for (int e = 0; e < kWideGroup; ++e) acc[tb][e] = 0.f;
    }
    // two aligned float4 per row when the row pitch and the base allow it
    const bool full8 = (E % 4 == 0) && e0 + kWideGroup <= E && ((uintptr_t)p.Wr & 15u) == 0;
    for (int d0 = tid; d0 < D; d0 += UNROLL * kRouterThreads) {
        float xv[UNROLL][TB];
        float wv[UNROLL][kWideGroup];
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
            if (full8) {
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
                if (in) {
                    const float4* r = reinterpret_cast<const float4*>(p.Wr + (size_t)d * E + e0);
                    a = __ldg(r);
                    b = __ldg(r + 1);
                }
                wv[u][0] = a.x; wv[u][1] = a.y; wv[u][2] = a.z; wv[u][3] = a.w;
                wv[u][4] = b.x; wv[u][5] = b.y; wv[u][6] = b.z; wv[u][7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < kWideGroup; ++e)
                    wv[u][e] = (in && e0 + e < E) ? __ldg(p.Wr + (size_t)d * E + e0 + e) : 0.f;
            }
            gv[u] = (in && gate) ? __ldg(p.gate_vec + d) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int d = d0 + u * kRouterThreads;
            if (d < D) {
#pragma unroll
                for (int tb = 0; tb < TB; ++tb) {
#pragma unroll
                    for (int e = 0; e < kWideGroup; ++e) acc[tb][e] = fmaf(xv[u][tb], wv[u][e], acc[tb][e]);
                    if (gate) gacc[tb] = fmaf(xv[u][tb], gv[u], gacc[tb]);
                    if (lead && p.xin && tb < ntb) p.xin[(size_t)(t0 + tb) * D + d] = xv[u][tb];
                }
            }
        }
    }
#pragma unroll
    for (int tb = 0; tb < TB; ++tb) {
#pragma unroll
        for (int e = 0; e < kWideGroup; ++e) {
            const float v = warp_tree(acc[tb][e]);
            if (lane == 0) red[warp][tb * kWideGroup + e] = v;
        }
        if (gate) {
            const float v = warp_tree(gacc[tb]);
            if (lane == 0) red[warp][TB * kWideGroup + tb] = v;
        }
    }
    __syncthreads();
    // this CTA's logits into the leader's shared memory
    float* lead_logits = cl.map_shared_rank(logits, 0);
    if (tid < TB * kWideGroup) {
        const int tb = tid / kWideGroup, e = tid % kWideGroup;
        if (tb < ntb && e0 + e < E) {
            float s[8];
            for (int w = 0; w < 8; ++w) s[w] = red[w][tid];
            lead_logits[tb * 64 + e0 + e] = tree8(s);
        }
    }
    if (gate && tid < ntb) {
        float s[8];
        for (int w = 0; w < 8; ++w) s[w] = red[w][TB * kWideGroup + tid];
        gate_s[tid] = 1.0f / (1.0f + expf(-tree8(s)));
    }
    cl.sync();  // every CTA's logits have landed in the leader
    if (!lead) return;

    // ---- top-k by rank and the softmax weights, one warp per token
    if (warp < ntb) {
        const int t = t0 + warp;
        const float* l = logits + warp * 64;
        const int k = p.k;
        const int ea = lane, eb = lane + 32;
        const float va = (ea < E && !isnan(l[ea])) ? l[ea] : -INFINITY;
        const float vb = (eb < E && !isnan(l[eb])) ? l[eb] : -INFINITY;
        int ra = 0, rb = 0;
        for (int e = 0; e < E; ++e) {
            const float v = isnan(l[e]) ? -INFINITY : l[e];
            ra += (v > va || (v == va && e < ea)) ? 1 : 0;
            rb += (v > vb || (v == vb && e < eb)) ? 1 : 0;
        }
        if (ea < E && ra < k) sid[warp][ra] = ea;
        if (eb < E && rb < k) sid[warp][rb] = eb;
        __syncwarp();
        const int first = sid[warp][0];
        const float mx = isnan(l[first]) ? -INFINITY : l[first];
        if (ea < E) ex[warp][ea] = expf(l[ea] - mx);
        if (eb < E) ex[warp][eb] = expf(l[eb] - mx);
        __syncwarp();
        float den = 0.f;
        if (lane == 0) {
            if (p.renorm) {
                for (int j = 0; j < k; ++j) den += ex[warp][sid[warp][j]];
            } else {
                for (int e = 0; e < E; ++e) den += ex[warp][e];
            }
        }
        den = __shfl_sync(0xffffffffu, den, 0);
        if (lane < k) {
            const int id = sid[warp][lane];
            p.ids[(size_t)t * k + lane] = id;
            p.w[(size_t)t * k + lane] = ex[warp][id] / den;
        }
        if (p.logits)
            for (int e = lane; e < E; e += 32) p.logits[(size_t)t * E + e] = l[e];
        if (lane == 0 && p.gate_vec && p.gate_out) p.gate_out[t] = gate_s[warp];
    }
}

template <int TB, int UNROLL>
static cudaError_t launch_router_wide(const RouterParams& p, cudaStream_t stream) {
    const int ctas = (p.E + kWideGroup - 1) / kWideGroup;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(ctas, (p.T + TB - 1) / TB);
    cfg.blockDim = dim3(kRouterThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ctas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, router_wide_kernel<TB, UNROLL>, p);
}

cudaError_t router_launch(const RouterParams& p, cudaStream_t stream) {
    if (p.T <= 0) return cudaSuccess;
    if (p.E <= 0 || p.E > 64 || p.k <= 0 || p.k > 16 || p.k > p.E || p.D <= 0)
        return cudaErrorInvalidValue;
    if (p.norm_w && (p.E > 8 || !p.rmsnorm)) return cudaErrorInvalidValue;
    // Few tokens: one token per CTA for parallelism; many: amortise Wr loads.
    const bool many = p.T > 64;
    if (p.E <= 8) return many ? launch_router<8, 4, 4>(p, stream) : launch_router<8, 1, 4>(p, stream);
    // wider routers: a cluster of E/8 CTAs per token block; one token per
    // block up to 64 tokens (more CTAs in flight), four beyond (fewer
    // re-reads of the router columns)
    return p.T > 64 ? launch_router_wide<4, 4>(p, stream) : launch_router_wide<1, 8>(p, stream);
}

}  // namespace glc
