// router.cu -- MoE router on sm_100a: optional RMSNorm ingress, gate GEMV
// (logits = xin . Wr), softmax, top-k with ties to the lower expert index,
// optional renormalisation, and the Qwen shared-expert sigmoid gate.
//
// The reference receives expert ids and weights as inputs
// (DistributedPipelineCoordinator.ExecuteStep, DistributedPipelineCoordinator.cs:72-78;
// GpuFirstExpertStageWorker.ProcessRoutedTopK, GpuFirstExpertStageWorker.cs:416-423);
// the router itself lives in the un-vendored model code.  Expert ids must be
// bit-exact against the CPU oracle, so every fp32 sum here uses one canonical
// order that the oracle replays: 256 strided fused partials, a xor butterfly
// inside each warp, and a fixed pairwise tree over the 8 warp sums.  Top-k is
// taken on the logits, so exp() differences cannot change the selection.
#include "common.cuh"
#include "kernels.h"

namespace glc {

constexpr int kRouterThreads = 256;
constexpr int kRouterMaxAcc = 64;  // tokens-per-CTA x experts held in registers

__device__ __forceinline__ float tree8(const float* s) {
    return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

template <int TBE>
__global__ void __launch_bounds__(kRouterThreads) router_kernel(const __grid_constant__ RouterParams p,
                                                                int tb_per_cta) {
    __shared__ float red[8][kRouterMaxAcc];
    __shared__ float logits[kRouterMaxAcc];
    __shared__ float rms_s[kRouterMaxAcc];
    __shared__ float gate_s[kRouterMaxAcc];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = p.E, D = p.D;
    const int t0 = blockIdx.x * tb_per_cta;
    const int ntb = min(tb_per_cta, p.T - t0);

    // RMSNorm scale per token (canonical sum of squares).
    for (int tb = 0; tb < ntb; ++tb) {
        const float* x = p.x + (size_t)(t0 + tb) * D;
        float rms = 1.0f;
        if (p.rmsnorm) {
            float a = 0.f;
            for (int d = tid; d < D; d += kRouterThreads) a = fmaf(x[d], x[d], a);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (lane == 0) red[warp][0] = a;
            __syncthreads();
            if (tid == 0) {
                float s[8];
                for (int w = 0; w < 8; ++w) s[w] = red[w][0];
                const float ss = tree8(s);
                rms_s[tb] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
            }
            __syncthreads();
            rms = rms_s[tb];
        }
        if (p.xin) {
            float* xo = p.xin + (size_t)(t0 + tb) * D;
            for (int d = tid; d < D; d += kRouterThreads) xo[d] = p.rmsnorm ? __fmul_rn(x[d], rms) : x[d];
        }
        if (tid == 0) rms_s[tb] = rms;
    }
    __syncthreads();

    // Gate GEMV partials.
    float acc[TBE];
#pragma unroll
    for (int i = 0; i < TBE; ++i) acc[i] = 0.f;
    float gacc[TBE];
#pragma unroll
    for (int i = 0; i < TBE; ++i) gacc[i] = 0.f;
    for (int d = tid; d < D; d += kRouterThreads) {
        const float* wr = p.Wr + (size_t)d * E;
#pragma unroll
        for (int i = 0; i < TBE; ++i) {
            const int tb = i / E, e = i - tb * E;
            if (tb < ntb) {
                const float xv = p.rmsnorm ? __fmul_rn(p.x[(size_t)(t0 + tb) * D + d], rms_s[tb])
                                           : p.x[(size_t)(t0 + tb) * D + d];
                acc[i] = fmaf(xv, __ldg(wr + e), acc[i]);
                if (p.gate_vec && e == 0) gacc[i] = fmaf(xv, __ldg(p.gate_vec + d), gacc[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < TBE; ++i) {
        float v = acc[i];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[warp][i] = v;
    }
    __syncthreads();
    if (tid < TBE && tid < ntb * E) {
        float s[8];
        for (int w = 0; w < 8; ++w) s[w] = red[w][tid];
        logits[tid] = tree8(s);
    }
    __syncthreads();
    if (p.gate_vec) {
#pragma unroll
        for (int i = 0; i < TBE; ++i) {
            float v = gacc[i];
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) red[warp][i] = v;
        }
        __syncthreads();
        if (tid < ntb) {
            float s[8];
            for (int w = 0; w < 8; ++w) s[w] = red[w][tid * E];
            const float g = tree8(s);
            gate_s[tid] = 1.0f / (1.0f + expf(-g));
        }
        __syncthreads();
    }

    // Softmax / top-k, one thread per token.
    if (tid < ntb) {
        const int t = t0 + tid;
        const float* l = logits + tid * E;
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

cudaError_t router_launch(const RouterParams& p, cudaStream_t stream) {
    if (p.T <= 0) return cudaSuccess;
    if (p.E <= 0 || p.E > 64 || p.k <= 0 || p.k > 16 || p.k > p.E || p.D <= 0)
        return cudaErrorInvalidValue;
    int tb = kRouterMaxAcc / p.E;
    if (tb < 1) tb = 1;
    if (tb > p.T) tb = p.T;
    const int grid = (p.T + tb - 1) / tb;
    // TBE template: smallest of {8, 16, 32, 64} covering tb * E.
    const int need = tb * p.E;
    if (need <= 8) router_kernel<8><<<grid, kRouterThreads, 0, stream>>>(p, tb);
    else if (need <= 16) router_kernel<16><<<grid, kRouterThreads, 0, stream>>>(p, tb);
    else if (need <= 32) router_kernel<32><<<grid, kRouterThreads, 0, stream>>>(p, tb);
    else router_kernel<64><<<grid, kRouterThreads, 0, stream>>>(p, tb);
    return cudaGetLastError();
}

}  // namespace glc
