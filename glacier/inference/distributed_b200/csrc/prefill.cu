// prefill.cu -- batched (T > 1) MoE path around the grouped tensor-core GEMMs:
//   * dispatch plan: token->expert histogram, exclusive offsets and a stable
//     permutation of the (token, slot) pairs grouped by expert (ascending pair
//     order inside an expert), plus the MMA group table (<= 32 or <= 64 tokens a group);
//   * operand split: one activation row per pair -> power-of-two row scale and
//     fp16 hi/lo halves written straight into the SWIZZLE_128B K-major tiles the
//     MMA reads (rows 0..N/2-1 hi, N/2..N-1 lo of each group);
//   * weighted combine: out[t] = (residual|0) + sum_j y[inv[t,j]] * w[t,j] in j
//     order (AccumulatorStageWorker.AccumulateWeightedExpert, StageWorkers.cs:152-160).
// The reference runs experts one token at a time (DistributedPipelineCoordinator.cs:
// 181-206, GpuFirstExpertStageWorker.cs:482-519); grouping by expert is what lets
// one read of an expert's weights serve all of its tokens.
#include "common.cuh"
#include "kernels.h"

namespace glc {

constexpr int kPlanThreads = 1024;

// count (optional, device): the pairs actually present, <= P (a batch sized
// on the device, e.g. the rows an expert-parallel exchange delivered).
__global__ void __launch_bounds__(kPlanThreads) dispatch_plan_kernel(const int* __restrict__ ids, int P, int E,
                                                                     DispatchPlan plan, const int* __restrict__ count,
                                                                     int gtok) {
    if (count) P = min(P, *count);
    __shared__ int s_count[64];
    __shared__ int s_off[65];
    __shared__ int s_run[64];
    __shared__ int s_warp[kPlanThreads / 32][64];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < 64) { s_count[tid] = 0; s_run[tid] = 0; }
    __syncthreads();
    for (int p = tid; p < P; p += kPlanThreads) {
        int e = ids[p];
        e = e < 0 ? 0 : (e >= E ? E - 1 : e);
        atomicAdd(&s_count[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        s_off[0] = 0;
        int g = 0, units = 0;
        for (int e = 0; e < E; ++e) {
            s_off[e + 1] = s_off[e] + s_count[e];
            plan.counts[e] = s_count[e];
            plan.grp_first[e] = g;
            for (int base = 0; base < s_count[e]; base += gtok) {
                const int nt = min(gtok, s_count[e] - base);
                const int N = 2 * ((nt + 7) / 8) * 8;
                plan.grp_e[g] = e;
                plan.grp_ntok[g] = nt;
                plan.grp_N[g] = N;
                plan.grp_pos0[g] = s_off[e] + base;
                plan.grp_units[g] = units;
                units += N;
                ++g;
            }
        }
        for (int e = 0; e <= E; ++e) plan.offsets[e] = s_off[e];
        plan.meta[0] = g;      // number of groups
        plan.meta[1] = units;  // sum of group N (B-tile rows)
    }
    __syncthreads();
    // Stable placement, chunk by chunk in pair order.
    for (int base = 0; base < P; base += kPlanThreads) {
        const int p = base + tid;
        int e = -1;
        if (p < P) {
            e = ids[p];
            e = e < 0 ? 0 : (e >= E ? E - 1 : e);
        }
        for (int i = tid; i < (kPlanThreads / 32) * 64; i += kPlanThreads) (&s_warp[0][0])[i] = 0;
        __syncthreads();
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
        if (p < P && rank_in_warp == 0) s_warp[warp][e] = __popc(same);
        __syncthreads();
        // exclusive prefix over warps for each expert, then advance the run
        if (tid < E) {
            int acc = 0;
            for (int w = 0; w < kPlanThreads / 32; ++w) {
                const int c = s_warp[w][tid];
                s_warp[w][tid] = acc;
                acc += c;
            }
            s_count[tid] = acc;  // chunk total (s_count no longer needed as histogram)
        }
        __syncthreads();
        if (p < P) {
            const int pos = s_off[e] + s_run[e] + s_warp[warp][e] + rank_in_warp;
            plan.perm[pos] = p;
            plan.inv[p] = pos;
        }
        __syncthreads();
        if (tid < E) s_run[tid] += s_count[tid];
        __syncthreads();
    }
}

// One CTA per pair position: row = src[row_of(pos)], scale to [2^14, 2^15),
// split into fp16 hi + lo and scatter into the group's swizzled B tiles.
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ src, int K, int kslots,
                                                         int src_is_token, DispatchPlan plan,
                                                         uint8_t* __restrict__ btiles, float* __restrict__ rscale,
                                                         const int* __restrict__ count) {
    if (count && (int)blockIdx.x >= *count) return;  // a position past the batch sized on the device
    __shared__ float smax[8];
    const int pos = blockIdx.x, tid = threadIdx.x;
    const int pair = plan.perm[pos];
    const float* x = src + (size_t)(src_is_token ? pair / kslots : pos) * K;
    float m = 0.f;
    for (int k = tid; k < K; k += 256) m = fmaxf(m, fabsf(x[k]));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((tid & 31) == 0) smax[tid >> 5] = m;
    __syncthreads();
    m = smax[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, smax[w]);
    // power-of-two scale: max/scale in [2^14, 2^15) keeps hi in fp16 range
    int ex = 0;
    if (m > 0.f && isfinite(m)) ex = ilogbf(m) - 14;
    const float inv = ldexpf(1.0f, -ex);
    // locate (group, slot)
    int lo = 0, hi = plan.meta[0] - 1;
    while (lo < hi) {  // last group with pos0 <= pos
        const int mid = (lo + hi + 1) >> 1;
        if (plan.grp_pos0[mid] <= pos) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int n = pos - plan.grp_pos0[g];
    const int N = plan.grp_N[g];
    const size_t gbase = (size_t)plan.grp_units[g] * 512u * (size_t)(K / 256);
    if (tid == 0) rscale[pos] = ldexpf(1.0f, ex);
    for (int k = tid; k < K; k += 256) {
        const float v = x[k] * inv;
        const __half h = __float2half_rn(v);
        const __half l = __float2half_rn(v - __half2float(h));
        const int s = k >> 8, c = (k >> 6) & 3, kk = k & 63, j = kk >> 3;
        const size_t sb = gbase + (size_t)s * N * 512 + (size_t)c * N * 128;
#pragma unroll
        for (int part = 0; part < 2; ++part) {
            const int r = part ? (N / 2 + n) : n;
            const int rr = r & 7;
            const size_t off = sb + (size_t)(r >> 3) * 1024 + rr * 128 + ((j ^ rr) << 4) + ((kk & 7) << 1);
            *reinterpret_cast<__half*>(btiles + off) = part ? l : h;
        }
    }
}

// Shared expert term of the combine (Qwen2-MoE): acc = (ysh * sg[t]) + acc
// after the routed slots, ysh the sum of nslices K-slice planes (slice order).
struct SharedCombine {
    const float* ysh;  // [nslices][T][D] or nullptr
    int nslices;
    long long stride;  // elements between planes
    const float* sg;   // [T] sigmoid gate values
};

// CTA (t, chunk): dimensions chunk * 256 + thread of token t.  Every load of
// a thread (its k expert rows and the shared expert's slices) is issued
// before the sums, which keep the k-ordered order (y * w) + acc, then the
// shared term (y_shared * gate) + acc.
constexpr int kCombineMaxK = 16, kCombineMaxSlices = 8;
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y, int D, int k,
                                                      const int* __restrict__ inv, const float* __restrict__ w,
                                                      const float* __restrict__ resid, float* __restrict__ out,
                                                      SharedCombine sh, const int* __restrict__ count) {
    const int t = blockIdx.x;
    if (count && t >= *count) return;  // a token past the batch sized on the device
    __shared__ int s_pos[kCombineMaxK];
    __shared__ float s_w[kCombineMaxK];
    if (threadIdx.x < k) {
        s_pos[threadIdx.x] = inv[t * k + threadIdx.x];
        s_w[threadIdx.x] = w[t * k + threadIdx.x];
    }
    __syncthreads();
    const int d = blockIdx.y * 256 + threadIdx.x;
    if (d >= D) return;
    float yv[kCombineMaxK], sv[kCombineMaxSlices];
#pragma unroll
    for (int j = 0; j < kCombineMaxK; ++j)
        if (j < k) yv[j] = __ldg(y + (size_t)s_pos[j] * D + d);
    const int ns = sh.ysh ? sh.nslices : 0;
#pragma unroll
    for (int s = 0; s < kCombineMaxSlices; ++s)
        if (s < ns) sv[s] = __ldg(sh.ysh + (size_t)s * sh.stride + (size_t)t * D + d);
    float acc = resid ? __ldg(resid + (size_t)t * D + d) : 0.f;
#pragma unroll
    for (int j = 0; j < kCombineMaxK; ++j)
        if (j < k) acc = __fadd_rn(__fmul_rn(yv[j], s_w[j]), acc);
    if (ns > 0) {
        float v = sv[0];
#pragma unroll
        for (int s = 1; s < kCombineMaxSlices; ++s)
            if (s < ns) v = __fadd_rn(v, sv[s]);
        acc = __fadd_rn(__fmul_rn(v, sh.sg[t]), acc);
    }
    out[(size_t)t * D + d] = acc;
}

cudaError_t dispatch_plan_launch(const int* ids, int P, int E, const DispatchPlan& plan, cudaStream_t st,
                                 const int* count, int group_tokens) {
    if (E > 64 || (group_tokens != kGroupTokens && group_tokens != kGroupTokensWide)) return cudaErrorInvalidValue;
    dispatch_plan_kernel<<<1, kPlanThreads, 0, st>>>(ids, P, E, plan, count, group_tokens);
    return cudaGetLastError();
}

cudaError_t split_rows_launch(const float* src, int P, int K, int kslots, int src_is_token, const DispatchPlan& plan,
                              uint8_t* btiles, float* rscale, cudaStream_t st, const int* count) {
    if (P <= 0) return cudaSuccess;
    split_rows_kernel<<<P, 256, 0, st>>>(src, K, kslots, src_is_token, plan, btiles, rscale, count);
    return cudaGetLastError();
}

cudaError_t combine_launch(const float* y, int T, int D, int k, const int* inv, const float* w, const float* resid,
                           float* out, cudaStream_t st, const float* ysh, int ysh_slices, long long ysh_stride,
                           const float* sg, const int* count) {
    if (T <= 0) return cudaSuccess;
    if (ysh && (ysh_slices < 1 || ysh_slices > kCombineMaxSlices || !sg)) return cudaErrorInvalidValue;
    if (k < 1 || k > kCombineMaxK) return cudaErrorInvalidValue;
    combine_kernel<<<dim3(T, (D + 255) / 256), 256, 0, st>>>(y, D, k, inv, w, resid, out,
                                                             SharedCombine{ysh, ysh_slices, ysh_stride, sg}, count);
    return cudaGetLastError();
}

}  // namespace glc
