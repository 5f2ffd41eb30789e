// decode_fused.cu -- one persistent launch for the whole MoE feed-forward layer
// of a few decode tokens on sm_100a.
//
// Replaces, for the decode step, the chain the reference runs per token:
// router (external model code) -> GpuFirstExpertStageWorker.ProcessRoutedTopK
// (GpuFirstExpertStageWorker.cs:416-583: per selected expert GemvQ4K gate/up,
// SwiGLU, GemvQ4K down, VecAddWeighted) -> residual add
// (DistributedPipelineCoordinator.cs:104-134).
//
// Why one launch: the layer is HBM-bound (Mixtral-8x7B shape, top-2: 199 MB
// of Q4_K weights per token) and three launches leave the weight stream idle
// at every boundary (launch ramp, x staging behind the bulk-copy flood, epilogue
// tail).  Here every CTA (one per SM, all resident) does:
//   1. stages the router [D][E] and x [T][D] in shared memory with two bulk
//      copies, and computes RMSNorm + router logits + top-k itself, in the
//      canonical reduction order of router.cu (8 warps, 256 strided fused
//      partials, xor butterfly, pairwise tree) -- so no grid-wide exchange
//      is needed and every CTA holds the same bit-exact expert ids;
//   2. gate/up GEMV + SwiGLU over its balanced share of the (pair, F) rows,
//      weights streamed by a producer warp through a ring of shared-memory
//      stages (cp.async.bulk + mbarriers, L2 evict-first);
//   3. meanwhile the producer runs straight on into this CTA's down-projection
//      rows, so the ring is full of down weights when the consumers reach the
//      grid barrier that publishes the activations;
//   4. down GEMV over its share of the (token, D) rows, all k slots, then the
//      weighted combine in k order (+ residual).
// The lane math and the per-row reduction order are those of gemv_q4k.cu, so
// the results are bit-identical to the three-launch path.
#include <algorithm>

#include "common.cuh"
#include "gemv_lane.cuh"
#include "kernels.h"

#ifndef GLC_FUSED_MAX_STAGES
#define GLC_FUSED_MAX_STAGES 8
#endif
// Largest router split (CTAs per cluster sharing the router rows): 2 or 1
// (1 turns the split off).  Clusters of four cannot all be resident at one
// CTA per SM on B200's 148 SMs, so a four-way split would never launch.
#ifndef GLC_FUSED_RSPLIT
#define GLC_FUSED_RSPLIT 2
#endif

namespace glc {

namespace {

constexpr int kRouterWidth = 256;  // threads of the canonical router reduction (8 warps)

// Index, in floats, of element d of a token's normalised input in the padded
// chunk-major layout the gate/up lanes read: chunk i = (d % 64) / 4 of unit
// u = d / 64 is float4 number i * (U + 1) + u (U = D / 64 units; the one-unit
// pad per chunk row keeps both the router's writes and the lanes' 16-byte
// reads free of shared-memory bank conflicts).  A token takes D + 64 floats.
__device__ __forceinline__ int xs_index(int d, int U) {
    return (((d & 63) >> 2) * (U + 1) + (d >> 6)) * 4 + (d & 3);
}

// RMSNorm scale of every token, threads 0..255, from the raw input xr [T][D]:
// canonical sum of squares (256 strided fused partials, warp butterfly,
// pairwise tree over the 8 warp sums), then 1 / sqrt(ss / D + eps).
template <bool NW, int TT, int DD>
__device__ void router_rms(const FusedDecodeParams& p, const float* xr, float* red, float* rms_s, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int D = DD ? DD : p.D, T = TT ? TT : p.T;
    float a[kFusedMaxTokens];
#pragma unroll
    for (int t = 0; t < kFusedMaxTokens; ++t) a[t] = 0.f;
#pragma unroll 4
    for (int d = tid; d < D; d += kRouterWidth) {
#pragma unroll
        for (int t = 0; t < kFusedMaxTokens; ++t)
            if (t < T) {
                const float v = xr[(size_t)t * D + d];
                a[t] = fmaf(v, v, a[t]);
            }
    }
#pragma unroll
    for (int t = 0; t < kFusedMaxTokens; ++t)
        if (t < T) {
            const float v = warp_tree(a[t]);
            if (lane == 0) red[t * 8 + warp] = v;
        }
    named_bar_sync(2, kRouterWidth);
    const float eps = NW ? p.norm_eps : 1e-5f;
    if (tid < T) rms_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tree8(red + tid * 8), (float)D), eps)));
    named_bar_sync(2, kRouterWidth);
}

// Normalised input element d of token t: (raw * rms) * w[d] (NW: p.norm_w
// is set), as router.cu.
template <bool NW>
__device__ __forceinline__ float norm_in(const FusedDecodeParams& p, float raw, float rms, int d) {
    float v = p.rmsnorm ? __fmul_rn(raw, rms) : raw;
    if (NW) v = __fmul_rn(v, __ldg(p.norm_w + d));
    return v;
}

// Thread-block cluster primitives (the router split).  At kernel start every
// thread arrives (relaxed) and later waits once, so no CTA writes a peer's
// shared memory before that peer has started; the second phase publishes the
// partial logits.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(const float* local, uint32_t rank, float v) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// Router logits split over the R = 2 CTAs of a cluster, threads 0..255.
// The canonical order of router.cu is 256 strided partials (partial j sums
// d = j, j + 256, ... in order), a butterfly per warp and the pairwise tree
// ((w0+w1)+(w2+w3))+((w4+w5)+(w6+w7)) over the 8 warp sums.  CTA r computes
// the partials of canonical warps [4r, 4r+4) on threads 0..127, from the
// router rows those partials read (NL = 128 rows out of every 256, staged
// compactly: row 256i + r*NL + l at local row i*NL + l), reduces its four
// warps' subtree and stores it, for every (token, expert), into slot r of lh
// in both CTAs of the cluster; once the cluster barrier has passed, each CTA
// completes the tree from the two subtree values (logits_from_halves).
// Threads 128..255 write the normalised input of the d this CTA's partials
// do not visit.
template <bool NW, int TT, int EE, int DD>
__device__ void router_logits_split(const FusedDecodeParams& p, const float* Wl, const float* xr, float* xs,
                                    float* red, float* lh, const float* rms_s, int tid, int rank) {
    constexpr int R = 2, NL = kRouterWidth / R;
    const int warp = tid >> 5, lane = tid & 31;
    const int D = DD ? DD : p.D, E = EE ? EE : p.E, T = TT ? TT : p.T, U = D >> 6;
    if (tid >= NL) {
        const int t2 = tid - NL, o = t2 < rank * NL ? t2 : t2 + NL;  // the d this CTA's partials skip
        for (int t = 0; t < T; ++t) {
            const float* xt = xr + (size_t)t * D;
            float* xo = xs + (size_t)t * (D + 64);
            const float rms = p.rmsnorm ? rms_s[t] : 1.0f;
            for (int d = o; d < D; d += kRouterWidth) xo[xs_index(d, U)] = norm_in<NW>(p, xt[d], rms, d);
        }
        return;
    }
    const int h = (E == 8) ? ((lane >> 2) & 1) : 0;
    const int j = rank * NL + tid;  // canonical partial of this thread
    for (int t = 0; t < T; ++t) {
        const float* xt = xr + (size_t)t * D;
        float* xo = xs + (size_t)t * (D + 64);
        const float rms = p.rmsnorm ? rms_s[t] : 1.0f;
        for (int e0 = 0; e0 < E; e0 += 8) {
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.f;
            if ((E & 3) == 0 && e0 + 8 <= E) {
#pragma unroll 4
                for (int i = 0, d = j; d < D; ++i, d += kRouterWidth) {
                    const float xv = norm_in<NW>(p, xt[d], rms, d);
                    if (e0 == 0) xo[xs_index(d, U)] = xv;
                    const float4* wr = reinterpret_cast<const float4*>(Wl + (size_t)(i * NL + tid) * E + e0);
                    const float4 f = wr[h], g = wr[h ^ 1];
                    const float4 lo = h ? g : f, hi = h ? f : g;
                    acc[0] = fmaf(xv, lo.x, acc[0]); acc[1] = fmaf(xv, lo.y, acc[1]);
                    acc[2] = fmaf(xv, lo.z, acc[2]); acc[3] = fmaf(xv, lo.w, acc[3]);
                    acc[4] = fmaf(xv, hi.x, acc[4]); acc[5] = fmaf(xv, hi.y, acc[5]);
                    acc[6] = fmaf(xv, hi.z, acc[6]); acc[7] = fmaf(xv, hi.w, acc[7]);
                }
            } else {
                for (int i = 0, d = j; d < D; ++i, d += kRouterWidth) {
                    const float xv = norm_in<NW>(p, xt[d], rms, d);
                    if (e0 == 0) xo[xs_index(d, U)] = xv;
                    const float* wr = Wl + (size_t)(i * NL + tid) * E + e0;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (e0 + e < E) acc[e] = fmaf(xv, wr[e], acc[e]);
                }
            }
            const float v = warp_tree8(acc, lane);
            if ((lane & 3) == 0) red[((lane >> 2) & 7) * 8 + warp] = v;
            named_bar_sync(2, NL);
            if (tid < 8 && e0 + tid < E) {
                const float* s = red + tid * 8;
                const float c = (s[0] + s[1]) + (s[2] + s[3]);  // this CTA's four canonical warps
                float* dst = lh + (size_t)(t * E + e0 + tid) * R + rank;
                for (int r = 0; r < R; ++r) st_cluster_f32(dst, (uint32_t)r, c);
            }
            named_bar_sync(2, NL);
        }
    }
}

// Logit (t, e) from the two subtree values of the split: the top of the
// canonical pairwise tree.
__device__ __forceinline__ float logits_from_halves(const float* c) { return c[0] + c[1]; }

// Router logits of every token, threads 0..255, in the canonical order of
// router.cu (256 strided fused partials over the normalised input, warp
// butterfly, pairwise tree over the 8 warp sums), eight experts per pass; the
// first pass also writes the normalised input to xs (xs_index layout).
template <bool NW, int TT, int EE, int DD>
__device__ void router_logits(const FusedDecodeParams& p, const float* Wr, const float* xr, float* xs,
                              float* red, float* logit, const float* rms_s, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int D = DD ? DD : p.D, E = EE ? EE : p.E, T = TT ? TT : p.T, U = D >> 6;
    // At E = 8 rows are 32 B apart across lanes; lanes 4..7 of each 8 read
    // their second half first so one 16-byte read covers all banks.
    const int h = (E == 8) ? ((lane >> 2) & 1) : 0;
    for (int t = 0; t < T; ++t) {
        const float* xt = xr + (size_t)t * D;
        float* xo = xs + (size_t)t * (D + 64);
        const float rms = p.rmsnorm ? rms_s[t] : 1.0f;
        for (int e0 = 0; e0 < E; e0 += 8) {
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.f;
            if ((E & 3) == 0 && e0 + 8 <= E) {
#pragma unroll 4
                for (int d = tid; d < D; d += kRouterWidth) {
                    const float raw = xt[d];
                    const float xv = norm_in<NW>(p, raw, rms, d);
                    if (e0 == 0) xo[xs_index(d, U)] = xv;
                    const float4* wr = reinterpret_cast<const float4*>(Wr + (size_t)d * E + e0);
                    const float4 f = wr[h], g = wr[h ^ 1];
                    const float4 lo = h ? g : f, hi = h ? f : g;
                    acc[0] = fmaf(xv, lo.x, acc[0]); acc[1] = fmaf(xv, lo.y, acc[1]);
                    acc[2] = fmaf(xv, lo.z, acc[2]); acc[3] = fmaf(xv, lo.w, acc[3]);
                    acc[4] = fmaf(xv, hi.x, acc[4]); acc[5] = fmaf(xv, hi.y, acc[5]);
                    acc[6] = fmaf(xv, hi.z, acc[6]); acc[7] = fmaf(xv, hi.w, acc[7]);
                }
            } else {
                for (int d = tid; d < D; d += kRouterWidth) {
                    const float raw = xt[d];
                    const float xv = norm_in<NW>(p, raw, rms, d);
                    if (e0 == 0) xo[xs_index(d, U)] = xv;
                    const float* wr = Wr + (size_t)d * E + e0;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (e0 + e < E) acc[e] = fmaf(xv, wr[e], acc[e]);
                }
            }
            const float v = warp_tree8(acc, lane);
            if ((lane & 3) == 0) red[((lane >> 2) & 7) * 8 + warp] = v;
            named_bar_sync(2, kRouterWidth);
            if (tid < 8 && e0 + tid < E) logit[t * E + e0 + tid] = tree8(red + tid * 8);
            named_bar_sync(2, kRouterWidth);
        }
    }
}

// Top-k of token t by one warp (E <= 64: lane l ranks experts l and l+32),
// then the softmax weights.  An expert's rank is the number of experts ahead
// of it in the order (logit descending, lower index first on ties, NaN as
// -inf), so the experts of rank < k come out in the order of the router
// kernel's repeated arg-max in router.cu; the weights use the same expf
// arguments and the same sequential fp32 sums, so ids and weights are
// bit-identical to it.  ex holds E floats of scratch.
template <int KK, int EE>
__device__ void topk_token_warp(const FusedDecodeParams& p, const float* l, int t, int* s_ids, float* s_w,
                                float* ex, int lane) {
    const int E = EE ? EE : p.E, k = KK ? KK : p.k;
    const int e0 = lane, e1 = lane + 32;
    const float v0 = (e0 < E && !isnan(l[e0])) ? l[e0] : -INFINITY;
    const float v1 = (e1 < E && !isnan(l[e1])) ? l[e1] : -INFINITY;
    int r0 = 0, r1 = 0;
#pragma unroll 8
    for (int e = 0; e < E; ++e) {  // unrolled: the shared-memory reads overlap
        const float v = isnan(l[e]) ? -INFINITY : l[e];
        r0 += (v > v0 || (v == v0 && e < e0)) ? 1 : 0;
        r1 += (v > v1 || (v == v1 && e < e1)) ? 1 : 0;
    }
    if (e0 < E && r0 < k) s_ids[t * k + r0] = e0;
    if (e1 < E && r1 < k) s_ids[t * k + r1] = e1;
    __syncwarp();
    const int first = s_ids[t * k];
    const float mx = isnan(l[first]) ? -INFINITY : l[first];
    if (e0 < E) ex[e0] = expf(l[e0] - mx);
    if (e1 < E) ex[e1] = expf(l[e1] - mx);
    __syncwarp();
    float den = 0.f;
    if (lane == 0) {
        if (p.renorm) {
#pragma unroll 4
            for (int j = 0; j < k; ++j) den += ex[s_ids[t * k + j]];
        } else {
#pragma unroll 8
            for (int e = 0; e < E; ++e) den += ex[e];
        }
    }
    den = __shfl_sync(0xffffffffu, den, 0);
    if (lane < k) s_w[t * k + lane] = ex[s_ids[t * k + lane]] / den;
}

// SPLIT: the router split over a 2-CTA cluster (launched with clusters of
// two); NW: weighted RMSNorm (p.norm_w set); TT, KK, EE, DD, FF: the token
// count, top-k, expert count, hidden and expert widths when they are known at
// compile time, 0 = from p (with D, F and k known, so is the lane layout).
// Separate instantiations keep the unsplit, unweighted kernel's code exactly
// what it is without them (measured: folding the split and the weighted norm
// in as runtime branches cost 1.6 us per launch at the Mixtral-8x7B shape;
// the one-token instantiation saved 0.5 us).  PDL: launched programmatically
// serialised behind the kernel that writes its input (FusedDecodeParams::pdl):
// the router weights are staged before the kernel waits for that one.
template <bool SPLIT, bool NW, int TT, int KK, int EE, int DD, int FF, bool PDL = false>
__global__ void __launch_bounds__(kFusedThreads, 1) moe_decode_fused_kernel(const __grid_constant__ FusedDecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_ok, s_okx, s_okw;
    float* xs = reinterpret_cast<float*>(smem + p.off_xs);
    float* pgu = reinterpret_cast<float*>(smem + p.off_pgu);
    float* pdn = reinterpret_cast<float*>(smem + p.off_pdn);
    float* red = reinterpret_cast<float*>(smem + p.off_red);
    float* logit = reinterpret_cast<float*>(smem + p.off_logit);
    float* rms_s = reinterpret_cast<float*>(smem + p.off_rms);
    int* s_ids = reinterpret_cast<int*>(smem + p.off_ids);
    float* s_w = reinterpret_cast<float*>(smem + p.off_w);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    const int S = p.stages;
    uint64_t* empty = full + S;
    uint64_t* xbar = empty + S;
    uint64_t* wbar = xbar + 1;
    uint64_t* go_bar = wbar + 1;  // the producer has issued its first ring's worth of stages

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = TT ? TT : p.T, D = DD ? DD : p.D, F = FF ? FF : p.F, k = KK ? KK : p.k, P = T * k,
              E = EE ? EE : p.E;
    // lane layout: fused_decode_configure's values (its formulas, with
    // stage_rows_for(2, G) = 2G and stage_rows_for(1, G) = 4G) when D, F and k
    // are constants; read from p at each use otherwise
    constexpr int kGuNsegw = DD ? ((DD >> 8) * 4 + 31) / 32 : 0;
    constexpr int kGuG = DD ? kFusedConsumerWarps / kGuNsegw : 0;
    constexpr int kGuR = DD ? 2 * kGuG : 0;
    constexpr int kDnNsegw = FF ? ((FF >> 8) * 4 + 31) / 32 : 0;
    constexpr int kDnG = FF ? kFusedConsumerWarps / kDnNsegw : 0;
    constexpr int kDnSplit = (FF && KK) ? ((kDnG % KK) == 0 ? 1 : 0) : 0;
    constexpr int kDnR = (FF && KK) ? (kDnSplit ? 4 * (kDnG / KK) : 4 * kDnG) : 0;
    const uint64_t lim = p.wait_limit_ns > 0 ? (uint64_t)p.wait_limit_ns : kWaitLimitNs;
    const int slot = p.slot_bytes;
    constexpr int R = SPLIT ? 2 : 1;  // router split over a cluster of R CTAs
    float* lh = reinterpret_cast<float*>(smem + p.off_lh);
    if (R > 1) cluster_arrive_relaxed();
    if constexpr (PDL) grid_dep_launch_dependents();

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kFusedConsumerWarps);
        }
        mbar_init(xbar, 1);
        mbar_init(wbar, 1);
        mbar_init(go_bar, 1);
        fence_mbar_init();
        s_ok = s_okx = s_okw = 1;
    }
    __syncthreads();

    // ---- 1. stage x and the router in the (still idle) stage ring, each with
    // its own barrier so the sum of squares runs while the router lands; then
    // RMSNorm, logits and top-k (every CTA)
    // this CTA's router rows: all of them, or under the split the NL = 256/R
    // rows r*NL .. of every 256 (see router_logits_split), a multiple of 256 B
    const int rank = R > 1 ? (int)cluster_rank() : 0;
    const uint32_t wb = (uint32_t)D * E * 4u / (uint32_t)R;
    const float* xraw = reinterpret_cast<const float*>(smem + wb);
    if (tid == 0) {
        const uint32_t xb = (uint32_t)T * D * 4u;
        auto stage_router = [&]() {
            mbar_arrive_expect_tx(wbar, wb);
            if (R == 1) {
                bulk_g2s_nohint(smem, p.Wr, wb, wbar);
            } else {
                const int NL = kRouterWidth / R;
                const uint32_t blk = (uint32_t)NL * E * 4u;
                for (int i = 0; i < (D >> 8); ++i)
                    bulk_g2s_nohint(smem + (size_t)i * blk, p.Wr + ((size_t)i * kRouterWidth + (size_t)rank * NL) * E,
                                    blk, wbar);
            }
        };
        if constexpr (PDL) {  // the router weights never depend on the kernel before; the input does
            stage_router();
            grid_dep_wait();
            mbar_arrive_expect_tx(xbar, xb);
            bulk_g2s_nohint(smem + wb, p.x, xb, xbar);
        } else {
            mbar_arrive_expect_tx(xbar, xb);
            bulk_g2s_nohint(smem + wb, p.x, xb, xbar);
            stage_router();
        }
    }
    if constexpr (PDL) grid_dep_wait();  // every thread: what the kernel before wrote is visible
    // Every CTA reports its end when the caller waits on host memory (see
    // FusedDecodeParams::done_ctr): its writes become visible system-wide
    // first, and the CTA that completes a multiple of the grid size publishes
    // the error word and then the launch's epoch (count / grid), so the
    // launch needs no per-call parameter and can be replayed from a graph.
    auto signal_done = [&]() {
        if (p.done_ctr && tid == 0) {
            __threadfence_system();
            const unsigned long long prev = atomicAdd(p.done_ctr, 1ull);
            if ((prev + 1) % gridDim.x == 0) {
                __threadfence();
                *reinterpret_cast<volatile int*>(p.host_err) = *reinterpret_cast<volatile int*>(p.err);
                __threadfence_system();
                *reinterpret_cast<volatile unsigned long long*>(p.host_done) = (prev + 1) / gridDim.x;
            }
        }
    };
    // this CTA's rows, independent of the routing: computed while the copies fly
    const long long gu_total = (long long)P * F, dn_total = (long long)T * D;
    const int g0 = (int)(gu_total * blockIdx.x / gridDim.x);
    const int g1 = (int)(gu_total * (blockIdx.x + 1) / gridDim.x);
    const int q0 = (int)(dn_total * blockIdx.x / gridDim.x);
    const int q1 = (int)(dn_total * (blockIdx.x + 1) / gridDim.x);
    const int rbG = (D >> 8) * 144, rbD = (F >> 8) * 144;
    // The residual this thread adds in the final combine, loaded now so its
    // latency is not on the launch's last step (rows q0 + tid, one per thread
    // when the CTA has no more rows than consumer threads).
    constexpr int NT = kFusedConsumerWarps * 32;
    float resid0 = 0.f;
    if (p.resid && tid < NT && tid < q1 - q0) resid0 = __ldg(p.resid + (size_t)q0 + tid);
    if (tid < kRouterWidth) {
        if (R > 1) cluster_wait();  // every CTA of the cluster has started (its shared memory may be written)
        // Each wait's outcome goes through its own flag and a barrier of the
        // 256 router threads, so all of them take the same branch.
        if (!mbar_wait_spin(xbar, 0, p.err, kDevTimeoutFull, lim)) s_okx = 0;
        named_bar_sync(2, kRouterWidth);
        const bool okx = s_okx != 0;
        if (okx && p.rmsnorm) router_rms<NW, TT, DD>(p, xraw, red, rms_s, tid);
        if (okx && !mbar_wait_spin(wbar, 0, p.err, kDevTimeoutFull, lim)) s_okw = 0;
        named_bar_sync(2, kRouterWidth);
        if (okx && s_okw != 0) {
            if (R > 1)
                router_logits_split<NW, TT, EE, DD>(p, reinterpret_cast<const float*>(smem), xraw, xs, red, lh, rms_s, tid, rank);
            else
                router_logits<NW, TT, EE, DD>(p, reinterpret_cast<const float*>(smem), xraw, xs, red, logit, rms_s, tid);
        } else if (tid == 0) {
            s_ok = 0;
        }
    } else if (R > 1) {
        cluster_wait();
    }
    // Under the split, the cluster barrier publishes every CTA's partial
    // logits (and, as it includes all of this CTA's threads, orders the
    // CTA's own shared-memory writes); after it no CTA touches a peer's
    // shared memory, so any CTA may exit.
    if (R > 1)
        cluster_sync_all();
    else
        __syncthreads();
    const bool staged = s_ok != 0;
    if (staged && warp < T) {
        if (R > 1) {
            for (int e = lane; e < E; e += 32)
                logit[warp * E + e] = logits_from_halves(lh + (size_t)(warp * E + e) * R);
            __syncwarp();
        }
        topk_token_warp<KK, EE>(p, logit + warp * E, warp, s_ids, s_w, red + warp * 64, lane);
    }
    __syncthreads();
    if (!staged) {  // uniform: every thread read the same s_ok
        if (tid == 0) {  // the staging copies land (bounded) before the CTA exits
            mbar_wait_spin(xbar, 0, nullptr, 0, lim);
            mbar_wait_spin(wbar, 0, nullptr, 0, lim);
        }
        signal_done();
        return;
    }
    if (blockIdx.x == 0) {
        if (tid < P) {
            p.ids[tid] = s_ids[tid];
            p.w[tid] = s_w[tid];
        }
        if (p.xin)
            for (int i = tid; i < T * D; i += kFusedThreads) {
                const int t = i / D, d = i - t * D;
                p.xin[i] = xs[(size_t)t * (D + 64) + xs_index(d, D >> 6)];
            }
    }

    if (warp == kFusedConsumerWarps) {
        // ------------------------------------------------------ producer warp
        if (lane == 0) {
            fence_proxy_async_smem();  // router reads of the ring before bulk writes into it
            const uint64_t pol = l2_evict_first_policy();
            bool ok = true;
            int issued = 0;  // stages issued so far
            const int nxt = for_each_stage_rows(F, 1, (DD ? kGuR : p.gu_R), g0, g1, 0, [&](int sidx, int seg, int, int rin, int nr, int) {
                if (!ok) return;
                const int buf = sidx % S;
                const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                if (!mbar_wait_spin(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty, lim)) { ok = false; return; }
                const int e = clamp_expert(s_ids[seg], E);
                const size_t off = (size_t)e * p.gu_expert_bytes + (size_t)rin * rbG;
                const uint32_t bytes = (uint32_t)(nr * rbG);
                uint8_t* dst = smem + (size_t)buf * slot;
                mbar_arrive_expect_tx(&full[buf], 2u * bytes);
                bulk_g2s(dst, p.gate + off, bytes, &full[buf], pol);
                bulk_g2s(dst + (size_t)(DD ? kGuR : p.gu_R) * rbG, p.up + off, bytes, &full[buf], pol);
                issued = sidx + 1;
                if (sidx == S - 1) mbar_arrive(go_bar);
            });
            if (issued < S) mbar_arrive(go_bar);  // fewer stages than the ring, or gave up
            // Down-projection stages: with the slot-split layout a stage holds the
            // same dn_R rows of all k selected experts (one copy each), else dn_R
            // rows of one expert.
            const int nsl = ((FF && KK) ? kDnSplit : p.dn_split) ? 1 : k, ncp = ((FF && KK) ? kDnSplit : p.dn_split) ? k : 1;
            for_each_stage_rows(D, nsl, ((FF && KK) ? kDnR : p.dn_R), q0, q1, nxt, [&](int sidx, int seg, int j, int rin, int nr, int) {
                if (!ok) return;
                const int buf = sidx % S;
                const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                if (!mbar_wait_spin(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty, lim)) { ok = false; return; }
                const uint32_t bytes = (uint32_t)(nr * rbD);
                mbar_arrive_expect_tx(&full[buf], bytes * ncp);
                for (int c = 0; c < ncp; ++c) {
                    const int e = clamp_expert(s_ids[seg * k + j + c], E);
                    bulk_g2s(smem + (size_t)buf * slot + (size_t)c * ((FF && KK) ? kDnR : p.dn_R) * rbD,
                             p.down + (size_t)e * p.dn_expert_bytes + (size_t)rin * rbD, bytes, &full[buf], pol);
                }
                issued = sidx + 1;
            });
            // On every path (this warp gave up, the consumers abandoned the
            // ring after a failed grid barrier, or normal completion) the
            // copies of the last stages issued land before this warp, and so
            // the CTA, can exit.
            drain_issued_stages(full, S, issued, lim);
        }
        return;
    }

    // ---------------------------------------------------------- consumer warps
    bool ok = true;
    int nxt;
    {  // ---- 2. gate/up + SwiGLU
        const int nsegw = (DD ? kGuNsegw : p.gu_nsegw), G = (DD ? kGuG : p.gu_G);
        const bool wact = warp < nsegw * G;  // warps outside the layout only pace the ring
        const int segw = warp % nsegw, grp = warp / nsegw;
        const int u = segw * 32 + lane;
        const bool active = wact && u < (D >> 8) * 4;
        const int sb = active ? (u >> 2) : 0, c = u & 3;
        XRegs xr;
        int cur = -1;
        // The consumers' input loads start once the producer's first copies
        // are out: their shared-memory traffic would otherwise hold up the
        // producer's barrier and copy operations at the start of the stream.
        if (!mbar_wait_spin(go_bar, 0, p.err, kDevTimeoutFull, lim)) ok = false;
        nxt = for_each_stage_rows(F, 1, (DD ? kGuR : p.gu_R), g0, g1, 0, [&](int sidx, int seg, int, int, int nr, int lr0) {
            if (!ok) return;
            const int t = seg / k;
            if (t != cur) {
                load_x<kXShared>(xr, reinterpret_cast<const float4*>(xs + (size_t)t * (D + 64)) + u, (D >> 6) + 1, active);
                cur = t;
            }
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull, lim)) { ok = false; return; }
            if (wact)
                consume_stage(smem + (size_t)buf * slot, nr, (DD ? kGuR : p.gu_R), 2, G, grp, rbG, sb, c, active, xr, lane,
                              [&](int i, int m, float v) { pgu[((size_t)(lr0 + i) * 2 + m) * nsegw + segw] = v; });
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        });
    }
    if (!ok) s_ok = 0;
    named_bar_sync(1, NT);
    {
        const int nsegw = (DD ? kGuNsegw : p.gu_nsegw);
        for (int lr = tid; lr < g1 - g0; lr += NT) {
            const int g = g0 + lr, seg = g / F, rin = g - seg * F;
            const float* pp = pgu + (size_t)lr * 2 * nsegw;
            float gs = 0.f, us = 0.f;
            for (int q = 0; q < nsegw; ++q) { gs += pp[q]; us += pp[nsegw + q]; }
            // chunk-major, so that the down-projection lanes load it coalesced
            p.act[(size_t)seg * F + chunk_major_index(rin >> 6, rin & 63, F >> 6)] = (gs / (1.0f + expf(-gs))) * us;
        }
    }
    named_bar_sync(1, NT);
    // ---- 3. publish the activations grid-wide (every CTA arrives, even after
    // a local timeout, so the others are not held for the full wait limit)
    if (tid == 0) {
        if ((int)blockIdx.x == p.stall_cta - 1) {
            s_ok = 0;  // failure-detection test: this CTA stays out of the barrier
        } else {
            const bool gok = grid_barrier(p.bar, gridDim.x, p.err, lim);
            if (!gok) s_ok = 0;
        }
    }
    named_bar_sync(1, NT);
    if (!s_ok) {
        signal_done();
        return;
    }

    {  // ---- 4. down projection, all k slots of each row, then the combine
        const int nsegw = (FF ? kDnNsegw : p.dn_nsegw), G = (FF ? kDnG : p.dn_G);
        const bool wact = warp < nsegw * G;
        const int segw = warp % nsegw, grp = warp / nsegw;
        // slot-split layout: group grp works on slot grp % k of every stage
        // (its activations loaded once per token), as group grp / k of G / k
        const int js = ((FF && KK) ? kDnSplit : p.dn_split) ? grp % k : 0;
        const int Gs = ((FF && KK) ? kDnSplit : p.dn_split) ? G / k : G, gs = ((FF && KK) ? kDnSplit : p.dn_split) ? grp / k : grp;
        const int u = segw * 32 + lane;
        const bool active = wact && u < (F >> 8) * 4;
        const int sb = active ? (u >> 2) : 0, c = u & 3;
        XRegs xr;
        int cur = -1;
        for_each_stage_rows(D, ((FF && KK) ? kDnSplit : p.dn_split) ? 1 : k, ((FF && KK) ? kDnR : p.dn_R), q0, q1, nxt, [&](int sidx, int seg, int j0, int, int nr, int lr0) {
            if (!ok) return;
            const int j = ((FF && KK) ? kDnSplit : p.dn_split) ? js : j0;
            const int pair = seg * k + j;
            if (pair != cur) {
                load_x<kXGlobalCG>(xr, reinterpret_cast<const float4*>(p.act + (size_t)pair * F) + u, F >> 6, active);
                cur = pair;
            }
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull, lim)) { ok = false; return; }
            const uint8_t* st = smem + (size_t)buf * slot + (((FF && KK) ? kDnSplit : p.dn_split) ? (size_t)j * ((FF && KK) ? kDnR : p.dn_R) * rbD : 0);
            if (wact)
                consume_stage(st, nr, ((FF && KK) ? kDnR : p.dn_R), 1, Gs, gs, rbD, sb, c, active, xr, lane,
                              [&](int i, int, float v) { pdn[((size_t)(lr0 + i) * k + j) * nsegw + segw] = v; });
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        });
    }
    if (!ok) s_ok = 0;
    named_bar_sync(1, NT);
    if (!s_ok) {
        signal_done();
        return;
    }
    {
        const int nsegw = (FF ? kDnNsegw : p.dn_nsegw);
        for (int lr = tid; lr < q1 - q0; lr += NT) {
            const int g = q0 + lr, t = g / D, rin = g - t * D;
            const size_t o = (size_t)t * D + rin;
            float acc = p.resid ? (lr == tid ? resid0 : p.resid[o]) : 0.f;
            const float* pp = pdn + (size_t)lr * k * nsegw;
            for (int jj = 0; jj < k; ++jj) {
                float s = 0.f;
                for (int q = 0; q < nsegw; ++q) s += pp[jj * nsegw + q];
                acc = __fadd_rn(__fmul_rn(s, s_w[t * k + jj]), acc);
            }
            p.out[o] = acc;
        }
    }
    if (p.done_ctr) {
        named_bar_sync(1, NT);  // every consumer's output written before the CTA reports
        signal_done();
    }
}

size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Whether the configured launch has widths D, F and the lane layout that an
// instantiation with those widths (and p.k) derives at compile time.
bool layout_is(const FusedDecodeParams& p, int D, int F) {
    if (p.D != D || p.F != F || p.k < 1) return false;
    const int gn = ((D >> 8) * 4 + 31) / 32, gG = kFusedConsumerWarps / gn;
    const int dn = ((F >> 8) * 4 + 31) / 32, dG = kFusedConsumerWarps / dn;
    const int split = (dG % p.k == 0) ? 1 : 0;
    return p.gu_nsegw == gn && p.gu_G == gG && p.gu_R == 2 * gG && p.dn_nsegw == dn && p.dn_G == dG &&
           p.dn_split == split && p.dn_R == (split ? 4 * (dG / p.k) : 4 * dG);
}

// Whether grid / R clusters of R CTAs (kernel fn, smem bytes each) can all
// be resident at once; cached per device and shared-memory size.
bool clusters_fit(const void* fn, int dev, int R, size_t smem, int grid) {
    struct Entry {
        size_t smem;
        int clusters;
    };
    static Entry cache[kMaxDevices] = {};  // R = 2
    Entry& c = cache[dev];
    if (c.smem != smem) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kFusedThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = (unsigned)R;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = 1;
        cfg.attrs = a;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
        c.smem = smem;
        c.clusters = n;
    }
    return (long long)c.clusters * R >= grid;
}

}  // namespace

int fused_decode_configure(FusedDecodeParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid) {
    const int T = p.T, D = p.D, F = p.F, E = p.E, k = p.k;
    if (T < 1 || T > kFusedMaxTokens || E < 1 || E > 64 || k < 1 || k > 16 || k > E) return -1;
    if (D <= 0 || F <= 0 || (D & 255) || (F & 255) || num_sms < 1) return -1;
    if (((uintptr_t)p.x | (uintptr_t)p.Wr) & 15u) return -1;
    if (!p.gate || !p.up || !p.down || !p.act || !p.out || !p.ids || !p.w || !p.bar) return -1;
    const int gu_nsegw = ((D >> 8) * 4 + 31) / 32, dn_nsegw = ((F >> 8) * 4 + 31) / 32;
    if (gu_nsegw > kFusedConsumerWarps || dn_nsegw > kFusedConsumerWarps) return -1;
    const int gu_G = kFusedConsumerWarps / gu_nsegw, dn_G = kFusedConsumerWarps / dn_nsegw;
    const int rbG = (D >> 8) * 144, rbD = (F >> 8) * 144;
    // One pass of four row-units per warp per stage.  Down projection: when
    // top-k divides the group count, every stage holds the same rows of all k
    // selected experts and each group keeps one slot (slot-split layout).
    const int dn_split = (dn_G % k == 0) ? 1 : 0;
    const int gu_R = stage_rows_for(2, gu_G);
    const int dn_R = dn_split ? stage_rows_for(1, dn_G / k) : stage_rows_for(1, dn_G);
    const size_t slot = std::max((size_t)2 * gu_R * rbG, (size_t)(dn_split ? k : 1) * dn_R * rbD);
    const int g = num_sms;
    const long long P = (long long)T * k;
    const long long gu_rows = (P * F + g - 1) / g, dn_rows = ((long long)T * D + g - 1) / g;
    // everything but the ring, in order after it
    size_t o = 0;
    const size_t o_xs = o;    o = align16(o + (size_t)T * (D + 64) * 4);
    const size_t o_pgu = o;   o = align16(o + (size_t)gu_rows * 2 * gu_nsegw * 4);
    const size_t o_pdn = o;   o = align16(o + (size_t)dn_rows * k * dn_nsegw * 4);
    const size_t o_red = o;   o = align16(o + (size_t)kFusedMaxTokens * 64 * 4);
    const size_t o_logit = o; o = align16(o + (size_t)T * E * 4);
    const size_t o_rms = o;   o = align16(o + (size_t)T * 4);
    const size_t o_ids = o;   o = align16(o + (size_t)P * 4);
    const size_t o_w = o;     o = align16(o + (size_t)P * 4);
    const int R = p.rsplit > 1 ? p.rsplit : 1;
    if (R != 1 && R != 2) return -1;
    const size_t o_lh = o;    o = align16(o + (R > 1 ? (size_t)T * E * R * 4 : 0));
    const size_t o_bars = o;
    const size_t fixed = o + (2 * GLC_FUSED_MAX_STAGES + 3) * 8;
    if (fixed >= smem_limit) return -1;
    int S = (int)((smem_limit - fixed) / slot);
    if (S > GLC_FUSED_MAX_STAGES) S = GLC_FUSED_MAX_STAGES;
    if (S < 2) return -1;
    const size_t ring = (size_t)S * slot;
    const size_t wr_bytes = (size_t)D * E * 4 / R;  // this CTA's router rows
    if (wr_bytes + (size_t)T * D * 4 > ring) return -1;  // router rows and raw input are staged in the ring
    if ((size_t)T * D * 4 >= (1u << 20) || wr_bytes >= (1u << 20)) return -1;  // one mbarrier transaction each
    p.gu_nsegw = gu_nsegw; p.gu_G = gu_G; p.gu_R = gu_R;
    p.dn_nsegw = dn_nsegw; p.dn_G = dn_G; p.dn_R = dn_R; p.dn_split = dn_split;
    p.stages = S;
    p.slot_bytes = (int)slot;
    p.off_xs = (int)(ring + o_xs);
    p.off_pgu = (int)(ring + o_pgu);
    p.off_pdn = (int)(ring + o_pdn);
    p.off_red = (int)(ring + o_red);
    p.off_logit = (int)(ring + o_logit);
    p.off_rms = (int)(ring + o_rms);
    p.off_ids = (int)(ring + o_ids);
    p.off_w = (int)(ring + o_w);
    p.off_lh = (int)(ring + o_lh);
    p.rsplit = R;
    p.off_bars = (int)(ring + o_bars);
    *smem_bytes = ring + o_bars + (2 * (size_t)S + 3) * 8;
    *grid = g;
    return 0;
}

cudaError_t fused_decode_launch(const FusedDecodeParams& p0, int num_sms, cudaStream_t stream) {
    // a shared expert, or a router too large to stage: the wide kernel
    if (p0.Fs > 0) return wide_decode_launch(p0, num_sms, stream);
    FusedDecodeParams p = p0;
    // the kernel instantiations: [split][weighted norm][one token]
    using Kernel = void (*)(FusedDecodeParams);
    static const Kernel kernels[2][2][2] = {
        {{moe_decode_fused_kernel<false, false, 0, 0, 0, 0, 0>, moe_decode_fused_kernel<false, false, 1, 0, 0, 0, 0>},
         {moe_decode_fused_kernel<false, true, 0, 0, 0, 0, 0>, moe_decode_fused_kernel<false, true, 1, 0, 0, 0, 0>}},
        {{moe_decode_fused_kernel<true, false, 0, 0, 0, 0, 0>, moe_decode_fused_kernel<true, false, 1, 0, 0, 0, 0>},
         {moe_decode_fused_kernel<true, true, 0, 0, 0, 0, 0>, moe_decode_fused_kernel<true, true, 1, 0, 0, 0, 0>}}};
    // Mixtral-8x7B decode (one token, top-2 of 8 experts, D = 4096, F = 14336,
    // unsplit, unweighted norm), the same routing at other widths, and a
    // Mixtral-8x22B decoder layer's feed-forward (D = 6144, F = 16384: the
    // router split, the weighted norm)
    static const Kernel mixtral_decode = moe_decode_fused_kernel<false, false, 1, 2, 8, 4096, 14336>;
    static const Kernel top2of8_decode = moe_decode_fused_kernel<false, false, 1, 2, 8, 0, 0>;
    static const Kernel mixtral22b_ffn = moe_decode_fused_kernel<true, true, 1, 2, 8, 6144, 16384>;
    static const Kernel mixtral_decode_pdl = moe_decode_fused_kernel<false, false, 1, 2, 8, 4096, 14336, true>;
    static int smem_optin[kMaxDevices] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem_optin[dev] == 0) {
        int v = 0;
        e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        // static __shared__ of the kernel (s_ok) comes out of the same budget
        v -= 1024;
        for (int s = 0; s < 2; ++s)
            for (int w = 0; w < 2; ++w)
                for (int t = 0; t < 2; ++t) {
                    e = cudaFuncSetAttribute(kernels[s][w][t], cudaFuncAttributeMaxDynamicSharedMemorySize, v);
                    if (e != cudaSuccess) return e;
                }
        for (Kernel kf : {mixtral_decode, top2of8_decode, mixtral22b_ffn, mixtral_decode_pdl}) {
            e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
            if (e != cudaSuccess) return e;
        }
        smem_optin[dev] = v;
    }
    const int nw = p.norm_w ? 1 : 0, one = p.T == 1 ? 1 : 0;
    // The smallest router split R (1, then 2 when GLC_FUSED_RSPLIT allows)
    // for which the layer fits and all grid / R clusters of R CTAs can be
    // resident at once (the grid barrier needs every CTA resident).  No split
    // when the router fits: measured on B200 at the Mixtral-8x7B shape, the
    // split launch took 46.5-46.6 us per step against 45.3 us unsplit (same
    // box); it is what lets a router of twice the rows (Mixtral-8x22B,
    // D = 6144) run in one launch at all.
    size_t smem = 0;
    int grid = 0, R = 1;
    for (; R <= GLC_FUSED_RSPLIT; R <<= 1) {
        p.rsplit = R;
        if (fused_decode_configure(p, num_sms, (size_t)smem_optin[dev], &smem, &grid) != 0) continue;
        if (R == 1 || (grid % R == 0 && clusters_fit((const void*)kernels[1][nw][one], dev, R, smem, grid))) break;
    }
    if (R > GLC_FUSED_RSPLIT) return wide_decode_launch(p0, num_sms, stream);  // cudaErrorNotSupported when that does not fit either
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    const bool top2of8 = p.T == 1 && p.k == 2 && p.E == 8;
    // (a fixed-width instantiation only when the configured lane layout is the one it has built in)
    Kernel kf = kernels[R > 1 ? 1 : 0][nw][one];
    if (top2of8 && R == 1 && !nw)
        kf = layout_is(p, 4096, 14336) ? mixtral_decode : top2of8_decode;
    else if (top2of8 && R == 2 && nw && layout_is(p, 6144, 16384))
        kf = mixtral22b_ffn;
    // programmatic serialisation behind the input's writer only where the
    // instantiation waits for it (the others run in plain stream order)
    const bool pdl = p.pdl && kf == mixtral_decode;
    if (pdl) kf = mixtral_decode_pdl;
    cudaLaunchAttribute attr[3];
    int na = 0;
    attr[na].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barrier needs it
    attr[na++].val.cooperative = 1;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (R > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)R;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kf, p);
}

}  // namespace glc
