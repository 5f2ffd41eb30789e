// decode_wide.cu -- one persistent launch for the MoE feed-forward layer of a
// few decode tokens when the layer is "wide": a router too large to stage in
// shared memory (64 experts x 3584 x fp32 = 917 KB) and/or a Qwen2-MoE shared
// expert gated by sigmoid(x . g).
//
// Replaces, for the decode step, the chain router (external model code) ->
// GpuFirstExpertStageWorker.ProcessRoutedTopK (GpuFirstExpertStageWorker.cs:
// 416-583: per selected expert gate/up GEMV, SwiGLU, down GEMV, weighted
// accumulation) -> residual add (DistributedPipelineCoordinator.cs:104-134),
// plus the shared expert of the model code.
//
// Layout of one launch (one CTA per SM, all resident, 16 warps):
//   warp 15 (router): CTAs 2c and 2c + 1 compute the logit of expert c (the
//     shared-expert gate as column E) for every token in the canonical
//     reduction order of router.cu (256 strided fused partials -- here
//     virtual warps of one real warp, each lane running 4 of the partial
//     chains -- a xor butterfly per virtual warp, a pairwise tree over the
//     8), publishing the 8 virtual-warp sums as epoch-tagged 64-bit slots;
//     every CTA's router warp reads them (one memory round trip), ranks the
//     experts (ties to the lower index, NaN as -inf) and forms the softmax
//     weights exactly as router.cu, so ids and weights are bit-identical to it.
//     Its router column is loaded before the weight stream fills the memory
//     system: under a saturated stream every later memory round trip costs
//     several microseconds.
//   warp 14 (producer): streams this CTA's share of the SHARED expert's
//     gate/up rows first -- they do not depend on the routing, so the weight
//     stream starts at once and the routing is hidden behind it -- then,
//     once its router warp has the ids, its share of the routed experts'
//     gate/up rows, then the down-projection rows.  cp.async.bulk into a ring
//     of shared-memory stages on mbarriers, L2 evict-first, no multicast.
//   warps 0..13 (consumers): gate/up GEMV of the raw input (the lane math of
//     gemv_lane.cuh quantises each 32-block by its own maximum, so the norm
//     scale factors out of every row sum and is applied in the SwiGLU
//     epilogue), activations to global memory; grid
//     barrier; down projection: every output row is read as k routed slots
//     of F/64 lane units each plus the shared row of Fs/64 units, one lane per
//     unit (Qwen2-57B: 8 x 40 = 320 = 10 warps, and 320 for the shared row),
//     so each lane keeps one slot's activations in registers for the whole
//     phase; per-slot warp partial sums are added in a fixed order and
//     combined in k order: acc = resid; acc = (s_j * w_j) + acc ...;
//     acc = (s_shared * sigmoid gate) + acc (the oracle's order).
#include <algorithm>

#include "common.cuh"
#include "gemv_lane.cuh"
#include "kernels.h"

namespace glc {

namespace {

constexpr int kWConsumerWarps = 14;
constexpr int kWProducer = kWConsumerWarps;
constexpr int kWRouter = kWConsumerWarps + 1;
constexpr int kWThreads = (kWConsumerWarps + 2) * 32;
constexpr int kWNT = kWConsumerWarps * 32;
constexpr int kWMaxK = 16;
constexpr int kRouterThreadsC = 256;  // threads of the canonical router reduction

__device__ __forceinline__ int xs_index_w(int d, int U) {
    return (((d & 63) >> 2) * (U + 1) + (d >> 6)) * 4 + (d & 3);
}

__device__ __forceinline__ float rms_scale(float ss, int D) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), 1e-5f)));
}

// QW: the Qwen2-57B-A14B decode shape (one token, 64 experts, top-8, D = 3584,
// F = 2560, shared expert Fs = 20480) with wide_decode_configure's lane layout
// for it (gate/up: 2 lane segments, 6 warp groups, 12 stage rows; down: 4
// stage rows, slot units 40, shared units 320 on 10 + 10 warps, 2 partial
// sums per slot, 26 per row) built in as constants; the launch uses it only
// when the configured layout is exactly that.  Otherwise every value comes
// from the parameters.
template <bool QW>
__global__ void __launch_bounds__(kWThreads, 1) moe_decode_wide_kernel(const __grid_constant__ FusedDecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_ok, s_route_ok;
    __shared__ int s_ids[kFusedMaxTokens * kWMaxK];
    __shared__ float s_w[kFusedMaxTokens * kWMaxK];
    __shared__ float s_sg[kFusedMaxTokens];
    __shared__ float s_rms[kFusedMaxTokens];
    __shared__ float s_red[kFusedMaxTokens * 8];
    __shared__ float s_ex[64];
    __shared__ int s_rank[kWMaxK];
    float* xs = reinterpret_cast<float*>(smem + p.off_xs);
    float* pgu = reinterpret_cast<float*>(smem + p.off_pgu);
    float* pdn = reinterpret_cast<float*>(smem + p.off_pdn);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    const int S = p.stages;
    uint64_t* empty = full + S;
    uint64_t* route_mb = empty + S;  // the router warp's ids are in shared memory
    uint64_t* go_bar = route_mb + 1;  // the producer has issued its first ring's worth of stages
    uint64_t* xbar = go_bar + 1;      // the raw input has landed in shared memory
    float* xraw = reinterpret_cast<float*>(smem + p.off_red);  // [T][D] raw input

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int T = QW ? 1 : p.T, D = QW ? 3584 : p.D, F = QW ? 2560 : p.F, Fs = QW ? 20480 : p.Fs,
              k = QW ? 8 : p.k, E = QW ? 64 : p.E;
    const uint64_t lim = p.wait_limit_ns > 0 ? (uint64_t)p.wait_limit_ns : kWaitLimitNs;
    const int slot = p.slot_bytes;
    const int G = gridDim.x, b = blockIdx.x;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWConsumerWarps);
        }
        mbar_init(route_mb, 1);
        mbar_init(go_bar, 1);
        mbar_init(xbar, 1);
        fence_mbar_init();
        s_ok = 1;
        s_route_ok = 1;
        // the layer input in one bulk copy (the RMSNorm and the router read it)
        const uint32_t xb = (uint32_t)(p.T * p.D * 4);
        mbar_arrive_expect_tx(xbar, xb);
        bulk_g2s_nohint(xraw, p.x, xb, xbar);
    }
    __syncthreads();

    // work shares: gate/up rows of the shared expert [sh0, sh1) of T*Fs and of
    // the routed pairs [r0, r1) of T*k*F; down rows [q0, q1) of T*D
    const long long shTot = (long long)T * Fs, rTot = (long long)T * k * F, qTot = (long long)T * D;
    const int sh0 = (int)(shTot * b / G), sh1 = (int)(shTot * (b + 1) / G);
    const int r0 = (int)(rTot * b / G), r1 = (int)(rTot * (b + 1) / G);
    const int q0 = (int)(qTot * b / G), q1 = (int)(qTot * (b + 1) / G);
    const int nsh = sh1 - sh0;
    const int rbG = (D >> 8) * 144, rbD = (F >> 8) * 144, rbS = (Fs >> 8) * 144;

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

    if (warp == kWRouter) {
        // ------------------------------------------------------- router warp
        // Two CTAs per router column (expert c, or the shared gate as column
        // E): CTA 2c + h computes the partial sums of the 4 virtual warps
        // 4h .. 4h + 3 of the canonical 256-thread order (thread tid = 32 w +
        // lane runs d = tid, tid + 256, ... increasing, fused multiply-adds),
        // each reduced by the xor butterfly, and publishes them tagged with
        // the launch's epoch; every router warp then reads the 8 virtual-warp
        // sums of every column and adds them by the pairwise tree -- the
        // logits of router.cu bit for bit.  The router column is loaded before
        // the weight stream fills the memory system; the RMSNorm scale comes
        // from the staged input in shared memory.
        const bool has_gate = Fs > 0 && p.sh_gate_vec != nullptr;
        const int ncols = E + (has_gate ? 1 : 0);
        const int col = b >> 1, half = b & 1;
        unsigned long long prev = 0;
        if (lane == 0) prev = atomicAdd(p.route_bar, 1ull);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        const unsigned long long epoch = (prev / (unsigned long long)G + 1ull) & 0xFFFFFFFFull;
        bool rok = true;
        if (col < ncols) {
            constexpr int kRS = 14;  // d-steps of 256 held in registers per batch
            const float* wc = col < E ? p.Wr + col : p.sh_gate_vec;
            const size_t ws = col < E ? (size_t)E : 1;
            const int nsteps = D >> 8;
            float a[kFusedMaxTokens][4];
#pragma unroll
            for (int t = 0; t < kFusedMaxTokens; ++t)
#pragma unroll
                for (int w = 0; w < 4; ++w) a[t][w] = 0.f;
            float rms[kFusedMaxTokens];
            for (int s0 = 0; s0 < nsteps; s0 += kRS) {
                float wv[kRS][4];
#pragma unroll
                for (int s = 0; s < kRS; ++s)
#pragma unroll
                    for (int w = 0; w < 4; ++w) {
                        const int d = (s0 + s) * 256 + 32 * (4 * half + w) + lane;
                        wv[s][w] = (s0 + s < nsteps) ? __ldg(wc + (size_t)d * ws) : 0.f;
                    }
                if (s0 == 0) {
                    // the input has landed: RMSNorm scale of every token, canonical
                    if (!mbar_wait(xbar, 0, p.err, kDevTimeoutFull, lim)) { rok = false; break; }
#pragma unroll
                    for (int t = 0; t < kFusedMaxTokens; ++t) {
                        rms[t] = 1.0f;
                        if (t < T && p.rmsnorm) {
                            float q[8];
#pragma unroll
                            for (int w = 0; w < 8; ++w) q[w] = 0.f;
                            for (int s = 0; s < nsteps; ++s)
#pragma unroll
                                for (int w = 0; w < 8; ++w) {
                                    const float v = xraw[(size_t)t * D + s * 256 + 32 * w + lane];
                                    q[w] = fmaf(v, v, q[w]);
                                }
                            const float v = warp_tree8(q, lane);
                            float sw[8];
#pragma unroll
                            for (int w = 0; w < 8; ++w) sw[w] = __shfl_sync(0xffffffffu, v, 4 * w);
                            rms[t] = rms_scale(tree8(sw), D);
                        }
                    }
                }
#pragma unroll
                for (int s = 0; s < kRS; ++s)
                    if (s0 + s < nsteps)
#pragma unroll
                        for (int t = 0; t < kFusedMaxTokens; ++t)
                            if (t < T)
#pragma unroll
                                for (int w = 0; w < 4; ++w) {
                                    const float raw = xraw[(size_t)t * D + (s0 + s) * 256 + 32 * (4 * half + w) + lane];
                                    const float xv = p.rmsnorm ? __fmul_rn(raw, rms[t]) : raw;
                                    a[t][w] = fmaf(xv, wv[s][w], a[t][w]);
                                }
            }
            if (rok) {
#pragma unroll
                for (int t = 0; t < kFusedMaxTokens; ++t)
                    if (t < T) {
                        // zeros in values 4..7: lanes 4w (w < 4) hold virtual warp 4 half + w's sum
                        const float a8[8] = {a[t][0], a[t][1], a[t][2], a[t][3], 0.f, 0.f, 0.f, 0.f};
                        const float v = warp_tree8(a8, lane);
                        if ((lane & 3) == 0 && lane < 16) {
                            const unsigned long long tagged = (epoch << 32) | (unsigned long long)__float_as_uint(v);
                            unsigned long long* slot_p =
                                p.route_slots + ((size_t)t * (E + 1) + col) * 8 + 4 * half + (lane >> 2);
                            asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(slot_p), "l"(tagged) : "memory");
                        }
                    }
            }
        }
        // every column's 8 partial sums of this launch, then the top-k.  Each
        // 64-bit slot holds the epoch and the value together, so relaxed
        // loads suffice, and all of a lane's columns are polled in one loop
        // (one memory round trip when they are ready).
        const uint64_t t0 = global_timer_ns();
        for (int t = 0; t < T && rok; ++t) {
            const int ca = lane, cb = lane + 32;
            const unsigned long long* base = p.route_slots + (size_t)t * (E + 1) * 8;
            const bool wa = ca < E, wb = cb < E, wg = lane == 0 && has_gate;
            float sa[8], sb[8], sg8[8];
            bool got = false;
            while (true) {
                bool all = true;
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    unsigned long long va = 0, vb = 0, vg = 0;
                    if (wa) asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(va) : "l"(base + (size_t)ca * 8 + w) : "memory");
                    if (wb) asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(vb) : "l"(base + (size_t)cb * 8 + w) : "memory");
                    if (wg) asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(vg) : "l"(base + (size_t)E * 8 + w) : "memory");
                    all = all && (!wa || (va >> 32) == epoch) && (!wb || (vb >> 32) == epoch) && (!wg || (vg >> 32) == epoch);
                    sa[w] = __uint_as_float((uint32_t)va);
                    sb[w] = __uint_as_float((uint32_t)vb);
                    sg8[w] = __uint_as_float((uint32_t)vg);
                }
                if (all) { got = true; break; }
                if (global_timer_ns() - t0 > lim) break;
            }
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) atomicExch(p.err, kDevTimeoutGrid);
                rok = false;
                break;
            }
            const float la = wa ? tree8(sa) : 0.f, lb = wb ? tree8(sb) : 0.f, lg = wg ? tree8(sg8) : 0.f;
            const int ea = ca, eb = cb;
            const float va = (ea < E && !isnan(la)) ? la : -INFINITY;
            const float vb = (eb < E && !isnan(lb)) ? lb : -INFINITY;
            int ra = 0, rb = 0;
            for (int e = 0; e < E; ++e) {
                const float le = __shfl_sync(0xffffffffu, e < 32 ? la : lb, e & 31);
                const float v = isnan(le) ? -INFINITY : le;
                ra += (v > va || (v == va && e < ea)) ? 1 : 0;
                rb += (v > vb || (v == vb && e < eb)) ? 1 : 0;
            }
            if (ea < E && ra < k) s_rank[ra] = ea;
            if (eb < E && rb < k) s_rank[rb] = eb;
            __syncwarp();
            const int first = s_rank[0];
            const float lf = first < 32 ? __shfl_sync(0xffffffffu, la, first) : __shfl_sync(0xffffffffu, lb, first - 32);
            const float mx = isnan(lf) ? -INFINITY : lf;
            if (ea < E) s_ex[ea] = expf(la - mx);
            if (eb < E) s_ex[eb] = expf(lb - mx);
            __syncwarp();
            float den = 0.f;
            if (lane == 0) {
                if (p.renorm) {
                    for (int j = 0; j < k; ++j) den += s_ex[s_rank[j]];
                } else {
#pragma unroll 8
                    for (int e = 0; e < E; ++e) den += s_ex[e];
                }
            }
            den = __shfl_sync(0xffffffffu, den, 0);
            if (lane < k) {
                const int id = s_rank[lane];
                const float wv = s_ex[id] / den;
                s_ids[t * k + lane] = id;
                s_w[t * k + lane] = wv;
                if (b == 0) {
                    p.ids[t * k + lane] = id;
                    p.w[t * k + lane] = wv;
                }
            }
            if (lane == 0) s_sg[t] = has_gate ? 1.0f / (1.0f + expf(-lg)) : 0.f;
            __syncwarp();
        }
        if (!rok && lane == 0) s_route_ok = 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(route_mb);
        return;
    }

    if (warp == kWProducer) {
        // ------------------------------------------------------ producer warp
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            bool ok = true;
            int issued = 0;
            auto ring_wait = [&](int sidx, int& buf) {
                buf = sidx % S;
                const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                if (!mbar_wait_spin(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty, lim)) { ok = false; return false; }
                return true;
            };
            auto mark_issued = [&](int sidx) {
                issued = sidx + 1;
                if (sidx == S - 1) mbar_arrive(go_bar);
            };
            // shared-expert gate/up rows: no routing needed
            int nxt = for_each_stage_rows(Fs > 0 ? Fs : 1, 1, (QW ? 12 : p.gu_R), sh0, sh1, 0, [&](int sidx, int, int, int rin, int nr, int) {
                int buf;
                if (!ok || !ring_wait(sidx, buf)) return;
                const size_t off = (size_t)rin * rbG;
                const uint32_t bytes = (uint32_t)(nr * rbG);
                uint8_t* dst = smem + (size_t)buf * slot;
                mbar_arrive_expect_tx(&full[buf], 2u * bytes);
                bulk_g2s(dst, p.sh_gate + off, bytes, &full[buf], pol);
                bulk_g2s(dst + (size_t)(QW ? 12 : p.gu_R) * rbG, p.sh_up + off, bytes, &full[buf], pol);
                mark_issued(sidx);
            });
            // the routed rows need the ids
            if (ok && (!mbar_wait(route_mb, 0, p.err, kDevTimeoutFull, lim) || !s_route_ok)) ok = false;
            nxt = for_each_stage_rows(F, 1, (QW ? 12 : p.gu_R), r0, r1, nxt, [&](int sidx, int seg, int, int rin, int nr, int) {
                int buf;
                if (!ok || !ring_wait(sidx, buf)) return;
                const int e = clamp_expert(s_ids[seg], E);
                const size_t off = (size_t)e * p.gu_expert_bytes + (size_t)rin * rbG;
                const uint32_t bytes = (uint32_t)(nr * rbG);
                uint8_t* dst = smem + (size_t)buf * slot;
                mbar_arrive_expect_tx(&full[buf], 2u * bytes);
                bulk_g2s(dst, p.gate + off, bytes, &full[buf], pol);
                bulk_g2s(dst + (size_t)(QW ? 12 : p.gu_R) * rbG, p.up + off, bytes, &full[buf], pol);
                mark_issued(sidx);
            });
            if (issued < S) mbar_arrive(go_bar);  // fewer stages than the ring, or gave up
            // routed down rows: dn_R rows of each of the k slots
            nxt = for_each_stage_rows(D, 1, (QW ? 4 : p.dn_R), q0, q1, nxt, [&](int sidx, int t, int, int rin, int nr, int) {
                int buf;
                if (!ok || !ring_wait(sidx, buf)) return;
                const uint32_t bytes = (uint32_t)(nr * rbD);
                mbar_arrive_expect_tx(&full[buf], bytes * k);
                for (int j = 0; j < k; ++j) {
                    const int e = clamp_expert(s_ids[t * k + j], E);
                    bulk_g2s(smem + (size_t)buf * slot + (size_t)j * (QW ? 4 : p.dn_R) * rbD,
                             p.down + (size_t)e * p.dn_expert_bytes + (size_t)rin * rbD, bytes, &full[buf], pol);
                }
                issued = sidx + 1;
            });
            if (Fs > 0)
                for_each_stage_rows(D, 1, (QW ? 4 : p.dn_R), q0, q1, nxt, [&](int sidx, int, int, int rin, int nr, int) {
                    int buf;
                    if (!ok || !ring_wait(sidx, buf)) return;
                    const uint32_t bytes = (uint32_t)(nr * rbS);
                    mbar_arrive_expect_tx(&full[buf], bytes);
                    bulk_g2s(smem + (size_t)buf * slot, p.sh_down + (size_t)rin * rbS, bytes, &full[buf], pol);
                    issued = sidx + 1;
                });
            drain_issued_stages(full, S, issued, lim);
        }
        return;
    }

    // -------------------------------------------------------- consumer warps
    // The RAW input in the padded chunk-major layout the gate/up lanes read:
    // the lanes quantise it per 32-block (scale-free, so x and x * rms give
    // the same integers up to rounding) and the RMSNorm scale, a factor of
    // every gate/up row sum, is applied in the SwiGLU epilogue -- the weight
    // stream does not wait for the norm.
    {
        const int U = D >> 6;
        if (!mbar_wait_spin(xbar, 0, p.err, kDevTimeoutFull, lim)) s_ok = 0;
        for (int t = 0; t < T; ++t)
            for (int d = tid; d < D; d += kWNT) xs[(size_t)t * (D + 64) + xs_index_w(d, U)] = xraw[(size_t)t * D + d];
        named_bar_sync(1, kWNT);
    }
    // residual of this thread's first output row, loaded ahead of the end
    float resid0 = 0.f;
    if (p.resid && tid < q1 - q0) resid0 = __ldg(p.resid + (size_t)q0 + tid);

    bool ok = true;
    int nxt;
    {  // ---- gate/up + SwiGLU: the shared expert's rows, then the routed pairs'
        const int nsegw = (QW ? 2 : p.gu_nsegw), Gg = (QW ? 6 : p.gu_G);
        const bool wact = warp < nsegw * Gg;
        const int segw = warp % nsegw, grp = warp / nsegw;
        const int u = segw * 32 + lane;
        const bool active = wact && u < (D >> 8) * 4;
        const int sb = active ? (u >> 2) : 0, c = u & 3;
        XRegs xr;
        int cur = -1;
        if (!mbar_wait_spin(go_bar, 0, p.err, kDevTimeoutFull, lim)) ok = false;
        auto consume = [&](int sidx, int t, int nr, int lrow0) {
            if (!ok) return;
            if (t != cur) {
                load_x<kXShared>(xr, reinterpret_cast<const float4*>(xs + (size_t)t * (D + 64)) + u, (D >> 6) + 1, active);
                cur = t;
            }
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull, lim)) { ok = false; return; }
            if (wact)
                consume_stage(smem + (size_t)buf * slot, nr, (QW ? 12 : p.gu_R), 2, Gg, grp, rbG, sb, c, active, xr, lane,
                              [&](int i, int m, float v) { pgu[((size_t)(lrow0 + i) * 2 + m) * nsegw + segw] = v; });
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        };
        nxt = for_each_stage_rows(Fs > 0 ? Fs : 1, 1, (QW ? 12 : p.gu_R), sh0, sh1, 0,
                                  [&](int sidx, int t, int, int, int nr, int lr0) { consume(sidx, t, nr, lr0); });
        nxt = for_each_stage_rows(F, 1, (QW ? 12 : p.gu_R), r0, r1, nxt,
                                  [&](int sidx, int seg, int, int, int nr, int lr0) { consume(sidx, seg / k, nr, nsh + lr0); });
    }
    if (!ok) s_ok = 0;
    // RMSNorm scale of every token (canonical: 256 strided partials, warp
    // butterfly, pairwise tree), from the staged input
    if (tid < kRouterThreadsC && p.rmsnorm) {
        float a[kFusedMaxTokens];
#pragma unroll
        for (int t = 0; t < kFusedMaxTokens; ++t) a[t] = 0.f;
        for (int d = tid; d < D; d += kRouterThreadsC)
#pragma unroll
            for (int t = 0; t < kFusedMaxTokens; ++t)
                if (t < T) {
                    const float v = xraw[(size_t)t * D + d];
                    a[t] = fmaf(v, v, a[t]);
                }
#pragma unroll
        for (int t = 0; t < kFusedMaxTokens; ++t)
            if (t < T) {
                const float v = warp_tree(a[t]);
                if (lane == 0) s_red[t * 8 + warp] = v;
            }
    }
    named_bar_sync(1, kWNT);
    if (tid < T) s_rms[tid] = p.rmsnorm ? rms_scale(tree8(s_red + tid * 8), D) : 1.0f;
    named_bar_sync(1, kWNT);
    if (b == 0 && p.xin)
        for (int i = tid; i < T * D; i += kWNT) p.xin[i] = p.rmsnorm ? __fmul_rn(xraw[i], s_rms[i / D]) : xraw[i];
    {
        const int nsegw = (QW ? 2 : p.gu_nsegw);
        const int nrow = nsh + (r1 - r0);
        for (int lr = tid; lr < nrow; lr += kWNT) {
            const float* pp = pgu + (size_t)lr * 2 * nsegw;
            float gs = 0.f, us = 0.f;
            for (int q = 0; q < nsegw; ++q) { gs += pp[q]; us += pp[nsegw + q]; }
            const int tok = lr < nsh ? (sh0 + lr) / Fs : (r0 + (lr - nsh)) / F / k;
            gs = __fmul_rn(gs, s_rms[tok]);  // the row sums of the raw input, scaled by the norm
            us = __fmul_rn(us, s_rms[tok]);
            const float a = (gs / (1.0f + expf(-gs))) * us;
            if (lr < nsh) {
                const int g = sh0 + lr, t = g / Fs, rin = g - t * Fs;
                p.act_sh[(size_t)t * Fs + chunk_major_index(rin >> 6, rin & 63, Fs >> 6)] = a;
            } else {
                const int g = r0 + (lr - nsh), seg = g / F, rin = g - seg * F;
                p.act[(size_t)seg * F + chunk_major_index(rin >> 6, rin & 63, F >> 6)] = a;
            }
        }
    }
    named_bar_sync(1, kWNT);
    // ---- the activations grid-wide (every CTA arrives, even after a local
    // timeout, so the others are not held for the full wait limit)
    if (tid == 0) {
        if (b == p.stall_cta - 1) {
            s_ok = 0;  // failure-detection test: this CTA stays out of the barrier
        } else if (!grid_barrier(p.bar, gridDim.x, p.err, lim)) {
            s_ok = 0;
        }
    }
    named_bar_sync(1, kWNT);
    // the ids and weights (route_mb completed long before; this wait orders
    // the router warp's shared-memory writes before the reads below)
    if (!mbar_wait_spin(route_mb, 0, p.err, kDevTimeoutFull, lim) || !s_route_ok) ok = false;
    if (!s_ok || !ok) {
        signal_done();
        return;
    }

    const int PR = (QW ? 26 : p.dn_row_parts);
    // The shared row's lanes: unit L of Fs / 64 (its activations are loaded
    // when its sub-phase starts: holding both sets of activations at once
    // would not fit the registers).
    const int Us = (QW ? 320 : p.dn_Us);
    const int Ls = warp * 32 + lane;
    const bool act_s = Fs > 0 && warp < (QW ? 10 : p.dn_nws) && Ls < Us;
    XRegs xr_s;
    int cur_s = -1;
    auto load_shared_x = [&](int t) {
        load_x<kXGlobalCG>(xr_s, reinterpret_cast<const float4*>(p.act_sh + (size_t)t * Fs) + (act_s ? Ls : 0), Us, act_s);
        cur_s = t;
    };
    {  // ---- down projection, routed slots: lane unit L -> slot L / Ur, unit L % Ur
        const int Ur = (QW ? 40 : p.dn_Ur), Pr = (QW ? 2 : p.dn_Pr);
        const int L = warp * 32 + lane;
        const bool wact = warp < (QW ? 10 : p.dn_nwr);
        const int j = L / Ur, unit = L - (L / Ur) * Ur;
        const bool active = wact && j < k;
        const int jA = (warp * 32) / Ur;                // first slot in this warp
        const int partA = warp - (jA * Ur) / 32;         // this warp's part index of slot jA
        const bool hasB = (warp * 32 + 31) / Ur > jA && jA + 1 < k;
        const int sb = active ? (unit >> 2) : 0, c = unit & 3;
        XRegs xr;
        int cur = -1;
        nxt = for_each_stage_rows(D, 1, (QW ? 4 : p.dn_R), q0, q1, nxt, [&](int sidx, int t, int, int, int nr, int lr0) {
            if (!ok) return;
            if (t != cur) {
                load_x<kXGlobalCG>(xr, reinterpret_cast<const float4*>(p.act + (size_t)(t * k + (active ? j : 0)) * F) + unit,
                                   Ur, active);
                cur = t;
            }
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull, lim)) { ok = false; return; }
            if (wact) {
                const uint8_t* st = smem + (size_t)buf * slot + (size_t)(active ? j : 0) * (QW ? 4 : p.dn_R) * rbD;
                float va[4], vb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ii = i < nr ? i : nr - 1;
                    const float r = row_unit(st + (size_t)ii * rbD, sb, c, xr);
                    const float v = (active && i < nr) ? r : 0.f;
                    va[i] = (j == jA) ? v : 0.f;
                    vb[i] = (j == jA) ? 0.f : v;
                }
                const float ra = warp_reduce4(va, lane);
                const float rb = hasB ? warp_reduce4(vb, lane) : 0.f;
                if ((lane & 7) == 0) {
                    const int i = lane >> 3;
                    if (i < nr) {
                        float* pr = pdn + (size_t)(lr0 + i) * PR;
                        pr[jA * Pr + partA] = ra;
                        if (hasB) pr[(jA + 1) * Pr] = rb;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        });
    }
    if (Fs > 0) {  // ---- down projection, the shared row: lane unit L of Fs / 64
        const bool wact = warp < (QW ? 10 : p.dn_nws);
        const int sb = act_s ? (Ls >> 2) : 0, c = Ls & 3;
        for_each_stage_rows(D, 1, (QW ? 4 : p.dn_R), q0, q1, nxt, [&](int sidx, int t, int, int, int nr, int lr0) {
            if (!ok) return;
            if (t != cur_s) load_shared_x(t);
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull, lim)) { ok = false; return; }
            if (wact)
                consume_stage(smem + (size_t)buf * slot, nr, (QW ? 4 : p.dn_R), 1, 1, 0, rbS, sb, c, act_s, xr_s, lane,
                              [&](int i, int, float v) { pdn[(size_t)(lr0 + i) * PR + k * (QW ? 2 : p.dn_Pr) + warp] = v; });
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        });
    }
    if (!ok) s_ok = 0;
    named_bar_sync(1, kWNT);
    if (!s_ok) {
        signal_done();
        return;
    }
    {  // ---- combine in k order (+ residual, + gated shared expert)
        const int Ur = (QW ? 40 : p.dn_Ur), Pr = (QW ? 2 : p.dn_Pr);
        for (int lr = tid; lr < q1 - q0; lr += kWNT) {
            const int g = q0 + lr, t = g / D, rin = g - t * D;
            const size_t o = (size_t)t * D + rin;
            float acc = p.resid ? (lr == tid ? resid0 : p.resid[o]) : 0.f;
            const float* pr = pdn + (size_t)lr * PR;
            for (int jj = 0; jj < k; ++jj) {
                const int np = (jj * Ur + Ur - 1) / 32 - (jj * Ur) / 32 + 1;
                float s = 0.f;
                for (int q = 0; q < np; ++q) s += pr[jj * Pr + q];
                acc = __fadd_rn(__fmul_rn(s, s_w[t * k + jj]), acc);
            }
            if (Fs > 0) {
                float s = 0.f;
                for (int q = 0; q < (QW ? 10 : p.dn_nws); ++q) s += pr[k * Pr + q];
                acc = __fadd_rn(__fmul_rn(s, s_sg[t]), acc);
            }
            p.out[o] = acc;
        }
    }
    if (p.done_ctr) {
        named_bar_sync(1, kWNT);
        signal_done();
    }
}

size_t align16w(size_t v) { return (v + 15) & ~size_t(15); }

}  // namespace

int wide_decode_configure(FusedDecodeParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid) {
    const int T = p.T, D = p.D, F = p.F, E = p.E, k = p.k, Fs = p.Fs;
    if (T < 1 || T > kFusedMaxTokens || E < 1 || E > 64 || k < 1 || k > kWMaxK || k > E) return -1;
    if (D <= 0 || F <= 0 || (D & 255) || (F & 255) || Fs < 0 || (Fs & 255) || num_sms < 2 * (E + 1)) return -1;
    if (!p.gate || !p.up || !p.down || !p.act || !p.out || !p.ids || !p.w || !p.bar || !p.route_bar || !p.route_slots)
        return -1;
    if (Fs > 0 && (!p.sh_gate || !p.sh_up || !p.sh_down || !p.sh_gate_vec || !p.act_sh)) return -1;
    if (p.norm_w) return -1;  // the weighted RMSNorm is the fused kernel's only
    // gate/up lanes: D/64 units per row, whole warps per row
    const int gu_nsegw = ((D >> 6) + 31) / 32;
    if (gu_nsegw > kWConsumerWarps) return -1;
    // down lanes: k slots of F/64 units (each slot at least a warp wide, so a
    // warp holds parts of at most two slots) and the shared row's Fs/64 units
    const int Ur = F >> 6, Us = Fs >> 6;
    if (Ur < 32) return -1;
    const int nwr = (k * Ur + 31) / 32, nws = (Us + 31) / 32;
    if (nwr > kWConsumerWarps || nws > kWConsumerWarps) return -1;
    int Pr = 0;
    for (int j = 0; j < k; ++j) Pr = std::max(Pr, (j * Ur + Ur - 1) / 32 - (j * Ur) / 32 + 1);
    const int row_parts = k * Pr + (Fs > 0 ? nws : 0);
    const int rbG = (D >> 8) * 144, rbD = (F >> 8) * 144, rbS = (Fs >> 8) * 144;
    const int dn_R = 4;  // one pass of four row units per warp (one warp group)
    const size_t dn_stage = std::max((size_t)k * dn_R * rbD, (size_t)dn_R * rbS);
    const int g = num_sms;
    const long long gu_rows = ((long long)T * Fs + g - 1) / g + ((long long)T * k * F + g - 1) / g;
    const long long dn_rows = ((long long)T * D + g - 1) / g;
    size_t o = 0;
    const size_t o_xs = o;  o = align16w(o + (size_t)T * (D + 64) * 4);
    const size_t o_x = o;   o = align16w(o + (size_t)T * D * 4);
    const size_t o_pgu = o; o = align16w(o + (size_t)gu_rows * 2 * gu_nsegw * 4);
    const size_t o_pdn = o; o = align16w(o + (size_t)dn_rows * row_parts * 4);
    const size_t o_bars = o;
    const size_t fixed = o + (2 * 8 + 4) * 8;
    if (fixed >= smem_limit) return -1;
    // Warp groups of the gate/up phase: more groups make bigger stages, fewer
    // make more of them in the same shared memory.  The weight stream of each
    // phase is bounded by the bytes it keeps in flight (all stages but the one
    // being consumed), so pick the group count that minimises
    // sum over phases of phase bytes / bytes in flight.
    const double gu_bytes = (double)T * (Fs + (double)k * F) * 2 * rbG;
    const double dn_bytes = (double)T * D * ((double)k * rbD + (Fs > 0 ? rbS : 0));
    int gu_G = 0, S = 0;
    size_t slot = 0;
    double best = 0.0;
    for (int Gc = kWConsumerWarps / gu_nsegw; Gc >= 1; --Gc) {
        const size_t gu_stage = (size_t)2 * stage_rows_for(2, Gc) * rbG;
        const size_t sl = std::max(gu_stage, dn_stage);
        int Sc = (int)((smem_limit - fixed) / sl);
        if (Sc > 8) Sc = 8;
        if (Sc < 2) continue;
        const double cost = gu_bytes / ((double)(Sc - 1) * gu_stage) + dn_bytes / ((double)(Sc - 1) * dn_stage);
        if (gu_G == 0 || cost < best * 0.98) {
            gu_G = Gc; S = Sc; slot = sl; best = cost;
        }
    }
    if (gu_G == 0) return -1;
    if (((uintptr_t)p.x & 15u) || ((size_t)T * D * 4) >= (1u << 20)) return -1;  // one bulk copy of the input
    const int gu_R = stage_rows_for(2, gu_G);
    const size_t ring = (size_t)S * slot;
    p.wide = 1;
    p.gu_nsegw = gu_nsegw; p.gu_G = gu_G; p.gu_R = gu_R;
    p.dn_R = dn_R; p.dn_split = 0; p.dn_nsegw = 0; p.dn_G = 1;
    p.dn_Ur = Ur; p.dn_Pr = Pr; p.dn_nwr = nwr; p.dn_Us = Us; p.dn_nws = nws; p.dn_row_parts = row_parts;
    p.stages = S;
    p.slot_bytes = (int)slot;
    p.off_xs = (int)(ring + o_xs);
    p.off_red = (int)(ring + o_x);
    p.off_pgu = (int)(ring + o_pgu);
    p.off_pdn = (int)(ring + o_pdn);
    p.off_bars = (int)(ring + o_bars);
    *smem_bytes = ring + o_bars + (2 * (size_t)S + 4) * 8;
    *grid = g;
    return 0;
}

cudaError_t wide_decode_launch(const FusedDecodeParams& p0, int num_sms, cudaStream_t stream) {
    FusedDecodeParams p = p0;
    static int smem_optin[kMaxDevices] = {0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem_optin[dev] == 0) {
        int v = 0;
        e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        v -= 2048;  // the kernel's static shared memory comes out of the same budget
        for (auto kf : {moe_decode_wide_kernel<false>, moe_decode_wide_kernel<true>}) {
            e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
            if (e != cudaSuccess) return e;
        }
        smem_optin[dev] = v;
    }
    size_t smem = 0;
    int grid = 0;
    if (wide_decode_configure(p, num_sms, (size_t)smem_optin[dev], &smem, &grid) != 0) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kWThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid-wide waits need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool qw = p.T == 1 && p.D == 3584 && p.F == 2560 && p.Fs == 20480 && p.k == 8 && p.E == 64 &&
                    p.gu_nsegw == 2 && p.gu_G == 6 && p.gu_R == 12 && p.dn_R == 4 && p.dn_Ur == 40 && p.dn_Pr == 2 &&
                    p.dn_nwr == 10 && p.dn_Us == 320 && p.dn_nws == 10 && p.dn_row_parts == 26;
    return cudaLaunchKernelEx(&cfg, qw ? moe_decode_wide_kernel<true> : moe_decode_wide_kernel<false>, p);
}

}  // namespace glc
