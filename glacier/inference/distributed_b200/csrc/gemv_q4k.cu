// gemv_q4k.cu -- Q4_K dequant-fused GEMV for decode on sm_100a CUDA cores.
//
// Replaces QuantKernels.MatVecMul(Q4_K, ...) (external; call sites
// CpuWarmExpertPoolWorker.cs:379, GpuFirstExpertStageWorker.cs:734-737) and the
// D3D12 GemvQ4K / SwiGLU / VecAddWeighted dispatch chain of
// GpuFirstExpertStageWorker.ProcessRoutedTopK (GpuFirstExpertStageWorker.cs:482-519).
//
// Design (HBM-bound; ~0.56 byte per weight):
//   * Persistent CTAs, one per SM; each owns a contiguous, balanced range of the
//     flattened row space, so no wave-quantisation tail.
//   * A producer warp streams whole weight rows (contiguous GGUF rows: 2304 B at
//     K=4096, 8064 B at K=14336) into a ring of shared-memory stages with 1-D
//     bulk async copies (cp.async.bulk, TMA engine) completed on mbarriers,
//     with an L2 evict-first policy (weights are read once).
//   * Consumer warps never touch global weights; the lane math (int16
//     activations x 4-bit quants on dp2a) is in gemv_lane.cuh.
//   * Lane partials are reduced by warp shuffles, the per-segment sums are
//     kept in shared memory and summed in fixed order at the end (deterministic).
//   * Epilogues: plain store; gate/up pair -> SwiGLU act = silu(g)*u; down rows
//     of the k experts of a token -> weighted combine acc = (y*w)+acc in k order
//     (+ residual), i.e. AccumulatorStageWorker.AccumulateWeightedExpert.
//   * Down projection, when top-k divides the warp-group count: every stage
//     holds the same rows of all k selected experts (one copy each) and warp
//     group g computes slot g % k, keeping that slot's activations in
//     registers for the whole launch (no reload mid-stream, no half-empty
//     stage at each slot's end).  Each row's reduction order is unchanged.
#include <algorithm>

#include "common.cuh"
#include "gemv_lane.cuh"
#include "kernels.h"

// Pipeline shape knobs (stage count bound, L2 streaming hint).  A stage holds
// one pass of four row-units per warp; the ring takes as many stages as the
// shared-memory opt-in limit leaves room for after the partial sums, up to the
// bound.  At the Mixtral shapes a stage is 64.5 KB, so that is 3 stages: with
// 2, one stage loads while the other is consumed and the copies in flight
// cover only half the latency-bandwidth product of an SM.
#ifndef GLC_GEMV_MAX_STAGES
#define GLC_GEMV_MAX_STAGES 8
#endif
#ifndef GLC_GEMV_L2_HINT
#define GLC_GEMV_L2_HINT 1
#endif

namespace glc {

template <bool SPLIT, bool FIX, class F>
__device__ __forceinline__ void for_each_stage(const GemvParams& p, int R, int r0, int r1, F&& f) {
    for_each_stage_rows(p.rows, (!FIX && p.mode == kGemvDownCombine && !SPLIT) ? p.kslots : 1, R, r0, r1, 0, f);
}

// SPLIT: the slot-split down layout (p.split); NORM: the folded RMSNorm
// (p.norm_w); KK > 0: a plain one-input launch with K = KK, whose mode, lane
// layout and stage rows (gemv_configure's values) are then compile-time
// constants; separate instantiations so the other modes keep their code.
template <bool SPLIT, bool NORM, int KK>
__global__ void __launch_bounds__(kGemvMaxThreads, 1) q4k_gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool FIX = KK > 0;
    constexpr int kNsegw = FIX ? (((KK >> 8) * 4) + 31) / 32 : 0;
    constexpr int kG = FIX ? kGemvMaxConsumerWarps / kNsegw : 0;
    constexpr int kNw = FIX ? kNsegw * kG : 0;
    constexpr int kR = FIX ? 4 * kG : 0;  // stage_rows_for(1, G)
    const int NM = ((FIX ? (int)kGemvPlain : p.mode) == kGemvGateUp) ? 2 : 1;
    const int NMP = ((FIX ? (int)kGemvPlain : p.mode) == kGemvGateUp) ? 2 : ((FIX ? (int)kGemvPlain : p.mode) == kGemvDownCombine ? p.kslots : 1);
    const int NCP = SPLIT ? p.kslots : 1;  // expert copies per stage
    const int rowBytes = ((FIX ? KK : p.K) >> 8) * 144;
    const int R = (FIX ? kR : p.stage_rows);
    const int stage_bytes = NM * NCP * R * rowBytes;
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    float* part = reinterpret_cast<float*>(empty + S);
    float* nss = reinterpret_cast<float*>(smem + p.nss_off);  // [nsegw] sums of x^2 (norm_w set)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = (FIX ? kNw : p.nw);
    const long long total = (long long)(FIX ? 1 : p.nseg) * p.rows;
    const int r0 = (int)(total * blockIdx.x / gridDim.x);
    const int r1 = (int)(total * (blockIdx.x + 1) / gridDim.x);

    // The next programmatically serialised kernel of the stream may be
    // launched at once (its blocks take SMs as this grid's leave them, and it
    // waits for this grid's completion before it reads what this one writes):
    // its launch is then off the critical path.
    grid_dep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ------------------------------------------------------ producer warp
        // Launched behind another kernel with programmatic serialisation, the
        // weight stream of a plain GEMV starts at once (no kernel writes
        // weights); the other modes first wait for the expert ids.
        if ((FIX ? (int)kGemvPlain : p.mode) != kGemvPlain) grid_dep_wait();
        if (lane == 0) {
            const uint64_t pol = GLC_GEMV_L2_HINT ? l2_evict_first_policy() : 0ull;
            bool ok = true;
            int issued = 0;  // stages issued so far
            for_each_stage<SPLIT, FIX>(p, R, r0, r1, [&](int sidx, int seg, int j, int rin, int nr, int) {
                if (!ok) return;
                const int buf = sidx % S;
                const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                if (!mbar_wait_spin(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty)) { ok = false; return; }
                issued = sidx + 1;
                const uint8_t* srcA;
                const uint8_t* srcB = nullptr;
                if ((FIX ? (int)kGemvPlain : p.mode) == kGemvPlain) {
                    srcA = p.A + (size_t)rin * rowBytes;
                } else if ((FIX ? (int)kGemvPlain : p.mode) == kGemvGateUp) {
                    const int e = clamp_expert(__ldg(p.ids + seg), p.num_experts);
                    srcA = p.A + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                    srcB = p.B + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                } else if (!SPLIT) {
                    const int e = clamp_expert(__ldg(p.ids + seg * p.kslots + j), p.num_experts);
                    srcA = p.A + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                } else {
                    srcA = nullptr;  // one copy per slot below
                }
                const uint32_t bytes = (uint32_t)(nr * rowBytes);
                uint8_t* dst = smem + (size_t)buf * stage_bytes;
                if (SPLIT) {
                    mbar_arrive_expect_tx(&full[buf], bytes * NCP);
                    for (int c = 0; c < NCP; ++c) {
                        const int e = clamp_expert(__ldg(p.ids + seg * p.kslots + c), p.num_experts);
                        const uint8_t* src = p.A + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                        if (GLC_GEMV_L2_HINT) bulk_g2s(dst + (size_t)c * R * rowBytes, src, bytes, &full[buf], pol);
                        else bulk_g2s_nohint(dst + (size_t)c * R * rowBytes, src, bytes, &full[buf]);
                    }
                    return;
                }
                mbar_arrive_expect_tx(&full[buf], bytes * NM);
                if (GLC_GEMV_L2_HINT) {
                    bulk_g2s(dst, srcA, bytes, &full[buf], pol);
                    if (NM == 2) bulk_g2s(dst + (size_t)R * rowBytes, srcB, bytes, &full[buf], pol);
                } else {
                    bulk_g2s_nohint(dst, srcA, bytes, &full[buf]);
                    if (NM == 2) bulk_g2s_nohint(dst + (size_t)R * rowBytes, srcB, bytes, &full[buf]);
                }
            });
            // the copies in flight land before this warp, and so the CTA, exits
            drain_issued_stages(full, S, issued, kWaitLimitNs);
        }
        return;
    }

    // ---------------------------------------------------------- consumer warps
    const int nsegw = (FIX ? kNsegw : p.nsegw);
    const int segw = warp % nsegw, grp0 = warp / nsegw, G0 = NW / nsegw;
    // slot-split layout: group grp0 works on slot js of every stage, as group
    // grp of G per slot
    const int js = SPLIT ? grp0 % p.kslots : 0;
    const int G = SPLIT ? G0 / p.kslots : G0, grp = SPLIT ? grp0 / p.kslots : grp0;
    const int U = ((FIX ? KK : p.K) >> 8) * 4;
    const int u = segw * 32 + lane;
    const bool active = u < U;
    const int sb = active ? (u >> 2) : 0, c = u & 3;
    XRegs xr;
    int cur_x = -1;
    bool ok = true;
    grid_dep_wait();  // the input is the previous kernel's output
    // one input for the whole CTA (plain mode): staged once, coalesced, in the
    // partial-sum region before any partial sum is written
    const bool staged = (FIX ? (int)kGemvPlain : p.mode) == kGemvPlain && (FIX ? 1 : p.nseg) == 1;
    if (staged) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(part);
        stage_x_shared<kXGlobalRO>(p.x, NORM ? p.norm_w : nullptr, (FIX ? KK : p.K), xs, nss, threadIdx.x, NW * 32);
        named_bar_sync(1, NW * 32);
        read_x_shared(xr, xs, U, u, active);
        named_bar_sync(1, NW * 32);
        cur_x = 0;
    }
    for_each_stage<SPLIT, FIX>(p, R, r0, r1, [&](int sidx, int seg, int j, int, int nr, int lr0) {
        if (!ok) return;
        const int jj = SPLIT ? js : j;
        const int xid = ((FIX ? (int)kGemvPlain : p.mode) == kGemvPlain) ? 0
                        : ((FIX ? (int)kGemvPlain : p.mode) == kGemvGateUp ? seg / p.kslots : seg * p.kslots + jj);
        if (xid != cur_x) {
            if constexpr (NORM) {  // one segment: xid is 0
                float ss;
                load_x_norm<kXGlobalRO>(xr, reinterpret_cast<const float4*>(p.x) + 16 * u,
                                        reinterpret_cast<const float4*>(p.norm_w) + 16 * u, active, ss);
                ss = warp_tree(ss);
                if (grp0 == 0 && lane == 0) nss[segw] = ss;
            } else {
                load_x<kXGlobalRO>(xr, reinterpret_cast<const float4*>(p.x + (size_t)xid * (FIX ? KK : p.K)) + 16 * u, 1, active);
            }
            cur_x = xid;
        }
        const int buf = sidx % S;
        const uint32_t ph = (uint32_t)(sidx / S) & 1u;
        if (!mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull)) { ok = false; return; }
        const uint8_t* st = smem + (size_t)buf * stage_bytes + (SPLIT ? (size_t)js * R * rowBytes : 0);
        consume_stage(st, nr, R, NM, G, grp, rowBytes, sb, c, active, xr, lane, [&](int i, int m, float v) {
            const int slot = ((FIX ? (int)kGemvPlain : p.mode) == kGemvDownCombine) ? jj : m;
            part[((size_t)(lr0 + i) * NMP + slot) * nsegw + segw] = v;
        });
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
    });

    named_bar_sync(1, NW * 32);
    if (!ok) return;

    // ------------------------------------------------------------ epilogue
    float rinv = 1.0f;
    if constexpr (NORM) {
        float ss = 0.f;  // per-warp sums when staged, per-segment sums otherwise
        for (int q = 0; q < (staged ? NW : nsegw); ++q) ss += nss[q];
        rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)(FIX ? KK : p.K)), p.norm_eps)));
    }
    const int nrows = r1 - r0;
    for (int lr = threadIdx.x; lr < nrows; lr += NW * 32) {
        const int g = r0 + lr;
        const int seg = g / p.rows, rin = g - seg * p.rows;
        const float* pp = part + (size_t)lr * NMP * nsegw;
        if ((FIX ? (int)kGemvPlain : p.mode) == kGemvPlain) {
            float s = 0.f;
            for (int q = 0; q < nsegw; ++q) s += pp[q];
            p.y[rin] = NORM ? __fmul_rn(s, rinv) : s;
        } else if ((FIX ? (int)kGemvPlain : p.mode) == kGemvGateUp) {
            float gs = 0.f, us = 0.f;
            for (int q = 0; q < nsegw; ++q) { gs += pp[q]; us += pp[nsegw + q]; }
            if constexpr (NORM) {
                gs = __fmul_rn(gs, rinv);
                us = __fmul_rn(us, rinv);
            }
            p.y[(size_t)seg * p.rows + rin] = (gs / (1.0f + expf(-gs))) * us;
        } else {
            const size_t o = (size_t)seg * p.rows + rin;
            float acc = p.accumulate ? p.y[o] : (p.resid ? p.resid[o] : 0.f);
            for (int jj = 0; jj < p.kslots; ++jj) {
                float s = 0.f;
                for (int q = 0; q < nsegw; ++q) s += pp[jj * nsegw + q];
                acc = __fadd_rn(__fmul_rn(s, __ldg(p.cw + seg * p.kslots + jj)), acc);
            }
            p.y[o] = acc;
        }
    }
}

// ---------------------------------------------------------------- host side
int gemv_configure(GemvParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid) {
    if (p.K <= 0 || (p.K & 255) || p.rows <= 0 || p.nseg <= 0) return -1;
    const int U = (p.K >> 8) * 4;
    const int nsegw = (U + 31) / 32;
    if (nsegw > kGemvMaxConsumerWarps) return -1;  // K > 24576 not supported by the warp layout
    const int G = kGemvMaxConsumerWarps / nsegw;
    p.nsegw = nsegw;
    p.nw = nsegw * G;
    const int NM = (p.mode == kGemvGateUp) ? 2 : 1;
    const int NMP = (p.mode == kGemvGateUp) ? 2 : (p.mode == kGemvDownCombine ? p.kslots : 1);
    const int rowBytes = (p.K >> 8) * 144;
    p.split = (p.mode == kGemvDownCombine && p.kslots > 1 && G % p.kslots == 0) ? 1 : 0;
    const int NCP = p.split ? p.kslots : 1;
    p.stage_rows = stage_rows_for(NM, p.split ? G / p.kslots : G);  // one pass of four row-units per warp
    const size_t stage_bytes = (size_t)NM * NCP * p.stage_rows * rowBytes;
    const long long total = (long long)p.nseg * p.rows;
    int range_cap = (int)(16384 / (NMP * nsegw * 4));
    int g = num_sms;
    if ((total + g - 1) / g > range_cap) g = (int)((total + range_cap - 1) / range_cap);
    if (g > total) g = (int)total;
    if (p.norm_w && (p.nseg != 1 || p.mode == kGemvDownCombine)) return -1;
    // the per-CTA row sums, then the norm's per-segment sums of squares
    size_t part_bytes = (size_t)((total + g - 1) / g) * NMP * nsegw * sizeof(float);
    if (p.mode == kGemvPlain && p.nseg == 1) part_bytes = std::max(part_bytes, xs_bytes(p.K));  // staged input
    part_bytes += 32 * sizeof(float);
    const size_t per_stage = stage_bytes + 2 * sizeof(uint64_t);
    if (smem_limit < part_bytes + 2 * per_stage) return -1;
    int S = (int)((smem_limit - part_bytes) / per_stage);
    if (S > GLC_GEMV_MAX_STAGES) S = GLC_GEMV_MAX_STAGES;
    const size_t bytes = (size_t)S * per_stage + part_bytes;
    p.stages = S;
    p.nss_off = (int)(bytes - 32 * sizeof(float));
    *smem_bytes = bytes;
    *grid = g;
    return 0;
}

cudaError_t gemv_launch(const GemvParams& p0, int num_sms, cudaStream_t stream) {
    GemvParams p = p0;
    size_t smem = 0;
    int grid = 0;
    static int smem_optin[kMaxDevices] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (smem_optin[dev] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaError_t e = cudaSuccess;
        for (auto kf : {q4k_gemv_kernel<false, false, 0>, q4k_gemv_kernel<true, false, 0>, q4k_gemv_kernel<false, true, 0>,
                        q4k_gemv_kernel<false, false, 4096>, q4k_gemv_kernel<false, false, 14336>})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
        if (e != cudaSuccess) return e;
        smem_optin[dev] = v;
    }
    const size_t smem_limit = (size_t)smem_optin[dev];
    if (gemv_configure(p, num_sms, smem_limit, &smem, &grid) != 0) return cudaErrorInvalidValue;
    // Programmatic stream serialisation: a GEMV behind another kernel starts
    // on each SM as soon as that kernel's CTA there has left (and a plain
    // GEMV streams its weights at once), instead of after the whole grid
    // and a launch gap; the kernel waits before reading what came before.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((p.nw + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.split) return cudaLaunchKernelEx(&cfg, q4k_gemv_kernel<true, false, 0>, p);
    if (p.norm_w) return cudaLaunchKernelEx(&cfg, q4k_gemv_kernel<false, true, 0>, p);
    // a plain one-input GEMV at K = 4096 or 14336 (the Mixtral gate/up and
    // down rows): the instantiation with K built in, when the configured
    // layout is the one it derives
    if (p.mode == kGemvPlain && p.nseg == 1 && (p.K == 4096 || p.K == 14336)) {
        const int nsegw = ((p.K >> 8) * 4 + 31) / 32, G = kGemvMaxConsumerWarps / nsegw;
        if (p.nsegw == nsegw && p.nw == nsegw * G && p.stage_rows == 4 * G)
            return cudaLaunchKernelEx(&cfg, p.K == 4096 ? q4k_gemv_kernel<false, false, 4096>
                                                        : q4k_gemv_kernel<false, false, 14336>, p);
    }
    return cudaLaunchKernelEx(&cfg, q4k_gemv_kernel<false, false, 0>, p);
}

}  // namespace glc
