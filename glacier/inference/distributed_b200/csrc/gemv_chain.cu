// gemv_chain.cu -- a chain of Q4_K GEMVs in one persistent launch on sm_100a.
//
// The sequence of MatVecMul calls a decode step makes (the D3D12 GemvQ4K /
// SwiGLU / VecAddWeighted dispatch chain of GpuFirstExpertStageWorker.
// ProcessRoutedTopK, GpuFirstExpertStageWorker.cs:482-519; QuantKernels.
// MatVecMul, call shape CpuWarmExpertPoolWorker.cs:379) as ONE launch: each
// job is y = W x, y += W x, or y = SiLU(Wg x) * (Wu x), optionally on an
// RMSNorm'd input, and a job may read what earlier jobs wrote.
//
// Why one launch: a stand-alone GEMV streams its weights at the HBM rate only
// between its ramp and its tail; back to back, each launch's consumers must
// wait for the whole previous grid before they read their input, so every
// launch pays the slowest CTA of the one before plus a ramp.  Here one
// producer warp per SM streams the weight rows of ALL jobs through the
// shared-memory ring (weights never depend on activations), and only the
// consumer warps stop at the grid-wide barrier in front of a job whose input
// is an earlier job's output -- by then the ring already holds that job's
// first stages, so the consumers resume at compute speed while the copies
// catch up.  Measured per dependent job boundary on B200: ~2 us barrier
// (the slowest CTA's arrival and the polls) and ~1.5 us input staging.
//
// Per job the layout is the stand-alone GEMV's (gemv_q4k.cu, gemv_lane.cuh):
// lane u of a row owns one 32-byte quant chunk, nsegw warps cover a row, G
// groups of warps take four row-units per stage; rows of a job are split
// evenly over the CTAs.  A job's input is staged once per CTA
// (stage_x_shared: coalesced reads, int16 codes in shared memory) and each
// row's reduction order is the stand-alone kernel's, so a job's output is
// bit-identical to glc_gemv_q4k_dev's.  Launched cooperatively (all CTAs
// resident, one per SM) and programmatically serialised behind the kernel
// before it.
#include <algorithm>

#include "common.cuh"
#include "gemv_lane.cuh"
#include "kernels.h"

namespace glc {

namespace {

constexpr int kChainWarps = kGemvMaxConsumerWarps;      // consumer warps
constexpr int kChainThreads = (kChainWarps + 1) * 32;   // + the producer warp
constexpr int kNormSlots = 32;                          // per-warp sums of x^2 of a normed job
// (Measured on B200 with the input staged: holding the producer back at a
// dependent job until the consumers hold its input, or prefetching the
// stages beyond the ring into L2 so that HBM keeps streaming through the
// wait, made both GEMV shapes slower; the ring runs free.)
// KK, OPK: every job's K and op when the launch's jobs share them (known at
// compile time: the lane layout and loop bounds become constants), 0 / -1 =
// each job's own.
template <int KK, int OPK>
__device__ __forceinline__ void job_layout(const GemvJob& jb, int& nsegw, int& G, int& R, int& NM, int& rowBytes) {
    const int K = KK ? KK : jb.K;
    const int U = (K >> 8) * 4;
    nsegw = (U + 31) / 32;
    G = kChainWarps / nsegw;
    NM = ((OPK >= 0 ? OPK : (int)jb.op) == kChainGateUp) ? 2 : 1;
    R = stage_rows_for(NM, G);
    rowBytes = (K >> 8) * 144;
}

template <int KK, int OPK>
__global__ void __launch_bounds__(kChainThreads, 1) q4k_gemv_chain_kernel(const __grid_constant__ GemvChainParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * p.slot_bytes);
    uint64_t* empty = full + S;
    float* nss = reinterpret_cast<float*>(empty + S);  // [kNormSlots] per-warp sums of x^2
    // (dynamic shared memory only: the opt-in limit is set for the dynamic size)
    int& s_ok = *reinterpret_cast<int*>(nss + kNormSlots);
    // one region, used in turn: the staged input (xs_bytes(K)) while the
    // lanes read it, then the job's per-row partial sums (p.part_floats)
    float* part = nss + kNormSlots + 4;
    uint32_t* xs = reinterpret_cast<uint32_t*>(part);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    grid_dep_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kChainWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kChainWarps) {
        // ---------------------------------------------------- producer warp
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int sidx = 0;
            bool ok = true;
            for (int j = 0; j < p.njobs && ok; ++j) {
                const GemvJob& jb = p.jobs[j];
                int nsegw, G, R, NM, rowBytes;
                job_layout<KK, OPK>(jb, nsegw, G, R, NM, rowBytes);
                const int r0 = (int)((long long)jb.N * blockIdx.x / gridDim.x);
                const int r1 = (int)((long long)jb.N * (blockIdx.x + 1) / gridDim.x);
                for (int c = r0; c < r1 && ok; c += R) {
                    const int nr = min(R, r1 - c);
                    const int buf = sidx % S;
                    const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                    if (!mbar_wait_spin(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty)) { ok = false; break; }
                    ++sidx;
                    const uint32_t bytes = (uint32_t)(nr * rowBytes);
                    uint8_t* dst = smem + (size_t)buf * p.slot_bytes;
                    mbar_arrive_expect_tx(&full[buf], bytes * NM);
                    bulk_g2s(dst, jb.A + (size_t)c * rowBytes, bytes, &full[buf], pol);
                    if (NM == 2) bulk_g2s(dst + (size_t)R * rowBytes, jb.B + (size_t)c * rowBytes, bytes, &full[buf], pol);
                }
            }
            // the copies in flight land before this warp, and so the CTA, exits
            drain_issued_stages(full, S, sidx, kWaitLimitNs);
        }
        return;
    }

    // ------------------------------------------------------ consumer warps
    grid_dep_wait();  // the first job's input may be the previous kernel's output
    int sidx = 0;
    bool ok = true;
    for (int j = 0; j < p.njobs; ++j) {
        const GemvJob& jb = p.jobs[j];
        int nsegw, G, R, NM, rowBytes;
        job_layout<KK, OPK>(jb, nsegw, G, R, NM, rowBytes);
        const int r0 = (int)((long long)jb.N * blockIdx.x / gridDim.x);
        const int r1 = (int)((long long)jb.N * (blockIdx.x + 1) / gridDim.x);
        // the previous job's epilogue has read the region (partial sums)
        named_bar_sync(1, kChainWarps * 32);
        if (jb.after_previous && j > 0) {
            // every CTA's outputs of the earlier jobs before this job's input
            if (threadIdx.x == 0) s_ok = (ok && grid_barrier(p.bar, gridDim.x, p.err)) ? 1 : 0;
            named_bar_sync(1, kChainWarps * 32);
            if (!s_ok) ok = false;  // the barrier gave up (recorded): no further waits, no stores
        }
        const int segw = warp % nsegw, grp = warp / nsegw;
        const bool in_layout = grp < G;
        const int U = ((KK ? KK : jb.K) >> 8) * 4;
        const int u = segw * 32 + lane;
        const bool active = in_layout && u < U;
        const int sb = active ? (u >> 2) : 0, c = u & 3;
        XRegs xr;
        stage_x_shared<kXGlobalCG>(jb.x, jb.norm_w, (KK ? KK : jb.K), xs, nss, threadIdx.x, kChainWarps * 32);
        named_bar_sync(1, kChainWarps * 32);
        read_x_shared(xr, xs, U, u, active);
        float rinv = 1.0f;
        if (jb.norm_w) {
            float ss = 0.f;
            for (int q = 0; q < kChainWarps; ++q) ss += nss[q];
            rinv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)(KK ? KK : jb.K)), jb.norm_eps)));
        }
        named_bar_sync(1, kChainWarps * 32);  // every lane holds its input: the region takes partial sums now
        for (int c0 = r0; c0 < r1; c0 += R) {
            const int nr = min(R, r1 - c0);
            const int buf = sidx % S;
            const uint32_t ph = (uint32_t)(sidx / S) & 1u;
            ++sidx;
            if (ok && !mbar_wait_spin(&full[buf], ph, p.err, kDevTimeoutFull)) ok = false;
            if (ok && in_layout) {
                const uint8_t* st = smem + (size_t)buf * p.slot_bytes;
                const int lr0 = c0 - r0;
                consume_stage(st, nr, R, NM, G, grp, rowBytes, sb, c, active, xr, lane, [&](int i, int m, float v) {
                    part[((size_t)(lr0 + i) * NM + m) * nsegw + segw] = v;
                });
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        }
        named_bar_sync(1, kChainWarps * 32);  // the job's partial sums are in place
        if (ok) {
            for (int lr = threadIdx.x; lr < r1 - r0; lr += kChainWarps * 32) {
                const float* pp = part + (size_t)lr * NM * nsegw;
                const int row = r0 + lr;
                if (NM == 2) {
                    float gs = 0.f, us = 0.f;
                    for (int q = 0; q < nsegw; ++q) { gs += pp[q]; us += pp[nsegw + q]; }
                    if (jb.norm_w) {
                        gs = __fmul_rn(gs, rinv);
                        us = __fmul_rn(us, rinv);
                    }
                    jb.y[row] = (gs / (1.0f + expf(-gs))) * us;
                } else {
                    float s = 0.f;
                    for (int q = 0; q < nsegw; ++q) s += pp[q];
                    if (jb.norm_w) s = __fmul_rn(s, rinv);
                    // y += W x as the down-combine epilogue with one unit-weight slot: (s * 1) + y
                    jb.y[row] = ((OPK >= 0 ? OPK : (int)jb.op) == kChainAdd) ? __fadd_rn(__fmul_rn(s, 1.0f), jb.y[row]) : s;
                }
            }
        }
    }
}

}  // namespace

size_t gemv_chain_smem_bytes(const GemvChainParams& p) {
    return (size_t)p.stages * (p.slot_bytes + 2 * sizeof(uint64_t)) + (kNormSlots + 4) * sizeof(float) +
           (size_t)p.part_floats * sizeof(float);
}

// Fills the derived fields (ring shape, partial-sum space) and checks the jobs.
int gemv_chain_configure(GemvChainParams& p, int grid, size_t smem_limit, size_t* smem_bytes) {
    if (p.njobs <= 0 || p.njobs > kMaxChainJobs || grid <= 0) return -1;
    int slot = 0, part = 0;  // part: floats of the shared region (partial sums or the staged input)
    for (int j = 0; j < p.njobs; ++j) {
        const GemvJob& jb = p.jobs[j];
        if (jb.K <= 0 || (jb.K & 255) || jb.N <= 0 || !jb.A || !jb.x || !jb.y) return -1;
        if (jb.op != kChainSet && jb.op != kChainAdd && jb.op != kChainGateUp) return -1;
        if (jb.op == kChainGateUp && !jb.B) return -1;
        const int U = (jb.K >> 8) * 4;
        const int nsegw = (U + 31) / 32;
        if (nsegw > kChainWarps || nsegw > kNormSlots) return -1;
        const int G = kChainWarps / nsegw;
        const int NM = (jb.op == kChainGateUp) ? 2 : 1;
        const int rowBytes = (jb.K >> 8) * 144;
        slot = std::max(slot, NM * stage_rows_for(NM, G) * rowBytes);
        const int rows_per_cta = (jb.N + grid - 1) / grid;
        part = std::max(part, rows_per_cta * NM * nsegw);
        part = std::max(part, (int)(xs_bytes(jb.K) / sizeof(float)));
    }
    p.slot_bytes = (slot + 127) / 128 * 128;
    p.part_floats = part;
    const size_t fixed = (kNormSlots + 4) * sizeof(float) + (size_t)part * sizeof(float);
    const size_t per_stage = (size_t)p.slot_bytes + 2 * sizeof(uint64_t);
    if (smem_limit < fixed + 2 * per_stage) return -1;
    int S = (int)((smem_limit - fixed) / per_stage);
    if (S > 8) S = 8;
    p.stages = S;
    *smem_bytes = gemv_chain_smem_bytes(p);
    return 0;
}

namespace {
using Kernel = void (*)(GemvChainParams);
// the generic kernel, and instantiations for launches whose jobs all share
// one (K, op): the Q4_K GEMV at K = 4096 (Mixtral gate/up rows), 14336
// (Mixtral down rows) and 6144 (Mixtral-8x22B projections)
const Kernel kChainGeneric = q4k_gemv_chain_kernel<0, -1>;
const Kernel kChainK4096Set = q4k_gemv_chain_kernel<4096, kChainSet>;
const Kernel kChainK14336Set = q4k_gemv_chain_kernel<14336, kChainSet>;
const Kernel kChainK6144Set = q4k_gemv_chain_kernel<6144, kChainSet>;
const Kernel kChainK6144Add = q4k_gemv_chain_kernel<6144, kChainAdd>;

Kernel pick_chain_kernel(const GemvChainParams& p) {
    const int K = p.jobs[0].K, op = p.jobs[0].op;
    for (int j = 1; j < p.njobs; ++j)
        if (p.jobs[j].K != K || p.jobs[j].op != op) return kChainGeneric;
    if (op == kChainSet && K == 4096) return kChainK4096Set;
    if (op == kChainSet && K == 14336) return kChainK14336Set;
    if (op == kChainSet && K == 6144) return kChainK6144Set;
    if (op == kChainAdd && K == 6144) return kChainK6144Add;
    return kChainGeneric;
}
}  // namespace

cudaError_t gemv_chain_launch(GemvChainParams p, int num_sms, cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static int smem_optin[kMaxDevices] = {0};
    if (smem_optin[dev] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        for (Kernel kf : {kChainGeneric, kChainK4096Set, kChainK14336Set, kChainK6144Set, kChainK6144Add}) {
            cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
            if (e != cudaSuccess) return e;
        }
        smem_optin[dev] = v;
    }
    size_t smem = 0;
    if (gemv_chain_configure(p, num_sms, (size_t)smem_optin[dev], &smem) != 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(kChainThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barrier needs it
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, pick_chain_kernel(p), p);
}

}  // namespace glc
