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
//   * Consumer warps never touch global weights.  Lane u of a row owns one
//     32-byte quant chunk c of super-block sb (64 weights, two 32-weight
//     sub-blocks).  The lane's 64 activations are quantised once per input
//     vector to int16 with one fp32 scale per 32-block (error <= 2^-16 of the
//     block max), kept in registers, and every 8 weights cost 2 LOPs + 4 dp2a
//     (int16 x uint8 -> int32): no per-weight float conversion.
//     y_row = sum_sb d*(sc_a*s_a*Ia + sc_b*s_b*Ib/16) - dmin*(m_a*Sa + m_b*Sb)
//     where Ia/Ib are the integer dot products and Sa/Sb the fp32 sums of the
//     32 activations of each sub-block (the Q4_K min term).
//   * Lane partials are reduced by warp shuffles, the per-segment sums are
//     kept in shared memory and summed in fixed order at the end (deterministic).
//   * Epilogues: plain store; gate/up pair -> SwiGLU act = silu(g)*u; down rows
//     of the k experts of a token -> weighted combine acc = (y*w)+acc in k order
//     (+ residual), i.e. AccumulatorStageWorker.AccumulateWeightedExpert.
#include "common.cuh"
#include "kernels.h"

namespace glc {

template <class F>
__device__ __forceinline__ void for_each_stage(const GemvParams& p, int r0, int r1, F&& f) {
    int pos = r0, sidx = 0;
    const int nslots = (p.mode == kGemvDownCombine) ? p.kslots : 1;
    while (pos < r1) {
        const int seg = pos / p.rows;
        const int seg_end = min(r1, (seg + 1) * p.rows);
        for (int j = 0; j < nslots; ++j)
            for (int c = pos; c < seg_end; c += p.stage_rows)
                f(sidx++, seg, j, c - seg * p.rows, min(p.stage_rows, seg_end - c), c - r0);
        pos = seg_end;
    }
}

struct XRegs {
    int xa[16];
    int xb[16];
    float sA, sB16, sumA, sumB;
};

// Quantise one 32-block of activations to 16 int16 pairs; returns the block
// scale (max|x| / 32767) and the fp32 block sum.
__device__ __forceinline__ void quant_block32(const float4* xp, int (&dst)[16], float& scale, float& sum) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(xp + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
    float mx = 0.f, s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { mx = fmaxf(mx, fabsf(v[i])); s += v[i]; }
    const float inv = mx > 0.f ? 32767.0f / mx : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int q0 = __float2int_rn(v[2 * i] * inv);
        const int q1 = __float2int_rn(v[2 * i + 1] * inv);
        dst[i] = (q0 & 0xFFFF) | (q1 << 16);
    }
    scale = mx * (1.0f / 32767.0f);
    sum = s;
}

// Quantise the lane's 64 activations (two 32-blocks) to int16 pairs.
__device__ __forceinline__ void load_x(XRegs& r, const float* xrow, int sb, int c, bool active) {
    if (!active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) r.xa[i] = r.xb[i] = 0;
        r.sA = r.sB16 = r.sumA = r.sumB = 0.f;
        return;
    }
    const float4* xp = reinterpret_cast<const float4*>(xrow + sb * 256 + 64 * c);
    float sB;
    quant_block32(xp, r.xa, r.sA, r.sumA);
    quant_block32(xp + 8, r.xb, sB, r.sumB);
    r.sB16 = sB * 0.0625f;
}

// One lane's contribution to one row: chunk c of super-block sb.
__device__ __forceinline__ float row_unit(const uint8_t* row, int sb, int c, const XRegs& r) {
    const uint8_t* blk = row + sb * 144;
    const uint4 h = lds128(blk);
    const uint4 q0 = lds128(blk + 16 + 32 * c);
    const uint4 q1 = lds128(blk + 32 + 32 * c);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int ia = 0, ib = 0;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t lo = w[m] & 0x0F0F0F0Fu;
        const uint32_t hi = w[m] & 0xF0F0F0F0u;
        ia = dp2a_lo(r.xa[2 * m], lo, ia);
        ia = dp2a_hi(r.xa[2 * m + 1], lo, ia);
        ib = dp2a_lo(r.xb[2 * m], hi, ib);
        ib = dp2a_hi(r.xb[2 * m + 1], hi, ib);
    }
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const int sh = (c & 1) * 16;
    const uint32_t Y = h.y >> sh, Z = h.z >> sh, W = h.w >> sh;
    uint32_t scp, mp;
    if (c < 2) {
        scp = Y & 0x3F3Fu;
        mp = Z & 0x3F3Fu;
    } else {
        scp = (W & 0x0F0Fu) | ((Y >> 2) & 0x3030u);
        mp = ((W >> 4) & 0x0F0Fu) | ((Z >> 2) & 0x3030u);
    }
    const float sc0 = (float)(scp & 0xFFu), sc1 = (float)((scp >> 8) & 0xFFu);
    const float m0 = (float)(mp & 0xFFu), m1 = (float)((mp >> 8) & 0xFFu);
    const float fa = (float)ia * r.sA;
    const float fb = (float)ib * r.sB16;
    return d * (fa * sc0 + fb * sc1) - dmin * (m0 * r.sumA + m1 * r.sumB);
}

__device__ __forceinline__ int clamp_expert(int e, int E) { return e < 0 ? 0 : (e >= E ? E - 1 : e); }

__global__ void __launch_bounds__(kGemvMaxThreads, 1) q4k_gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NM = (p.mode == kGemvGateUp) ? 2 : 1;
    const int NMP = (p.mode == kGemvGateUp) ? 2 : (p.mode == kGemvDownCombine ? p.kslots : 1);
    const int rowBytes = (p.K >> 8) * 144;
    const int R = p.stage_rows;
    const int stage_bytes = NM * R * rowBytes;
    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    float* part = reinterpret_cast<float*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NW = p.nw;
    const long long total = (long long)p.nseg * p.rows;
    const int r0 = (int)(total * blockIdx.x / gridDim.x);
    const int r1 = (int)(total * (blockIdx.x + 1) / gridDim.x);

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
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            bool ok = true;
            for_each_stage(p, r0, r1, [&](int sidx, int seg, int j, int rin, int nr, int) {
                if (!ok) return;
                const int buf = sidx % S;
                const uint32_t ph = (uint32_t)(sidx / S) & 1u;
                if (!mbar_wait(&empty[buf], ph ^ 1u, p.err, kDevTimeoutEmpty)) { ok = false; return; }
                const uint8_t* srcA;
                const uint8_t* srcB = nullptr;
                if (p.mode == kGemvPlain) {
                    srcA = p.A + (size_t)rin * rowBytes;
                } else if (p.mode == kGemvGateUp) {
                    const int e = clamp_expert(__ldg(p.ids + seg), p.num_experts);
                    srcA = p.A + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                    srcB = p.B + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                } else {
                    const int e = clamp_expert(__ldg(p.ids + seg * p.kslots + j), p.num_experts);
                    srcA = p.A + (size_t)e * p.expert_bytes + (size_t)rin * rowBytes;
                }
                const uint32_t bytes = (uint32_t)(nr * rowBytes);
                uint8_t* dst = smem + (size_t)buf * stage_bytes;
                mbar_arrive_expect_tx(&full[buf], bytes * NM);
                bulk_g2s(dst, srcA, bytes, &full[buf], pol);
                if (NM == 2) bulk_g2s(dst + (size_t)R * rowBytes, srcB, bytes, &full[buf], pol);
            });
        }
        return;
    }

    // ---------------------------------------------------------- consumer warps
    const int nsegw = p.nsegw;
    const int segw = warp % nsegw, grp = warp / nsegw, G = NW / nsegw;
    const int U = (p.K >> 8) * 4;
    const int u = segw * 32 + lane;
    const bool active = u < U;
    const int sb = active ? (u >> 2) : 0, c = u & 3;
    XRegs xr;
    int cur_x = -1;
    bool ok = true;
    for_each_stage(p, r0, r1, [&](int sidx, int seg, int j, int, int nr, int lr0) {
        if (!ok) return;
        const int xid = (p.mode == kGemvPlain) ? 0
                        : (p.mode == kGemvGateUp ? seg / p.kslots : seg * p.kslots + j);
        if (xid != cur_x) {
            load_x(xr, p.x + (size_t)xid * p.K, sb, c, active);
            cur_x = xid;
        }
        const int buf = sidx % S;
        const uint32_t ph = (uint32_t)(sidx / S) & 1u;
        if (!mbar_wait(&full[buf], ph, p.err, kDevTimeoutFull)) { ok = false; return; }
        const uint8_t* st = smem + (size_t)buf * stage_bytes;
        for (int i = grp; i < nr; i += G) {
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                if (m >= NM) break;
                float v = active ? row_unit(st + (size_t)(m * R + i) * rowBytes, sb, c, xr) : 0.f;
                v = warp_sum(v);
                if (lane == 0) {
                    const int slot = (p.mode == kGemvDownCombine) ? j : m;
                    part[((size_t)(lr0 + i) * NMP + slot) * nsegw + segw] = v;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
    });

    named_bar_sync(1, NW * 32);
    if (!ok) return;

    // ------------------------------------------------------------ epilogue
    const int nrows = r1 - r0;
    for (int lr = threadIdx.x; lr < nrows; lr += NW * 32) {
        const int g = r0 + lr;
        const int seg = g / p.rows, rin = g - seg * p.rows;
        const float* pp = part + (size_t)lr * NMP * nsegw;
        if (p.mode == kGemvPlain) {
            float s = 0.f;
            for (int q = 0; q < nsegw; ++q) s += pp[q];
            p.y[rin] = s;
        } else if (p.mode == kGemvGateUp) {
            float gs = 0.f, us = 0.f;
            for (int q = 0; q < nsegw; ++q) { gs += pp[q]; us += pp[nsegw + q]; }
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
    if (nsegw > 16) return -1;  // K > 32768 not supported by the register layout
    const int G = (16 / nsegw) > 0 ? 16 / nsegw : 1;
    p.nsegw = nsegw;
    p.nw = nsegw * G;
    const int NM = (p.mode == kGemvGateUp) ? 2 : 1;
    const int NMP = (p.mode == kGemvGateUp) ? 2 : (p.mode == kGemvDownCombine ? p.kslots : 1);
    const int rowBytes = (p.K >> 8) * 144;
    int rpg = 32768 / (NM * G * rowBytes);
    rpg = rpg < 1 ? 1 : (rpg > 4 ? 4 : rpg);
    p.stage_rows = G * rpg;
    const size_t stage_bytes = (size_t)NM * p.stage_rows * rowBytes;
    int S = (int)((160 * 1024) / stage_bytes);
    S = S < 2 ? 2 : (S > 8 ? 8 : S);
    const long long total = (long long)p.nseg * p.rows;
    int range_cap = (int)(16384 / (NMP * nsegw * 4));
    int g = num_sms;
    if ((total + g - 1) / g > range_cap) g = (int)((total + range_cap - 1) / range_cap);
    if (g > total) g = (int)total;
    size_t bytes = (size_t)S * stage_bytes + 2 * S * sizeof(uint64_t) +
                   (size_t)((total + g - 1) / g) * NMP * nsegw * sizeof(float);
    while (bytes > smem_limit && S > 2) {
        --S;
        bytes -= stage_bytes + 2 * sizeof(uint64_t);
    }
    if (bytes > smem_limit) return -1;
    p.stages = S;
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
        cudaError_t e = cudaFuncSetAttribute(q4k_gemv_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, v);
        if (e != cudaSuccess) return e;
        smem_optin[dev] = v;
    }
    const size_t smem_limit = (size_t)smem_optin[dev];
    if (gemv_configure(p, num_sms, smem_limit, &smem, &grid) != 0) return cudaErrorInvalidValue;
    q4k_gemv_kernel<<<grid, (p.nw + 1) * 32, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace glc
