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
//     sub-blocks A and B); its activations are prepared once per input vector
//     and kept in registers.  Sub-block A runs on integer dot products (dp2a),
//     sub-block B on fp32 FMAs with a conversion-free nibble decode (see
//     XRegs), which balances the two pipes.
//     y_row = sum_sb d*(sc_a*A + sc_b*B) - dmin*(m_a*Sa + m_b*Sb), where A/B
//     are the sub-block dot products sum q*x and Sa/Sb the fp32 sums of the
//     32 activations of each sub-block (the Q4_K min term).
//   * Lane partials are reduced by warp shuffles, the per-segment sums are
//     kept in shared memory and summed in fixed order at the end (deterministic).
//   * Epilogues: plain store; gate/up pair -> SwiGLU act = silu(g)*u; down rows
//     of the k experts of a token -> weighted combine acc = (y*w)+acc in k order
//     (+ residual), i.e. AccumulatorStageWorker.AccumulateWeightedExpert.
#include "common.cuh"
#include "kernels.h"

// Pipeline shape knobs (bytes of weights per stage, bytes of the stage ring,
// stage count bound, L2 streaming hint).
#ifndef GLC_GEMV_STAGE_TARGET
#define GLC_GEMV_STAGE_TARGET 65536
#endif
#ifndef GLC_GEMV_RING_BYTES
#define GLC_GEMV_RING_BYTES (192 * 1024)
#endif
#ifndef GLC_GEMV_MAX_STAGES
#define GLC_GEMV_MAX_STAGES 8
#endif
#ifndef GLC_GEMV_MATH
#define GLC_GEMV_MATH 0  // 0: dp2a for both sub-blocks; 1: dp2a + fp32 FMA split
#endif
#ifndef GLC_GEMV_L2_HINT
#define GLC_GEMV_L2_HINT 1
#endif

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

#if GLC_GEMV_MATH == 0
// Lane math, integer form: the lane's 64 activations are quantised once per
// input vector to int16 with one fp32 scale per 32-block (error <= 2^-16 of
// the block max) and kept in registers; every 8 weights cost 2 LOPs and 4
// dp2a (int16 x uint8 -> int32), with no per-weight float conversion.
//   y_row += d*(sc_a*s_a*Ia + sc_b*s_b*Ib/16) - dmin*(m_a*Sa + m_b*Sb)
struct XRegs {
    int xa[16];
    int xb[16];
    float sA, sB16, sumA, sumB;
};

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

__device__ __forceinline__ float row_unit(const uint8_t* row, int sb, int c, const XRegs& r) {
    const uint8_t* blk = row + sb * 144;
    const uint4 h = lds128(blk);
    const uint4 q0 = lds128(blk + 16 + 32 * c);
    const uint4 q1 = lds128(blk + 32 + 32 * c);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int ia0 = 0, ia1 = 0, ib0 = 0, ib1 = 0;  // four short accumulation chains
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t lo = w[m] & 0x0F0F0F0Fu;
        const uint32_t hi = w[m] & 0xF0F0F0F0u;
        ia0 = dp2a_lo(r.xa[2 * m], lo, ia0);
        ia1 = dp2a_hi(r.xa[2 * m + 1], lo, ia1);
        ib0 = dp2a_lo(r.xb[2 * m], hi, ib0);
        ib1 = dp2a_hi(r.xb[2 * m + 1], hi, ib1);
    }
    const int ia = ia0 + ia1, ib = ib0 + ib1;
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
    return d * (((float)ia * r.sA) * sc0 + ((float)ib * r.sB16) * sc1) - dmin * (m0 * r.sumA + m1 * r.sumB);
}
#else
// The 64 weights a lane owns per row are split across two execution pipes so
// neither limits the HBM stream:
//  * sub-block A (low nibbles): integer dot products, activations as int16
//    with one fp32 scale per 32-block (error <= 2^-16 of the block max):
//    1 LOP + 2 dp2a (int16 x uint8 -> int32) per 4 weights;
//  * sub-block B (high nibbles): nibble -> float without a conversion
//    instruction.  Any bit pattern b < 2^24 read as an fp32 is exactly
//    b * 2^-149 (the subnormal binade and the first normal binade share the
//    ulp 2^-149), so (word & (0xF << sh)) is the float q * 2^(sh-149) after one
//    AND; the activation is pre-scaled by 2^(125-sh-E) (E bounds |x| of the
//    32-block), so each fused multiply-add adds q * x * 2^(-24-E) exactly up to
//    the fp32 rounding of the sum.  High-nibble shifts inside a qs word:
//    {4, 12, 20} for bytes 0..2 and 12 for byte 3 after >> 16.
// dp2a alone saturates the slow integer-dot-product / conversion pipe on
// sm_100, float FMAs alone cost about 2 issue slots per weight; half and half
// keeps both below the HBM time.
struct XRegs {
    int xa[16];     // sub-block A: int16 pairs (4m,4m+1), (4m+2,4m+3)
    float xb[32];   // sub-block B: pre-scaled fp32 activations
    float sA;       // A: block scale max|x|/32767
    float fB;       // B: 2^(24+E)
    float sumA, sumB;
};

__device__ __forceinline__ void load_block32(const float4* xp, float (&v)[32], float& mx, float& sum) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(xp + i);
        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
    mx = 0.f;
    sum = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { mx = fmaxf(mx, fabsf(v[i])); sum += v[i]; }
}

// Prepare the lane's 64 activations (two 32-blocks).
__device__ __forceinline__ void load_x(XRegs& r, const float* xrow, int sb, int c, bool active) {
    if (!active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) r.xa[i] = 0;
#pragma unroll
        for (int i = 0; i < 32; ++i) r.xb[i] = 0.f;
        r.sA = r.fB = r.sumA = r.sumB = 0.f;
        return;
    }
    const float4* xp = reinterpret_cast<const float4*>(xrow + sb * 256 + 64 * c);
    {
        float v[32], mx;
        load_block32(xp, v, mx, r.sumA);
        const float inv = mx > 0.f ? 32767.0f / mx : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int q0 = __float2int_rn(v[2 * i] * inv);
            const int q1 = __float2int_rn(v[2 * i + 1] * inv);
            r.xa[i] = (q0 & 0xFFFF) | (q1 << 16);
        }
        r.sA = mx * (1.0f / 32767.0f);
    }
    {
        float v[32], mx;
        load_block32(xp + 8, v, mx, r.sumB);
        const int E = mx > 0.f ? ((int)((__float_as_uint(mx) >> 23) & 0xFFu) - 126) : 0;
        const float s4 = ldexpf(1.0f, 121 - E), s12 = ldexpf(1.0f, 113 - E), s20 = ldexpf(1.0f, 105 - E);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            r.xb[4 * m] = v[4 * m] * s4;
            r.xb[4 * m + 1] = v[4 * m + 1] * s12;
            r.xb[4 * m + 2] = v[4 * m + 2] * s20;
            r.xb[4 * m + 3] = v[4 * m + 3] * s12;
        }
        r.fB = ldexpf(1.0f, 24 + E);
    }
}

// One lane's contribution to one row: chunk c of super-block sb.
__device__ __forceinline__ float row_unit(const uint8_t* row, int sb, int c, const XRegs& r) {
    const uint8_t* blk = row + sb * 144;
    const uint4 h = lds128(blk);
    const uint4 q0 = lds128(blk + 16 + 32 * c);
    const uint4 q1 = lds128(blk + 32 + 32 * c);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int ia = 0;
    float b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t x = w[m];
        const uint32_t lo = x & 0x0F0F0F0Fu;
        ia = dp2a_lo(r.xa[2 * m], lo, ia);
        ia = dp2a_hi(r.xa[2 * m + 1], lo, ia);
        b0 = fmaf(__uint_as_float(x & 0xF0u), r.xb[4 * m], b0);
        b1 = fmaf(__uint_as_float(x & 0xF000u), r.xb[4 * m + 1], b1);
        b0 = fmaf(__uint_as_float(x & 0xF00000u), r.xb[4 * m + 2], b0);
        b1 = fmaf(__uint_as_float((x >> 16) & 0xF000u), r.xb[4 * m + 3], b1);
    }
    const float accB = b0 + b1;
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
    return d * (((float)ia * r.sA) * sc0 + (accB * r.fB) * sc1) - dmin * (m0 * r.sumA + m1 * r.sumB);
}
#endif

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
            const uint64_t pol = GLC_GEMV_L2_HINT ? l2_evict_first_policy() : 0ull;
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
                if (GLC_GEMV_L2_HINT) {
                    bulk_g2s(dst, srcA, bytes, &full[buf], pol);
                    if (NM == 2) bulk_g2s(dst + (size_t)R * rowBytes, srcB, bytes, &full[buf], pol);
                } else {
                    bulk_g2s_nohint(dst, srcA, bytes, &full[buf]);
                    if (NM == 2) bulk_g2s_nohint(dst + (size_t)R * rowBytes, srcB, bytes, &full[buf]);
                }
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
        // Up to four independent row-units per warp per pass (rows x matrices),
        // all computed before one interleaved shuffle reduction, so the
        // dependent-latency chains of different rows overlap.
        for (int i0 = grp; i0 < nr; i0 += 2 * G) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + (u >> 1) * G, m = u & 1;
                v[u] = (active && m < NM && i < nr) ? row_unit(st + (size_t)(m * R + i) * rowBytes, sb, c, xr) : 0.f;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] += __shfl_xor_sync(0xffffffffu, v[u], off);
            if (lane == 0) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + (u >> 1) * G, m = u & 1;
                    if (m < NM && i < nr) {
                        const int slot = (p.mode == kGemvDownCombine) ? j : m;
                        part[((size_t)(lr0 + i) * NMP + slot) * nsegw + segw] = v[u];
                    }
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
    if (nsegw > kGemvMaxConsumerWarps) return -1;  // K > 24576 not supported by the warp layout
    const int G = kGemvMaxConsumerWarps / nsegw;
    p.nsegw = nsegw;
    p.nw = nsegw * G;
    const int NM = (p.mode == kGemvGateUp) ? 2 : 1;
    const int NMP = (p.mode == kGemvGateUp) ? 2 : (p.mode == kGemvDownCombine ? p.kslots : 1);
    const int rowBytes = (p.K >> 8) * 144;
    int rpg = GLC_GEMV_STAGE_TARGET / (NM * G * rowBytes);
    rpg = rpg < 1 ? 1 : (rpg > 4 ? 4 : rpg);
    p.stage_rows = G * rpg;
    const size_t stage_bytes = (size_t)NM * p.stage_rows * rowBytes;
    int S = (int)((size_t)GLC_GEMV_RING_BYTES / stage_bytes);
    S = S < 2 ? 2 : (S > GLC_GEMV_MAX_STAGES ? GLC_GEMV_MAX_STAGES : S);
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
