// gemv_lane.cuh -- per-lane Q4_K dot-product math shared by the decode GEMV
// (gemv_q4k.cu) and the fused decode layer kernel (decode_fused.cu).
//
// Lane u of a row owns one 32-byte quant chunk c of super-block sb = u / 4
// (64 weights: sub-block A = low nibbles, sub-block B = high nibbles of the
// chunk; GGUF Q4_K super-block = d f16 | dmin f16 | 12 B packed 6-bit
// scales/mins | 128 B quants).  Its 64 activations are quantised once per
// input vector to int16 with one fp32 scale per 32-block (error <= 2^-16 of the
// block max) and kept in registers; every 8 weights then cost 2 LOPs and
// 4 dp2a (int16 x uint8 -> int32), with no per-weight float conversion:
//   y_row += d*(sc_a*s_a*Ia + sc_b*s_b*Ib/16) - dmin*(m_a*Sa + m_b*Sb)
// where Ia/Ib are the integer sub-block dot products, s_a/s_b the block scales
// and Sa/Sb the fp32 sums of the block's activations (the Q4_K min term).
#pragma once

#include "common.cuh"

namespace glc {

// Where the activations are read from: read-only global data (ld.global.nc),
// global data written earlier in the same launch by other CTAs (ld.global.cg,
// coherent at L2), or shared memory.
enum XSource : int { kXGlobalRO = 0, kXGlobalCG = 1, kXShared = 2 };

template <int SRC>
__device__ __forceinline__ float4 ldx4(const float4* p) {
    if constexpr (SRC == kXGlobalRO) return __ldg(p);
    else if constexpr (SRC == kXGlobalCG) return __ldcg(p);
    else return *p;
}

struct XRegs {
    int xa[16];
    int xb[16];
    float sA, sB16, sumA, sumB;
};

__device__ __forceinline__ void quant_block32(const float4 (&t)[8], int (&dst)[16], float& scale, float& sum) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[4 * i] = t[i].x; v[4 * i + 1] = t[i].y; v[4 * i + 2] = t[i].z; v[4 * i + 3] = t[i].w;
    }
    float mx = 0.f, s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { mx = fmaxf(mx, fabsf(v[i])); s += v[i]; }
    const float inv = mx > 0.f ? 32767.0f / mx : 0.f;
    // Round to nearest even without a float-to-int conversion (a low-rate
    // pipe that a whole CTA quantising at once would queue on): adding
    // 1.5 * 2^23 to |v * inv| <= 32767 leaves the rounded integer in the low
    // 16 bits of the sum's bit pattern, the same value __float2int_rn gives.
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float t0 = __fadd_rn(__fmul_rn(v[2 * i], inv), 12582912.0f);
        const float t1 = __fadd_rn(__fmul_rn(v[2 * i + 1], inv), 12582912.0f);
        dst[i] = (int)__byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x5410);
    }
    scale = mx * (1.0f / 32767.0f);
    sum = s;
}

// Prepare the lane's 64 activations: its 16 float4 chunks are xp[0], xp[stride],
// ..., xp[15*stride] (all 16 loads are issued before any is used).  Row-major
// vectors use xp = x + 16*u, stride 1; the chunk-major layout (chunk i of unit u
// at float4 index i*U + u, U = K/64 units) uses xp = x + u, stride U, so a
// warp's loads of one chunk are contiguous.
template <int SRC>
__device__ __forceinline__ void load_x(XRegs& r, const float4* xp, int stride, bool active) {
    if (!active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) r.xa[i] = r.xb[i] = 0;
        r.sA = r.sB16 = r.sumA = r.sumB = 0.f;
        return;
    }
    float4 ta[8], tb[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ta[i] = ldx4<SRC>(xp + i * stride);
#pragma unroll
    for (int i = 0; i < 8; ++i) tb[i] = ldx4<SRC>(xp + (8 + i) * stride);
    float sB;
    quant_block32(ta, r.xa, r.sA, r.sumA);
    quant_block32(tb, r.xb, sB, r.sumB);
    r.sB16 = sB * 0.0625f;
}

// load_x of a row-major input that is RMSNorm'd with weights w: the lane's
// values are x * w (w read at the same float4 indices) and ss receives the
// lane's sum of the raw x^2 (in element order), from which the caller forms
// the norm's scale.
template <int SRC>
__device__ __forceinline__ void load_x_norm(XRegs& r, const float4* xp, const float4* wp, bool active, float& ss) {
    ss = 0.f;
    if (!active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) r.xa[i] = r.xb[i] = 0;
        r.sA = r.sB16 = r.sumA = r.sumB = 0.f;
        return;
    }
    // one 32-block at a time (x and w of a block: 64 registers)
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
        float4 t[8], w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = ldx4<SRC>(xp + 8 * blk + i);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = __ldg(wp + 8 * blk + i);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            ss = fmaf(t[i].x, t[i].x, ss); ss = fmaf(t[i].y, t[i].y, ss);
            ss = fmaf(t[i].z, t[i].z, ss); ss = fmaf(t[i].w, t[i].w, ss);
            t[i] = make_float4(__fmul_rn(t[i].x, w[i].x), __fmul_rn(t[i].y, w[i].y), __fmul_rn(t[i].z, w[i].z),
                               __fmul_rn(t[i].w, w[i].w));
        }
        if (blk == 0) {
            quant_block32(t, r.xa, r.sA, r.sumA);
        } else {
            float sB;
            quant_block32(t, r.xb, sB, r.sumB);
            r.sB16 = sB * 0.0625f;
        }
    }
}

// ---- the input staged once per CTA --------------------------------------
// load_x has every lane read its own 64 consecutive floats (a warp's 16-byte
// loads then touch 32 lines each) and every warp group of a CTA repeat it;
// for a row-major input that nothing has laid out for the lanes, a CTA then
// issues ~K/2 line requests to L2 for a K-float vector, and 148 CTAs doing so
// at once took ~10 us per input.  Here the CTA's threads read the vector once,
// coalesced (thread t of n reads float4 t, t + n, ...), form each 32-block's
// maximum and sum with shuffles among its 8 threads, quantise to int16 as
// quant_block32 does, and write every lane's registers transposed into shared
// memory (word w of unit u at w * xs_stride(U) + u, conflict-free); each lane
// then reads its 36 words.  The block sums are formed in a different order
// from quant_block32's, so values can differ from load_x's in the last bit.
constexpr int kXsWords = 36;  // xa[16], xb[16], sA, sB16, sumA, sumB

__host__ __device__ inline int xs_stride(int U) { return (U + 31) / 32 * 32 + 1; }
__host__ __device__ inline size_t xs_bytes(int K) { return (size_t)kXsWords * xs_stride(K / 64) * 4; }

// nthr threads (a multiple of 32) starting at thread 0 of the CTA; x, w
// 16-byte aligned.  w may be null.  With w, ss_warp[warp] receives the warp's
// sum of the raw x^2 (threads add their values in load order, then a warp
// butterfly), from which the caller forms the RMSNorm scale.
template <int SRC>
__device__ __forceinline__ void stage_x_shared(const float* x, const float* w, int K, uint32_t* xs, float* ss_warp,
                                               int tid, int nthr) {
    const int F4 = K >> 2, U = K >> 6, st = xs_stride(U);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float ss = 0.f;
    for (int f0 = 0; f0 < F4; f0 += 8 * nthr) {
        // every load of the pass (input and norm weights) issued before any is used: one L2 round trip
        float4 v[8], g[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int f = f0 + k * nthr + tid;
            v[k] = f < F4 ? ldx4<SRC>(x4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
            g[k] = (w && f < F4) ? __ldg(w4 + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int f = f0 + k * nthr + tid;  // F4 is a multiple of 64: an 8-thread group is in or out together
            if (f0 + k * nthr >= F4) break;
            float4 a = v[k];
            if (w) {
                ss = fmaf(a.x, a.x, ss); ss = fmaf(a.y, a.y, ss); ss = fmaf(a.z, a.z, ss); ss = fmaf(a.w, a.w, ss);
                a = make_float4(__fmul_rn(a.x, g[k].x), __fmul_rn(a.y, g[k].y), __fmul_rn(a.z, g[k].z),
                                __fmul_rn(a.w, g[k].w));
            }
            float mx = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
            float sm = ((a.x + a.y) + a.z) + a.w;
#pragma unroll
            for (int o = 1; o <= 4; o <<= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                sm += __shfl_xor_sync(0xffffffffu, sm, o);
            }
            if (f < F4) {
                const float inv = mx > 0.f ? 32767.0f / mx : 0.f;
                const float t0 = __fadd_rn(__fmul_rn(a.x, inv), 12582912.0f);
                const float t1 = __fadd_rn(__fmul_rn(a.y, inv), 12582912.0f);
                const float t2 = __fadd_rn(__fmul_rn(a.z, inv), 12582912.0f);
                const float t3 = __fadd_rn(__fmul_rn(a.w, inv), 12582912.0f);
                const int u = f >> 4, q = f & 15, blk = q >> 3, wi = blk * 16 + (q & 7) * 2;
                xs[wi * st + u] = __byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x5410);
                xs[(wi + 1) * st + u] = __byte_perm(__float_as_uint(t2), __float_as_uint(t3), 0x5410);
                if ((q & 7) == 0) {
                    const float scale = mx * (1.0f / 32767.0f);
                    xs[(32 + blk) * st + u] = __float_as_uint(blk ? scale * 0.0625f : scale);
                    xs[(34 + blk) * st + u] = __float_as_uint(sm);
                }
            }
        }
    }
    if (w) {
        ss = warp_tree(ss);
        if ((tid & 31) == 0) ss_warp[tid >> 5] = ss;
    }
}

__device__ __forceinline__ void read_x_shared(XRegs& r, const uint32_t* xs, int U, int u, bool active) {
    const int st = xs_stride(U);
    if (!active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) r.xa[i] = r.xb[i] = 0;
        r.sA = r.sB16 = r.sumA = r.sumB = 0.f;
        return;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        r.xa[i] = (int)xs[i * st + u];
        r.xb[i] = (int)xs[(16 + i) * st + u];
    }
    r.sA = __uint_as_float(xs[32 * st + u]);
    r.sB16 = __uint_as_float(xs[33 * st + u]);
    r.sumA = __uint_as_float(xs[34 * st + u]);
    r.sumB = __uint_as_float(xs[35 * st + u]);
}

// Float index of element w (0..63) of unit u in the chunk-major layout.
__device__ __forceinline__ int chunk_major_index(int u, int w, int U) { return ((w >> 2) * U + u) * 4 + (w & 3); }

// One lane's contribution to one row held in shared memory: chunk c of super-block sb.
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
    // 6-bit scale / min of sub-blocks 2c and 2c+1 (GGUF get_scale_min_k4),
    // two at a time from the 12 packed bytes held in h.y, h.z, h.w.
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

// Four per-lane values reduced across the warp with 6 shuffles (a transposing
// butterfly): lane L ends up holding the warp sum of value (L >> 3) & 3.
__device__ __forceinline__ float warp_reduce4(const float (&v)[4], int lane) {
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1;
    float a0 = b4 ? v[2] : v[0], a1 = b4 ? v[3] : v[1];
    const float s0 = b4 ? v[0] : v[2], s1 = b4 ? v[1] : v[3];
    a0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    a1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    float b = b3 ? a1 : a0;
    const float s = b3 ? a0 : a1;
    b += __shfl_xor_sync(0xffffffffu, s, 8);
    b += __shfl_xor_sync(0xffffffffu, b, 4);
    b += __shfl_xor_sync(0xffffffffu, b, 2);
    b += __shfl_xor_sync(0xffffffffu, b, 1);
    return b;
}

// Rows a stage holds so that every warp of a G-group layout does exactly one
// pass of four row-units: 2G rows of each of 2 matrices, or 4G rows of one.
__host__ __device__ inline int stage_rows_for(int NM, int G) { return NM == 2 ? 2 * G : 4 * G; }

// One warp's share of a shared-memory stage of nr <= stage_rows_for(NM, G)
// rows (NM matrices of R rows each, matrix m at row offset m*R): four
// row-units (rows grp and grp+G of both matrices, or rows grp + {0,1,2,3}*G)
// computed unconditionally (rows past nr re-read row nr-1 and are discarded)
// so their dependent-latency chains interleave, then one 6-shuffle reduction.
// store(i, m, v) is called by lanes 0, 8, 16, 24 with the warp's segment sum
// of row i of matrix m.
template <class Store>
__device__ __forceinline__ void consume_stage(const uint8_t* st, int nr, int R, int NM, int G, int grp,
                                              int rowBytes, int sb, int c, bool active, const XRegs& xr,
                                              int lane, Store&& store) {
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int i = (NM == 2) ? grp + (u >> 1) * G : grp + u * G;
        const int m = (NM == 2) ? (u & 1) : 0;
        const int ii = i < nr ? i : nr - 1;
        const float r = row_unit(st + (size_t)(m * R + ii) * rowBytes, sb, c, xr);
        v[u] = (active && i < nr) ? r : 0.f;
    }
    const float b = warp_reduce4(v, lane);
    if ((lane & 7) == 0) {
        const int j = lane >> 3;
        const int i = (NM == 2) ? grp + (j >> 1) * G : grp + j * G;
        const int m = (NM == 2) ? (j & 1) : 0;
        if (i < nr) store(i, m, b);
    }
}

// Walks the stages of rows [r0, r1) of a flattened (segment, row) space with
// `rows` rows per segment: within a segment, for each of `nslots` slots, chunks
// of at most stage_rows rows.  f(sidx, seg, slot, row_in_seg, nrows, local_row0)
// with sidx counting up from sidx0; returns the next stage index.
template <class F>
__device__ __forceinline__ int for_each_stage_rows(int rows, int nslots, int stage_rows, int r0, int r1,
                                                   int sidx0, F&& f) {
    int pos = r0, sidx = sidx0;
    while (pos < r1) {
        const int seg = pos / rows;
        const int seg_end = min(r1, (seg + 1) * rows);
        for (int j = 0; j < nslots; ++j)
            for (int c = pos; c < seg_end; c += stage_rows)
                f(sidx++, seg, j, c - seg * rows, min(stage_rows, seg_end - c), c - r0);
        pos = seg_end;
    }
    return sidx;
}

__device__ __forceinline__ int clamp_expert(int e, int E) { return e < 0 ? 0 : (e >= E ? E - 1 : e); }

}  // namespace glc
