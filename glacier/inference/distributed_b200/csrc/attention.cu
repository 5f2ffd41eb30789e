// attention.cu -- decode attention over an fp16 KV cache with grouped-query
// heads and rotary position embedding, for the attention half of a decode
// stage (the caller side of IClusterStageModel.ForwardStage,
// IClusterStageModel.cs:19; the reference's attention body is in its external
// model package, Program.cs:1390).
//
// One token at position pos: q [Hq][128] and the token's k, v [Hkv][128]
// (fp32, before rotation) come in; RoPE (NeoX / rotate-half pairing (i, i+64),
// theta^(-2i/128) frequencies, angles in double) rotates q and k; the rotated
// k and v are stored in the caches as fp16 at row pos; the output is
// softmax(q.K^T / sqrt(128)) V over positions 0..pos, query head h reading KV
// head h / G (G = Hq / Hkv query heads per KV head).
//
// HBM-bound (the cache rows are read once: 2 x Hkv x (pos+1) x 256 B): the
// sequence is split into chunks of 64 positions, one CTA per (KV head, chunk),
// so every byte of K and V read serves all G query heads of its group.  A CTA
// stages its chunk in shared memory (K rows padded to 272 B so the per-position
// 16-byte reads are conflict-free), computes the G x 64 scores, the chunk's
// softmax statistics and unnormalised output, and writes them to a workspace;
// a second launch, one CTA per query head, merges the chunks (flash-decoding).
// Merging in the last CTA of each KV head instead (an atomic count) measured
// slower: 8 CTAs then merge 5 heads each on the critical path.  The CTA whose
// chunk holds pos builds the new rows from the inputs (fp16-rounded as stored)
// instead of reading them, and writes them to the caches.  Each thread issues
// all its row loads before storing any, so a CTA's 32 KB are in flight at once.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace glc {

namespace {

constexpr int kHd = 128;        // head dimension
constexpr int kChunk = 64;      // positions per CTA
constexpr int kKStride = 136;   // halves per staged K row (272 B)
constexpr int kAttnThreads = 128;

// RoPE of pair i (0..63) at position pos: cos and sin of pos * theta^(-2i/128),
// the angle formed and reduced to [-pi, pi] in double, then sincosf.
__device__ __forceinline__ void rope_cs(int pos, float theta, int i, float& c, float& s) {
    const double inv = exp(-(double)(2 * i) / (double)kHd * log((double)theta));
    double ang = (double)pos * inv;
    ang -= 6.283185307179586 * rint(ang * 0.15915494309189535);
    sincosf((float)ang, &s, &c);
}

__global__ void __launch_bounds__(kAttnThreads) attn_decode_split_kernel(const AttnParams p) {
    __shared__ __align__(16) __half ks[kChunk * kKStride];
    __shared__ __align__(16) __half vs[kChunk * kHd];
    __shared__ float qs[kAttnMaxGroup * kHd];
    __shared__ float sc[kAttnMaxGroup * kChunk];
    __shared__ float cs_c[kHd / 2], cs_s[kHd / 2];

    const int g = blockIdx.x, chunk = blockIdx.y, tid = threadIdx.x;
    const int G = p.n_heads / p.n_kv_heads;
    const int pos = p.pos_dev ? *p.pos_dev : p.pos;  // graph replays read the position from device memory
    if (chunk * kChunk > pos) return;                // a chunk past the position (device-position launches)
    const int L = pos + 1;
    const int p0 = chunk * kChunk, np = min(kChunk, L - p0);
    // the chunk's K and V rows already in the cache, all loads in flight first
    const size_t head_off = (size_t)g * p.max_len * kHd;
    const int nold = min(np, pos - p0);
    constexpr int kLd = kChunk * (kHd / 8) / kAttnThreads;  // 16-byte loads per thread and matrix
    uint4 kr[kLd], vr[kLd];
#pragma unroll
    for (int j = 0; j < kLd; ++j) {
        const int idx = tid + j * kAttnThreads, r = idx / (kHd / 8), c8 = idx - r * (kHd / 8);
        if (r < nold) {
            const size_t src = head_off + (size_t)(p0 + r) * kHd + c8 * 8;
            kr[j] = __ldg(reinterpret_cast<const uint4*>(p.k_cache + src));
            vr[j] = __ldg(reinterpret_cast<const uint4*>(p.v_cache + src));
        }
    }
    if (tid < kHd / 2) rope_cs(pos, p.theta, tid, cs_c[tid], cs_s[tid]);
    __syncthreads();

    // rotated, scaled queries of this group
    const float scale = rsqrtf((float)kHd);
    for (int idx = tid; idx < G * (kHd / 2); idx += kAttnThreads) {
        const int h = idx / (kHd / 2), i = idx - h * (kHd / 2);
        const float* qh = p.q + (size_t)(g * G + h) * kHd;
        const float a = qh[i], b = qh[i + kHd / 2];
        qs[h * kHd + i] = (a * cs_c[i] - b * cs_s[i]) * scale;
        qs[h * kHd + i + kHd / 2] = (b * cs_c[i] + a * cs_s[i]) * scale;
    }
#pragma unroll
    for (int j = 0; j < kLd; ++j) {
        const int idx = tid + j * kAttnThreads, r = idx / (kHd / 8), c8 = idx - r * (kHd / 8);
        if (r < nold) {
            *reinterpret_cast<uint4*>(ks + r * kKStride + c8 * 8) = kr[j];
            *reinterpret_cast<uint4*>(vs + r * kHd + c8 * 8) = vr[j];
        }
    }
    // the row of pos comes from the inputs
    if (pos >= p0 && pos < p0 + kChunk && tid < kHd / 2) {
        const int r = pos - p0, i = tid;
        const float* kn = p.k_new + (size_t)g * kHd;
        const float* vn = p.v_new + (size_t)g * kHd;
        const float a = kn[i], b = kn[i + kHd / 2];
        const __half k0 = __float2half_rn(a * cs_c[i] - b * cs_s[i]);
        const __half k1 = __float2half_rn(b * cs_c[i] + a * cs_s[i]);
        const __half v0 = __float2half_rn(vn[i]), v1 = __float2half_rn(vn[i + kHd / 2]);
        ks[r * kKStride + i] = k0;
        ks[r * kKStride + i + kHd / 2] = k1;
        vs[r * kHd + i] = v0;
        vs[r * kHd + i + kHd / 2] = v1;
        const size_t dst = head_off + (size_t)pos * kHd;
        p.k_cache[dst + i] = __half_as_ushort(k0);
        p.k_cache[dst + i + kHd / 2] = __half_as_ushort(k1);
        p.v_cache[dst + i] = __half_as_ushort(v0);
        p.v_cache[dst + i + kHd / 2] = __half_as_ushort(v1);
    }
    __syncthreads();

    // scores: thread t -> position t % 64, heads t / 64, t / 64 + 2, ...
    {
        const int r = tid & (kChunk - 1), h0 = tid >> 6;
        float acc[kAttnMaxGroup / 2];
#pragma unroll
        for (int j = 0; j < kAttnMaxGroup / 2; ++j) acc[j] = 0.f;
        if (r < np) {
#pragma unroll 4
            for (int c8 = 0; c8 < kHd / 8; ++c8) {
                const uint4 raw = *reinterpret_cast<const uint4*>(ks + r * kKStride + c8 * 8);
                const __half2* hp = reinterpret_cast<const __half2*>(&raw);
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(hp[e]);
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int j = 0; j < kAttnMaxGroup / 2; ++j) {
                    const int h = h0 + 2 * j;
                    if (h < G) {
                        const float* qh = qs + h * kHd + c8 * 8;
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[j] = fmaf(qh[e], kf[e], acc[j]);
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kAttnMaxGroup / 2; ++j) {
            const int h = h0 + 2 * j;
            if (h < G) sc[h * kChunk + r] = (r < np) ? acc[j] : -INFINITY;
        }
    }
    __syncthreads();

    // per head: chunk maximum and sum of exponentials (one warp per head)
    __shared__ float mh[kAttnMaxGroup], lh[kAttnMaxGroup];
    {
        const int warp = tid >> 5, lane = tid & 31;
        for (int h = warp; h < G; h += kAttnThreads / 32) {
            float* s = sc + h * kChunk;
            float m = fmaxf(s[lane], s[lane + 32]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float e0 = (lane < np) ? __expf(s[lane] - m) : 0.f;
            const float e1 = (lane + 32 < np) ? __expf(s[lane + 32] - m) : 0.f;
            s[lane] = e0;
            s[lane + 32] = e1;
            float l = e0 + e1;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) { mh[h] = m; lh[h] = l; }
        }
    }
    __syncthreads();

    // unnormalised output of the chunk: thread t -> dimension t, all G heads
    {
        float acc[kAttnMaxGroup];
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h) acc[h] = 0.f;
        for (int r = 0; r < np; ++r) {
            const float v = __half2float(vs[r * kHd + tid]);
#pragma unroll
            for (int h = 0; h < kAttnMaxGroup; ++h)
                if (h < G) acc[h] = fmaf(sc[h * kChunk + r], v, acc[h]);
        }
        float* ws = p.work + ((size_t)g * p.nchunks + chunk) * G * (kHd + 2);
#pragma unroll
        for (int h = 0; h < kAttnMaxGroup; ++h)
            if (h < G) {
                ws[h * (kHd + 2) + tid] = acc[h];
                if (tid == 0) {
                    ws[h * (kHd + 2) + kHd] = mh[h];
                    ws[h * (kHd + 2) + kHd + 1] = lh[h];
                }
            }
    }
}

// Merge of the chunks of query head blockIdx.x (flash-decoding): warp 0 turns
// the chunks' (max, sum) statistics into weights exp(m_c - M) / sum_c l_c
// exp(m_c - M); then thread t sums dimension t over the chunks, the partials
// read independently (at most 64 chunks).
__global__ void __launch_bounds__(kAttnThreads) attn_combine_kernel(const AttnParams p) {
    __shared__ float wts[kChunk];
    const int hq = blockIdx.x, tid = threadIdx.x;
    const int G = p.n_heads / p.n_kv_heads, g = hq / G, h = hq - g * G;
    const int nact = ((p.pos_dev ? *p.pos_dev : p.pos) + kChunk) / kChunk;  // chunks written (<= p.nchunks)
    const size_t cstride = (size_t)G * (kHd + 2);
    const float* bh = p.work + (size_t)g * p.nchunks * cstride + (size_t)h * (kHd + 2);
    if (tid < 32) {
        const int lane = tid;
        const float m0 = lane < nact ? __ldg(bh + lane * cstride + kHd) : -INFINITY;
        const float m1 = lane + 32 < nact ? __ldg(bh + (lane + 32) * cstride + kHd) : -INFINITY;
        const float l0 = lane < nact ? __ldg(bh + lane * cstride + kHd + 1) : 0.f;
        const float l1 = lane + 32 < nact ? __ldg(bh + (lane + 32) * cstride + kHd + 1) : 0.f;
        float M = fmaxf(m0, m1);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float f0 = lane < nact ? __expf(m0 - M) : 0.f;
        const float f1 = lane + 32 < nact ? __expf(m1 - M) : 0.f;
        float l = l0 * f0 + l1 * f1;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        wts[lane] = f0 / l;
        wts[lane + 32] = f1 / l;
    }
    __syncthreads();
    float acc = 0.f;
#pragma unroll 8
    for (int c = 0; c < nact; ++c) acc = fmaf(__ldg(bh + c * cstride + tid), wts[c], acc);
    p.out[(size_t)hq * kHd + tid] = acc;
}


}  // namespace

// Partials [n_kv_heads][chunks][G][130] floats: a chunk's 128 unnormalised
// outputs, its score maximum and its sum of exponentials.
size_t attn_workspace_bytes(int n_heads, int n_kv_heads, int max_len) {
    const int G = n_kv_heads > 0 ? n_heads / n_kv_heads : 0;
    const int nchunks = (max_len + kChunk - 1) / kChunk;
    return (size_t)n_kv_heads * nchunks * G * (kHd + 2) * sizeof(float);
}

cudaError_t attn_decode_launch(AttnParams p, cudaStream_t stream) {
    if (p.head_dim != kHd || p.n_kv_heads <= 0 || p.n_heads % p.n_kv_heads) return cudaErrorInvalidValue;
    const int G = p.n_heads / p.n_kv_heads;
    if (G > kAttnMaxGroup || p.max_len > kAttnMaxLen) return cudaErrorInvalidValue;
    if (!p.pos_dev && (p.pos < 0 || p.pos >= p.max_len)) return cudaErrorInvalidValue;
    // a device position (0 <= *pos_dev < max_len, the caller's contract) gets
    // the launch shape of max_len: the same launch serves every position
    p.nchunks = p.pos_dev ? (p.max_len + kChunk - 1) / kChunk : (p.pos + 1 + kChunk - 1) / kChunk;
    attn_decode_split_kernel<<<dim3(p.n_kv_heads, p.nchunks), kAttnThreads, 0, stream>>>(p);
    attn_combine_kernel<<<p.n_heads, kAttnThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace glc
