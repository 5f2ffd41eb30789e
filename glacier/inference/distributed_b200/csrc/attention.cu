// attention.cu -- decode attention over an fp16 KV cache with grouped-query
// heads and rotary position embedding, for the attention half of a decode
// stage (the caller side of IClusterStageModel.ForwardStage,
// IClusterStageModel.cs:19; the reference's attention body is in its external
// model package, Program.cs:1390).
//
// One token at position pos: q [Hq][128] and the token's k, v [Hkv][128]
// (fp32, before rotation; optional biases added on load) come in; RoPE (NeoX /
// rotate-half pairing (i, i+64), theta^(-2i/128) frequencies, angles in
// double) rotates q and k; the rotated k and v are stored in the caches as
// fp16 at row pos; the output is softmax(q.K^T / sqrt(128)) V over positions
// 0..pos, query head h reading KV head h / G (G = Hq / Hkv query heads per KV
// head).
//
// HBM-bound (the cache rows are read once: 2 x Hkv x (pos+1) x 256 B), one
// launch: a thread-block cluster of C CTAs per KV head (C = 16 where the GPU
// can place such clusters, else 8) splits positions 0..pos evenly; each CTA
// stages its rows in rounds of 128 positions in shared memory (K rows padded
// to 272 B so the per-position 16-byte reads are conflict-free), computes the
// G x 128 scores with every K and V byte serving all G query heads, keeps a
// running maximum, sum of exponentials and unnormalised output per head, and
// leaves them in its shared memory; after a cluster barrier each CTA merges a
// 1/C slice of the KV head's G x 128 outputs from its peers' shared memory
// (flash-decoding, merged in rank order).  No workspace round trip and no
// second launch.  The CTA whose range holds pos builds that row from the
// inputs (fp16-rounded as stored) instead of reading it and writes it to the
// caches.
//
// Launched behind the QKV projection with programmatic stream serialisation:
// the cache rows below pos do not depend on that kernel, so every CTA issues
// its first round of row loads before it waits for the projection's output.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace glc {

namespace {

constexpr int kHd = 128;        // head dimension
constexpr int kRound = 128;     // positions staged per CTA round
constexpr int kKStride = 136;   // halves per staged K row (272 B)
constexpr int kAttnThreads = 256;
constexpr int kHeadsPerHalf = kAttnMaxGroup / 2;  // heads per thread half (heads half, half + 2, ...)
constexpr int kLd = kRound * (kHd / 8) / kAttnThreads;  // 16-byte loads per thread and matrix per round

struct AttnSmem {
    __half ks[kRound * kKStride];
    __half vs[kRound * kHd];
    float qs[kAttnMaxGroup * kHd];
    float sc[kAttnMaxGroup * kRound];
    float acc[kAttnMaxGroup * kHd];  // this CTA's unnormalised output (read by the cluster's merge)
    float m[kAttnMaxGroup];          // running score maximum per head (read by the merge)
    float l[kAttnMaxGroup];          // running sum of exponentials per head (read by the merge)
    float corr[kAttnMaxGroup];       // rescale of the previous rounds' output
    float cs_c[kHd / 2], cs_s[kHd / 2];
};

// RoPE of pair i (0..63) at position pos: cos and sin of pos * theta^(-2i/128),
// the angle formed and reduced to [-pi, pi] in double, then sincosf.
__device__ __forceinline__ void rope_cs(int pos, float theta, int i, float& c, float& s) {
    const double inv = exp(-(double)(2 * i) / (double)kHd * log((double)theta));
    double ang = (double)pos * inv;
    ang -= 6.283185307179586 * rint(ang * 0.15915494309189535);
    sincosf((float)ang, &s, &c);
}

__device__ __forceinline__ float ld_bias(const float* b, int i) { return b ? __ldg(b + i) : 0.f; }

template <int C>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);

    grid_dep_launch_dependents();
    const int r = (int)cl.block_rank(), g = blockIdx.y, tid = threadIdx.x;
    const int G = p.n_heads / p.n_kv_heads;
    // the position word is written before the kernel this launch follows starts
    const int pos = p.pos_dev ? *p.pos_dev : p.pos;
    const int L = pos + 1;
    const int lo = (int)((long long)r * L / C), hi = (int)((long long)(r + 1) * L / C);
    const size_t head_off = (size_t)g * p.max_len * kHd;
    const int half = tid >> 7, row_t = tid & (kRound - 1);

    float acc[kHeadsPerHalf];
#pragma unroll
    for (int j = 0; j < kHeadsPerHalf; ++j) acc[j] = 0.f;
    if (tid < kAttnMaxGroup) {
        S.m[tid] = -INFINITY;
        S.l[tid] = 0.f;
    }

    bool first = true;
    for (int base = lo; base < hi || first; base += kRound) {
        const int np = max(0, min(kRound, hi - base));
        const int nold = max(0, min(np, pos - base));  // rows already in the cache
        uint4 kr[kLd], vr[kLd];
#pragma unroll
        for (int j = 0; j < kLd; ++j) {
            const int idx = tid + j * kAttnThreads, rr = idx / (kHd / 8), c8 = idx - rr * (kHd / 8);
            if (rr < nold) {
                const size_t src = head_off + (size_t)(base + rr) * kHd + c8 * 8;
                kr[j] = __ldg(reinterpret_cast<const uint4*>(p.k_cache + src));
                vr[j] = __ldg(reinterpret_cast<const uint4*>(p.v_cache + src));
            }
        }
        if (first) {
            if (tid < kHd / 2) rope_cs(pos, p.theta, tid, S.cs_c[tid], S.cs_s[tid]);
            __syncthreads();
            grid_dep_wait();  // q, k and v are the previous kernel's output
            const float scale = rsqrtf((float)kHd);
            for (int idx = tid; idx < G * (kHd / 2); idx += kAttnThreads) {
                const int h = idx / (kHd / 2), i = idx - h * (kHd / 2);
                const int o = (g * G + h) * kHd;
                const float a = __ldg(p.q + o + i) + ld_bias(p.bq, o + i);
                const float b = __ldg(p.q + o + i + kHd / 2) + ld_bias(p.bq, o + i + kHd / 2);
                S.qs[h * kHd + i] = (a * S.cs_c[i] - b * S.cs_s[i]) * scale;
                S.qs[h * kHd + i + kHd / 2] = (b * S.cs_c[i] + a * S.cs_s[i]) * scale;
            }
            first = false;
        }
        if (np == 0) break;  // an empty range: the partials stay (-inf, 0, 0)
        const int np4 = (np + 3) & ~3;
#pragma unroll
        for (int j = 0; j < kLd; ++j) {
            const int idx = tid + j * kAttnThreads, rr = idx / (kHd / 8), c8 = idx - rr * (kHd / 8);
            if (rr < nold) {
                *reinterpret_cast<uint4*>(S.ks + rr * kKStride + c8 * 8) = kr[j];
                *reinterpret_cast<uint4*>(S.vs + rr * kHd + c8 * 8) = vr[j];
            } else if (rr >= np && rr < np4) {  // rows the value loop reads past the range: zero
                *reinterpret_cast<uint4*>(S.vs + rr * kHd + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        // the row of pos comes from the inputs
        if (pos >= base && pos < base + np && tid < kHd / 2) {
            const int rr = pos - base, i = tid, o = g * kHd;
            const float a = __ldg(p.k_new + o + i) + ld_bias(p.bk, o + i);
            const float b = __ldg(p.k_new + o + i + kHd / 2) + ld_bias(p.bk, o + i + kHd / 2);
            const __half k0 = __float2half_rn(a * S.cs_c[i] - b * S.cs_s[i]);
            const __half k1 = __float2half_rn(b * S.cs_c[i] + a * S.cs_s[i]);
            const __half v0 = __float2half_rn(__ldg(p.v_new + o + i) + ld_bias(p.bv, o + i));
            const __half v1 = __float2half_rn(__ldg(p.v_new + o + i + kHd / 2) + ld_bias(p.bv, o + i + kHd / 2));
            S.ks[rr * kKStride + i] = k0;
            S.ks[rr * kKStride + i + kHd / 2] = k1;
            S.vs[rr * kHd + i] = v0;
            S.vs[rr * kHd + i + kHd / 2] = v1;
            const size_t dst = head_off + (size_t)pos * kHd;
            p.k_cache[dst + i] = __half_as_ushort(k0);
            p.k_cache[dst + i + kHd / 2] = __half_as_ushort(k1);
            p.v_cache[dst + i] = __half_as_ushort(v0);
            p.v_cache[dst + i + kHd / 2] = __half_as_ushort(v1);
        }
        __syncthreads();

        // scores: thread t -> position t % 128, heads t / 128, t / 128 + 2, ...
        {
            float a[kHeadsPerHalf];
#pragma unroll
            for (int j = 0; j < kHeadsPerHalf; ++j) a[j] = 0.f;
            if (row_t < np) {
#pragma unroll 4
                for (int c8 = 0; c8 < kHd / 8; ++c8) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(S.ks + row_t * kKStride + c8 * 8);
                    const __half2* hp = reinterpret_cast<const __half2*>(&raw);
                    float kf[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(hp[e]);
                        kf[2 * e] = f.x;
                        kf[2 * e + 1] = f.y;
                    }
#pragma unroll
                    for (int j = 0; j < kHeadsPerHalf; ++j) {
                        const int h = half + 2 * j;
                        if (h < G) {
                            const float4 q0 = *reinterpret_cast<const float4*>(S.qs + h * kHd + c8 * 8);
                            const float4 q1 = *reinterpret_cast<const float4*>(S.qs + h * kHd + c8 * 8 + 4);
                            a[j] = fmaf(q0.x, kf[0], a[j]);
                            a[j] = fmaf(q0.y, kf[1], a[j]);
                            a[j] = fmaf(q0.z, kf[2], a[j]);
                            a[j] = fmaf(q0.w, kf[3], a[j]);
                            a[j] = fmaf(q1.x, kf[4], a[j]);
                            a[j] = fmaf(q1.y, kf[5], a[j]);
                            a[j] = fmaf(q1.z, kf[6], a[j]);
                            a[j] = fmaf(q1.w, kf[7], a[j]);
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kHeadsPerHalf; ++j) {
                const int h = half + 2 * j;
                if (h < G) S.sc[h * kRound + row_t] = (row_t < np) ? a[j] : -INFINITY;
            }
        }
        __syncthreads();

        // per head (one warp each): the round's maximum, exponentials and sum,
        // folded into the running statistics
        {
            const int warp = tid >> 5, lane = tid & 31;
            if (warp < G) {
                float* s = S.sc + warp * kRound;
                float v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = s[lane + 32 * q];
                float mc = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
                const float mold = S.m[warp];
                const float M = fmaxf(mold, mc);
                float ls = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float e = (lane + 32 * q < np) ? __expf(v[q] - M) : 0.f;
                    s[lane + 32 * q] = e;
                    ls += e;
                }
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
                __syncwarp();
                if (lane == 0) {
                    const float cr = (mold == -INFINITY) ? 0.f : __expf(mold - M);
                    S.corr[warp] = cr;
                    S.l[warp] = S.l[warp] * cr + ls;
                    S.m[warp] = M;
                }
            }
        }
        __syncthreads();

        // unnormalised output: thread t -> dimension t % 128, heads t / 128 + 2j
        {
            const int d = row_t;
#pragma unroll
            for (int j = 0; j < kHeadsPerHalf; ++j) {
                const int h = half + 2 * j;
                if (h < G) acc[j] *= S.corr[h];
            }
            for (int rr = 0; rr < np4; rr += 4) {
                float v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = __half2float(S.vs[(rr + q) * kHd + d]);
#pragma unroll
                for (int j = 0; j < kHeadsPerHalf; ++j) {
                    const int h = half + 2 * j;
                    if (h < G) {
                        const float4 e = *reinterpret_cast<const float4*>(S.sc + h * kRound + rr);
                        acc[j] = fmaf(e.x, v[0], acc[j]);
                        acc[j] = fmaf(e.y, v[1], acc[j]);
                        acc[j] = fmaf(e.z, v[2], acc[j]);
                        acc[j] = fmaf(e.w, v[3], acc[j]);
                    }
                }
            }
        }
        __syncthreads();  // the next round overwrites the staged rows and scores
    }
#pragma unroll
    for (int j = 0; j < kHeadsPerHalf; ++j) {
        const int h = half + 2 * j;
        if (h < G) S.acc[h * kHd + row_t] = acc[j];
    }

    // merge: CTA r writes outputs [r, r + 1) * G * 128 / C of this KV head
    cl.sync();
    const int GH = G * kHd;
    const int o0 = r * GH / C, o1 = (r + 1) * GH / C;
    for (int o = o0 + tid; o < o1; o += kAttnThreads) {
        const int h = o / kHd;
        float mp[C];
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const AttnSmem* peer = cl.map_shared_rank(&S, c);
            mp[c] = peer->m[h];
            M = fmaxf(M, mp[c]);
        }
        float lsum = 0.f, a = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const AttnSmem* peer = cl.map_shared_rank(&S, c);
            const float f = (mp[c] == -INFINITY) ? 0.f : __expf(mp[c] - M);
            lsum = fmaf(peer->l[h], f, lsum);
            a = fmaf(peer->acc[o], f, a);
        }
        p.out[(size_t)g * GH + o] = a / lsum;
    }
    cl.sync();  // every CTA's partials stay in place until the merge has read them
}

template <int C>
cudaError_t launch_cluster(const AttnParams& p, cudaStream_t stream) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(C, p.n_kv_heads);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<C>, p);
}

// Per device: 16-CTA clusters when the GPU can place one (non-portable size),
// else 8.  0 = not yet decided.
int g_cluster[kMaxDevices] = {0};

cudaError_t pick_cluster(int dev, int* c) {
    if (g_cluster[dev]) {
        *c = g_cluster[dev];
        return cudaSuccess;
    }
    const int smem = (int)sizeof(AttnSmem);
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_decode_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int n16 = 0;
    if (cudaFuncSetAttribute(attn_decode_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
        cudaSuccess) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(16, 8);
        cfg.blockDim = dim3(kAttnThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 16;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n16, attn_decode_kernel<16>, &cfg) != cudaSuccess) n16 = 0;
    }
    cudaGetLastError();  // a refused query leaves no sticky error
    g_cluster[dev] = n16 >= 1 ? 16 : 8;
    *c = g_cluster[dev];
    return cudaSuccess;
}

}  // namespace

// The kernel keeps its partial results in shared memory; the workspace is a
// reserved, unused argument of the C ABI.
size_t attn_workspace_bytes(int, int, int) { return 256; }

cudaError_t attn_decode_launch(AttnParams p, cudaStream_t stream) {
    if (p.head_dim != kHd || p.n_kv_heads <= 0 || p.n_heads % p.n_kv_heads) return cudaErrorInvalidValue;
    const int G = p.n_heads / p.n_kv_heads;
    if (G > kAttnMaxGroup || p.max_len <= 0 || p.max_len > kAttnMaxLen) return cudaErrorInvalidValue;
    if (!p.pos_dev && (p.pos < 0 || p.pos >= p.max_len)) return cudaErrorInvalidValue;
    if (p.n_kv_heads > 65535) return cudaErrorInvalidValue;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    int c = 8;
    cudaError_t e = pick_cluster(dev, &c);
    if (e != cudaSuccess) return e;
    return c == 16 ? launch_cluster<16>(p, stream) : launch_cluster<8>(p, stream);
}

}  // namespace glc
