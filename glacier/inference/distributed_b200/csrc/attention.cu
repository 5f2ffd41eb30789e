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
// stages its rows in rounds of 128 positions in shared memory and runs the
// two products of the round on the tensor cores (mma.sync m16n8k16, fp16
// operands, fp32 accumulation): scores S = Q K^T with the G query heads
// padded to 16 rows, and O += P V.  The fp32 operands are split into two
// fp16 halves (q = q_hi + q_lo, p = p_hi + p_lo, two products each), so the
// products carry ~22 bits of q and p against the fp16 cache values; the
// softmax is online over the rounds in fp32.  Each CTA leaves its running
// maximum, sum of exponentials and unnormalised output in shared memory;
// after a cluster barrier each CTA merges a 1/C slice of the KV head's
// G x 128 outputs from its peers' shared memory (flash-decoding, merged in
// rank order).  No workspace round trip and no second launch.  The CTA whose
// range holds pos builds that row from the inputs (fp16-rounded as stored)
// instead of reading it and writes it to the caches.
//
// Launched behind the QKV projection with programmatic stream serialisation:
// the cache rows below pos do not depend on that kernel, so every CTA issues
// its first round of row loads before it waits for the projection's output.
#include <cmath>
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace glc {

namespace {

constexpr int kHd = 128;        // head dimension
constexpr int kRound = 128;     // positions staged per CTA round
constexpr int kRow = 136;       // halves per staged row (272 B: ldmatrix rows conflict-free)
constexpr int kSRow = 132;      // floats per score row
constexpr int kAttnThreads = 256;
constexpr int kLd = kRound * (kHd / 8) / kAttnThreads;  // 16-byte loads per thread and matrix per round

struct AttnSmem {
    __half ks[kRound * kRow];        // K rows of the round (positions x dims)
    __half vs[kRound * kRow];        // V rows of the round
    __half qh[16 * kRow], ql[16 * kRow];  // rotated, scaled queries: fp16 high and low halves (rows >= G zero)
    __half ph[16 * kRow], pl[16 * kRow];  // exponentials of the round: fp16 high and low halves (rows >= G zero)
    float sc[16 * kSRow];            // scores of the round
    // received from every CTA r of the cluster (written by r into this CTA's
    // shared memory): its unnormalised outputs of this CTA's slice, and its
    // running maximum and sum of exponentials per head
    float rcv_acc[16][kAttnMaxGroup * kHd / 8];
    float rcv_m[16][kAttnMaxGroup];
    float rcv_l[16][kAttnMaxGroup];
    float m[16];                     // running score maximum per head
    float l[16];                     // running sum of exponentials per head
    float corr[16];                  // rescale of the previous rounds' output
    float cs_c[kHd / 2], cs_s[kHd / 2];
};

// RoPE of pair i (0..63) at position pos: cos and sin of pos * theta^(-2i/128)
// (the frequency formed on the host in double), the angle formed and reduced
// to [-pi, pi] in double, then sincosf.
__device__ __forceinline__ void rope_cs(int pos, double inv_freq, float& c, float& s) {
    double ang = (double)pos * inv_freq;
    ang -= 6.283185307179586 * rint(ang * 0.15915494309189535);
    sincosf((float)ang, &s, &c);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_older() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ float ld_bias(const float* b, int i) { return b ? __ldg(b + i) : 0.f; }

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(const void* p, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_trans(const void* p, uint32_t& r0, uint32_t& r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_u32(p)));
}
// d += a * b, m16n8k16, fp16 operands, fp32 accumulators
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The A fragment (16 x 16, rows r, cols k0..k0+15) of a [16][kRow] fp16 tile.
__device__ __forceinline__ void load_a(const __half* t, int k0, int lane, uint32_t (&a)[4]) {
    const int r = (lane & 7) + ((lane >> 3) & 1) * 8, c = k0 + (lane >> 4) * 8;
    ldsm_x4(t + r * kRow + c, a[0], a[1], a[2], a[3]);
}

template <int C>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);

    grid_dep_launch_dependents();
    const int r = (int)cl.block_rank(), g = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = p.n_heads / p.n_kv_heads;
    // the position word is written before the kernel this launch follows starts
    const int pos = p.pos_dev ? *p.pos_dev : p.pos;
    const int L = pos + 1;
    const int lo = (int)((long long)r * L / C), hi = (int)((long long)(r + 1) * L / C);
    const size_t head_off = (size_t)g * p.max_len * kHd;

    // padded query / exponential rows (>= G) stay zero; running statistics
    for (int i = tid; i < 16 * kRow; i += kAttnThreads) {
        S.qh[i] = S.ql[i] = S.ph[i] = S.pl[i] = __float2half_rn(0.f);
    }
    if (tid < 16) {
        S.m[tid] = -INFINITY;
        S.l[tid] = 0.f;
        S.corr[tid] = 1.f;  // padded rows keep 1 (their outputs stay zero)
    }
    // output accumulators: rows lane/4 and lane/4 + 8 (heads), dims 16 warp + 8 t + 2 (lane % 4) + {0, 1}
    float o[2][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[t][e] = 0.f;

    bool first = true;
    for (int base = lo; base < hi || first; base += kRound) {
        const int np = max(0, min(kRound, hi - base));
        const int nold = max(0, min(np, pos - base));  // rows already in the cache
        // the round's cache rows straight into shared memory (no register
        // staging), K rows in one copy group and V rows in the next, so the
        // scores start while V is in flight; rows past the range are zeroed
        // (their weights are zero)
#pragma unroll
        for (int j = 0; j < kLd; ++j) {
            const int idx = tid + j * kAttnThreads, rr = idx / (kHd / 8), c8 = idx - rr * (kHd / 8);
            if (rr < nold)
                cp_async16(S.ks + rr * kRow + c8 * 8, p.k_cache + head_off + (size_t)(base + rr) * kHd + c8 * 8);
            else if (rr >= np)
                *reinterpret_cast<uint4*>(S.ks + rr * kRow + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
        cp_async_commit();
#pragma unroll
        for (int j = 0; j < kLd; ++j) {
            const int idx = tid + j * kAttnThreads, rr = idx / (kHd / 8), c8 = idx - rr * (kHd / 8);
            if (rr < nold)
                cp_async16(S.vs + rr * kRow + c8 * 8, p.v_cache + head_off + (size_t)(base + rr) * kHd + c8 * 8);
            else if (rr >= np)
                *reinterpret_cast<uint4*>(S.vs + rr * kRow + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
        }
        cp_async_commit();
        if (first) {
            if (tid < kHd / 2) rope_cs(pos, p.inv_freq[tid], S.cs_c[tid], S.cs_s[tid]);
            __syncthreads();
            grid_dep_wait();  // q, k and v are the previous kernel's output
            const float scale = rsqrtf((float)kHd);
            for (int idx = tid; idx < G * (kHd / 2); idx += kAttnThreads) {
                const int h = idx / (kHd / 2), i = idx - h * (kHd / 2);
                const int o_ = (g * G + h) * kHd;
                const float a = __ldg(p.q + o_ + i) + ld_bias(p.bq, o_ + i);
                const float b = __ldg(p.q + o_ + i + kHd / 2) + ld_bias(p.bq, o_ + i + kHd / 2);
                const float q0 = (a * S.cs_c[i] - b * S.cs_s[i]) * scale;
                const float q1 = (b * S.cs_c[i] + a * S.cs_s[i]) * scale;
                const __half h0 = __float2half_rn(q0), h1 = __float2half_rn(q1);
                S.qh[h * kRow + i] = h0;
                S.qh[h * kRow + i + kHd / 2] = h1;
                S.ql[h * kRow + i] = __float2half_rn(q0 - __half2float(h0));
                S.ql[h * kRow + i + kHd / 2] = __float2half_rn(q1 - __half2float(h1));
            }
            first = false;
        }
        if (np == 0) {  // an empty range: the partials stay (-inf, 0, 0)
            cp_async_wait_all();
            break;
        }
        // the row of pos comes from the inputs
        if (pos >= base && pos < base + np && tid < kHd / 2) {
            const int rr = pos - base, i = tid, o_ = g * kHd;
            const float a = __ldg(p.k_new + o_ + i) + ld_bias(p.bk, o_ + i);
            const float b = __ldg(p.k_new + o_ + i + kHd / 2) + ld_bias(p.bk, o_ + i + kHd / 2);
            const __half k0 = __float2half_rn(a * S.cs_c[i] - b * S.cs_s[i]);
            const __half k1 = __float2half_rn(b * S.cs_c[i] + a * S.cs_s[i]);
            const __half v0 = __float2half_rn(__ldg(p.v_new + o_ + i) + ld_bias(p.bv, o_ + i));
            const __half v1 = __float2half_rn(__ldg(p.v_new + o_ + i + kHd / 2) + ld_bias(p.bv, o_ + i + kHd / 2));
            S.ks[rr * kRow + i] = k0;
            S.ks[rr * kRow + i + kHd / 2] = k1;
            S.vs[rr * kRow + i] = v0;
            S.vs[rr * kRow + i + kHd / 2] = v1;
            const size_t dst = head_off + (size_t)pos * kHd;
            p.k_cache[dst + i] = __half_as_ushort(k0);
            p.k_cache[dst + i + kHd / 2] = __half_as_ushort(k1);
            p.v_cache[dst + i] = __half_as_ushort(v0);
            p.v_cache[dst + i + kHd / 2] = __half_as_ushort(v1);
        }
        cp_async_wait_older();  // this thread's K rows have landed
        __syncthreads();

        // scores S = Q K^T: warp w -> positions 16 w .. 16 w + 15 (two n-tiles
        // of 8); the q_hi and q_lo products in separate accumulators (four
        // independent MMA chains instead of two), added at the end
        {
            float sacc[2][4], sacl[2][4];
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) sacc[t][e] = sacl[t][e] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < kHd; k0 += 16) {
                uint32_t ah[4], al[4];
                load_a(S.qh, k0, lane, ah);
                load_a(S.ql, k0, lane, al);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int n0 = 16 * warp + 8 * t;
                    uint32_t b0, b1;
                    ldsm_x2(S.ks + (n0 + (lane & 7)) * kRow + k0 + ((lane >> 3) & 1) * 8, b0, b1);
                    mma16816(sacc[t], ah, b0, b1);
                    mma16816(sacl[t], al, b0, b1);
                }
            }
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) sacc[t][e] += sacl[t][e];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int col = 16 * warp + 8 * t + (lane & 3) * 2, row = lane >> 2;
                S.sc[row * kSRow + col] = col < np ? sacc[t][0] : -INFINITY;
                S.sc[row * kSRow + col + 1] = col + 1 < np ? sacc[t][1] : -INFINITY;
                S.sc[(row + 8) * kSRow + col] = col < np ? sacc[t][2] : -INFINITY;
                S.sc[(row + 8) * kSRow + col + 1] = col + 1 < np ? sacc[t][3] : -INFINITY;
            }
        }
        __syncthreads();

        // per head (one warp each): the round's maximum, exponentials (fp16
        // halves for the tensor cores) and sum, folded into the running statistics
        if (warp < G) {
            const float* s = S.sc + warp * kSRow;
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = s[lane + 32 * q];
            float mc = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
            const float mold = S.m[warp];
            const float M = fmaxf(mold, mc);
            float ls = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int c = lane + 32 * q;
                const float e = (c < np) ? __expf(v[q] - M) : 0.f;
                const __half eh = __float2half_rn(e);
                S.ph[warp * kRow + c] = eh;
                S.pl[warp * kRow + c] = __float2half_rn(e - __half2float(eh));
                ls += e;
            }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
            __syncwarp();
            if (lane == 0) {
                const float cr = (mold == -INFINITY) ? 0.f : __expf(mold - M);
                S.corr[warp] = cr;
                S.l[warp] = S.l[warp] * cr + ls;
                S.m[warp] = M;
            }
        }
        cp_async_wait_all();  // this thread's V rows have landed
        __syncthreads();

        // O = O * corr + P V: warp w -> dims 16 w .. 16 w + 15 (two n-tiles
        // of 8); the round's p_lo products in their own accumulators, added
        // after the loop
        {
            const int row = lane >> 2;
            const float c0 = S.corr[row], c1 = S.corr[row + 8];
            float ol[2][4];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                o[t][0] *= c0;
                o[t][1] *= c0;
                o[t][2] *= c1;
                o[t][3] *= c1;
#pragma unroll
                for (int e = 0; e < 4; ++e) ol[t][e] = 0.f;
            }
#pragma unroll
            for (int k0 = 0; k0 < kRound; k0 += 16) {
                uint32_t ah[4], al[4];
                load_a(S.ph, k0, lane, ah);
                load_a(S.pl, k0, lane, al);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int d0 = 16 * warp + 8 * t;
                    uint32_t b0, b1;
                    ldsm_x2_trans(S.vs + (k0 + (lane & 7) + ((lane >> 3) & 1) * 8) * kRow + d0, b0, b1);
                    mma16816(o[t], ah, b0, b1);
                    mma16816(ol[t], al, b0, b1);
                }
            }
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[t][e] += ol[t][e];
        }
        __syncthreads();  // the next round overwrites the staged rows, scores and exponentials
    }
    // merge (flash-decoding): CTA q of the cluster owns outputs [q, q + 1) *
    // slice of this KV head (slice = G * 128 / C); every CTA writes its
    // partials for each owner into that owner's shared memory, then one
    // cluster barrier, then each owner merges in rank order from its own
    // shared memory and writes the outputs.
    const int GH = G * kHd, slice = GH / C;
    {
        const int row = lane >> 2;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int d = 16 * warp + 8 * t + (lane & 3) * 2;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int h = row + 8 * hh;
                if (h < G) {
                    const int oi = h * kHd + d, owner = oi / slice, off = oi - owner * slice;
                    float* dst = cl.map_shared_rank(&S.rcv_acc[r][off], owner);
                    dst[0] = o[t][2 * hh];
                    dst[1] = o[t][2 * hh + 1];  // d even, slice even: the pair stays with one owner
                }
            }
        }
        if (tid < C * G) {
            const int owner = tid / G, h = tid - owner * G;
            *cl.map_shared_rank(&S.rcv_m[r][h], owner) = S.m[h];
            *cl.map_shared_rank(&S.rcv_l[r][h], owner) = S.l[h];
        }
    }
    cl.sync();  // every CTA's partials are in their owners' shared memory
    for (int off = tid; off < slice; off += kAttnThreads) {
        const int oi = r * slice + off, h = oi / kHd;
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < C; ++c) M = fmaxf(M, S.rcv_m[c][h]);
        float lsum = 0.f, a = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const float mc = S.rcv_m[c][h];
            const float f = (mc == -INFINITY) ? 0.f : __expf(mc - M);
            lsum = fmaf(S.rcv_l[c][h], f, lsum);
            a = fmaf(S.rcv_acc[c][off], f, a);
        }
        p.out[(size_t)g * GH + oi] = a / lsum;
    }
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

// Per device: how many 16-CTA (non-portable size) and 8-CTA clusters of this
// kernel the GPU can hold at once; 0 = not yet measured.
struct ClusterFit {
    int n16 = 0, n8 = 0;
    bool done = false;
};
ClusterFit g_fit[kMaxDevices];

template <int C>
int max_clusters() {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(C, 8);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<C>, &cfg) != cudaSuccess) n = 0;
    return n;
}

cudaError_t cluster_fit(int dev, ClusterFit** out) {
    ClusterFit& f = g_fit[dev];
    if (!f.done) {
        const int smem = (int)sizeof(AttnSmem);
        cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_decode_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        f.n8 = max_clusters<8>();
        if (cudaFuncSetAttribute(attn_decode_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
            cudaSuccess)
            f.n16 = max_clusters<16>();
        cudaGetLastError();  // a refused query leaves no sticky error
        f.done = true;
    }
    *out = &f;
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
    for (int i = 0; i < kHd / 2; ++i)
        p.inv_freq[i] = std::exp(-(double)(2 * i) / (double)kHd * std::log((double)p.theta));
    ClusterFit* f = nullptr;
    cudaError_t e = cluster_fit(dev, &f);
    if (e != cudaSuccess) return e;
    // 16-CTA clusters only when all of the launch's clusters fit at once (a
    // second wave of clusters would double the time)
    return f->n16 >= p.n_kv_heads ? launch_cluster<16>(p, stream) : launch_cluster<8>(p, stream);
}

}  // namespace glc
