// grouped_mma.cu -- grouped expert GEMM for the batched (prefill) MoE path on
// sm_100a tensor cores (tcgen05 + TMEM), with Q4_K weights dequantised on the
// fly.  Replaces the per-token expert loop behind IClusterStageModel.ForwardBatchStage
// (IClusterStageModel.cs:24) for MoE layers.
//
// One work item = (group g of <= 32 tokens routed to expert e, 128 output rows;
// <= 64 tokens in the wide layout below).
//   D[128 x N] = A[128 x K] * B[N x K]^T,  A = expert weight rows (fp16 values
//   d*sc*q - dmin*m, one rounding), B = the group's activations as fp16 hi/lo
//   halves (N = 2 * roundup8(ntok)); the epilogue adds the hi and lo columns and
//   applies the row's power-of-two scale, so activations keep ~22 bits.
//
// Warp roles (512 threads, one CTA per SM, persistent over work items):
//   w0      TMA: raw Q4_K tiles (2-D tensor map, box 144 B x 128 rows, one
//           super-block) into the raw ring, completing on raw_full[stage]; a
//           raw stage is refilled as soon as the dequantisers have read it.
//   w15     loads the B tile of each super-block (1-D bulk copy) into a
//           separate 2-stage ring that the MMA issuers release; keeping B out
//           of the raw ring lets the weight prefetch run up to 4 (gate/up) or
//           8 (down) super-blocks ahead of the dequantisers.  No multicast.
//   w1..w8  dequantise, two groups of four warps (one TMEM lane quarter each).
//           Work comes in A units of 128 TMEM columns = 16 MMAs of K 16: half a
//           super-block of both matrices (gate/up), or a whole super-block of
//           the one matrix (down); the groups take alternate units.  A warp
//           turns its 32 rows of the unit into fp16 pairs (PRMT + LOP3 nibble ->
//           1024+q half trick, two HFMA2s, exact q*sc) and stores them to TMEM
//           with tcgen05.st: A never touches shared memory, which keeps
//           shared-memory traffic at ~2x the HBM bytes.
//   w9, w14 the two MMA issuers (w9 also allocates TMEM).  Issuer i owns
//           accumulator i and issues the MMAs of sub-unit i of every A unit
//           (gate/up: matrix i; down: K half i of each super-block), A from
//           TMEM, B from a SWIZZLE_128B shared-memory descriptor, committing
//           the unit's slot back to the dequantisers when its MMAs complete.
//           An issuing thread's own shared-memory accesses (mbarrier waits)
//           wait behind its queued MMAs (~260 cycles each, measured); with two
//           issuers one waits while the other's MMAs run, which holds the
//           tensor core near its ~44-cycle floor per M=128 MMA.
//   w10..13 epilogue: tcgen05.ld of the accumulators, SwiGLU (gate/up) or the
//           sum of the two K halves (down), coalesced fp32 stores per token.
// TMEM columns: accumulator i at [64i, +64); a ring of three A units at
// [128 + 128u, +128).  The unit size is set by the tensor core: an M=128
// kind::f16 MMA costs ~44 cycles for any N <= 64 (measured), and a wait +
// fence + commit between every 8 MMAs nearly doubled that, so each hand-off
// covers 16 MMAs; the ring lets dequantisation run up to two units ahead.
// Wide layout (groups of <= 64 tokens, N <= 128): accumulator i at
// [128i, +128), two A units at [256 + 128u, +128), B stages of 128 rows.  A
// group's weights are dequantised once for up to 64 tokens instead of once
// per 32; each output is the same fp32 sum over the same K order.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace glc {

constexpr int kTcThreads = 16 * 32;
constexpr int kBStages = 2;          // B-tile ring, separate from the raw-weight ring
constexpr unsigned kPollNs = 64;     // sleep between polls of the roles that wait most (see mbar_wait_backoff)
constexpr int kRawTile = 128 * 144;          // one super-block x 128 rows
constexpr uint32_t kTmemCols = 512;

// TMEM and B-ring layout of the narrow (WIDE = false) and wide instantiations.
template <bool WIDE>
struct TcLayout {
    static constexpr int kNMax = WIDE ? 128 : 64;                 // MMA N: hi + lo columns of the group
    static constexpr uint32_t kAccStride = WIDE ? 128u : 64u;     // TMEM columns of one accumulator
    static constexpr uint32_t kAccCols = 2u * kAccStride;         // both accumulators
    static constexpr int kAUnits = WIDE ? 2 : 3;                  // TMEM A ring of 128-column units
    static constexpr int kBStageBytes = kNMax * 512;              // N_max rows x 256 K x fp16
    static_assert(kAccCols + 128u * kAUnits <= kTmemCols, "TMEM layout exceeds the allocation");
};

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (fp16 x fp16 -> fp32).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

#define TC_ST32(taddr, r)                                                                                  \
    asm volatile(                                                                                          \
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16," \
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                  \
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),  \
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),       \
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),      \
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                   \
        : "memory")

#define TC_LD32(taddr, r)                                                                                  \
    asm volatile(                                                                                          \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16," \
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                             \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),   \
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),         \
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),       \
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),       \
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                                                           \
        : "r"(taddr)                                                                                      \
        : "memory")

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// SWIZZLE_128B K-major shared-memory matrix descriptor (sm_100 format):
// start>>4 [0,14), LBO>>4 [16,30) (unused for swizzled K-major, 1), SBO>>4
// [32,46) = 1024 B between 8-row groups, version 1 at [46,48), layout 2 at [61,64).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint64_t a = smem_u32(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((1024ull >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, M = 128.
__device__ __forceinline__ uint32_t idesc_f16(int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// fp16x2 bit patterns of constants
constexpr uint32_t kH2_1024 = 0x64006400u, kH2_m1024 = 0xE400E400u, kH2_1_16 = 0x2C002C00u, kH2_m64 = 0xD400D400u;

// One super-block row's header: d and -dmin as fp16x2, and the 12 bytes of
// packed 6-bit scales / mins (GGUF Q4_K).
struct Q4kRowHdr {
    uint32_t dd, ndm, y, z, w;
};

// Plain (schedulable) 16-byte shared-memory load: the compiler may issue a
// unit's loads back to back, so one queueing delay behind MMAs covers all of them.
__device__ __forceinline__ uint4 ld_sh128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ Q4kRowHdr make_hdr(const uint4 h) {
    Q4kRowHdr r;
    r.dd = (h.x & 0xFFFFu) | (h.x << 16);
    const uint32_t nm = (h.x >> 16) ^ 0x8000u;
    r.ndm = nm | (nm << 16);
    r.y = h.y;
    r.z = h.z;
    r.w = h.w;
    return r;
}

// Dequantise one 64-weight chunk (qs bytes [32c, 32c+32) of a super-block row)
// into 32 packed fp16 pairs: words 0..15 = sub-block 2c (K 0..31 of the chunk),
// words 16..31 = sub-block 2c+1 (K 32..63).  weight = d*(sc*q) - dmin*m with
// sc*q exact (the 1024+q half trick and two HFMA2s) and -dmin*m one rounding.
// The per-sub-block factors are built without conversion instructions: PRMT
// puts a 6-bit scale or min x into the mantissa of 1024 + x and one fp16
// subtraction leaves x exactly; every later product is exact except dmin*m,
// rounded once like a float -> half conversion of the exact product.
// q0, q1: qs bytes [32c, 32c+16) and [32c+16, 32c+32) of the row.
__device__ __forceinline__ void dequant_chunk(const Q4kRowHdr& hd, const uint4 q0, const uint4 q1, int c,
                                              uint32_t (&r)[32]) {
    // 6-bit scale / min of sub-blocks 2c and 2c+1 (get_scale_min_k4): bytes 0 and 1
    const int sh = (c & 1) * 16;
    const uint32_t Y = hd.y >> sh, Z = hd.z >> sh, W = hd.w >> sh;
    uint32_t scp, mp;
    if (c < 2) {
        scp = Y & 0x3F3Fu;
        mp = Z & 0x3F3Fu;
    } else {
        scp = (W & 0x0F0Fu) | ((Y >> 2) & 0x3030u);
        mp = ((W >> 4) & 0x0F0Fu) | ((Z >> 2) & 0x3030u);
    }
    const uint32_t a_lo = hsub2_u(prmt(scp, 0x64u, 0x4040u), kH2_1024);           // sc0
    const uint32_t a_hi = hfma2_u(prmt(scp, 0x64u, 0x4141u), kH2_1_16, kH2_m64);  // sc1 / 16
    const uint32_t b_lo = hmul2_u(a_lo, kH2_m1024);                                // -1024 sc0
    const uint32_t b_hi = hmul2_u(a_hi, kH2_m1024);                                // -64 sc1
    const uint32_t n_lo = hmul2_u(hsub2_u(prmt(mp, 0x64u, 0x4040u), kH2_1024), hd.ndm);  // -dmin m0
    const uint32_t n_hi = hmul2_u(hsub2_u(prmt(mp, 0x64u, 0x4141u), kH2_1024), hd.ndm);  // -dmin m1
    const uint32_t dd = hd.dd;
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t t0 = prmt(w[i], 0u, 0x4140u);  // bytes 0,1 -> halves
        const uint32_t t1 = prmt(w[i], 0u, 0x4342u);  // bytes 2,3 -> halves
        const uint32_t l0 = (t0 & 0x000F000Fu) | 0x64006400u;
        const uint32_t l1 = (t1 & 0x000F000Fu) | 0x64006400u;
        const uint32_t g0 = (t0 & 0x00F000F0u) | 0x64006400u;
        const uint32_t g1 = (t1 & 0x00F000F0u) | 0x64006400u;
        r[2 * i] = hfma2_u(hfma2_u(l0, a_lo, b_lo), dd, n_lo);
        r[2 * i + 1] = hfma2_u(hfma2_u(l1, a_lo, b_lo), dd, n_lo);
        r[16 + 2 * i] = hfma2_u(hfma2_u(g0, a_hi, b_hi), dd, n_hi);
        r[16 + 2 * i + 1] = hfma2_u(hfma2_u(g1, a_hi, b_hi), dd, n_hi);
    }
}

#define TC_LD8(taddr, r)                                                                                  \
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"                 \
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
                   "=r"(r[7])                                                                              \
                 : "r"(taddr)                                                                              \
                 : "memory")

// Epilogue of one row for the group's tokens.  Accumulator i (TMEM columns
// [ACS i, +ACS)) holds hi columns [0, HALF) and lo columns [HALF, 2 HALF).
// Gate/up (nm = 2): accumulator 0 = gate, 1 = up, SwiGLU.  Down (nm = 1): the
// two accumulators are the two K halves of every super-block, added in fixed
// order.  The tensor core waits for the accumulators to be released
// (acc_empty) before the next work item, so up to 16 tokens (64 registers)
// are loaded in one go and released before any arithmetic; wider groups go
// in passes of 8 tokens (released after the last pass's loads).
template <int HALF, uint32_t ACS>
__device__ __forceinline__ void epilogue_item(uint32_t trow, int nm, int ntok, const float* rs, float* o, int stride,
                                              uint64_t* acc_empty, int lane) {
    constexpr int PASS = (HALF <= 16) ? HALF : 8;
#pragma unroll
    for (int p0 = 0; p0 < HALF; p0 += PASS) {
        uint32_t ah[PASS], al[PASS], bh[PASS], bl[PASS];
#pragma unroll
        for (int c = 0; c < PASS; c += 8) {
            TC_LD8(trow + (uint32_t)(p0 + c), (&ah[c]));
            TC_LD8(trow + (uint32_t)(HALF + p0 + c), (&al[c]));
            TC_LD8(trow + ACS + (uint32_t)(p0 + c), (&bh[c]));
            TC_LD8(trow + ACS + (uint32_t)(HALF + p0 + c), (&bl[c]));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (p0 + PASS >= HALF) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
        }
#pragma unroll
        for (int i = 0; i < PASS; ++i) {
            const int n = p0 + i;
            if (n < ntok) {
                const float sc = __ldg(rs + n);
                const float gh = __uint_as_float(ah[i]), gl = __uint_as_float(al[i]);
                const float uh = __uint_as_float(bh[i]), ul = __uint_as_float(bl[i]);
                float v;
                if (nm == 2) {
                    const float g = (gh + gl) * sc, u = (uh + ul) * sc;
                    v = (g / (1.0f + expf(-g))) * u;
                } else {
                    v = ((gh + uh) + (gl + ul)) * sc;
                }
                o[(size_t)n * stride] = v;
            }
        }
    }
}

// Work item -> (group g, 128-row tile mt, K slice ks) and the K slice's
// super-blocks [s0, s1).  The K slice is the fastest-varying index; every
// role of the CTA walks the same items in the same order.
struct ItemCoords {
    int g, mt, ks, s0, s1;
};
__device__ __forceinline__ ItemCoords item_coords(int item, int mtiles, int ksplit, int nsb) {
    ItemCoords c;
    c.ks = item % ksplit;
    const int r = item / ksplit;
    c.g = r / mtiles;
    c.mt = r - c.g * mtiles;
    c.s0 = (int)((long long)nsb * c.ks / ksplit);
    c.s1 = (int)((long long)nsb * (c.ks + 1) / ksplit);
    return c;
}

template <bool WIDE>
__global__ void __launch_bounds__(kTcThreads, 1)
    grouped_q4k_mma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ GroupedParams p, int stages) {
    using L = TcLayout<WIDE>;
    constexpr int kAUnits = L::kAUnits;
    constexpr uint32_t kAccCols = L::kAccCols;
    constexpr int kBStageBytes = L::kBStageBytes;
    // shared memory: [kBStages][kBStageBytes] B ring (1024-aligned) | [S][nm][kRawTile] raw ring | mbarriers
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    const int S = stages;
    uint8_t* bst = smem;
    uint8_t* raw = bst + (size_t)kBStages * kBStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(raw + (size_t)S * p.nm * kRawTile);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = bars + S;
    uint64_t* b_full = bars + 2 * S;
    uint64_t* b_empty = b_full + kBStages;
    uint64_t* a_full = b_empty + kBStages;
    uint64_t* a_empty = a_full + kAUnits;
    uint64_t* acc_full = a_empty + kAUnits;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* mma_drain = acc_empty + 1;  // one per MMA issuer: its MMAs done before an early exit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_drain + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nm = p.nm;
    const int nsb = p.K >> 8;
    const int mtiles = p.rows_per_e >> 7;
    const int ngroups = p.plan.meta[0];
    const int ksplit = p.ksplit > 0 ? p.ksplit : 1;
    const int nitems = ngroups * mtiles * ksplit;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 8);
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 2);
        }
        for (int u = 0; u < kAUnits; ++u) {
            mbar_init(&a_full[u], 4);
            mbar_init(&a_empty[u], 2);
        }
        mbar_init(acc_full, 2);
        mbar_init(acc_empty, 4);
        mbar_init(&mma_drain[0], 1);
        mbar_init(&mma_drain[1], 1);
        fence_mbar_init();
    }
    if (warp == 9) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------- raw TMA
        if (lane == 0) {
            bool ok = true;
            int it = 0;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const ItemCoords ic = item_coords(item, mtiles, ksplit, nsb);
                // a group wider than this layout's B stage (a plan built for
                // the wide layout given to the narrow one): every role stops
                // at the same item, nothing of it issued
                if (p.plan.grp_N[ic.g] > L::kNMax) { atomicExch(p.err, kDevBadArg); break; }
                const int e = p.plan.grp_e[ic.g];
                const int row0 = e * p.rows_per_e + ic.mt * 128;
                for (int s = ic.s0; s < ic.s1; ++s, ++it) {
                    const int stg = it % S;
                    const uint32_t ph = (uint32_t)(it / S) & 1u;
                    if (!mbar_wait_backoff(&raw_empty[stg], ph ^ 1u, p.err, kDevTimeoutEmpty, kPollNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&raw_full[stg], (uint32_t)(nm * kRawTile));
                    uint8_t* rdst = raw + (size_t)stg * nm * kRawTile;
                    tma_load_2d(rdst, &tmA, s * 144, row0, &raw_full[stg]);
                    if (nm == 2) tma_load_2d(rdst + kRawTile, &tmB, s * 144, row0, &raw_full[stg]);
                }
            }
            // the tiles in flight land before the CTA can exit (also when the
            // dequantisers abandoned the ring after a failed wait)
            drain_issued_stages(raw_full, S, it, kWaitLimitNs);
        }
    } else if (warp == 15) {
        // ------------------------------------------------------------ B tiles
        if (lane == 0) {
            bool ok = true;
            int it = 0;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const ItemCoords ic = item_coords(item, mtiles, ksplit, nsb);
                const int N = p.plan.grp_N[ic.g];
                if (N > L::kNMax) break;
                const uint8_t* bsrc = p.btiles + (size_t)p.plan.grp_units[ic.g] * 512u * nsb;
                for (int s = ic.s0; s < ic.s1; ++s, ++it) {
                    const int stg = it % kBStages;
                    const uint32_t ph = (uint32_t)(it / kBStages) & 1u;
                    if (!mbar_wait_backoff(&b_empty[stg], ph ^ 1u, p.err, kDevTimeoutEmpty, kPollNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&b_full[stg], (uint32_t)(N * 512));
                    bulk_g2s_plain(bst + (size_t)stg * kBStageBytes, bsrc + (size_t)s * N * 512, (uint32_t)(N * 512),
                                   &b_full[stg]);
                }
            }
            drain_issued_stages(b_full, kBStages, it, kWaitLimitNs);
        }
    } else if (warp >= 1 && warp <= 8) {
        // ------------------------------------------------------- dequantise
        const int grp = (warp - 1) >> 2;       // takes units u with u % 2 == grp
        const int q = warp & 3;                // TMEM lane quarter of this warp
        const int row = 32 * q + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
        const int upsb = (nm == 2) ? 2 : 1;    // units per super-block
        bool ok = true;
        int it = 0, u = 0;                     // super-block and unit counters over all items
        for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
            const ItemCoords ic = item_coords(item, mtiles, ksplit, nsb);
            if (p.plan.grp_N[ic.g] > L::kNMax) break;
            for (int s = ic.s0; s < ic.s1 && ok; ++s, ++it) {
                const int stg = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (!mbar_wait(&raw_full[stg], ph, p.err, kDevTimeoutFull)) { ok = false; break; }
                const uint8_t* rsrc = raw + (size_t)stg * nm * kRawTile + (size_t)row * 144;
                for (int j = 0; j < upsb; ++j, ++u) {
                    if ((u & 1) != grp) continue;
                    const int slot = u % kAUnits;
                    const uint32_t uph = ((uint32_t)(u / kAUnits) & 1u) ^ 1u;
                    if (!mbar_wait(&a_empty[slot], uph, p.err, kDevTimeoutEmpty)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t tcol = kAccCols + 128u * (uint32_t)slot;
                    // sub-unit v (64 columns): matrix v of half j (gate/up), or half v of matrix 0 (down)
                    // all of the unit's shared-memory reads first: 2 row headers + 8 quant words
                    uint4 hw[2], qw[2][2][2];
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const int m = (nm == 2) ? v : 0, hh = (nm == 2) ? j : v;
                        const uint8_t* blk = rsrc + (size_t)m * kRawTile;
                        hw[v] = ld_sh128(blk);
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const int c = 2 * hh + cc;
                            qw[v][cc][0] = ld_sh128(blk + 16 + 32 * c);
                            qw[v][cc][1] = ld_sh128(blk + 32 + 32 * c);
                        }
                    }
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const int hh = (nm == 2) ? j : v;
                        const Q4kRowHdr hd = make_hdr(hw[v]);
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            uint32_t r[32];
                            dequant_chunk(hd, qw[v][cc][0], qw[v][cc][1], 2 * hh + cc, r);
                            TC_ST32(trow + tcol + 64u * v + 32u * cc, r);
                        }
                    }
                    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[slot]);
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&raw_empty[stg]);
            }
        }
    } else if (warp == 9 || warp == 14) {
        // ---------------------------------------------------------------- MMA
        const int v = (warp == 9) ? 0 : 1;     // this issuer's accumulator / sub-unit
        if (lane == 0) {
            bool ok = true;
            int it = 0, u = 0, icount = 0;
            const int upsb = (nm == 2) ? 2 : 1;
            const uint32_t dcol = tmem + L::kAccStride * (uint32_t)v;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++icount) {
                const ItemCoords ic = item_coords(item, mtiles, ksplit, nsb);
                const int N = p.plan.grp_N[ic.g];
                if (N > L::kNMax) break;
                const uint32_t idesc = idesc_f16(N);
                const uint32_t cstride = (uint32_t)N * 128u;  // bytes between the 4 K chunks of the B tile
                if (!mbar_wait_backoff(acc_empty, ((uint32_t)icount & 1u) ^ 1u, p.err, kDevTimeoutEmpty, kPollNs)) { ok = false; break; }
                tc_fence_after();
                for (int s = ic.s0; s < ic.s1 && ok; ++s, ++it) {
                    const int stg = it % kBStages;
                    const uint32_t ph = (uint32_t)(it / kBStages) & 1u;
                    if (!mbar_wait_backoff(&b_full[stg], ph, p.err, kDevTimeoutFull, kPollNs)) { ok = false; break; }
                    // descriptor of the stage's B tile; K steps add their byte offset >> 4
                    // to the start-address field (addresses stay below 2^18)
                    const uint64_t bbase = sw128_desc(bst + (size_t)stg * kBStageBytes);
                    for (int j = 0; j < upsb; ++j, ++u) {
                        const int slot = u % kAUnits;
                        if (!mbar_wait_backoff(&a_full[slot], (uint32_t)(u / kAUnits) & 1u, p.err, kDevTimeoutFull, kPollNs)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int hh = (nm == 2) ? j : v;  // K half of the super-block
                        const bool first = (s == ic.s0) && (nm == 1 || j == 0);
                        const uint32_t acol = tmem + kAccCols + 128u * (uint32_t)slot + 64u * (uint32_t)v;
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk) {
                            const uint32_t off = (uint32_t)(2 * hh + (kk >> 2)) * cstride + (uint32_t)(kk & 3) * 32u;
                            tc_mma_ts(dcol, acol + 8u * kk, bbase + (off >> 4), idesc, (first && kk == 0) ? 0u : 1u);
                        }
                        tc_commit(&a_empty[slot]);
                    }
                    if (!ok) break;
                    tc_commit(&b_empty[stg]);
                }
                if (ok) tc_commit(acc_full);
            }
            if (!ok) {
                // gave up: every MMA this thread issued completes before the
                // CTA frees its tensor memory and exits
                tc_commit(&mma_drain[v]);
                mbar_wait(&mma_drain[v], 0, nullptr, 0, kWaitLimitNs);
            }
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int row = 32 * q + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
        bool ok = true;
        int icount = 0;
        for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++icount) {
            const ItemCoords ic = item_coords(item, mtiles, ksplit, nsb);
            const int g = ic.g, mt = ic.mt;
            const int N = p.plan.grp_N[g];
            const int ntok = p.plan.grp_ntok[g];
            const int pos0 = p.plan.grp_pos0[g];
            if (N > L::kNMax) break;
            if (!mbar_wait_backoff(acc_full, (uint32_t)icount & 1u, p.err, kDevTimeoutFull, kPollNs)) { ok = false; break; }
            tc_fence_after();
            // a K slice writes its partial sums to its own plane of the output
            float* o = p.out + (size_t)ic.ks * (size_t)p.part_stride + (size_t)pos0 * p.rows_per_e +
                       (size_t)mt * 128 + row;
            const float* rs = p.rscale + pos0;
            constexpr uint32_t A = L::kAccStride;
            switch (N) {  // hi columns [0, N/2), lo columns [N/2, N) of each accumulator
                case 16: epilogue_item<8, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                case 32: epilogue_item<16, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                case 48: epilogue_item<24, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                case 64: epilogue_item<32, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                default:
                    if constexpr (WIDE) {
                        switch (N) {
                            case 80: epilogue_item<40, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                            case 96: epilogue_item<48, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                            case 112: epilogue_item<56, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                            default: epilogue_item<64, A>(trow, nm, ntok, rs, o, p.rows_per_e, acc_empty, lane); break;
                        }
                    }
                    break;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int make_q4k_tensor_map(void* tmap64, const void* base, long long rows, int row_bytes) {
    static PFN_encodeTiled fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess || !ptr)
            return -1;
        fn = (PFN_encodeTiled)ptr;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {144, 128};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(reinterpret_cast<CUtensorMap*>(tmap64), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                    dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -2;
}

cudaError_t grouped_launch(const void* tmapA, const void* tmapB, const GroupedParams& p, int max_items, int num_sms,
                           cudaStream_t st) {
    if ((p.K & 255) || (p.rows_per_e & 127) || (p.nm != 1 && p.nm != 2)) return cudaErrorInvalidValue;
    // K slices only for the plain projection (the SwiGLU epilogue needs whole sums)
    if (p.ksplit < 1 || (p.ksplit > 1 && p.nm != 1) || p.ksplit > (p.K >> 8)) return cudaErrorInvalidValue;
    const bool wide = p.wide != 0;
    static int optin[2][kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    const void* fn = wide ? (const void*)grouped_q4k_mma_kernel<true> : (const void*)grouped_q4k_mma_kernel<false>;
    if (!optin[wide][dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v);
        if (e != cudaSuccess) return e;
        optin[wide][dev] = v;
    }
    const size_t bring = (size_t)kBStages * (wide ? TcLayout<true>::kBStageBytes : TcLayout<false>::kBStageBytes);
    const size_t per_stage = (size_t)p.nm * kRawTile;
    const size_t fixed = 1024 + 512;  // alignment slack + mbarriers + TMEM address slot
    int S = (int)(((size_t)optin[wide][dev] - fixed - bring) / per_stage);
    if (S > 8) S = 8;
    if (S < 2) return cudaErrorInvalidValue;
    const size_t smem = fixed + bring + (size_t)S * per_stage;
    int grid = num_sms;
    if (max_items < grid) grid = max_items > 0 ? max_items : 1;
    const CUtensorMap* a = reinterpret_cast<const CUtensorMap*>(tmapA);
    const CUtensorMap* b = reinterpret_cast<const CUtensorMap*>(tmapB ? tmapB : tmapA);
    if (wide)
        grouped_q4k_mma_kernel<true><<<grid, kTcThreads, smem, st>>>(*a, *b, p, S);
    else
        grouped_q4k_mma_kernel<false><<<grid, kTcThreads, smem, st>>>(*a, *b, p, S);
    return cudaGetLastError();
}

}  // namespace glc
