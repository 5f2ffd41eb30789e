// common.cuh -- device helpers shared by the sm_100a kernels: mbarrier pipeline
// primitives, 1-D bulk async copies (cp.async.bulk, the TMA bulk path), integer
// dot products and bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kernels.h"  // device error codes

namespace glc {

// Upper bound on any device-side wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and records `code` in *err) if the phase does
// not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) break;
    }
    if (err) atomicExch(err, code);
    return false;
}

// Bounded wait that polls with the non-suspending test_wait.  For kernels
// whose waiting warps have no working neighbours to take issue slots from
// (every consumer waits on the same stage): a thread suspended in try_wait
// resumes measurably later than the phase completes.  Same bound and error
// reporting as mbar_wait.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err, int code,
                                               uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 32; ++i)
            if (mbar_test_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) break;
    }
    if (err) atomicExch(err, code);
    return false;
}

// Bounded wait for threads that share their SM sub-partition with warps doing
// the real work: between polls the thread sleeps `ns` nanoseconds instead of
// spinning, so it does not take issue slots from them.  Same bound and error
// reporting as mbar_wait.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* err, int code, unsigned ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        __nanosleep(ns);
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) break;
    }
    if (err) atomicExch(err, code);
    return false;
}

// Called by a producer thread before it returns, on every path: waits
// (bounded, suspending polls, nothing recorded) until the copies of the last
// min(issued, S) stages of a ring of S stages (stage i on full[i % S], phase
// i / S) have landed, so the CTA can never exit with bulk copies still writing
// into its shared memory -- also when the consumers abandon the ring (a
// timed-out grid barrier) while the producer has issued everything.  On the
// normal path those phases completed long ago and every wait returns at once.
__device__ __forceinline__ void drain_issued_stages(uint64_t* full, int S, int issued, uint64_t limit_ns) {
    for (int st = issued > S ? issued - S : 0; st < issued; ++st)
        mbar_wait(&full[st % S], (uint32_t)(st / S) & 1u, nullptr, 0, limit_ns);
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while the kernel before it on the stream is still
// running: it must call grid_dep_wait() before touching anything that kernel
// writes (or reads and this one writes); grid_dep_wait returns once that
// kernel has completed and its memory is visible.  grid_dep_launch_dependents
// lets the next such kernel be scheduled once every CTA of this one has
// called it or exited.  Both are no-ops for a kernel launched without the
// attribute, or without such a dependent.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// L2 policy for data read once (streamed expert weights).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// Two-way int16 x uint8 dot products with int32 accumulation.
//   lo: c + a.h0 * b.byte0 + a.h1 * b.byte1
//   hi: c + a.h0 * b.byte2 + a.h1 * b.byte3
__device__ __forceinline__ int dp2a_lo(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Orders this thread's earlier generic-proxy accesses of shared memory before
// its later async-proxy (bulk copy) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long atom_add_acq_rel_gpu_u64(unsigned long long* p, unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}

// Grid-wide barrier for a launch whose CTAs are all resident (one per SM),
// on a 64-bit arrival counter that only ever grows: every launch adds exactly
// nblocks arrivals, so arrival number `prev` belongs to barrier instance
// prev / nblocks, which completes when the counter reaches the next multiple
// of nblocks.  One atomic round trip to arrive, polling to leave, no reset.
// Called by ONE thread per CTA after the CTA's participating threads have
// synchronised; the caller synchronises them again afterwards.  No separate
// fences: the arrival is a release at gpu scope (acq_rel atomic) and the poll
// an acquire, and the CTA barriers on either side carry the other threads'
// writes before the release and their reads after the acquire (causality
// order is transitive across the CTA barrier).  Waits at most kWaitLimitNs,
// then records kDevTimeoutGrid and returns false (the host must then clear
// the counter before the next launch).
__device__ __forceinline__ bool grid_barrier(unsigned long long* ctr, unsigned nblocks, int* err,
                                             uint64_t limit_ns = kWaitLimitNs) {
    const unsigned long long prev = atom_add_acq_rel_gpu_u64(ctr, 1ull);
    const unsigned long long target = (prev / nblocks + 1) * nblocks;
    if (prev + 1 == target) return true;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu_u64(ctr) < target) {
        if (global_timer_ns() - t0 > limit_ns) {
            if (err) atomicExch(err, kDevTimeoutGrid);
            return false;
        }
        __nanosleep(32);  // keeps the pollers from crowding out the last arrivals at the counter's L2 slice
    }
    return true;
}

// Canonical router reduction steps (the CPU oracle replays the same order):
// a xor butterfly inside a warp and a fixed pairwise tree over 8 warp sums.
__device__ __forceinline__ float warp_tree(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Eight per-lane values reduced across the warp with 9 shuffles instead of
// 8 x 5: at the 16, 8 and 4 levels each lane keeps half of its values and
// trades the other half with its partner, then the 2 and 1 levels add.  Every
// value is summed over the same lane pairs at every level as warp_tree, and
// fp32 addition is commutative, so each sum is bit-identical to warp_tree's.
// Lane L ends up holding the sum of value (L >> 2) & 7.
__device__ __forceinline__ float warp_tree8(const float (&v)[8], int lane) {
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    float a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = b4 ? v[4 + i] : v[i], send = b4 ? v[i] : v[4 + i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float b[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = b3 ? a[2 + i] : a[i], send = b3 ? a[i] : a[2 + i];
        b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float c = (b2 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, b2 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

__device__ __forceinline__ float tree8(const float* s) {
    return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace glc
