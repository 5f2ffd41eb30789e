// ep.cu -- expert-parallel dispatch helpers.
//
// The reference has no expert parallelism: a token's experts run one after
// another on one worker (DistributedPipelineCoordinator.cs:181-206).  With the
// experts of a layer split into contiguous shards, one per rank
// (expert e lives on rank e / (E / world)), a rank's (token, slot) pairs are
// grouped by destination rank -- a stable counting sort of the rank keys,
// done by dispatch_plan_kernel -- and the activation row of each pair is
// gathered into a send buffer in that order, with its global expert id.
#include "common.cuh"
#include "kernels.h"

namespace glc {

__global__ void __launch_bounds__(256) ep_rank_keys_kernel(const int* __restrict__ ids, int P, int epr, int world,
                                                           int* __restrict__ keys) {
    const int p = blockIdx.x * 256 + threadIdx.x;
    if (p >= P) return;
    int r = ids[p];
    r = r < 0 ? 0 : r / epr;
    keys[p] = r >= world ? world - 1 : r;
}

// One CTA per send position: rows[pos] = xin[perm[pos] / k], row_ids[pos] = ids[perm[pos]].
__global__ void __launch_bounds__(256) ep_gather_kernel(const float* __restrict__ xin, const int* __restrict__ ids,
                                                        int D, int k, const int* __restrict__ perm,
                                                        float* __restrict__ rows, int* __restrict__ row_ids) {
    const int pos = blockIdx.x;
    const int pair = perm[pos];
    const float* src = xin + (size_t)(pair / k) * D;
    float* dst = rows + (size_t)pos * D;
    if ((D & 3) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
    } else {
        for (int i = threadIdx.x; i < D; i += 256) dst[i] = src[i];
    }
    if (threadIdx.x == 0) row_ids[pos] = ids[pair];
}

// Global expert ids -> indices into this rank's shard [begin, begin + count), clamped
// like GpuFirstExpertStageWorker.ProcessRoutedTopK clamps ids (GpuFirstExpertStageWorker.cs:452).
__global__ void __launch_bounds__(256) localize_ids_kernel(const int* __restrict__ ids, int n, int begin, int count,
                                                           int* __restrict__ out) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= n) return;
    const int e = ids[i] - begin;
    out[i] = e < 0 ? 0 : (e >= count ? count - 1 : e);
}

__global__ void __launch_bounds__(256) fill_kernel(float* __restrict__ p, int n, float v) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < n) p[i] = v;
}

// ---------------------------------------------------------------------------
// Fixed-capacity exchange blocks (no host read of the counts): the block a
// rank sends to peer p holds [int32 count | pad to 16 B][int32 expert id x
// cap, padded to 16 B][fp32 row x cap]; `cap` is the worst case of one rank's
// pairs to one peer, so every block has the same size on every rank and the
// all-to-all is one grouped send/receive of equal blocks.

__host__ __device__ inline size_t ep_ids_off() { return 16; }
__host__ __device__ inline size_t ep_rows_off(int cap) { return 16 + (((size_t)cap * 4 + 15) & ~(size_t)15); }
size_t ep_block_bytes(int cap, int D) { return ep_rows_off(cap) + (size_t)cap * D * 4; }

// One CTA per send position (or one CTA when there are none): the row and the
// global expert id of pair perm[pos] into slot pos - offsets[p] of the block
// for its rank p; block 0 also writes every block's count.
__global__ void __launch_bounds__(256) ep_pack_kernel(const float* __restrict__ xin, const int* __restrict__ ids, int P,
                                                      int D, int k, int world, int cap, const int* __restrict__ keys,
                                                      DispatchPlan plan, uint8_t* __restrict__ blocks, size_t bb) {
    const int pos = blockIdx.x;
    if (pos == 0 && threadIdx.x < world)
        *reinterpret_cast<int*>(blocks + (size_t)threadIdx.x * bb) = P > 0 ? plan.counts[threadIdx.x] : 0;
    if (pos >= P) return;
    const int pair = plan.perm[pos];
    const int p = keys[pair];
    const int slot = pos - plan.offsets[p];
    uint8_t* blk = blocks + (size_t)p * bb;
    const float4* s4 = reinterpret_cast<const float4*>(xin + (size_t)(pair / k) * D);
    float4* d4 = reinterpret_cast<float4*>(blk + ep_rows_off(cap) + (size_t)slot * D * 4);
    for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
    if (threadIdx.x == 0) reinterpret_cast<int*>(blk + ep_ids_off())[slot] = ids[pair];
}

// Received blocks -> contiguous rows in source order: slot s of source q
// goes to row R_q + s (R_q = rows of the sources before q); the expert id is
// localised to this rank's shard [begin, begin + count) (clamped, like
// GpuFirstExpertStageWorker.ProcessRoutedTopK clamps ids).  CTA (s, q); the
// first CTA writes the total row count and the source offsets.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* __restrict__ blocks, size_t bb, int world,
                                                        int cap, int D, int begin, int count, float* __restrict__ rows,
                                                        int* __restrict__ local_ids, int* __restrict__ src_off) {
    __shared__ int s_base, s_n;
    const int s = blockIdx.x, q = blockIdx.y;
    if (threadIdx.x == 0) {
        int base = 0;
        for (int r = 0; r < q; ++r) base += *reinterpret_cast<const int*>(blocks + (size_t)r * bb);
        s_base = base;
        s_n = *reinterpret_cast<const int*>(blocks + (size_t)q * bb);
        if (s == 0 && q == 0) {
            int acc = 0;
            for (int r = 0; r < world; ++r) {
                src_off[r] = acc;
                acc += *reinterpret_cast<const int*>(blocks + (size_t)r * bb);
            }
            src_off[world] = acc;  // total rows received
        }
    }
    __syncthreads();
    if (s >= s_n) return;
    const uint8_t* blk = blocks + (size_t)q * bb;
    const float4* s4 = reinterpret_cast<const float4*>(blk + ep_rows_off(cap) + (size_t)s * D * 4);
    float4* d4 = reinterpret_cast<float4*>(rows + (size_t)(s_base + s) * D);
    for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
    if (threadIdx.x == 0) {
        const int e = reinterpret_cast<const int*>(blk + ep_ids_off())[s] - begin;
        local_ids[s_base + s] = e < 0 ? 0 : (e >= count ? count - 1 : e);
    }
}

// Expert outputs back into per-source blocks of rows: y[R_q + s] -> out
// block q slot s (the order the source sent them in).  CTA (s, q).
__global__ void __launch_bounds__(256) ep_repack_kernel(const float* __restrict__ y, const int* __restrict__ src_off,
                                                        int cap, int D, float* __restrict__ out) {
    const int s = blockIdx.x, q = blockIdx.y;
    if (s >= src_off[q + 1] - src_off[q]) return;
    const float4* s4 = reinterpret_cast<const float4*>(y + (size_t)(src_off[q] + s) * D);
    float4* d4 = reinterpret_cast<float4*>(out + ((size_t)q * cap + s) * D);
    for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
}

// This rank's expert outputs, received as per-peer blocks, into send order:
// y_back[pos] = blocks[p][pos - offsets[p]] with p the rank of pair perm[pos].
__global__ void __launch_bounds__(256) ep_unblock_kernel(const float* __restrict__ blocks, int cap, int D,
                                                         const int* __restrict__ keys, DispatchPlan plan,
                                                         float* __restrict__ y_back) {
    const int pos = blockIdx.x;
    const int p = keys[plan.perm[pos]];
    const int slot = pos - plan.offsets[p];
    const float4* s4 = reinterpret_cast<const float4*>(blocks + ((size_t)p * cap + slot) * D);
    float4* d4 = reinterpret_cast<float4*>(y_back + (size_t)pos * D);
    for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
}

// ---------------------------------------------------------------------------
// Exchange over a peer window (comm_window: every rank's buffer mapped in
// every rank over NVLink).  Instead of packing blocks locally for a grouped
// NCCL send, the pack kernel writes each block straight into its
// destination's window, and the repack kernel writes each expert output row
// straight into its home rank's window: only the pairs actually routed cross
// NVLink.  Window layout (the same on every rank):
//   [0, 1024)     flags: uint64 [2 phases][64 sources], the epoch of the
//                 source's last completed write of that phase
//   [1024, 1032)  two uint32 launch counters (this rank's own)
//   disp(parity)  world blocks of ep_block_bytes(cap, D), by source rank
//   ret(parity)   world x cap rows of D floats, by source rank and slot
// The areas are double-buffered by the parity of the exchange's epoch: a rank
// cannot start exchange n + 2 before every peer has finished exchange n + 1
// (it needs their returns of n + 1), so a peer never writes an area its
// owner is still reading.

constexpr size_t kWinFlags = 0, kWinCtr = 1024, kWinData = 2048;

size_t ep_win_disp_off(int parity, int world, int cap, int D) {
    return kWinData + (size_t)parity * world * ep_block_bytes(cap, D);
}
size_t ep_win_ret_off(int parity, int world, int cap, int D) {
    return kWinData + 2 * (size_t)world * ep_block_bytes(cap, D) + (size_t)parity * world * cap * D * 4;
}
size_t ep_window_bytes(int world, int cap, int D) { return ep_win_ret_off(2, world, cap, D); }

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Called by every CTA of a launch after its writes: each CTA's writes are
// fenced at system scope before it counts itself done; the last one (which
// also returns the counter to 0 for the next launch, ordered after this one
// on the stream) fences again and publishes the epoch in flag[phase][me] of
// every rank's window.
__device__ void signal_when_done(uint8_t* own, void* const* peers, int world, int me, int phase,
                                 unsigned long long epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        unsigned* ctr = reinterpret_cast<unsigned*>(own + kWinCtr) + phase;
        const unsigned prev = atomicAdd(ctr, 1u);
        if (prev == gridDim.x * gridDim.y - 1) {
            *ctr = 0u;
            __threadfence_system();
            for (int p = 0; p < world; ++p)
                st_release_sys_u64(reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(peers[p]) + kWinFlags) +
                                       phase * 64 + me,
                                   epoch);
        }
    }
}

// ep_pack_kernel with the block for rank p written into rank p's window
// (source slot me of its dispatch area), then the dispatch flags.
__global__ void __launch_bounds__(256) ep_pack_peer_kernel(const float* __restrict__ xin, const int* __restrict__ ids,
                                                           int P, int D, int k, int world, int me, int cap,
                                                           const int* __restrict__ keys, DispatchPlan plan,
                                                           void* const* __restrict__ peers, size_t disp_off,
                                                           size_t bb, uint8_t* own, unsigned long long epoch) {
    const int pos = blockIdx.x;
    if (pos == 0 && threadIdx.x < world)
        *reinterpret_cast<int*>(static_cast<uint8_t*>(peers[threadIdx.x]) + disp_off + (size_t)me * bb) =
            P > 0 ? plan.counts[threadIdx.x] : 0;
    if (pos < P) {
        const int pair = plan.perm[pos];
        const int p = keys[pair];
        const int slot = pos - plan.offsets[p];
        uint8_t* blk = static_cast<uint8_t*>(peers[p]) + disp_off + (size_t)me * bb;
        const float4* s4 = reinterpret_cast<const float4*>(xin + (size_t)(pair / k) * D);
        float4* d4 = reinterpret_cast<float4*>(blk + ep_rows_off(cap) + (size_t)slot * D * 4);
        for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
        if (threadIdx.x == 0) reinterpret_cast<int*>(blk + ep_ids_off())[slot] = ids[pair];
    }
    signal_when_done(own, peers, world, me, 0, epoch);
}

// ep_repack_kernel with row s of source q written into rank q's window
// (source slot me of its return area), then the return flags.
__global__ void __launch_bounds__(256) ep_repack_peer_kernel(const float* __restrict__ y,
                                                             const int* __restrict__ src_off, int world, int me,
                                                             int cap, int D, void* const* __restrict__ peers,
                                                             size_t ret_off, uint8_t* own, unsigned long long epoch) {
    const int s = blockIdx.x, q = blockIdx.y;
    if (s < src_off[q + 1] - src_off[q]) {
        const float4* s4 = reinterpret_cast<const float4*>(y + (size_t)(src_off[q] + s) * D);
        float4* d4 = reinterpret_cast<float4*>(static_cast<uint8_t*>(peers[q]) + ret_off +
                                               ((size_t)me * cap + s) * D * 4);
        for (int i = threadIdx.x; i < (D >> 2); i += 256) d4[i] = s4[i];
    }
    signal_when_done(own, peers, world, me, 1, epoch);
}

// Waits (bounded) until every rank has published `epoch` for `phase` in this
// rank's window; on time-out records kDevTimeoutGrid and returns, so the
// launch sequence ends and the host reports the error.
__global__ void ep_wait_kernel(const uint8_t* own, int world, int phase, unsigned long long epoch, int* err) {
    const int p = threadIdx.x;
    if (p >= world) return;
    const unsigned long long* f = reinterpret_cast<const unsigned long long*>(own + kWinFlags) + phase * 64 + p;
    if (ld_acquire_sys_u64(f) >= epoch) return;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys_u64(f) < epoch) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            if (err) atomicExch(err, kDevTimeoutGrid);
            return;
        }
        __nanosleep(64);
    }
}

cudaError_t ep_pack_peer_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world,
                                int me, int cap, int* keys, const DispatchPlan& plan, void* const* peers, int parity,
                                unsigned long long epoch, uint8_t* own, cudaStream_t st) {
    const int P = T * k;
    if (world < 1 || world > 64 || me < 0 || me >= world || num_experts % world || (D & 3) || P > cap)
        return cudaErrorInvalidValue;
    if (P > 0) {
        ep_rank_keys_kernel<<<(P + 255) / 256, 256, 0, st>>>(ids, P, num_experts / world, world, keys);
        const cudaError_t e = dispatch_plan_launch(keys, P, world, plan, st);
        if (e != cudaSuccess) return e;
    }
    ep_pack_peer_kernel<<<P > 0 ? P : 1, 256, 0, st>>>(xin, ids, P, D, k, world, me, cap, keys, plan, peers,
                                                         ep_win_disp_off(parity, world, cap, D),
                                                         ep_block_bytes(cap, D), own, epoch);
    return cudaGetLastError();
}

cudaError_t ep_repack_peer_launch(const float* y, const int* src_off, int world, int me, int cap, int D,
                                  void* const* peers, int parity, unsigned long long epoch, uint8_t* own,
                                  cudaStream_t st) {
    ep_repack_peer_kernel<<<dim3(cap, world), 256, 0, st>>>(y, src_off, world, me, cap, D, peers,
                                                            ep_win_ret_off(parity, world, cap, D), own, epoch);
    return cudaGetLastError();
}

cudaError_t ep_wait_launch(const uint8_t* own, int world, int phase, unsigned long long epoch, int* err,
                           cudaStream_t st) {
    ep_wait_kernel<<<1, 64, 0, st>>>(own, world, phase, epoch, err);
    return cudaGetLastError();
}

cudaError_t ep_pack_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world, int cap,
                           int* keys, const DispatchPlan& plan, uint8_t* blocks, cudaStream_t st) {
    const int P = T * k;
    if (world < 1 || world > 64 || num_experts % world || (D & 3) || P > cap) return cudaErrorInvalidValue;
    if (P > 0) {
        ep_rank_keys_kernel<<<(P + 255) / 256, 256, 0, st>>>(ids, P, num_experts / world, world, keys);
        const cudaError_t e = dispatch_plan_launch(keys, P, world, plan, st);
        if (e != cudaSuccess) return e;
    }
    ep_pack_kernel<<<P > 0 ? P : 1, 256, 0, st>>>(xin, ids, P, D, k, world, cap, keys, plan, blocks,
                                                    ep_block_bytes(cap, D));
    return cudaGetLastError();
}

cudaError_t ep_unpack_launch(const uint8_t* blocks, int world, int cap, int D, int begin, int count, float* rows,
                             int* local_ids, int* src_off, cudaStream_t st) {
    ep_unpack_kernel<<<dim3(cap, world), 256, 0, st>>>(blocks, ep_block_bytes(cap, D), world, cap, D, begin, count,
                                                       rows, local_ids, src_off);
    return cudaGetLastError();
}

cudaError_t ep_repack_launch(const float* y, const int* src_off, int world, int cap, int D, float* out,
                             cudaStream_t st) {
    ep_repack_kernel<<<dim3(cap, world), 256, 0, st>>>(y, src_off, cap, D, out);
    return cudaGetLastError();
}

cudaError_t ep_unblock_launch(const float* blocks, int P, int cap, int D, const int* keys, const DispatchPlan& plan,
                              float* y_back, cudaStream_t st) {
    if (P <= 0) return cudaSuccess;
    ep_unblock_kernel<<<P, 256, 0, st>>>(blocks, cap, D, keys, plan, y_back);
    return cudaGetLastError();
}

cudaError_t ep_dispatch_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world,
                               int* keys, const DispatchPlan& plan, float* rows, int* row_ids, cudaStream_t st) {
    const int P = T * k;
    if (P <= 0) return cudaSuccess;
    if (world < 1 || world > 64 || num_experts % world) return cudaErrorInvalidValue;
    ep_rank_keys_kernel<<<(P + 255) / 256, 256, 0, st>>>(ids, P, num_experts / world, world, keys);
    cudaError_t e = dispatch_plan_launch(keys, P, world, plan, st);
    if (e != cudaSuccess) return e;
    ep_gather_kernel<<<P, 256, 0, st>>>(xin, ids, D, k, plan.perm, rows, row_ids);
    return cudaGetLastError();
}

cudaError_t localize_ids_launch(const int* ids, int n, int begin, int count, int* out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    localize_ids_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, n, begin, count, out);
    return cudaGetLastError();
}

cudaError_t fill_launch(float* p, int n, float v, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    fill_kernel<<<(n + 255) / 256, 256, 0, st>>>(p, n, v);
    return cudaGetLastError();
}

}  // namespace glc
