// kernels.h -- host-visible launch interfaces of the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct glc_comm;  // NCCL communicator of the C ABI (comm.cu)

namespace glc {

// Device-side error codes written to the per-handle error word.
enum : int {
    kDevOk = 0,
    kDevTimeoutFull = 1,   // consumer gave up waiting for a stage to land
    kDevTimeoutEmpty = 2,  // producer gave up waiting for a stage to be released
    kDevBadArg = 3,
    kDevTimeoutGrid = 4,   // a CTA gave up waiting at a grid-wide barrier
};


constexpr int kMaxDevices = 64;
#ifndef GLC_GEMV_WARPS
#define GLC_GEMV_WARPS 15
#endif
constexpr int kGemvMaxConsumerWarps = GLC_GEMV_WARPS;
constexpr int kGemvMaxThreads = (kGemvMaxConsumerWarps + 1) * 32;  // + 1 producer warp

enum GemvMode : int {
    kGemvPlain = 0,        // y[N] = W x
    kGemvGateUp = 1,       // act[p][F] = silu(W1_e x_t) * (W3_e x_t), pair p = (t, j)
    kGemvDownCombine = 2,  // out[t][D] = (resid|0|out) + sum_j (W2_{e_tj} act_tj) * w_tj
};

struct GemvParams {
    int mode;
    int K;             // input length (multiple of 256)
    int rows;          // rows per segment (N, F or D)
    int nseg;          // segments: 1, pairs P, or tokens T
    int kslots;        // slots per token (gate/up: pair -> token = p / kslots)
    int num_experts;   // clamp bound for expert ids
    const uint8_t* A;  // W / gate_exps / down_exps
    const uint8_t* B;  // up_exps (gate/up mode)
    long long expert_bytes;
    const int* ids;    // gate/up: [P]; down: [T * kslots]
    const float* cw;   // down: combine weights [T * kslots]
    const float* x;    // plain [K]; gate/up [T][K]; down [P][K]
    const float* resid;  // down: [T][D] or nullptr
    float* y;
    int* err;          // device error word (bounded waits)
    int accumulate;    // down: start from the existing y instead of resid / 0
    // plain / gate-up with one segment: when set, the input is RMSNorm(x) *
    // norm_w; the lanes take x * norm_w and the epilogue scales each row sum
    // by 1 / sqrt(mean(x^2) + norm_eps), the sum of squares formed by every
    // CTA in the same order
    const float* norm_w = nullptr;
    float norm_eps = 0.f;
    // filled by gemv_configure; split: down mode with the slot-split stage
    // layout (every stage holds the same stage_rows rows of all kslots
    // experts, warp group g computes slot g % kslots)
    int nsegw, nw, stage_rows, stages, split;
    int nss_off;  // shared-memory byte offset of the norm's sums of squares
};

int gemv_configure(GemvParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid);

// A chain of Q4_K GEMVs in one persistent launch (gemv_chain.cu).
enum GemvChainOp : int { kChainSet = 0, kChainAdd = 1, kChainGateUp = 2 };
constexpr int kMaxChainJobs = 64;
struct GemvJob {          // 56 bytes: 64 jobs and the rest stay under 4 KB of kernel parameters
    const uint8_t* A;      // Q4_K [N][K/256*144] (gate rows for kChainGateUp)
    const uint8_t* B;      // up rows (kChainGateUp)
    const float* x;        // [K]
    float* y;              // [N]
    const float* norm_w;   // nullptr, or the input is RMSNorm(x) * norm_w
    float norm_eps;
    int K, N;
    unsigned short op;
    unsigned short after_previous;  // x may be an earlier job's output: grid-wide barrier first
};
struct GemvChainParams {
    GemvJob jobs[kMaxChainJobs];
    int njobs;
    unsigned long long* bar;  // grid barrier counter (grows only; one counter per grid size)
    int* err;                 // device error word (bounded waits)
    // filled by gemv_chain_configure
    int stages, slot_bytes, part_floats;
};
static_assert(sizeof(GemvChainParams) <= 4096, "chain parameters fit the classic kernel-parameter limit");
int gemv_chain_configure(GemvChainParams& p, int grid, size_t smem_limit, size_t* smem_bytes);
cudaError_t gemv_chain_launch(GemvChainParams p, int num_sms, cudaStream_t stream);

// Decode attention of one token over fp16 K/V caches (attention.cu).
constexpr int kAttnMaxGroup = 8;    // query heads per KV head
constexpr int kAttnMaxLen = 32768;  // cache rows (at most 4096 positions per CTA of an 8-CTA cluster)
struct AttnParams {
    const float* q;        // [n_heads][head_dim] before rotation
    const float* k_new;    // [n_kv_heads][head_dim] before rotation
    const float* v_new;    // [n_kv_heads][head_dim]
    uint16_t* k_cache;     // fp16 [n_kv_heads][max_len][head_dim] (rotated keys), row pos written
    uint16_t* v_cache;     // fp16 [n_kv_heads][max_len][head_dim], row pos written
    float* out;            // [n_heads][head_dim]
    float* work;           // attn_workspace_bytes() (reserved)
    int n_heads, n_kv_heads, head_dim, max_len, pos;
    float theta;
    // When set, the position is read here (a launch any position can replay).
    // The kernel reads it before it waits for the kernel it is launched
    // behind, so the word must be written before that kernel starts.
    const int* pos_dev = nullptr;
    // optional biases added to q, k_new and v_new as they are read
    const float* bq = nullptr;
    const float* bk = nullptr;
    const float* bv = nullptr;
    // theta^(-2i/128) for pair i, in double (filled by attn_decode_launch)
    double inv_freq[64];
};
size_t attn_workspace_bytes(int n_heads, int n_kv_heads, int max_len);
cudaError_t attn_decode_launch(AttnParams p, cudaStream_t stream);
cudaError_t gemv_launch(const GemvParams& p, int num_sms, cudaStream_t stream);

// Router: gate GEMV + softmax + top-k (+ renormalise) with optional RMSNorm
// ingress; canonical reduction order shared with the CPU oracle.
struct RouterParams {
    const float* x;      // [T][D]
    const float* Wr;     // [D][E]
    int T, D, E, k;
    int renorm;
    int rmsnorm;
    float* xin;          // [T][D] normalised input (or copy of x); may be nullptr
    float* logits;       // [T][E] or nullptr
    int* ids;            // [T][k]
    float* w;            // [T][k]
    const float* gate_vec;  // shared-expert gate [D] or nullptr
    float* gate_out;        // [T] sigmoid(xin . gate_vec)
    // E <= 8 with rmsnorm: when set, xin = RMSNorm(x) * norm_w with epsilon
    // norm_eps (a decoder layer's weighted feed-forward norm); else the
    // unweighted norm with epsilon 1e-5
    const float* norm_w = nullptr;
    float norm_eps = 0.f;
};
cudaError_t router_launch(const RouterParams& p, cudaStream_t stream);

// Whole MoE layer for a few decode tokens in ONE persistent launch (one CTA
// per SM, all resident): router (every CTA, canonical order), gate/up GEMV +
// SwiGLU, grid barrier, down GEMV + k-ordered combine (+ residual).  Results
// are bit-identical to router_launch + gemv_launch(gate/up) + gemv_launch(down).
constexpr int kFusedConsumerWarps = 14;
constexpr int kFusedThreads = (kFusedConsumerWarps + 1) * 32;  // + 1 producer warp
constexpr int kFusedMaxTokens = 4;

struct FusedDecodeParams {
    const float* x;       // [T][D] layer input (16-byte aligned)
    const float* Wr;      // [D][E] router (16-byte aligned)
    const float* resid;   // [T][D] or nullptr
    const uint8_t* gate;  // [E][F][D/256*144]
    const uint8_t* up;
    const uint8_t* down;  // [E][D][F/256*144]
    long long gu_expert_bytes, dn_expert_bytes;
    float* act;           // [T*k][F] SwiGLU activations (scratch)
    float* out;           // [T][D]
    float* xin;           // [T][D] normalised input, or nullptr
    int* ids;             // [T][k] expert ids
    float* w;             // [T][k] combine weights
    unsigned long long* bar;  // grid-barrier arrival counter (8-byte aligned), zero at first use
    int* err;
    // Host-visible completion, for a caller that waits on host memory instead
    // of the stream: when done_ctr is set, every CTA adds 1 to it as it
    // finishes, and the one that completes a multiple of the grid size copies
    // *err to *host_err and then writes the launch's epoch (the count over the
    // grid size: launches since the counter was last cleared) to *host_done
    // (both mapped host memory; out/ids/w may be mapped host memory too).
    unsigned long long* done_ctr;
    unsigned long long* host_done;
    int* host_err;
    // Failure-detection tests: wait_limit_ns > 0 replaces the 4 s limit of every
    // device-side wait of the launch, and CTA stall_cta - 1 (stall_cta > 0;
    // 0 = none) stays out of the grid barrier, so the other CTAs' wait there
    // runs out and is reported.
    long long wait_limit_ns;
    int stall_cta;
    int T, D, F, E, k, renorm, rmsnorm;
    // Weighted RMSNorm (rmsnorm set): the input is x * rms * norm_w[d] with
    // eps = norm_eps, as router.cu's norm_w; nullptr = unweighted, eps 1e-5.
    const float* norm_w;
    float norm_eps;
    // x (and resid) are written by the kernel launched just before on the
    // stream: where an instantiation can, the launch is programmatically
    // serialised behind it and stages the router weights before waiting.
    int pdl;
    // Qwen2-MoE shared expert (Fs > 0): rows [Fs][D/256*144] gate/up,
    // [D][Fs/256*144] down, gate vector [D]; act_sh [T][Fs] scratch.  A layer
    // with a shared expert, or whose router does not fit the shared-memory
    // staging, runs the wide kernel (decode_wide.cu), which also needs
    // route_slots [T][E+1][8] scratch (epoch-tagged partial logits, cleared
    // together with route_bar) and route_bar, a launch counter.
    const uint8_t* sh_gate;
    const uint8_t* sh_up;
    const uint8_t* sh_down;
    const float* sh_gate_vec;
    int Fs;
    float* act_sh;
    unsigned long long* route_slots;
    unsigned long long* route_bar;
    // filled by fused_decode_configure
    int gu_nsegw, gu_G, gu_R, dn_nsegw, dn_G, dn_R, dn_split, stages, slot_bytes;
    int off_xs, off_pgu, off_pdn, off_red, off_logit, off_rms, off_ids, off_w, off_bars;
    // router split over a cluster of rsplit CTAs (1 or 2; set at launch):
    // each stages 1/rsplit of the router rows; off_lh holds the rsplit partial
    // logits of every (token, expert) gathered over distributed shared memory
    int rsplit, off_lh;
    // wide kernel: down-phase lane layout (units of 64 weights per routed slot
    // / shared row, warps covering them, partial-sum slots per output row)
    int wide, dn_Ur, dn_Pr, dn_nwr, dn_Us, dn_nws, dn_row_parts;
};
// Returns 0 and fills the launch shape when the layer fits the fused kernel
// (T <= kFusedMaxTokens, E <= 64, router and input staged in shared memory),
// -1 otherwise (callers then use the separate launches).
int fused_decode_configure(FusedDecodeParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid);
// Returns cudaErrorNotSupported when the layer does not fit (see above).
cudaError_t fused_decode_launch(const FusedDecodeParams& p, int num_sms, cudaStream_t stream);
// The wide kernel (decode_wide.cu): same contract.
int wide_decode_configure(FusedDecodeParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid);
cudaError_t wide_decode_launch(const FusedDecodeParams& p, int num_sms, cudaStream_t stream);

// ---------------------------------------------------------------- batched path
constexpr int kGroupTokens = 32;      // tokens per MMA group (N = 2*roundup8(ntok) <= 64)
constexpr int kGroupTokensWide = 64;  // the wide layout's (N <= 128; see GroupedParams::wide)

// Device-resident dispatch plan (all arrays device memory).
struct DispatchPlan {
    int* counts;      // [E]
    int* offsets;     // [E+1]
    int* perm;        // [P] position -> pair
    int* inv;         // [P] pair -> position
    int* grp_first;   // [E] first group of expert e
    int* grp_e;       // [Gmax]
    int* grp_ntok;    // [Gmax]
    int* grp_N;       // [Gmax] MMA N (hi + lo rows, multiple of 16)
    int* grp_pos0;    // [Gmax] first position of the group
    int* grp_units;   // [Gmax] prefix sum of N over earlier groups (B-tile rows)
    int* meta;        // [2] = {groups, total units}
};
inline int plan_max_groups(int P, int E) { return E + P / kGroupTokens + 1; }

// count (optional, device memory): the pairs actually present, <= P; the
// split and combine below take the same pointer and skip the rest.
// group_tokens: the most tokens of one expert in one MMA group (kGroupTokens,
// or kGroupTokensWide for the grouped kernel's wide layout).
cudaError_t dispatch_plan_launch(const int* ids, int P, int E, const DispatchPlan& plan, cudaStream_t st,
                                 const int* count = nullptr, int group_tokens = kGroupTokens);
// B tiles: per group, per super-block s of K: [4 chunks][N rows][128 B] SWIZZLE_128B.
cudaError_t split_rows_launch(const float* src, int P, int K, int kslots, int src_is_token,
                              const DispatchPlan& plan, uint8_t* btiles, float* rscale, cudaStream_t st,
                              const int* count = nullptr);
// out[t] = (resid|0) + sum_j y[inv[t,j]] * w[t,j] in j order, then, with ysh,
// + (sum of ysh's K-slice planes) * sg[t] (the shared expert).
cudaError_t combine_launch(const float* y, int T, int D, int k, const int* inv, const float* w,
                           const float* resid, float* out, cudaStream_t st, const float* ysh = nullptr,
                           int ysh_slices = 1, long long ysh_stride = 0, const float* sg = nullptr,
                           const int* count = nullptr);

// Grouped expert GEMM on tcgen05 tensor cores (weights dequantised into TMEM).
struct GroupedParams {
    int K;             // reduction length (D for gate/up, F for down)
    int rows_per_e;    // output rows per expert (F for gate/up, D for down)
    int nm;            // 2: gate+up with SwiGLU epilogue; 1: down projection
    int num_experts;   // experts held in the weight tensors (row bound)
    DispatchPlan plan;
    const uint8_t* btiles;
    const float* rscale;  // [P] power-of-two row scales of the B operand
    float* out;           // nm=2: act [P][F]; nm=1: y [P][D] (K slice ks: out + ks * part_stride)
    int* err;
    int ksplit = 1;       // nm=1 only: K split into ksplit slices of whole super-blocks,
    long long part_stride = 0;  // each writing partial sums to its own plane (elements apart)
    // Groups of up to kGroupTokensWide tokens (the plan built with that group
    // size): accumulators of 128 TMEM columns, a ring of two A units instead
    // of three, B stages of 128 rows.  Each output column is the same sum as
    // in the narrow layout, so the results are identical; fewer groups mean
    // each expert's weights are dequantised fewer times.
    int wide = 0;
};
// Tensor maps are built once per weight tensor (2-D [rows][rowBytes] uint8, box 144 x 128).
int make_q4k_tensor_map(void* tmap64, const void* base, long long rows, int row_bytes);
cudaError_t grouped_launch(const void* tmapA, const void* tmapB, const GroupedParams& p, int max_items,
                           int num_sms, cudaStream_t st);

// Expert parallelism: pairs grouped by destination rank (rank = expert / (E/world)),
// stable, with the activation row and global expert id of each pair gathered in
// that order.  plan.counts/offsets/perm/inv receive the per-rank histogram,
// offsets and permutation; keys is scratch [T*k].
cudaError_t ep_dispatch_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world,
                               int* keys, const DispatchPlan& plan, float* rows, int* row_ids, cudaStream_t st);
cudaError_t localize_ids_launch(const int* ids, int n, int begin, int count, int* out, cudaStream_t st);
// Fixed-capacity expert-parallel exchange (ep.cu): per-peer blocks of
// ep_block_bytes(cap, D) = [count][cap expert ids][cap rows], cap = the most
// pairs one rank can send one peer, so the all-to-all needs no host read.
size_t ep_block_bytes(int cap, int D);
cudaError_t ep_pack_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world, int cap,
                           int* keys, const DispatchPlan& plan, uint8_t* blocks, cudaStream_t st);
// rows [world*cap][D] in source order, local expert ids, src_off [world+1]
// (src_off[world] = rows received, the device count of the expert batch)
cudaError_t ep_unpack_launch(const uint8_t* blocks, int world, int cap, int D, int begin, int count, float* rows,
                             int* local_ids, int* src_off, cudaStream_t st);
cudaError_t ep_repack_launch(const float* y, const int* src_off, int world, int cap, int D, float* out,
                             cudaStream_t st);
// Exchange over a peer window (see ep.cu): layout, and the pack / repack
// kernels that write into the peers' windows and publish an epoch flag, and
// the bounded wait for every peer's flag.
size_t ep_window_bytes(int world, int cap, int D);
size_t ep_win_disp_off(int parity, int world, int cap, int D);
size_t ep_win_ret_off(int parity, int world, int cap, int D);
cudaError_t ep_pack_peer_launch(const float* xin, const int* ids, int T, int D, int k, int num_experts, int world,
                                int me, int cap, int* keys, const DispatchPlan& plan, void* const* peers, int parity,
                                unsigned long long epoch, uint8_t* own, cudaStream_t st);
cudaError_t ep_repack_peer_launch(const float* y, const int* src_off, int world, int me, int cap, int D,
                                  void* const* peers, int parity, unsigned long long epoch, uint8_t* own,
                                  cudaStream_t st);
cudaError_t ep_wait_launch(const uint8_t* own, int world, int phase, unsigned long long epoch, int* err,
                           cudaStream_t st);
cudaError_t ep_unblock_launch(const float* blocks, int P, int cap, int D, const int* keys, const DispatchPlan& plan,
                              float* y_back, cudaStream_t st);
cudaError_t fill_launch(float* p, int n, float v, cudaStream_t st);

// Wire codec (QuantizationKernels), one CTA per token.
cudaError_t wire_quantize_launch(int mode, const float* x, int T, int D, uint8_t* out,
                                 cudaStream_t stream);
cudaError_t wire_dequantize_launch(int mode, const uint8_t* in, int T, int D, float* out,
                                   cudaStream_t stream);

int set_last_error(int code, const char* msg);

// ---------------------------------------------------------------- communicator (comm.cu)
int comm_world(const glc_comm* c);
int comm_rank(const glc_comm* c);
int32_t* comm_host_counts(glc_comm* c);  // pinned [2 * world]
void* comm_scratch(glc_comm* c, int slot, size_t bytes);
int comm_alltoall_i32(glc_comm* c, const int32_t* send, int32_t* recv, cudaStream_t st);
// Peer window of at least `bytes` on every rank (collective); GLC_ERR_UNSUPPORTED
// when it cannot be mapped on every rank or is turned off (glc_comm_peer_exchange).
int comm_window(glc_comm* c, size_t bytes, cudaStream_t st, uint8_t** own, void* const** d_peers);
unsigned long long comm_window_next_epoch(glc_comm* c);
int comm_alltoallv(glc_comm* c, const void* send, const size_t* soff, const size_t* scnt, void* recv,
                   const size_t* roff, const size_t* rcnt, cudaStream_t st);

}  // namespace glc
