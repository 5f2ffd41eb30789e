/*
 * glacier_b200.h -- C ABI of libglacier_b200.so, the B200 (sm_100a) backend for
 * the quantized Mixture-of-Experts feed-forward hot path of
 * Glacier.Inference.Distributed.
 *
 * Conventions
 *   - Every function returns an int status: GLC_OK (0) or a negative GLC_ERR_*.
 *     glc_last_error() returns a thread-local message for the last failure.
 *   - Pointers are HOST memory unless the function name ends in _dev; _dev
 *     functions take DEVICE pointers and a cudaStream_t passed as void*, and
 *     return without synchronising the stream.
 *   - The library never frees caller memory, never calls exit() and never traps.
 *   - A glc_moe handle owns one device and one stream. On the glc_moe_*_dev
 *     entry points a NULL stream selects the handle's own (non-blocking)
 *     stream; a caller working on the legacy default stream passes
 *     cudaStreamLegacy.  Entry points without a handle use the stream as
 *     given (NULL is the legacy default stream).  Calls on one handle must
 *     be serialised by the caller (the reference serialises GPU work with
 *     lock(_gpuLock), GpuFirstExpertStageWorker.cs:447). Handles on different
 *     devices are independent.
 *   - Weight blobs use the GGUF layout the reference uses:
 *     [expert][rows][rowBytes] (CpuWarmExpertPoolWorker.cs:247-253), Q4_K rows
 *     of K/256 super-blocks of 144 bytes.
 */
#ifndef GLACIER_B200_H
#define GLACIER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLC_ABI_VERSION 1

/* status codes */
#define GLC_OK 0
#define GLC_ERR_INVALID_ARG -1   /* ArgumentException / ArgumentOutOfRangeException */
#define GLC_ERR_CUDA -2
#define GLC_ERR_OOM -3
#define GLC_ERR_UNSUPPORTED -4   /* NotSupportedException (e.g. K % 256 != 0 for Q4_K) */
#define GLC_ERR_DISPOSED -5      /* ObjectDisposedException */
#define GLC_ERR_NCCL -6
#define GLC_ERR_TIMEOUT -7       /* a bounded device-side wait gave up */
#define GLC_ERR_STATE -8

/* GGUF tensor types accepted for expert weights (GGUF type ids). */
#define GLC_GGUF_Q4_K 12

/* wire precision modes (WirePrecisionMode, Protocol/FusedActivationHeader.cs:12-18) */
#define GLC_WIRE_FP32 0
#define GLC_WIRE_FP16 1
#define GLC_WIRE_INT8 2
#define GLC_WIRE_FP8_E4M3 3

/* layer-forward flags */
#define GLC_FWD_RMSNORM 1u   /* xin = RMSNorm(x), no weight, eps 1e-5 (StageWorkers.cs:89-91) */
#define GLC_FWD_RESIDUAL 2u  /* out = x + sum_k w_k y_k (DistributedPipelineCoordinator.cs:104-134) */
#define GLC_FWD_DECODE 4u    /* force the per-pair GEMV path (default for T == 1) */
#define GLC_FWD_BATCHED 8u   /* force the grouped tensor-core path (default for T > 1) */
#define GLC_FWD_UNFUSED 16u  /* decode path: router, gate/up and down as three launches instead of
                                the single fused layer launch (same results, bit for bit) */

typedef struct glc_moe glc_moe;

/* Shapes of one MoE layer family.  Replaces the constructor arguments of
 * GpuFirstExpertStageWorker (GpuFirstExpertStageWorker.cs:109-124) and
 * CpuWarmExpertPoolWorker (CpuWarmExpertPoolWorker.cs:89-100). */
typedef struct glc_moe_desc {
    int32_t hidden_dim;      /* D (multiple of 256) */
    int32_t expert_ffn_dim;  /* F (multiple of 256) */
    int32_t num_experts;     /* E, total routed experts of the layer */
    int32_t top_k;           /* k */
    int32_t shared_ffn_dim;  /* Fs of the sigmoid-gated shared expert, 0 = none */
    int32_t renormalize;     /* 1: softmax -> top-k -> renormalise; 0: plain softmax weights */
    int32_t weight_type;     /* GLC_GGUF_Q4_K */
    int32_t device;          /* CUDA ordinal */
    int32_t num_layers;      /* layers held by the handle (header.LayerIndex is clamped) */
    int32_t max_tokens;      /* largest T passed to glc_moe_forward* */
    int32_t expert_begin;    /* first expert held on this device (expert parallelism) */
    int32_t expert_count;    /* experts held on this device (0 = all E) */
} glc_moe_desc;

/* Host-side weights of one layer (copied to HBM by glc_moe_load_layer).
 * gate/up: [expert_count][F][rowBytes(D)]; down: [expert_count][D][rowBytes(F)];
 * router: fp32 [D][E]; shared_*: one expert of width Fs; shared_gate: fp32 [D]. */
typedef struct glc_layer_weights {
    const void* gate_exps;
    const void* up_exps;
    const void* down_exps;
    const float* router;
    const void* shared_gate;
    const void* shared_up;
    const void* shared_down;
    const float* shared_gate_vec;
} glc_layer_weights;

/* ---- library ---- */
int glc_abi_version(void);
const char* glc_last_error(void);
int glc_device_count(int32_t* count);
/* GetRowBytes for Q4_K (the external GgufTypes.GetRowBytes, CpuWarmExpertPoolWorker.cs:133). */
int64_t glc_q4k_row_bytes(int32_t k);

/* ---- MoE handle lifecycle (GpuFirstExpertStageWorker ctor / Dispose, :109-167, :785-834) ---- */
int glc_moe_create(const glc_moe_desc* desc, glc_moe** out);
int glc_moe_destroy(glc_moe* h);
int glc_moe_load_layer(glc_moe* h, int32_t layer, const glc_layer_weights* w);
/* Fill a layer with the documented seeded synthetic weights (SplitMix64 streams,
 * Q4_K d/dmin = fp16(|N(0,sigma_d)|), uniform 6-bit scales/mins and 4-bit quants,
 * router N(0, 0.02), shared gate N(0, 0.02)).  Only this device's experts are made. */
int glc_moe_synth_layer(glc_moe* h, int32_t layer, uint64_t seed);

/* Expert residency, GpuFirstExpertStageWorker's GPU slot cache
 * (GpuFirstExpertStageWorker.cs:144-151, 344-407).  Called after
 * glc_moe_create and before the first layer is loaded, it keeps every layer's
 * routed experts in pinned host memory and `slots` of them at a time in HBM
 * (clamped to [1, num_experts], as GpuFirstExpertStageWorker.cs:144; router and
 * shared expert stay resident).  A forward routes first, then brings each
 * selected expert into a slot -- a hit when it is there, else the least
 * recently used slot not used by this call is refilled from host memory --
 * and runs the expert kernels on the slots: results equal the fully resident
 * layer's bit for bit.  Loading layer 0 stages its first experts
 * (WarmInitialGpuSlots, GpuFirstExpertStageWorker.cs:344-352).  A call that
 * routes to more distinct experts than there are slots returns
 * GLC_ERR_UNSUPPORTED (the reference sends those to its CPU pool; this
 * library has no CPU path).  With slots the decode step is not one fused
 * launch and a forward waits on the host for its routing; expert-parallel
 * calls, glc_moe_graph_build and glc_moe_layer_device_ptrs are then not
 * available, and expert-parallel shards cannot use slots.  One stream per
 * handle: a refilled slot is written behind the work queued on it. */
int glc_moe_set_expert_slots(glc_moe* h, int32_t slots);
/* Router lookahead prefetch (PrefetchLookaheadExperts,
 * GpuFirstExpertStageWorker.cs:388-407): stages the listed experts of `layer`
 * into slots, asynchronously on the handle's stream (ids clamped; a no-op
 * without expert slots). */
int glc_moe_prefetch_experts(glc_moe* h, int32_t layer, const int32_t* expert_ids, int32_t n);
/* out4 = {slot capacity (num_experts when every expert is resident), VRAM
 * hits, host-to-HBM expert transfers, lookahead prefetches}: the
 * GpuResidentSlotCapacity, GpuVramHitCount, GpuPcieTransferCount and
 * LookaheadPrefetchCount of GpuFirstExpertStageWorker.GetTelemetry
 * (GpuFirstExpertStageWorker.cs:763-783); a hit or transfer is counted per
 * (token, slot) pair. */
int glc_moe_expert_residency(glc_moe* h, int64_t* out4);
/* Device pointers of a resident layer (for the _dev raw primitives). */
int glc_moe_layer_device_ptrs(glc_moe* h, int32_t layer, const void** gate, const void** up,
                              const void** down, const float** router);

/* Telemetry (the CUDA-event counterpart of StageTelemetry / GpuFirstWorkerTelemetry,
 * Program.cs:28, GpuFirstExpertStageWorker.cs:21-31): when enabled, every
 * forward records an event after each kernel; glc_moe_kernel_times returns the
 * device milliseconds of each kernel of the last forward, in launch order
 * (router, gate/up, down[, shared gate/up, shared down]). */
int glc_moe_set_profiling(glc_moe* h, int32_t enable);
int glc_moe_kernel_times(glc_moe* h, float* ms, int32_t max_kernels, int32_t* n_kernels);
/* Reads and clears the device error word of the handle (GLC_ERR_TIMEOUT when a
 * bounded device-side wait gave up during an asynchronous _dev call). */
int glc_moe_poll_error(glc_moe* h);
/* Failure-detection test hook: the next fused decode launch of this handle
 * leaves CTA `cta` out of its grid barrier and gives every device-side wait of
 * the launch `wait_limit_ns` instead of 4 s, so the other CTAs' wait runs out;
 * that launch reports GLC_ERR_TIMEOUT (the host-buffer forward, or
 * glc_moe_poll_error) and clears the device words, after which the handle
 * works normally.  One launch only. */
int glc_moe_debug_stall(glc_moe* h, int32_t cta, int64_t wait_limit_ns);

/* ---- per-expert stage worker: IInferenceStageWorker.ProcessActivation
 *      (IInferenceStageWorker.cs:43; zero-alloc overload CpuWarmExpertPoolWorker.cs:232).
 *      y = W2 * SwiGLU(W1 x, W3 x) for expert `expert` (clamped to [0,E)) of
 *      layer `layer` (clamped). x, y: host fp32 [D]. ---- */
int glc_expert_forward(glc_moe* h, int32_t layer, int32_t expert, const float* x, float* y);
int glc_expert_forward_dev(glc_moe* h, int32_t layer, int32_t expert, const float* x, float* y,
                           void* stream);

/* ---- routed top-k: GpuFirstExpertStageWorker.ProcessRoutedTopK (:416-423).
 *      out = sum_j w[j] * Expert_{ids[j]}(x), accumulated in j order; out cleared
 *      first; k == 0 gives zeros; ids clamped to [0,E). Host fp32 [D]. ---- */
int glc_routed_topk(glc_moe* h, int32_t layer, const float* x, const int32_t* ids,
                    const float* w, int32_t k, float* out);

/* ---- full MoE layer for T tokens: router (gate GEMV + softmax + top-k +
 *      renormalise), dispatch, experts, combine. x, out: fp32 [T][D]; ids_out
 *      int32 [T][k], w_out fp32 [T][k] (either may be NULL).  T == 1 runs the
 *      decode path (dequant-fused GEMV kernels); T > 1 the batched path.
 *      Host-buffer form: for shapes the fused decode launch takes, the first
 *      call of each (layer, T, flags) captures the input copy and the launch
 *      into a graph that later calls replay (up to 64 shapes per handle,
 *      replaced round robin); results are the same either way. ---- */
int glc_moe_forward(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags,
                    float* out, int32_t* ids_out, float* w_out);
int glc_moe_forward_dev(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags,
                        float* out, int32_t* ids_out, float* w_out, void* stream);

/* ---- one-submission decode step: the CUDA-graph counterpart of the single
 *      D3D12 command list GpuFirstExpertStageWorker records per call
 *      (GpuFirstExpertStageWorker.cs:463-534).  build captures
 *      glc_moe_forward_dev(layer, x, T, flags, out) into a graph held by the
 *      handle (pointers are baked in; refill x between launches); launch
 *      replays it on `stream`.  A second build replaces the first. ---- */
int glc_moe_graph_build(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags,
                        float* out);
int glc_moe_graph_launch(glc_moe* h, void* stream);

/* ---- raw primitive: QuantKernels.MatVecMul(Q4_K, W, x, y, nCols=K, nRows=N)
 *      (call shape CpuWarmExpertPoolWorker.cs:379). K % 256 != 0 -> GLC_ERR_UNSUPPORTED;
 *      W and x 16-byte aligned. ---- */
int glc_gemv_q4k_dev(const void* W, const float* x, float* y, int32_t K, int32_t N, void* stream);

/* ---- a chain of MatVecMul calls in one launch: the GemvQ4K / SwiGLU /
 *      VecAddWeighted dispatch sequence of a decode step
 *      (GpuFirstExpertStageWorker.cs:482-519) with the weights of every job
 *      streamed back to back.  Jobs run in order; a job with after_previous
 *      set may read what earlier jobs of the chain wrote (a grid-wide wait
 *      precedes it).  Device pointers; at most 64 jobs; K % 256 == 0;
 *      W, W_up, x, norm_w 16-byte aligned.  Each job's output is bit-identical to
 *      glc_gemv_q4k_dev's (op SET, no norm).  Asynchronous on `stream`. ---- */
#define GLC_GEMV_SET 0      /* y = W x */
#define GLC_GEMV_ADD 1      /* y = y + W x */
#define GLC_GEMV_GATE_UP 2  /* y = SiLU(W x) * (W_up x) */
typedef struct glc_gemv_job {
    const void* W;        /* Q4_K [N][K/256*144] (the gate rows for GATE_UP) */
    const void* W_up;     /* Q4_K [N][K/256*144] up rows (GATE_UP), else NULL */
    const float* x;       /* [K] */
    float* y;             /* [N] */
    const float* norm_w;  /* NULL, or [K]: the input is RMSNorm(x) * norm_w */
    float norm_eps;       /* RMSNorm epsilon (norm_w set) */
    int32_t K;
    int32_t N;
    int32_t op;           /* GLC_GEMV_* */
    int32_t after_previous;
} glc_gemv_job;
int glc_gemv_q4k_chain_dev(const glc_gemv_job* jobs, int32_t n, void* stream);
/* Reads and clears the device error word of glc_gemv_q4k_dev /
 * glc_gemv_q4k_chain_dev on the current device (synchronises the device):
 * GLC_ERR_TIMEOUT when a bounded device-side wait gave up, else GLC_OK. */
int glc_gemv_poll_error(void);

/* ---- decode attention of one token (the attention half of a decode stage;
 *      caller side IClusterStageModel.ForwardStage, IClusterStageModel.cs:19,
 *      body external in the reference, Program.cs:1390).  Device pointers:
 *      q [n_heads][128], k_new / v_new [n_kv_heads][128] fp32 before rotation;
 *      k_cache / v_cache fp16 [n_kv_heads][max_len][128] (16-byte aligned).
 *      RoPE (rotate-half pairs (i, i+64), frequencies theta^(-2i/128)) at
 *      position pos rotates q and k_new; row pos of the caches receives the
 *      rotated k and v as fp16; out [n_heads][128] = softmax(q.K^T/sqrt(128)) V
 *      over positions 0..pos, query head h reading KV head h / (n_heads /
 *      n_kv_heads).  head_dim must be 128; n_heads a multiple of n_kv_heads,
 *      at most 8 query heads per KV head; 0 <= pos < max_len <= 32768.
 *      workspace: glc_attn_workspace_bytes(n_heads, n_kv_heads, max_len) bytes
 *      of device memory (reserved: the kernel keeps its partial results on
 *      chip).  One launch on `stream` (a thread-block cluster per KV head). ---- */
int glc_attn_workspace_bytes(int32_t n_heads, int32_t n_kv_heads, int32_t max_len, uint64_t* bytes);
int glc_attn_decode_dev(const float* q, const float* k_new, const float* v_new, void* k_cache, void* v_cache,
                        int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_len, int32_t pos,
                        float rope_theta, float* out, void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- router alone (for tests and for callers that route elsewhere) ---- */
int glc_router_topk_dev(const float* x, const float* router_w, int32_t T, int32_t D, int32_t E,
                        int32_t k, int32_t renormalize, int32_t rmsnorm, float* xin_out,
                        float* logits_out, int32_t* ids_out, float* w_out, void* stream);

/* ---- token -> expert dispatch plan (the batched path's histogram / scan /
 *      stable permutation).  ids: [P] expert per (token, slot) pair; outputs
 *      counts [E], exclusive offsets [E+1], perm [P] (position -> pair, pairs
 *      grouped by expert in ascending pair order) and inv [P] (pair -> position).
 *      The reference has no batching: it runs experts one token at a time
 *      (DistributedPipelineCoordinator.cs:181-206).  Asynchronous on `stream`;
 *      its internal group table comes from CUDA's stream-ordered pool
 *      (cudaMallocAsync / cudaFreeAsync on `stream`). ---- */
int glc_dispatch_plan_dev(const int32_t* ids, int32_t P, int32_t E, int32_t* counts,
                          int32_t* offsets, int32_t* perm, int32_t* inv, void* stream);

/* ---- allocation-free dispatch plan.  No counterpart in the reference (its
 *      hosts never batch tokens per expert).  Same inputs, outputs and results
 *      as glc_dispatch_plan_dev, for callers that cannot allocate device memory
 *      on the hot path (cudaMalloc/cudaFree may synchronise the whole device,
 *      or the host budgets device memory itself): the scratch group table lives
 *      in a fixed 51 KB device array owned by the library, so the call
 *      allocates and frees nothing and does not synchronise `stream`.
 *      Limits: P <= 65536 pairs, E <= 64 experts (larger -> GLC_ERR_INVALID_ARG).
 *      The first call on a device looks up the array's address (make it before
 *      any stream capture).  Calls share the array: calls that overlap on the
 *      GPU race and must be serialised by the caller. ---- */
int glc_dispatch_plan_noalloc_dev(const int32_t* ids, int32_t P, int32_t E, int32_t* counts,
                                  int32_t* offsets, int32_t* perm, int32_t* inv, void* stream);

/* ---- expert parallelism.  No counterpart in the reference: it runs a token's
 *      experts one after another on one worker (DistributedPipelineCoordinator.cs:
 *      181-206) and moves activations between LAN nodes.  Here a layer's experts are
 *      split into contiguous shards, one per rank (glc_moe_desc.expert_begin /
 *      expert_count; expert e lives on rank e / (E / world)), and a step is
 *        route -> dispatch plan + gather -> all-to-all (caller, e.g. NCCL) ->
 *        experts -> reverse all-to-all -> combine.
 *      All pointers are device memory; every call is asynchronous on `stream`. ---- */

/* RMSNorm (GLC_FWD_RMSNORM) + router + top-k on the handle's layer router (all E
 * experts, replicated on every rank): xin_out [T][D] normalised input, ids_out
 * [T][k] global expert ids, w_out [T][k] combine weights.  Also records the
 * shared-expert gate for a later glc_moe_combine_dev on the same handle. */
int glc_moe_route_dev(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags,
                      float* xin_out, int32_t* ids_out, float* w_out, void* stream);

/* Pairs (t, j) grouped by destination rank, stable: rank_counts [world],
 * rank_offsets [world+1], perm [T*k] (send position -> pair), inv [T*k]
 * (pair -> send position); send_rows [T*k][D] = xin row of each pair in send
 * order, send_ids [T*k] its global expert id.  num_experts % world == 0,
 * world <= 64. */
int glc_moe_ep_dispatch_dev(glc_moe* h, const float* xin, const int32_t* ids, int32_t T, int32_t world,
                            int32_t* rank_counts, int32_t* rank_offsets, int32_t* perm, int32_t* inv,
                            float* send_rows, int32_t* send_ids, void* stream);

/* y_out[r] = expert_{expert_ids[r]}(rows[r]) (gate, up, SwiGLU, down; no combine)
 * for R rows whose global ids lie in this handle's shard (ids outside are
 * clamped into it).  R <= max_tokens * top_k.  flags: GLC_FWD_DECODE forces the
 * per-row GEMVs, GLC_FWD_BATCHED the grouped tensor-core GEMMs; default GEMV
 * for R == 1, grouped otherwise. */
int glc_moe_experts_dev(glc_moe* h, int32_t layer, const float* rows, const int32_t* expert_ids,
                        int32_t R, uint32_t flags, float* y_out, void* stream);

/* out[t] = (resid[t] | 0) + sum_j w[t][j] * y_back[inv[t*k+j]], in j order
 * (AccumulatorStageWorker.AccumulateWeightedExpert, StageWorkers.cs:152-160),
 * then + sigmoid-gated shared expert of xin when the layer has one. */
int glc_moe_combine_dev(glc_moe* h, int32_t layer, const float* y_back, const int32_t* inv,
                        const float* w, int32_t T, const float* resid, const float* xin, float* out,
                        void* stream);

/* ---- wire codec: QuantizationKernels (Protocol/QuantizationKernels.cs:57-163) ---- */
int32_t glc_wire_token_bytes(int32_t mode, int32_t dim);
int glc_wire_quantize(int32_t mode, const float* x, int32_t T, int32_t D, uint8_t* out,
                      size_t out_bytes);
int glc_wire_dequantize(int32_t mode, const uint8_t* in, size_t in_bytes, int32_t T, int32_t D,
                        float* out);
int glc_wire_quantize_dev(int32_t mode, const float* x, int32_t T, int32_t D, uint8_t* out,
                          void* stream);
int glc_wire_dequantize_dev(int32_t mode, const uint8_t* in, int32_t T, int32_t D, float* out,
                            void* stream);

/* ---- FusedActivationHeader (Protocol/FusedActivationHeader.cs:41-218) ---- */
typedef struct glc_fused_header {
    uint64_t sequence_id;
    int32_t token_index;
    int32_t layer_index;
    int32_t hidden_dim;
    uint8_t precision_mode;
    uint8_t flags;
    uint16_t batch_tokens;
    float scale;
} glc_fused_header;
int glc_fused_header_write(const glc_fused_header* h, uint8_t* out32);
int glc_fused_header_read(const uint8_t* in32, glc_fused_header* h);
int32_t glc_fused_header_payload_bytes(const glc_fused_header* h);

/* ---- Multi-GPU plumbing for hosts without torch.distributed (the C# host):
 *      an NCCL communicator inside the library (NCCL is loaded at first use).
 *      One process per GPU; the host moves the 128-byte id from one rank to
 *      the others (its own channel), then every rank calls glc_comm_create.
 *      NCCL is opened by soname ("libnccl.so.2"): a process that also loads
 *      another NCCL user (e.g. torch, with its own NCCL) loads that one first. ---- */
#define GLC_COMM_ID_BYTES 128
typedef struct glc_comm glc_comm;
int glc_comm_unique_id(uint8_t* id_out);
int glc_comm_create(const uint8_t* id, int32_t nranks, int32_t rank, int32_t device, glc_comm** out);
int glc_comm_destroy(glc_comm* c);
/* Expert-parallel exchanges over NVLink peer memory (default on): the first
 * glc_moe_ep_forward maps every rank's exchange window into every rank with
 * CUDA IPC (collective); the dispatch and return blocks are then written
 * straight into the destination's window by the pack kernels, with an epoch
 * flag per source, and only routed rows cross the links.  If any rank cannot
 * map every peer, or enable = 0 (call it on every rank alike, between
 * exchanges), the same blocks go through grouped NCCL send / receive.
 * enable < 0 changes nothing and returns 1 when the exchanges go over peer
 * memory (the window is mapped and the option on), else 0. */
int glc_comm_peer_exchange(glc_comm* c, int32_t enable);

/* Stage boundary, replacing the socket transport of a FusedActivationHeader and
 * its wire payload (FusedSocketTransport.cs:51-135, DistributedClusterSession.cs:1123):
 * glc_pp_send quantises x [T][D] on the GPU in hdr->precision_mode (T =
 * hdr->batch_tokens, 0 meaning 1; D = hdr->hidden_dim) and sends the 32-byte
 * header and the payload to `peer`; glc_pp_recv receives the header, sizes the
 * payload with GetPayloadByteCount (FusedActivationHeader.cs:109-125),
 * receives and dequantises it into x_out [T][hidden_dim] (T <= max_tokens).
 * Device pointers; NULL stream = the communicator's stream.  glc_pp_recv reads
 * the header on the host, so it returns after the header has arrived. */
int glc_pp_send(glc_comm* c, int32_t peer, const glc_fused_header* hdr, const float* x, void* stream);
/* Raw device bytes to / from `peer` over the communicator (the sampled token
 * a last stage hands back to the first, DistributedClusterSession.cs:775-830).
 * Asynchronous on `stream` (NULL = the communicator's stream). */
int glc_comm_send(glc_comm* c, int32_t peer, const void* buf, size_t bytes, void* stream);
int glc_comm_recv(glc_comm* c, int32_t peer, void* buf, size_t bytes, void* stream);
int glc_pp_recv(glc_comm* c, int32_t peer, glc_fused_header* hdr_out, float* x_out, int32_t max_tokens,
                int32_t hidden_dim, void* stream);

/* The expert-parallel layer in one call (the steps of the glc_moe_*_dev
 * functions above with the exchanges over `c`): h holds expert shard
 * comm_rank of comm_world (expert_begin = rank * E / world), every rank calls
 * it with its own T tokens (T may differ, 0 <= T <= max_tokens / comm_world:
 * size the handle's max_tokens as world x the largest per-rank batch), and
 * out [T][D], ids_out [T][k], w_out [T][k] equal the single-GPU layer's
 * batched path bit for bit (the rows a rank receives are a batch: they run on
 * the grouped tensor-core experts whatever the decode flag).  Device pointers
 * (ids_out, w_out may be NULL); NULL stream = the handle's stream.
 * Asynchronous: the exchange blocks are sized for the most pairs one rank can
 * send one peer and their counts are read on the device only, so nothing
 * waits on the host; over peer memory (glc_comm_peer_exchange) only the
 * routed rows are written, through NCCL the whole blocks move.  A rank whose T is out of range still
 * takes part in both exchanges with no pairs (its peers do not wait on it)
 * and returns GLC_ERR_INVALID_ARG.  With profiling on, glc_moe_kernel_times
 * returns the phases: route, dispatch, exchange out, experts, exchange back,
 * combine. */
int glc_moe_ep_forward(glc_moe* h, glc_comm* c, int32_t layer, const float* x, int32_t T, uint32_t flags,
                       float* out, int32_t* ids_out, float* w_out, void* stream);

/* ---- dense decoder pipeline stage: IClusterStageModel (Pipeline/IClusterStageModel.cs:9-36)
 *      for Qwen2-style dense layers.  A stage holds layers [layer_begin,
 *      layer_begin + layer_count) of a model with their fp16 KV caches (the
 *      reference splits a model's layers over nodes, DistributedClusterSession.cs:
 *      775-830), plus the embedding table on a first stage and the final norm
 *      and LM head on a last stage.  One token per call: ForwardStage
 *      (IClusterStageModel.cs:19). ---- */
typedef struct glc_stage glc_stage;
typedef struct glc_stage_desc {
    int32_t hidden_dim;    /* D (multiple of 256) */
    int32_t ffn_dim;       /* FF of the SwiGLU feed-forward (multiple of 256) */
    int32_t n_heads;       /* query heads (n_heads * 128 a multiple of 256) */
    int32_t n_kv_heads;    /* KV heads (n_heads / n_kv_heads <= 8) */
    int32_t head_dim;      /* 128 */
    int32_t layer_begin;   /* first global layer of the stage (names its synthetic weights) */
    int32_t layer_count;   /* layers held */
    int32_t max_len;       /* KV cache rows, <= 32768 */
    float rope_theta;      /* rotate-half RoPE base (1e6 for Qwen2.5) */
    float rms_eps;         /* RMSNorm epsilon (1e-6 for Qwen2.5) */
    int32_t vocab;         /* rows of the embedding / LM head tables */
    int32_t has_embedding; /* first stage: x = dequantised embedding row of the token */
    int32_t has_lm_head;   /* last stage: logits = LM_head * (RMSNorm(x) * final_norm) */
    int32_t device;
    /* Mixture-of-experts feed-forward (Mixtral-style layers, no q/k/v biases)
     * when num_experts > 0: h = RMSNorm(x) * w_ffn, fp32 router [D][E],
     * softmax top-k (renormalised when moe_renormalize), x += sum_j p_j
     * Down_j(SiLU(Gate_j h) * (Up_j h)); ffn_dim is then unused. */
    int32_t num_experts;   /* 0 (dense) or 2..8 */
    int32_t top_k;         /* 1..num_experts */
    int32_t expert_ffn_dim;  /* F of each expert (multiple of 256) */
    int32_t moe_renormalize;
} glc_stage_desc;
/* Host weights of one layer: norms fp32 [D]; wq Q4_K [n_heads*128][D], wk / wv
 * [n_kv_heads*128][D], wo [D][n_heads*128], w_gate / w_up [FF][D], w_down
 * [D][FF] (GGUF row layout); biases fp32 (NULL = zero). */
typedef struct glc_dense_layer_weights {
    const float* attn_norm;
    const void* wq;
    const void* wk;
    const void* wv;
    const float* bq;
    const float* bk;
    const float* bv;
    const void* wo;
    const float* ffn_norm;
    const void* w_gate;
    const void* w_up;
    const void* w_down;
} glc_dense_layer_weights;
int glc_stage_create(const glc_stage_desc* desc, glc_stage** out);
int glc_stage_destroy(glc_stage* h);
/* layer: index within the stage (0 .. layer_count - 1) */
int glc_stage_load_layer(glc_stage* h, int32_t layer, const glc_dense_layer_weights* w);
/* A mixture-of-experts layer: the attention weights and norms of w (its
 * biases and feed-forward matrices are ignored), the fp32 router [D][E] and
 * the experts' Q4_K gate / up [E][F][D] and down [E][D][F] (GGUF ffn_*_exps). */
int glc_stage_load_moe_layer(glc_stage* h, int32_t layer, const glc_dense_layer_weights* w, const float* router,
                             const void* gate_exps, const void* up_exps, const void* down_exps);
/* embedding Q4_K [vocab][D] (first stage), final_norm fp32 [D] and lm_head Q4_K
 * [vocab][D] (last stage); the others may be NULL. */
int glc_stage_load_io(glc_stage* h, const void* embedding, const float* final_norm, const void* lm_head);
/* The documented seeded synthetic weights (Q4_K fields as glc_moe_synth_layer
 * with sigma_d 0.001; norms 1 + N(0, 0.02); biases N(0, 0.02); in a
 * mixture-of-experts stage no biases, the router N(0, 0.02) and the experts). */
int glc_stage_synth_layer(glc_stage* h, int32_t layer, uint64_t seed);
int glc_stage_synth_io(glc_stage* h, uint64_t seed);
/* ResetKvCache (IClusterStageModel.cs:35): clears the caches (synchronous). */
int glc_stage_reset(glc_stage* h);
/* ForwardStage(token, pos, inputX, outputX, logits, computeLogits): one token
 * at position pos (0 <= pos < max_len) through the stage's layers, writing
 * row pos of every layer's KV cache.  Device pointers: x_in [D] (NULL on a
 * first stage: the embedding row of *token), x_out [D] (NULL = not needed),
 * logits [vocab] and token_out (the arg-max, lower index on ties) on a last
 * stage (NULL = not computed).  Asynchronous on `stream` (NULL = the stage's
 * stream); after the first call of each (embedding, logits) variant the
 * stage's kernels are replayed from a captured CUDA graph. */
int glc_stage_forward_dev(glc_stage* h, int32_t pos, const int32_t* token, const float* x_in, float* x_out,
                          float* logits, int32_t* token_out, void* stream);
/* Reads and clears the stage's device error word. */
int glc_stage_poll_error(glc_stage* h);
/* Copies rows [0, rows) of layer `layer`'s fp16 K and V caches to host
 * buffers k_out / v_out [n_kv_heads][rows][128] (synchronous; the rotated
 * keys and the values as stored). */
int glc_stage_read_kv_cache(glc_stage* h, int32_t layer, int32_t rows, void* k_out, void* v_out);

#ifdef __cplusplus
}
#endif
#endif
