// api.cu -- the C ABI of libglacier_b200.so (include/glacier_b200.h).
//
// Host orchestration of the sm_100a kernels behind the reference's operator
// API: IInferenceStageWorker.ProcessActivation (IInferenceStageWorker.cs:43),
// GpuFirstExpertStageWorker.ProcessRoutedTopK (GpuFirstExpertStageWorker.cs:416),
// the MoE layer step (DistributedPipelineCoordinator.ExecuteStep, :72) and the
// QuantizationKernels wire codec (Protocol/QuantizationKernels.cs:86-163).
// There is no CPU fallback: every compute entry point runs on the GPU or
// returns an error.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../../../include/glacier_b200.h"
#include "kernels.h"
#include "synth.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                        \
    do {                                                                                      \
        cudaError_t e_ = (expr);                                                              \
        if (e_ != cudaSuccess)                                                                \
            return fail(e_ == cudaErrorMemoryAllocation ? GLC_ERR_OOM : GLC_ERR_CUDA,         \
                        "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__,     \
                        __LINE__);                                                            \
    } while (0)

int64_t rowbytes(int k) { return (int64_t)(k / 256) * 144; }

int host_threads() {
    unsigned n = std::thread::hardware_concurrency();
    return n == 0 ? 1 : (int)std::min(n, 32u);
}

struct LayerDev {
    uint8_t* gate = nullptr;
    uint8_t* up = nullptr;
    uint8_t* down = nullptr;
    float* router = nullptr;
    uint8_t* sh_gate = nullptr;
    uint8_t* sh_up = nullptr;
    uint8_t* sh_down = nullptr;
    float* sh_gate_vec = nullptr;
    bool loaded = false;
    // 2-D TMA descriptors of the expert tensors ([E*rows][rowBytes], box 144 x 128)
    alignas(64) uint8_t tmap_gate[128];
    alignas(64) uint8_t tmap_up[128];
    alignas(64) uint8_t tmap_down[128];
    // the shared expert's ([Fs][D/256*144] gate/up, [D][Fs/256*144] down)
    alignas(64) uint8_t tmap_sh_gate[128];
    alignas(64) uint8_t tmap_sh_up[128];
    alignas(64) uint8_t tmap_sh_down[128];
    bool tmaps = false;
    bool host_experts = false;  // gate/up/down in pinned host memory (expert residency mode)
};

}  // namespace

namespace glc {
// Records the thread-local message returned by glc_last_error() for entry
// points defined in other translation units.
int set_last_error(int code, const char* msg) {
    g_last_error = msg;
    return code;
}
}  // namespace glc

// Device words at the head of a handle's result block: error word, grid-barrier
// counter and completion counter of the fused decode kernel.
constexpr int kErrWords = 8;
// K slices of the shared expert's batched down projection: enough 128-row x
// slice work items to cover the SMs when a few token groups give few tiles.
constexpr int kShSlicesMax = 8;

struct glc_moe {
    glc_moe_desc d{};
    int num_sms = 0;
    int disposed = 0;
    cudaStream_t stream = nullptr;
    std::vector<LayerDev> layers;
    // device workspace sized for max_tokens
    float* x = nullptr;        // [T][D]
    float* xin = nullptr;      // [T][D]
    float* out = nullptr;      // [T][D]
    float* act = nullptr;      // [T*k][F]
    float* act_sh = nullptr;   // [T][Fs]
    float* wts = nullptr;      // [T*k]
    float* gate_out = nullptr; // [T]
    unsigned long long* route_slots = nullptr;  // [T][E+1][8] epoch-tagged partial logits of the wide decode kernel
    int* ids = nullptr;        // [T*k]
    int* zeros_i = nullptr;    // [T] expert id 0 for the shared expert
    float* ones = nullptr;     // [T*k] unit combine weights (per-row expert outputs)
    int* ep_keys = nullptr;    // [T*k] destination-rank keys of the expert-parallel dispatch
    int* err = nullptr;        // [0] device error word; [2..3] grid-barrier counter (u64), [4..5] completion counter (u64) of the fused decode kernel
    // err, ids, wts and out are carved from one result block, in that order,
    // so the host-buffer forward returns all of them with one copy
    uint8_t* res = nullptr;
    size_t res_off_ids = 0, res_off_w = 0, res_off_out = 0, res_bytes = 0;
    // batched (T > 1) path
    glc::DispatchPlan plan{};
    int plan_gmax = 0;
    uint8_t* btiles = nullptr;  // swizzled fp16 hi/lo B tiles
    size_t btiles_bytes = 0;
    float* rscale = nullptr;    // [T*k]
    float* ysort = nullptr;     // [T*k][D]
    // the shared expert on the batched path: all T tokens as one expert's
    // groups, its down projection in K slices (partial planes summed by the combine)
    glc::DispatchPlan plan_sh{};
    int plan_sh_gmax = 0;
    float* rscale_sh = nullptr;  // [T]
    float* ysh = nullptr;        // [kShSlicesMax][T][D]
    // pinned host staging
    float* h_x = nullptr;
    const float* d_x_map = nullptr;  // device address of h_x (mapped), or null
    uint8_t* h_res = nullptr;  // pinned (and mapped) copy of the result block
    uint8_t* d_res_map = nullptr;  // device address of h_res
    // mapped completion words of the fused decode launch the host-buffer
    // forward waits on: [0] epoch of the last finished launch, [1] its error word
    unsigned long long* h_sig = nullptr;
    unsigned long long* d_sig_map = nullptr;
    unsigned long long host_epoch = 0;
    // failure-detection test hook (glc_moe_debug_stall), consumed by the next fused launch
    int debug_stall_cta = 0;           // CTA index + 1, 0 = none
    long long debug_wait_limit_ns = 0;
    int* h_ids = nullptr;
    float* h_w = nullptr;
    // Expert residency (glc_moe_set_expert_slots), GpuFirstExpertStageWorker's
    // GPU slot cache (GpuFirstExpertStageWorker.cs:144-151, 354-407): the routed
    // experts of every layer in pinned host memory, `slots` of them at a time
    // in an HBM pool, the least recently used out first.
    int slots = 0;
    uint8_t* pool_gate = nullptr;
    uint8_t* pool_up = nullptr;
    uint8_t* pool_down = nullptr;
    LayerDev pool_maps{};                       // tensor maps over the pool
    std::vector<long long> slot_key;            // layer * El + local expert held, or -1
    std::vector<unsigned long long> slot_used;  // call stamp of the last use
    unsigned long long slot_clock = 0;
    long long res_hits = 0, res_transfers = 0, res_prefetches = 0;
    int* d_slot_ids = nullptr;  // [max_tokens * k] slot of each (token, slot) pair
    int* h_slot_ids = nullptr;  // pinned
    // optional per-kernel CUDA-event timing of the last forward (launch order)
    int profiling = 0;
    int n_marks = 0;
    int mark_lock = 0;  // > 0: inner steps of a call that records its own phase marks
    cudaEvent_t marks[16] = {};
    // captured decode step
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    // the host-buffer forward's replayed steps (copy of h_x + fused launch),
    // one per (layer, T, flags) shape seen, replaced round robin when full
    struct FwdGraph {
        cudaGraphExec_t exec = nullptr;
        int layer = -1, T = 0;
        uint32_t flags = 0;
    };
    std::vector<FwdGraph> fwd_graphs;
    size_t fwd_next = 0;
};

namespace {

int check_handle(glc_moe* h) {
    if (!h) return fail(GLC_ERR_INVALID_ARG, "null handle");
    if (h->disposed) return fail(GLC_ERR_DISPOSED, "handle was destroyed");
    cudaError_t e = cudaSetDevice(h->d.device);
    if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "cudaSetDevice(%d): %s", h->d.device, cudaGetErrorString(e));
    return GLC_OK;
}

int local_experts(const glc_moe* h) { return h->d.expert_count > 0 ? h->d.expert_count : h->d.num_experts; }

LayerDev* layer_of(glc_moe* h, int layer) {
    // LayerIndex is clamped like CpuWarmExpertPoolWorker.cs:243.
    int n = (int)h->layers.size();
    int l = layer < 0 ? 0 : (layer >= n ? n - 1 : layer);
    return &h->layers[l];
}

// Records a timing mark on `st` when profiling is enabled (marks[i+1]-marks[i]
// is the device time of the i-th kernel of the last forward).
void mark(glc_moe* h, cudaStream_t st) {
    if (!h->profiling || h->mark_lock || h->n_marks >= 16) return;
    cudaEventRecord(h->marks[h->n_marks++], st);
}

// A phase boundary of a call that times its phases rather than its kernels.
void mark_phase(glc_moe* h, cudaStream_t st) {
    if (!h->profiling || h->n_marks >= 16) return;
    cudaEventRecord(h->marks[h->n_marks++], st);
}

int check_device_error(glc_moe* h) {
    int code = 0;
    CUDA_TRY(cudaMemcpy(&code, h->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code != 0) {
        // also clears the fused kernel's barrier and completion counters, which a
        // launch that gave up may leave mid-count, and the host's matching epoch
        cudaMemset(h->err, 0, kErrWords * sizeof(int));
        // the wide kernel's launch counter restarts, so its tagged slots must too
        cudaMemset(h->route_slots, 0, sizeof(unsigned long long) * h->d.max_tokens * (h->d.num_experts + 1) * 8);
        h->host_epoch = 0;
        if (h->h_sig) h->h_sig[0] = h->h_sig[1] = 0;
        if (code == glc::kDevBadArg)
            return fail(GLC_ERR_INVALID_ARG, "a kernel rejected its arguments (device code %d)", code);
        return fail(GLC_ERR_TIMEOUT, "device-side wait gave up (code %d)", code);
    }
    return GLC_OK;
}

// Decode-path expert launches: gate/up + SwiGLU over `npairs` (token, slot)
// pairs, then the down projection with the weighted combine per token.
int run_experts(glc_moe* h, LayerDev* L, const float* xin, int T, int k, const int* ids,
                const float* wts, const float* resid, float* out, cudaStream_t st) {
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, E = local_experts(h);
    glc::GemvParams g{};
    g.mode = glc::kGemvGateUp;
    g.K = D;
    g.rows = F;
    g.nseg = T * k;
    g.kslots = k;
    g.num_experts = E;
    g.A = L->gate;
    g.B = L->up;
    g.expert_bytes = (long long)F * rowbytes(D);
    g.ids = ids;
    g.x = xin;
    g.y = h->act;
    g.err = h->err;
    CUDA_TRY(glc::gemv_launch(g, h->num_sms, st));
    mark(h, st);
    glc::GemvParams dn{};
    dn.mode = glc::kGemvDownCombine;
    dn.K = F;
    dn.rows = D;
    dn.nseg = T;
    dn.kslots = k;
    dn.num_experts = E;
    dn.A = L->down;
    dn.expert_bytes = (long long)D * rowbytes(F);
    dn.ids = ids;
    dn.cw = wts;
    dn.x = h->act;
    dn.resid = resid;
    dn.y = out;
    dn.err = h->err;
    CUDA_TRY(glc::gemv_launch(dn, h->num_sms, st));
    mark(h, st);
    return GLC_OK;
}

int run_shared_expert(glc_moe* h, LayerDev* L, const float* xin, int T, float* out, cudaStream_t st) {
    const int D = h->d.hidden_dim, Fs = h->d.shared_ffn_dim;
    glc::GemvParams g{};
    g.mode = glc::kGemvGateUp;
    g.K = D;
    g.rows = Fs;
    g.nseg = T;
    g.kslots = 1;
    g.num_experts = 1;
    g.A = L->sh_gate;
    g.B = L->sh_up;
    g.expert_bytes = 0;
    g.ids = h->zeros_i;
    g.x = xin;
    g.y = h->act_sh;
    g.err = h->err;
    CUDA_TRY(glc::gemv_launch(g, h->num_sms, st));
    mark(h, st);
    glc::GemvParams dn{};
    dn.mode = glc::kGemvDownCombine;
    dn.K = Fs;
    dn.rows = D;
    dn.nseg = T;
    dn.kslots = 1;
    dn.num_experts = 1;
    dn.A = L->sh_down;
    dn.expert_bytes = 0;
    dn.ids = h->zeros_i;
    dn.cw = h->gate_out;
    dn.x = h->act_sh;
    dn.y = out;
    dn.accumulate = 1;
    dn.err = h->err;
    CUDA_TRY(glc::gemv_launch(dn, h->num_sms, st));
    mark(h, st);
    return GLC_OK;
}

int make_layer_tmaps(glc_moe* h, LayerDev& L) {
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, El = local_experts(h);
    // (host-resident routed experts are read through the slot pool's maps)
    if (!L.host_experts &&
        (glc::make_q4k_tensor_map(L.tmap_gate, L.gate, (long long)El * F, (int)rowbytes(D)) ||
         glc::make_q4k_tensor_map(L.tmap_up, L.up, (long long)El * F, (int)rowbytes(D)) ||
         glc::make_q4k_tensor_map(L.tmap_down, L.down, (long long)El * D, (int)rowbytes(F))))
        return fail(GLC_ERR_CUDA, "cuTensorMapEncodeTiled failed for the expert tensors");
    const int Fs = h->d.shared_ffn_dim;
    if (Fs > 0 && (glc::make_q4k_tensor_map(L.tmap_sh_gate, L.sh_gate, Fs, (int)rowbytes(D)) ||
                   glc::make_q4k_tensor_map(L.tmap_sh_up, L.sh_up, Fs, (int)rowbytes(D)) ||
                   glc::make_q4k_tensor_map(L.tmap_sh_down, L.sh_down, D, (int)rowbytes(Fs))))
        return fail(GLC_ERR_CUDA, "cuTensorMapEncodeTiled failed for the shared expert");
    L.tmaps = true;
    return GLC_OK;
}

// Layouts of the grouped tensor-core GEMMs for a batch of `pairs` (token,
// expert) pairs over `experts` experts.  Groups of up to 64 tokens (the wide
// kernel layout) once the batch averages 32 or more pairs per expert, where
// experts with more than 32 tokens are common and groups of 32 would
// dequantise their weights once per 32 tokens.  The down projection runs the
// wide kernel layout for either group size (it holds groups of 32 as well:
// the same time on the Mixtral 64-token batch, 3 % less on the Qwen2-57B
// 16-token one); gate/up, two matrices per raw stage, keeps the narrow
// layout's four raw stages (two in the wide one) for groups of 32, where the
// wide layout measured 4 % slower.  GLC_GROUPED_WIDE=0 / 1
// forces the narrow / wide layout everywhere (read on every call).  Every
// choice gives the same bits: an output is the same fp32 sum over the same K
// order in both layouts.
struct GroupedLayouts {
    bool wide_groups, gateup_wide, down_wide;
};
static GroupedLayouts grouped_layouts(int pairs, int experts) {
    const char* v = getenv("GLC_GROUPED_WIDE");
    if (v && (v[0] == '0' || v[0] == '1') && v[1] == 0) {
        const bool w = v[0] == '1';
        return {w, w, w};
    }
    const bool w = pairs > glc::kGroupTokens && pairs >= glc::kGroupTokens * experts;
    return {w, w, true};
}

// The shared expert of a batched call (T > 1) on the grouped tensor-core
// path: all T tokens are one expert's groups, so its weights are read once
// per launch whatever T is; the down projection (few 128-row tiles at small
// T) is split into K slices to fill the SMs.  Leaves the slice planes in
// h->ysh (their count in *slices) for the combine to add with the gate.
int run_shared_grouped(glc_moe* h, LayerDev* L, const float* xin, int T, int* slices, cudaStream_t st) {
    const int D = h->d.hidden_dim, Fs = h->d.shared_ffn_dim;
    if (!L->sh_gate || !L->tmaps) return fail(GLC_ERR_STATE, "layer has no shared expert tensor maps");
    const GroupedLayouts lay = grouped_layouts(T, 1);
    const int gtok = lay.wide_groups ? glc::kGroupTokensWide : glc::kGroupTokens;
    CUDA_TRY(glc::dispatch_plan_launch(h->zeros_i, T, 1, h->plan_sh, st, nullptr, gtok));
    mark(h, st);
    CUDA_TRY(glc::split_rows_launch(xin, T, D, 1, 1, h->plan_sh, h->btiles, h->rscale_sh, st));
    mark(h, st);
    const int gsh = (T + gtok - 1) / gtok;
    glc::GroupedParams sg{};
    sg.wide = lay.gateup_wide;
    sg.K = D;
    sg.rows_per_e = Fs;
    sg.nm = 2;
    sg.num_experts = 1;
    sg.plan = h->plan_sh;
    sg.btiles = h->btiles;
    sg.rscale = h->rscale_sh;
    sg.out = h->act_sh;
    sg.err = h->err;
    CUDA_TRY(glc::grouped_launch(L->tmap_sh_gate, L->tmap_sh_up, sg, gsh * (Fs / 128), h->num_sms, st));
    mark(h, st);
    CUDA_TRY(glc::split_rows_launch(h->act_sh, T, Fs, 1, 0, h->plan_sh, h->btiles, h->rscale_sh, st));
    mark(h, st);
    const int tiles = gsh * (D / 128);
    // K slices, when one slice of tiles leaves SMs idle: the count whose
    // items fill whole rounds of the SMs best (fewest rounds of 1/n-sized
    // items; the smaller count on a tie), e.g. 5 slices of 28 tiles = 140
    // items in one round rather than 6 = 168 items in two (Qwen2-57B shared
    // expert at 16 tokens: 36.8 -> 28.7 us).  With a full round of tiles
    // already (256 tokens), no slices: smaller items there measured slower
    // (each item ends with an accumulator drain).  The count (and so the
    // order of the partial sums) follows the narrow layout's tile count
    // whichever layout runs: both give the same bits.
    const int tiles_n = (T + glc::kGroupTokens - 1) / glc::kGroupTokens * (D / 128);
    const int nmax = tiles_n >= h->num_sms ? 1 : std::max(1, std::min(kShSlicesMax, Fs / 256));
    int n = 1;
    long long best_num = 1, best_den = 0;  // rounds / n of the best count so far (den 0: none yet)
    for (int c = 1; c <= nmax; ++c) {
        const long long rounds = ((long long)tiles_n * c + h->num_sms - 1) / h->num_sms;
        if (best_den == 0 || rounds * best_den < best_num * c) {
            best_num = rounds;
            best_den = c;
            n = c;
        }
    }
    glc::GroupedParams sd = sg;
    sd.K = Fs;
    sd.rows_per_e = D;
    sd.nm = 1;
    sd.out = h->ysh;
    sd.ksplit = n;
    sd.wide = lay.down_wide;
    sd.part_stride = (long long)T * D;
    CUDA_TRY(glc::grouped_launch(L->tmap_sh_down, nullptr, sd, tiles * n, h->num_sms, st));
    mark(h, st);
    *slices = n;
    return GLC_OK;
}

// Batched path (T > 1): dispatch plan, fp16 hi/lo operand tiles, grouped
// tcgen05 GEMMs (gate/up + SwiGLU, then down), k-ordered weighted combine.
// count (optional, device memory): the rows actually present of the T given
// (a batch sized on the device; T is then its upper bound).
int run_experts_grouped(glc_moe* h, LayerDev* L, const float* xin, int T, int k, const int* ids,
                        const float* wts, const float* resid, float* out, cudaStream_t st, bool with_shared,
                        const int* count = nullptr) {
    int rc = GLC_OK;
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, E = local_experts(h);
    const int P = T * k;
    if (!L->tmaps) return fail(GLC_ERR_STATE, "layer has no tensor maps");
    const GroupedLayouts lay = grouped_layouts(P, E);
    CUDA_TRY(glc::dispatch_plan_launch(ids, P, E, h->plan, st, count,
                                       lay.wide_groups ? glc::kGroupTokensWide : glc::kGroupTokens));
    mark(h, st);
    CUDA_TRY(glc::split_rows_launch(xin, P, D, k, 1, h->plan, h->btiles, h->rscale, st, count));
    mark(h, st);
    const int gmax = glc::plan_max_groups(P, E);
    glc::GroupedParams g{};
    g.wide = lay.gateup_wide;
    g.K = D;
    g.rows_per_e = F;
    g.nm = 2;
    g.num_experts = E;
    g.plan = h->plan;
    g.btiles = h->btiles;
    g.rscale = h->rscale;
    g.out = h->act;
    g.err = h->err;
    CUDA_TRY(glc::grouped_launch(L->tmap_gate, L->tmap_up, g, gmax * (F / 128), h->num_sms, st));
    mark(h, st);
    CUDA_TRY(glc::split_rows_launch(h->act, P, F, k, 0, h->plan, h->btiles, h->rscale, st, count));
    mark(h, st);
    glc::GroupedParams dn = g;
    dn.K = F;
    dn.rows_per_e = D;
    dn.nm = 1;
    dn.wide = lay.down_wide;
    dn.out = h->ysort;
    CUDA_TRY(glc::grouped_launch(L->tmap_down, nullptr, dn, gmax * (D / 128), h->num_sms, st));
    mark(h, st);
    const float* ysh = nullptr;
    int slices = 1;
    if (with_shared && h->d.shared_ffn_dim > 0) {
        rc = run_shared_grouped(h, L, xin, T, &slices, st);
        if (rc) return rc;
        ysh = h->ysh;
    }
    CUDA_TRY(glc::combine_launch(h->ysort, T, D, k, h->plan.inv, wts, resid, out, st, ysh, slices,
                                 (long long)T * D, h->gate_out, count));
    mark(h, st);
    return GLC_OK;
}

void free_layer(LayerDev& L) {
    if (L.host_experts) {
        cudaFreeHost(L.gate); cudaFreeHost(L.up); cudaFreeHost(L.down);
    } else {
        cudaFree(L.gate); cudaFree(L.up); cudaFree(L.down);
    }
    cudaFree(L.router);
    cudaFree(L.sh_gate); cudaFree(L.sh_up); cudaFree(L.sh_down); cudaFree(L.sh_gate_vec);
    L = LayerDev{};
}

int alloc_layer(glc_moe* h, LayerDev& L) {
    if (L.gate) return GLC_OK;
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, E = h->d.num_experts, El = local_experts(h);
    const size_t gsz = (size_t)El * F * rowbytes(D), dsz = (size_t)El * D * rowbytes(F);
    if (h->slots > 0) {  // routed experts stay in pinned host memory, paged into the slot pool
        L.host_experts = true;
        CUDA_TRY(cudaMallocHost(&L.gate, gsz));
        CUDA_TRY(cudaMallocHost(&L.up, gsz));
        CUDA_TRY(cudaMallocHost(&L.down, dsz));
    } else {
        CUDA_TRY(cudaMalloc(&L.gate, gsz));
        CUDA_TRY(cudaMalloc(&L.up, gsz));
        CUDA_TRY(cudaMalloc(&L.down, dsz));
    }
    CUDA_TRY(cudaMalloc(&L.router, sizeof(float) * (size_t)D * E));
    if (h->d.shared_ffn_dim > 0) {
        const int Fs = h->d.shared_ffn_dim;
        CUDA_TRY(cudaMalloc(&L.sh_gate, (size_t)Fs * rowbytes(D)));
        CUDA_TRY(cudaMalloc(&L.sh_up, (size_t)Fs * rowbytes(D)));
        CUDA_TRY(cudaMalloc(&L.sh_down, (size_t)D * rowbytes(Fs)));
        CUDA_TRY(cudaMalloc(&L.sh_gate_vec, sizeof(float) * D));
    }
    return GLC_OK;
}

// ---- expert residency (glc_moe_set_expert_slots)

// Slot holding local expert e of `layer`, loading it into the least recently
// used slot not yet used by this call (stamp) on a miss -- the three matrices
// copied from pinned host memory on `st`, behind the work already queued
// there that may still read the slot.  Returns the slot, -1 when every slot
// is in use by this call, -2 on a CUDA error (recorded).
int ensure_slot(glc_moe* h, int layer, int e, unsigned long long stamp, cudaStream_t st, bool* loaded) {
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, El = local_experts(h);
    const long long key = (long long)layer * El + e;
    *loaded = false;
    for (int s = 0; s < h->slots; ++s)
        if (h->slot_key[s] == key) {
            h->slot_used[s] = stamp;
            return s;
        }
    int victim = -1;
    for (int s = 0; s < h->slots; ++s)
        if (h->slot_used[s] < stamp && (victim < 0 || h->slot_used[s] < h->slot_used[victim])) victim = s;
    if (victim < 0) return -1;
    const size_t gsl = (size_t)F * rowbytes(D), dsl = (size_t)D * rowbytes(F);
    const LayerDev& L = h->layers[layer];
    h->slot_key[victim] = -1;  // until the copies are queued
    if (cudaMemcpyAsync(h->pool_gate + victim * gsl, L.gate + e * gsl, gsl, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(h->pool_up + victim * gsl, L.up + e * gsl, gsl, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(h->pool_down + victim * dsl, L.down + e * dsl, dsl, cudaMemcpyHostToDevice, st) != cudaSuccess) {
        fail(GLC_ERR_CUDA, "expert page-in copy: %s", cudaGetErrorString(cudaGetLastError()));
        return -2;
    }
    h->slot_key[victim] = key;
    h->slot_used[victim] = stamp;
    *loaded = true;
    return victim;
}

// A layer's routed experts were (re)written: its slots no longer hold them.
// Layer 0's first min(slots, experts) experts are then staged, as
// GpuFirstExpertStageWorker.WarmInitialGpuSlots (GpuFirstExpertStageWorker.cs:344-352)
// (not counted as transfers).
int warm_slots(glc_moe* h, int layer) {
    if (h->slots == 0) return GLC_OK;
    const int El = local_experts(h);
    for (int s = 0; s < h->slots; ++s)
        if (h->slot_key[s] >= 0 && h->slot_key[s] / El == layer) {
            h->slot_key[s] = -1;
            h->slot_used[s] = 0;
        }
    if (layer != 0) return GLC_OK;
    const unsigned long long stamp = ++h->slot_clock;
    for (int e = 0; e < std::min(h->slots, El); ++e) {
        bool loaded;
        if (ensure_slot(h, 0, e, stamp, h->stream, &loaded) < 0) return GLC_ERR_CUDA;
    }
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    return GLC_OK;
}

// After the router of a call on a residency-mode handle: the routed ids
// [P] to the host, every selected expert into a slot (hits and transfers
// counted per pair, as EnsureExpertInGpuSlot, GpuFirstExpertStageWorker.cs:354-385),
// and the slot of each pair back to the device for the expert kernels, which
// read the pool as their expert array.
int page_in(glc_moe* h, int layer, const int* ids_dev, int P, cudaStream_t st, const int** slot_ids) {
    const int El = local_experts(h);
    CUDA_TRY(cudaMemcpyAsync(h->h_slot_ids, ids_dev, sizeof(int) * P, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    const unsigned long long stamp = ++h->slot_clock;
    for (int i = 0; i < P; ++i) {
        int e = h->h_slot_ids[i];
        e = e < 0 ? 0 : (e >= El ? El - 1 : e);  // clamped like ProcessRoutedTopK
        bool loaded;
        const int sl = ensure_slot(h, layer, e, stamp, st, &loaded);
        if (sl == -1)
            return fail(GLC_ERR_UNSUPPORTED, "the call routes to more distinct experts than the %d expert slots",
                        h->slots);
        if (sl < 0) return GLC_ERR_CUDA;
        if (loaded) ++h->res_transfers;
        else ++h->res_hits;
        h->h_slot_ids[i] = sl;
    }
    CUDA_TRY(cudaMemcpyAsync(h->d_slot_ids, h->h_slot_ids, sizeof(int) * P, cudaMemcpyHostToDevice, st));
    *slot_ids = h->d_slot_ids;
    return GLC_OK;
}

// The layer as the expert kernels see it in residency mode: the slot pool
// as its expert array (router and shared expert its own).
LayerDev pool_view(const glc_moe* h, const LayerDev* L) {
    LayerDev V = *L;
    V.gate = h->pool_gate;
    V.up = h->pool_up;
    V.down = h->pool_down;
    std::memcpy(V.tmap_gate, h->pool_maps.tmap_gate, sizeof(V.tmap_gate));
    std::memcpy(V.tmap_up, h->pool_maps.tmap_up, sizeof(V.tmap_up));
    std::memcpy(V.tmap_down, h->pool_maps.tmap_down, sizeof(V.tmap_down));
    V.host_experts = false;
    return V;
}

// The layer and pair ids the expert kernels run on: as given, or in
// residency mode the selected experts paged into slots (ids [P] on the
// device) and the pool as the expert array (*V holds that view).
int expert_operands(glc_moe* h, LayerDev* L, const int* ids, int P, cudaStream_t st, LayerDev* V, LayerDev** LR,
                    const int** run_ids) {
    *LR = L;
    *run_ids = ids;
    if (!h->slots || P <= 0) return GLC_OK;
    const int rc = page_in(h, (int)(L - h->layers.data()), ids, P, st, run_ids);
    if (rc) return rc;
    *V = pool_view(h, L);
    *LR = V;
    return GLC_OK;
}

}  // namespace

extern "C" {

int glc_abi_version(void) { return GLC_ABI_VERSION; }

int glc_moe_set_expert_slots(glc_moe* h, int32_t slots) {
    int rc = check_handle(h);
    if (rc) return rc;
    for (const auto& L : h->layers)
        if (L.gate) return fail(GLC_ERR_STATE, "expert slots are set before the first layer is loaded");
    if (h->slots) return fail(GLC_ERR_STATE, "expert slots are already set");
    if (local_experts(h) != h->d.num_experts)
        return fail(GLC_ERR_UNSUPPORTED, "expert residency on an expert-parallel shard");
    const int E = h->d.num_experts, D = h->d.hidden_dim, F = h->d.expert_ffn_dim;
    slots = slots < 1 ? 1 : (slots > E ? E : slots);  // clamped like GpuFirstExpertStageWorker.cs:144
    const size_t gsl = (size_t)F * rowbytes(D), dsl = (size_t)D * rowbytes(F);
    CUDA_TRY(cudaSetDevice(h->d.device));
    CUDA_TRY(cudaMalloc(&h->pool_gate, slots * gsl));
    CUDA_TRY(cudaMalloc(&h->pool_up, slots * gsl));
    CUDA_TRY(cudaMalloc(&h->pool_down, slots * dsl));
    if (glc::make_q4k_tensor_map(h->pool_maps.tmap_gate, h->pool_gate, (long long)slots * F, (int)rowbytes(D)) ||
        glc::make_q4k_tensor_map(h->pool_maps.tmap_up, h->pool_up, (long long)slots * F, (int)rowbytes(D)) ||
        glc::make_q4k_tensor_map(h->pool_maps.tmap_down, h->pool_down, (long long)slots * D, (int)rowbytes(F)))
        return fail(GLC_ERR_CUDA, "cuTensorMapEncodeTiled failed for the expert slot pool");
    const size_t P = (size_t)h->d.max_tokens * h->d.top_k;
    CUDA_TRY(cudaMalloc(&h->d_slot_ids, sizeof(int) * P));
    CUDA_TRY(cudaMallocHost(&h->h_slot_ids, sizeof(int) * P));
    h->slot_key.assign(slots, -1);
    h->slot_used.assign(slots, 0);
    h->slots = slots;
    return GLC_OK;
}

int glc_moe_prefetch_experts(glc_moe* h, int32_t layer, const int32_t* expert_ids, int32_t n) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (h->slots == 0) return GLC_OK;  // every expert is resident
    if (n < 0 || (n > 0 && !expert_ids)) return fail(GLC_ERR_INVALID_ARG, "bad expert list");
    const int El = local_experts(h);
    const int l = (int)(layer_of(h, layer) - h->layers.data());
    if (!h->layers[l].loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", l);
    const unsigned long long stamp = ++h->slot_clock;
    for (int i = 0; i < n; ++i) {
        const int e = expert_ids[i] < 0 ? 0 : (expert_ids[i] >= El ? El - 1 : expert_ids[i]);
        bool loaded;
        const int sl = ensure_slot(h, l, e, stamp, h->stream, &loaded);
        if (sl == -2) return GLC_ERR_CUDA;
        if (sl == -1) break;  // every slot already taken by this prefetch
        if (loaded) ++h->res_prefetches;
    }
    return GLC_OK;
}

int glc_moe_expert_residency(glc_moe* h, int64_t* out4) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!out4) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    out4[0] = h->slots ? h->slots : local_experts(h);
    out4[1] = h->res_hits;
    out4[2] = h->res_transfers;
    out4[3] = h->res_prefetches;
    return GLC_OK;
}

const char* glc_last_error(void) { return g_last_error.c_str(); }

int glc_device_count(int32_t* count) {
    if (!count) return fail(GLC_ERR_INVALID_ARG, "null count");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return fail(GLC_ERR_CUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = n;
    return GLC_OK;
}

int64_t glc_q4k_row_bytes(int32_t k) {
    if (k <= 0 || (k % 256) != 0) return -1;
    return rowbytes(k);
}

int glc_moe_create(const glc_moe_desc* desc, glc_moe** out) {
    if (!desc || !out) return fail(GLC_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const glc_moe_desc& d = *desc;
    if (d.hidden_dim <= 0 || d.expert_ffn_dim <= 0 || d.num_experts <= 0)
        return fail(GLC_ERR_INVALID_ARG, "dimensions must be positive (D=%d F=%d E=%d)", d.hidden_dim,
                    d.expert_ffn_dim, d.num_experts);
    if (d.weight_type != GLC_GGUF_Q4_K)
        return fail(GLC_ERR_UNSUPPORTED, "weight type %d not supported (Q4_K = 12)", d.weight_type);
    if (d.hidden_dim % 256 || d.expert_ffn_dim % 256 || (d.shared_ffn_dim > 0 && d.shared_ffn_dim % 256))
        return fail(GLC_ERR_UNSUPPORTED, "Q4_K needs dimensions that are multiples of 256");
    if (d.top_k <= 0 || d.top_k > d.num_experts || d.top_k > 16 || d.num_experts > 64)
        return fail(GLC_ERR_INVALID_ARG, "top_k %d / num_experts %d out of range", d.top_k, d.num_experts);
    if (d.num_layers <= 0 || d.max_tokens <= 0) return fail(GLC_ERR_INVALID_ARG, "num_layers and max_tokens must be positive");
    if (d.expert_begin < 0 || d.expert_count < 0 || d.expert_begin + (d.expert_count ? d.expert_count : d.num_experts) > d.num_experts)
        return fail(GLC_ERR_INVALID_ARG, "expert shard out of range");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(GLC_ERR_CUDA, "no CUDA device");
    if (d.device < 0 || d.device >= ndev) return fail(GLC_ERR_INVALID_ARG, "device %d out of range", d.device);
    CUDA_TRY(cudaSetDevice(d.device));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, d.device));
    if (prop.major < 10) return fail(GLC_ERR_UNSUPPORTED, "device %d is sm_%d%d; sm_100a required", d.device, prop.major, prop.minor);

    glc_moe* h = new glc_moe();
    h->d = d;
    h->num_sms = prop.multiProcessorCount;
    h->layers.resize(d.num_layers);
    const size_t T = d.max_tokens, D = d.hidden_dim, F = d.expert_ffn_dim, k = d.top_k;
    const size_t Fs = d.shared_ffn_dim > 0 ? d.shared_ffn_dim : 0;
    auto cleanup = [&](int rc) { glc_moe_destroy(h); return rc; };
#define ALLOC(ptr, bytes)                                                                     \
    do {                                                                                      \
        cudaError_t e_ = cudaMalloc(&(ptr), (bytes));                                         \
        if (e_ != cudaSuccess) return cleanup(fail(GLC_ERR_OOM, "cudaMalloc %zu: %s", (size_t)(bytes), cudaGetErrorString(e_))); \
    } while (0)
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
        return cleanup(fail(GLC_ERR_CUDA, "cudaStreamCreate failed"));
    ALLOC(h->x, sizeof(float) * T * D);
    ALLOC(h->xin, sizeof(float) * T * D);
    ALLOC(h->act, sizeof(float) * T * k * F);
    if (Fs) ALLOC(h->act_sh, sizeof(float) * T * Fs);
    ALLOC(h->gate_out, sizeof(float) * T);
    ALLOC(h->route_slots, sizeof(unsigned long long) * T * (d.num_experts + 1) * 8);
    ALLOC(h->zeros_i, sizeof(int) * T);
    ALLOC(h->ones, sizeof(float) * T * k);
    ALLOC(h->ep_keys, sizeof(int) * T * k);
    {
        auto a16 = [](size_t v) { return (v + 15) & ~size_t(15); };
        h->res_off_ids = a16(kErrWords * sizeof(int));
        h->res_off_w = a16(h->res_off_ids + sizeof(int) * T * k);
        h->res_off_out = a16(h->res_off_w + sizeof(float) * T * k);
        h->res_bytes = h->res_off_out + sizeof(float) * T * D;
        ALLOC(h->res, h->res_bytes);
        h->err = reinterpret_cast<int*>(h->res);
        h->ids = reinterpret_cast<int*>(h->res + h->res_off_ids);
        h->wts = reinterpret_cast<float*>(h->res + h->res_off_w);
        h->out = reinterpret_cast<float*>(h->res + h->res_off_out);
    }
    {
        const size_t P = T * k;
        const int E = d.num_experts;
        const int gmax = glc::plan_max_groups((int)P, E);
        h->plan_gmax = gmax;
        ALLOC(h->plan.counts, sizeof(int) * E);
        ALLOC(h->plan.offsets, sizeof(int) * (E + 1));
        ALLOC(h->plan.perm, sizeof(int) * P);
        ALLOC(h->plan.inv, sizeof(int) * P);
        ALLOC(h->plan.grp_first, sizeof(int) * E);
        ALLOC(h->plan.grp_e, sizeof(int) * gmax);
        ALLOC(h->plan.grp_ntok, sizeof(int) * gmax);
        ALLOC(h->plan.grp_N, sizeof(int) * gmax);
        ALLOC(h->plan.grp_pos0, sizeof(int) * gmax);
        ALLOC(h->plan.grp_units, sizeof(int) * gmax);
        ALLOC(h->plan.meta, sizeof(int) * 2);
        // B tiles: sum_g N_g <= 2 * (P + 7 * groups) rows, 512 B per row per 256 of K
        const size_t units = 2 * (P + 7 * (size_t)gmax);
        h->btiles_bytes = units * 512 * (size_t)(std::max(D, F) / 256);
        if (Fs) {  // the shared expert's tiles (T tokens, K up to Fs) reuse the same buffer
            const int gsh = glc::plan_max_groups((int)T, 1);
            const size_t units_sh = 2 * (T + 7 * (size_t)gsh);
            h->btiles_bytes = std::max(h->btiles_bytes, units_sh * 512 * (size_t)(std::max(D, Fs) / 256));
            h->plan_sh_gmax = gsh;
            ALLOC(h->plan_sh.counts, sizeof(int));
            ALLOC(h->plan_sh.offsets, sizeof(int) * 2);
            ALLOC(h->plan_sh.perm, sizeof(int) * T);
            ALLOC(h->plan_sh.inv, sizeof(int) * T);
            ALLOC(h->plan_sh.grp_first, sizeof(int));
            ALLOC(h->plan_sh.grp_e, sizeof(int) * gsh);
            ALLOC(h->plan_sh.grp_ntok, sizeof(int) * gsh);
            ALLOC(h->plan_sh.grp_N, sizeof(int) * gsh);
            ALLOC(h->plan_sh.grp_pos0, sizeof(int) * gsh);
            ALLOC(h->plan_sh.grp_units, sizeof(int) * gsh);
            ALLOC(h->plan_sh.meta, sizeof(int) * 2);
            ALLOC(h->rscale_sh, sizeof(float) * T);
            ALLOC(h->ysh, sizeof(float) * kShSlicesMax * T * D);
        }
        ALLOC(h->btiles, h->btiles_bytes);
        ALLOC(h->rscale, sizeof(float) * P);
        ALLOC(h->ysort, sizeof(float) * P * D);
    }
#undef ALLOC
    cudaMemset(h->zeros_i, 0, sizeof(int) * T);
    if (glc::fill_launch(h->ones, T * k, 1.0f, h->stream) != cudaSuccess)
        return cleanup(fail(GLC_ERR_CUDA, "initialising the unit weights failed"));
    cudaMemset(h->err, 0, kErrWords * sizeof(int));
    if (cudaMallocHost(&h->h_x, sizeof(float) * T * D) != cudaSuccess ||
        cudaHostAlloc(&h->h_res, h->res_bytes, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostAlloc(&h->h_sig, 64, cudaHostAllocMapped) != cudaSuccess ||
        cudaMallocHost(&h->h_ids, sizeof(int) * T * k) != cudaSuccess ||
        cudaMallocHost(&h->h_w, sizeof(float) * T * k) != cudaSuccess)
        return cleanup(fail(GLC_ERR_OOM, "cudaMallocHost failed"));
    h->h_sig[0] = h->h_sig[1] = 0;
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_res_map), h->h_res, 0) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_sig_map), h->h_sig, 0) != cudaSuccess) {
        h->d_res_map = nullptr;  // no mapped host memory: the host-buffer forward copies instead
        h->d_sig_map = nullptr;
        cudaGetLastError();
    }
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(const_cast<float**>(&h->d_x_map)), h->h_x, 0) != cudaSuccess) {
        h->d_x_map = nullptr;  // the input then goes over with a host-to-device copy
        cudaGetLastError();
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return cleanup(fail(GLC_ERR_CUDA, "device sync failed"));
    *out = h;
    return GLC_OK;
}

int glc_moe_destroy(glc_moe* h) {
    if (!h) return GLC_OK;
    cudaSetDevice(h->d.device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    for (auto& L : h->layers) free_layer(L);
    for (auto& e : h->marks)
        if (e) cudaEventDestroy(e);
    if (h->graph_exec) cudaGraphExecDestroy(h->graph_exec);
    if (h->graph) cudaGraphDestroy(h->graph);
    for (auto& g : h->fwd_graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    cudaFree(h->x); cudaFree(h->xin); cudaFree(h->act); cudaFree(h->act_sh);
    cudaFree(h->gate_out); cudaFree(h->route_slots); cudaFree(h->zeros_i); cudaFree(h->res);
    cudaFree(h->ones); cudaFree(h->ep_keys);
    cudaFree(h->plan.counts); cudaFree(h->plan.offsets); cudaFree(h->plan.perm); cudaFree(h->plan.inv);
    cudaFree(h->plan.grp_first); cudaFree(h->plan.grp_e); cudaFree(h->plan.grp_ntok); cudaFree(h->plan.grp_N);
    cudaFree(h->plan.grp_pos0); cudaFree(h->plan.grp_units); cudaFree(h->plan.meta);
    cudaFree(h->btiles); cudaFree(h->rscale); cudaFree(h->ysort);
    cudaFree(h->plan_sh.counts); cudaFree(h->plan_sh.offsets); cudaFree(h->plan_sh.perm); cudaFree(h->plan_sh.inv);
    cudaFree(h->plan_sh.grp_first); cudaFree(h->plan_sh.grp_e); cudaFree(h->plan_sh.grp_ntok);
    cudaFree(h->plan_sh.grp_N); cudaFree(h->plan_sh.grp_pos0); cudaFree(h->plan_sh.grp_units);
    cudaFree(h->plan_sh.meta); cudaFree(h->rscale_sh); cudaFree(h->ysh);
    cudaFreeHost(h->h_x); cudaFreeHost(h->h_res); cudaFreeHost(h->h_sig); cudaFreeHost(h->h_ids); cudaFreeHost(h->h_w);
    cudaFree(h->pool_gate); cudaFree(h->pool_up); cudaFree(h->pool_down); cudaFree(h->d_slot_ids);
    cudaFreeHost(h->h_slot_ids);
    if (h->stream) cudaStreamDestroy(h->stream);
    h->disposed = 1;
    delete h;
    return GLC_OK;
}

int glc_moe_load_layer(glc_moe* h, int32_t layer, const glc_layer_weights* w) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!w || !w->gate_exps || !w->up_exps || !w->down_exps) return fail(GLC_ERR_INVALID_ARG, "null weight pointer");
    if (layer < 0 || layer >= h->d.num_layers) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    LayerDev& L = h->layers[layer];
    rc = alloc_layer(h, L);
    if (rc) return rc;
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, E = h->d.num_experts, El = local_experts(h);
    const size_t gsz = (size_t)El * F * rowbytes(D), dsz = (size_t)El * D * rowbytes(F);
    CUDA_TRY(cudaMemcpy(L.gate, w->gate_exps, gsz, cudaMemcpyDefault));  // HBM, or pinned host (residency mode)
    CUDA_TRY(cudaMemcpy(L.up, w->up_exps, gsz, cudaMemcpyDefault));
    CUDA_TRY(cudaMemcpy(L.down, w->down_exps, dsz, cudaMemcpyDefault));
    if (w->router) CUDA_TRY(cudaMemcpy(L.router, w->router, sizeof(float) * (size_t)D * E, cudaMemcpyHostToDevice));
    else CUDA_TRY(cudaMemset(L.router, 0, sizeof(float) * (size_t)D * E));
    if (h->d.shared_ffn_dim > 0) {
        const int Fs = h->d.shared_ffn_dim;
        if (!w->shared_gate || !w->shared_up || !w->shared_down || !w->shared_gate_vec)
            return fail(GLC_ERR_INVALID_ARG, "shared expert weights missing");
        CUDA_TRY(cudaMemcpy(L.sh_gate, w->shared_gate, (size_t)Fs * rowbytes(D), cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy(L.sh_up, w->shared_up, (size_t)Fs * rowbytes(D), cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy(L.sh_down, w->shared_down, (size_t)D * rowbytes(Fs), cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy(L.sh_gate_vec, w->shared_gate_vec, sizeof(float) * D, cudaMemcpyHostToDevice));
    }
    L.loaded = true;
    rc = make_layer_tmaps(h, L);
    return rc ? rc : warm_slots(h, layer);
}

int glc_moe_synth_layer(glc_moe* h, int32_t layer, uint64_t seed) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (layer < 0 || layer >= h->d.num_layers) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    LayerDev& L = h->layers[layer];
    rc = alloc_layer(h, L);
    if (rc) return rc;
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim, E = h->d.num_experts, El = local_experts(h);
    const int nt = host_threads();
    // Stage one matrix at a time through a host buffer.
    const size_t gsl = (size_t)F * rowbytes(D), dsl = (size_t)D * rowbytes(F);
    std::vector<uint8_t> buf(std::max(gsl, dsl));
    for (int el = 0; el < El; ++el) {
        const int e = h->d.expert_begin + el;
        glc::synth_q4k(seed, glc::expert_tag(e, 0), 0.01f, buf.data(), gsl / 144, nt);
        CUDA_TRY(cudaMemcpy(L.gate + el * gsl, buf.data(), gsl, cudaMemcpyDefault));
        glc::synth_q4k(seed, glc::expert_tag(e, 1), 0.01f, buf.data(), gsl / 144, nt);
        CUDA_TRY(cudaMemcpy(L.up + el * gsl, buf.data(), gsl, cudaMemcpyDefault));
        glc::synth_q4k(seed, glc::expert_tag(e, 2), 0.01f, buf.data(), dsl / 144, nt);
        CUDA_TRY(cudaMemcpy(L.down + el * dsl, buf.data(), dsl, cudaMemcpyDefault));
    }
    std::vector<float> r((size_t)D * E);
    glc::synth_normal(seed, glc::kTagRouter, 0.02f, r.data(), r.size(), nt);
    CUDA_TRY(cudaMemcpy(L.router, r.data(), sizeof(float) * r.size(), cudaMemcpyHostToDevice));
    if (h->d.shared_ffn_dim > 0) {
        const int Fs = h->d.shared_ffn_dim;
        const int se = glc::kSharedExpertIndex;
        const size_t sg = (size_t)Fs * rowbytes(D), sd = (size_t)D * rowbytes(Fs);
        std::vector<uint8_t> sb(std::max(sg, sd));
        glc::synth_q4k(seed, glc::expert_tag(se, 0), 0.01f, sb.data(), sg / 144, nt);
        CUDA_TRY(cudaMemcpy(L.sh_gate, sb.data(), sg, cudaMemcpyHostToDevice));
        glc::synth_q4k(seed, glc::expert_tag(se, 1), 0.01f, sb.data(), sg / 144, nt);
        CUDA_TRY(cudaMemcpy(L.sh_up, sb.data(), sg, cudaMemcpyHostToDevice));
        glc::synth_q4k(seed, glc::expert_tag(se, 2), 0.01f, sb.data(), sd / 144, nt);
        CUDA_TRY(cudaMemcpy(L.sh_down, sb.data(), sd, cudaMemcpyHostToDevice));
        std::vector<float> gv(D);
        glc::synth_normal(seed, glc::kTagSharedGate, 0.02f, gv.data(), D, 1);
        CUDA_TRY(cudaMemcpy(L.sh_gate_vec, gv.data(), sizeof(float) * D, cudaMemcpyHostToDevice));
    }
    L.loaded = true;
    rc = make_layer_tmaps(h, L);
    return rc ? rc : warm_slots(h, layer);
}

int glc_moe_set_profiling(glc_moe* h, int32_t enable) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (enable && !h->marks[0])
        for (auto& e : h->marks) CUDA_TRY(cudaEventCreate(&e));
    h->profiling = enable ? 1 : 0;
    if (!h->mark_lock) h->n_marks = 0;
    return GLC_OK;
}

int glc_moe_kernel_times(glc_moe* h, float* ms, int32_t max_kernels, int32_t* n_kernels) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!ms || !n_kernels) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const int n = h->n_marks > 1 ? h->n_marks - 1 : 0;
    *n_kernels = n;
    for (int i = 0; i < n && i < max_kernels; ++i) {
        CUDA_TRY(cudaEventSynchronize(h->marks[i + 1]));
        CUDA_TRY(cudaEventElapsedTime(&ms[i], h->marks[i], h->marks[i + 1]));
    }
    return GLC_OK;
}

int glc_moe_debug_stall(glc_moe* h, int32_t cta, int64_t wait_limit_ns) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (cta < 0 || cta >= h->num_sms) return fail(GLC_ERR_INVALID_ARG, "CTA %d outside the grid of %d", cta, h->num_sms);
    if (wait_limit_ns <= 0) return fail(GLC_ERR_INVALID_ARG, "the wait limit must be positive");
    h->debug_stall_cta = cta + 1;
    h->debug_wait_limit_ns = wait_limit_ns;
    return GLC_OK;
}

int glc_moe_poll_error(glc_moe* h) {
    int rc = check_handle(h);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    return check_device_error(h);
}

int glc_moe_layer_device_ptrs(glc_moe* h, int32_t layer, const void** gate, const void** up,
                              const void** down, const float** router) {
    int rc = check_handle(h);
    if (rc) return rc;
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    if (L->host_experts) return fail(GLC_ERR_STATE, "the routed experts are host-resident (expert slots)");
    if (gate) *gate = L->gate;
    if (up) *up = L->up;
    if (down) *down = L->down;
    if (router) *router = L->router;
    return GLC_OK;
}

int glc_expert_forward_dev(glc_moe* h, int32_t layer, int32_t expert, const float* x, float* y, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!x || !y) return fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    // ExpertId is clamped to [0, E) (CpuWarmExpertPoolWorker.cs:263).
    const int El = local_experts(h);
    int e = expert - h->d.expert_begin;
    e = e < 0 ? 0 : (e >= El ? El - 1 : e);
    h->h_ids[0] = e;
    h->h_w[0] = 1.0f;
    CUDA_TRY(cudaMemcpyAsync(h->ids, h->h_ids, sizeof(int), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(h->wts, h->h_w, sizeof(float), cudaMemcpyHostToDevice, st));
    const int* run_ids = nullptr;
    LayerDev V;
    LayerDev* LR = nullptr;
    rc = expert_operands(h, L, h->ids, 1, st, &V, &LR, &run_ids);
    if (rc) return rc;
    return run_experts(h, LR, x, 1, 1, run_ids, h->wts, nullptr, y, st);
}

int glc_expert_forward(glc_moe* h, int32_t layer, int32_t expert, const float* x, float* y) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!x || !y) return fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    const int D = h->d.hidden_dim;
    CUDA_TRY(cudaMemcpyAsync(h->x, x, sizeof(float) * D, cudaMemcpyHostToDevice, h->stream));
    rc = glc_expert_forward_dev(h, layer, expert, h->x, h->out, h->stream);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(y, h->out, sizeof(float) * D, cudaMemcpyDeviceToHost, h->stream));
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    return check_device_error(h);
}

int glc_routed_topk(glc_moe* h, int32_t layer, const float* x, const int32_t* ids, const float* w,
                    int32_t k, float* out) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!x || !out) return fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    const int D = h->d.hidden_dim;
    if (k <= 0 || !ids || !w) {  // empty selection -> zeros (GpuFirstExpertStageWorker.cs:431-437)
        std::memset(out, 0, sizeof(float) * D);
        return GLC_OK;
    }
    if (k > h->d.top_k * h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "k=%d exceeds workspace", k);
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    const int El = local_experts(h);
    for (int j = 0; j < k; ++j) {
        int e = ids[j] - h->d.expert_begin;
        h->h_ids[j] = e < 0 ? 0 : (e >= El ? El - 1 : e);
        h->h_w[j] = w[j];
    }
    cudaStream_t st = h->stream;
    CUDA_TRY(cudaMemcpyAsync(h->x, x, sizeof(float) * D, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(h->ids, h->h_ids, sizeof(int) * k, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(h->wts, h->h_w, sizeof(float) * k, cudaMemcpyHostToDevice, st));
    if (k > h->d.top_k * h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "k too large");
    const int* run_ids = nullptr;
    LayerDev V;
    LayerDev* LR = nullptr;
    rc = expert_operands(h, L, h->ids, k, st, &V, &LR, &run_ids);
    if (rc) return rc;
    rc = run_experts(h, LR, h->x, 1, k, run_ids, h->wts, nullptr, h->out, st);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(out, h->out, sizeof(float) * D, cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    return check_device_error(h);
}

namespace {

// The whole-layer fused decode launch serves this call (T tokens, flags).
// The host-buffer forward's input: the token in the pinned staging buffer,
// read through its mapped device address, into the device input -- the
// kernel in front of the fused decode launch, which is programmatically
// serialised behind it (stages its router weights meanwhile and waits for
// this kernel before reading the input).
// (256 threads: small enough that the fused launch's CTA fits beside it on its SM.)
__global__ void __launch_bounds__(256) copy_in_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                                      int n4) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the fused launch may start at once
    for (int i = threadIdx.x; i < n4; i += 256) dst[i] = src[i];
}

// The input of a host-buffer call onto the device: the copy kernel from the
// mapped staging buffer, or a host-to-device copy.
cudaError_t stage_input(glc_moe* h, size_t xbytes, cudaStream_t st) {
    if (h->d_x_map) {
        copy_in_kernel<<<1, 256, 0, st>>>(reinterpret_cast<const float4*>(h->d_x_map), reinterpret_cast<float4*>(h->x),
                                           (int)(xbytes / 16));
        return cudaGetLastError();
    }
    return cudaMemcpyAsync(h->x, h->h_x, xbytes, cudaMemcpyHostToDevice, st);
}

bool fused_applies(const glc_moe* h, int T, uint32_t flags) {
    const bool grouped = (flags & GLC_FWD_BATCHED) ? true : (flags & GLC_FWD_DECODE) ? false : (T > 1);
    // residency mode routes first and pages the selected experts in before they run
    return !grouped && !(flags & GLC_FWD_UNFUSED) && h->slots == 0;
}

// Fused-kernel parameters of a layer; the caller sets x, resid and out.
glc::FusedDecodeParams fused_params(glc_moe* h, const LayerDev* L, int T, uint32_t flags) {
    const int D = h->d.hidden_dim, F = h->d.expert_ffn_dim;
    glc::FusedDecodeParams fp{};
    fp.Wr = L->router;
    fp.gate = L->gate;
    fp.up = L->up;
    fp.down = L->down;
    fp.gu_expert_bytes = (long long)F * rowbytes(D);
    fp.dn_expert_bytes = (long long)D * rowbytes(F);
    fp.act = h->act;
    fp.xin = nullptr;
    fp.ids = h->ids;
    fp.w = h->wts;
    fp.bar = reinterpret_cast<unsigned long long*>(h->err + 2);
    // the wide kernel (shared expert, or a router too large to stage)
    fp.route_bar = reinterpret_cast<unsigned long long*>(h->err + 6);
    fp.route_slots = h->route_slots;
    fp.Fs = h->d.shared_ffn_dim > 0 ? h->d.shared_ffn_dim : 0;
    fp.sh_gate = L->sh_gate;
    fp.sh_up = L->sh_up;
    fp.sh_down = L->sh_down;
    fp.sh_gate_vec = L->sh_gate_vec;
    fp.act_sh = h->act_sh;
    fp.err = h->err;
    fp.T = T;
    fp.D = D;
    fp.F = F;
    fp.E = h->d.num_experts;
    fp.k = h->d.top_k;
    fp.renorm = h->d.renormalize;
    fp.rmsnorm = (flags & GLC_FWD_RMSNORM) ? 1 : 0;
    fp.stall_cta = h->debug_stall_cta;
    fp.wait_limit_ns = h->debug_wait_limit_ns;
    h->debug_stall_cta = 0;  // one launch only
    h->debug_wait_limit_ns = 0;
    return fp;
}

}  // namespace

int glc_moe_forward_dev(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags, float* out,
                        int32_t* ids_out, float* w_out, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (T <= 0) return GLC_OK;
    if (!x || !out) return fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    if (T > h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, h->d.max_tokens);
    if (local_experts(h) != h->d.num_experts)
        return fail(GLC_ERR_STATE, "full-layer forward on an expert shard needs the expert-parallel path");
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    const int D = h->d.hidden_dim, E = h->d.num_experts, k = h->d.top_k;
    // T == 1 (decode): dequant-fused GEMVs; T > 1: grouped tensor-core GEMMs.
    const bool grouped = (flags & GLC_FWD_BATCHED) ? true : (flags & GLC_FWD_DECODE) ? false : (T > 1);
    const float* resid = (flags & GLC_FWD_RESIDUAL) ? x : nullptr;
    if (fused_applies(h, T, flags)) {
        // Whole layer in one persistent launch when it fits (few tokens, router
        // and input small enough to stage in shared memory).
        glc::FusedDecodeParams fp = fused_params(h, L, T, flags);
        fp.x = x;
        fp.resid = resid;
        fp.out = out;
        if (!h->mark_lock) h->n_marks = 0;
        mark(h, st);
        const cudaError_t e = glc::fused_decode_launch(fp, h->num_sms, st);
        if (e == cudaSuccess) {
            mark(h, st);
            if (ids_out) CUDA_TRY(cudaMemcpyAsync(ids_out, h->ids, sizeof(int) * T * k, cudaMemcpyDeviceToDevice, st));
            if (w_out) CUDA_TRY(cudaMemcpyAsync(w_out, h->wts, sizeof(float) * T * k, cudaMemcpyDeviceToDevice, st));
            return GLC_OK;
        }
        if (e != cudaErrorNotSupported) return fail(GLC_ERR_CUDA, "fused decode launch: %s", cudaGetErrorString(e));
    }
    glc::RouterParams rp{};
    rp.x = x;
    rp.Wr = L->router;
    rp.T = T;
    rp.D = D;
    rp.E = E;
    rp.k = k;
    rp.renorm = h->d.renormalize;
    rp.rmsnorm = (flags & GLC_FWD_RMSNORM) ? 1 : 0;
    rp.xin = h->xin;
    rp.ids = h->ids;
    rp.w = h->wts;
    rp.gate_vec = h->d.shared_ffn_dim > 0 ? L->sh_gate_vec : nullptr;
    rp.gate_out = h->gate_out;
    if (!h->mark_lock) h->n_marks = 0;
    mark(h, st);
    CUDA_TRY(glc::router_launch(rp, st));
    mark(h, st);
    // residency mode: the selected experts into HBM slots, the kernels on the pool
    const int* run_ids = nullptr;
    LayerDev V;
    LayerDev* LR = nullptr;
    rc = expert_operands(h, L, h->ids, T * k, st, &V, &LR, &run_ids);
    if (rc) return rc;
    rc = grouped ? run_experts_grouped(h, LR, h->xin, T, k, run_ids, h->wts, resid, out, st, true)
                 : run_experts(h, LR, h->xin, T, k, run_ids, h->wts, resid, out, st);
    if (rc) return rc;
    if (h->d.shared_ffn_dim > 0 && !grouped) {  // the grouped path ran it already
        rc = run_shared_expert(h, LR, h->xin, T, out, st);
        if (rc) return rc;
    }
    if (ids_out) CUDA_TRY(cudaMemcpyAsync(ids_out, h->ids, sizeof(int) * T * k, cudaMemcpyDeviceToDevice, st));
    if (w_out) CUDA_TRY(cudaMemcpyAsync(w_out, h->wts, sizeof(float) * T * k, cudaMemcpyDeviceToDevice, st));
    return GLC_OK;
}

int glc_moe_route_dev(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags, float* xin_out,
                      int32_t* ids_out, float* w_out, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (T <= 0) return GLC_OK;
    if (!x || !xin_out || !ids_out || !w_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (T > h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, h->d.max_tokens);
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    glc::RouterParams rp{};
    rp.x = x;
    rp.Wr = L->router;
    rp.T = T;
    rp.D = h->d.hidden_dim;
    rp.E = h->d.num_experts;
    rp.k = h->d.top_k;
    rp.renorm = h->d.renormalize;
    rp.rmsnorm = (flags & GLC_FWD_RMSNORM) ? 1 : 0;
    rp.xin = xin_out;
    rp.ids = ids_out;
    rp.w = w_out;
    rp.gate_vec = h->d.shared_ffn_dim > 0 ? L->sh_gate_vec : nullptr;
    rp.gate_out = h->gate_out;
    CUDA_TRY(glc::router_launch(rp, stream ? (cudaStream_t)stream : h->stream));
    return GLC_OK;
}

int glc_moe_ep_dispatch_dev(glc_moe* h, const float* xin, const int32_t* ids, int32_t T, int32_t world,
                            int32_t* rank_counts, int32_t* rank_offsets, int32_t* perm, int32_t* inv,
                            float* send_rows, int32_t* send_ids, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (T <= 0) return GLC_OK;
    if (!xin || !ids || !rank_counts || !rank_offsets || !perm || !inv || !send_rows || !send_ids)
        return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (T > h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, h->d.max_tokens);
    if (world < 1 || world > 64 || h->d.num_experts % world)
        return fail(GLC_ERR_INVALID_ARG, "world=%d must divide the %d experts (and be <= 64)", world, h->d.num_experts);
    glc::DispatchPlan pl = h->plan;  // group-table scratch of the handle, outputs in the caller's buffers
    pl.counts = rank_counts;
    pl.offsets = rank_offsets;
    pl.perm = perm;
    pl.inv = inv;
    CUDA_TRY(glc::ep_dispatch_launch(xin, ids, T, h->d.hidden_dim, h->d.top_k, h->d.num_experts, world, h->ep_keys,
                                     pl, send_rows, send_ids, stream ? (cudaStream_t)stream : h->stream));
    return GLC_OK;
}

int glc_moe_experts_dev(glc_moe* h, int32_t layer, const float* rows, const int32_t* expert_ids, int32_t R,
                        uint32_t flags, float* y_out, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (R <= 0) return GLC_OK;
    if (!rows || !expert_ids || !y_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const int cap = h->d.max_tokens * h->d.top_k;
    if (R > cap) return fail(GLC_ERR_INVALID_ARG, "R=%d rows exceed the handle's %d pair slots", R, cap);
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    CUDA_TRY(glc::localize_ids_launch(expert_ids, R, h->d.expert_begin, local_experts(h), h->ids, st));
    // each row is its own "token" with one slot and unit weight: y = expert(row) exactly
    const bool grouped = (flags & GLC_FWD_BATCHED) ? true : (flags & GLC_FWD_DECODE) ? false : (R > 1);
    if (!h->mark_lock) h->n_marks = 0;
    mark(h, st);
    const int* run_ids = nullptr;
    LayerDev V;
    LayerDev* LR = nullptr;
    rc = expert_operands(h, L, h->ids, R, st, &V, &LR, &run_ids);
    if (rc) return rc;
    return grouped ? run_experts_grouped(h, LR, rows, R, 1, run_ids, h->ones, nullptr, y_out, st, false)
                   : run_experts(h, LR, rows, R, 1, run_ids, h->ones, nullptr, y_out, st);
}

int glc_moe_combine_dev(glc_moe* h, int32_t layer, const float* y_back, const int32_t* inv, const float* w,
                        int32_t T, const float* resid, const float* xin, float* out, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (T <= 0) return GLC_OK;
    if (!y_back || !inv || !w || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (T > h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, h->d.max_tokens);
    LayerDev* L = layer_of(h, layer);
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    if (h->d.shared_ffn_dim > 0) {
        if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
        if (!xin) return fail(GLC_ERR_INVALID_ARG, "the shared expert needs xin");
    }
    if (h->d.shared_ffn_dim > 0 && T > 1) {
        // batched: the shared expert on the grouped path, added by the combine
        int slices = 1;
        rc = run_shared_grouped(h, L, xin, T, &slices, st);
        if (rc) return rc;
        CUDA_TRY(glc::combine_launch(y_back, T, h->d.hidden_dim, h->d.top_k, inv, w, resid, out, st, h->ysh, slices,
                                     (long long)T * h->d.hidden_dim, h->gate_out));
        return GLC_OK;
    }
    CUDA_TRY(glc::combine_launch(y_back, T, h->d.hidden_dim, h->d.top_k, inv, w, resid, out, st));
    if (h->d.shared_ffn_dim > 0) {
        rc = run_shared_expert(h, L, xin, T, out, st);
        if (rc) return rc;
    }
    return GLC_OK;
}

int glc_moe_ep_forward(glc_moe* h, glc_comm* c, int32_t layer, const float* x, int32_t T, uint32_t flags,
                       float* out, int32_t* ids_out, float* w_out, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!c) return fail(GLC_ERR_INVALID_ARG, "null communicator");
    if (h->slots) return fail(GLC_ERR_UNSUPPORTED, "expert parallelism on a handle with expert slots");
    const int world = glc::comm_world(c), rank = glc::comm_rank(c);
    const int E = h->d.num_experts, El = local_experts(h);
    if (E % world || El * world != E || h->d.expert_begin != rank * El)
        return fail(GLC_ERR_STATE, "the handle must hold expert shard %d of %d (experts [%d, %d))", rank, world,
                    rank * (E / world), (rank + 1) * (E / world));
    LayerDev* L = layer_of(h, layer);
    if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    const int D = h->d.hidden_dim, k = h->d.top_k;
    // Every rank's batch holds at most Tc = max_tokens / world tokens (the
    // handle is sized world x the largest per-rank batch), so the most pairs
    // one rank can send one peer, cap, is the same on every rank: the
    // exchange is an all-to-all of equal fixed-size blocks whose counts
    // travel inside them and are used only on the device.  No host read.
    const int Tc = h->d.max_tokens / world;
    if (Tc < 1 || (D & 3)) return fail(GLC_ERR_STATE, "max_tokens=%d holds no token per rank of %d", h->d.max_tokens, world);
    const int cap = Tc * k;
    // A call that is invalid on this rank still takes part in both exchanges
    // with no pairs, so its peers do not wait on it; it reports afterwards.
    int bad = GLC_OK;
    if (T < 0 || T > Tc)
        bad = fail(GLC_ERR_INVALID_ARG,
                   "T=%d outside [0, %d]: an expert-parallel handle's max_tokens is world x the largest per-rank batch",
                   T, Tc);
    else if (T > 0 && (!x || !out))
        bad = fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    const int Tl = bad ? 0 : T, P = Tl * k;
    const size_t row = sizeof(float) * (size_t)D;
    const size_t bb = glc::ep_block_bytes(cap, D);
    auto scratch = [&](int slot, size_t bytes) { return glc::comm_scratch(c, slot, bytes); };
    // communicator scratch slots 2.. (0 and 1 hold stage-boundary payloads);
    // their sizes depend only on the handle and the world, so they are
    // allocated by the first call and reused
    float* xin = static_cast<float*>(scratch(2, (size_t)Tc * row));
    int32_t* ids = static_cast<int32_t*>(scratch(3, sizeof(int32_t) * cap));
    float* w = static_cast<float*>(scratch(4, sizeof(float) * cap));
    int32_t* ints = static_cast<int32_t*>(scratch(5, sizeof(int32_t) * (3 * (size_t)cap + 3 * (size_t)world + 2)));
    float* rows = static_cast<float*>(scratch(8, (size_t)world * cap * row));
    float* y = static_cast<float*>(scratch(9, (size_t)world * cap * row));
    float* y_back = static_cast<float*>(scratch(12, (size_t)cap * row));
    if (!xin || !ids || !w || !ints || !rows || !y || !y_back) return fail(GLC_ERR_OOM, "expert-parallel scratch");
    int32_t* counts = ints;                 // [world] pairs to each rank
    int32_t* offsets = counts + world;      // [world + 1]
    int32_t* perm = offsets + world + 1;    // [cap]
    int32_t* inv = perm + cap;              // [cap]
    int32_t* src_off = inv + cap;           // [world + 1] received rows per source, prefix
    glc::DispatchPlan pl = h->plan;  // group-table scratch of the handle, outputs here
    pl.counts = counts;
    pl.offsets = offsets;
    pl.perm = perm;
    pl.inv = inv;
    // The exchange: over the peer window when every rank has mapped every
    // other rank's (the blocks written straight into the destination's
    // memory, an epoch flag per source, only routed rows crossing NVLink),
    // else the same blocks through one grouped NCCL send / receive each way.
    uint8_t* win = nullptr;
    void* const* peers = nullptr;
    const int wr = glc::comm_window(c, glc::ep_window_bytes(world, cap, D), st, &win, &peers);
    if (wr != GLC_OK && wr != GLC_ERR_UNSUPPORTED) return wr;
    const bool peer = wr == GLC_OK;
    uint8_t *send = nullptr, *recv = nullptr;
    float *y_send = nullptr, *y_recv = nullptr;
    if (!peer) {
        send = static_cast<uint8_t*>(scratch(6, (size_t)world * bb));
        recv = static_cast<uint8_t*>(scratch(7, (size_t)world * bb));
        y_send = static_cast<float*>(scratch(10, (size_t)world * cap * row));
        y_recv = static_cast<float*>(scratch(11, (size_t)world * cap * row));
        if (!send || !recv || !y_send || !y_recv) return fail(GLC_ERR_OOM, "expert-parallel exchange buffers");
    }
    const unsigned long long epoch = peer ? glc::comm_window_next_epoch(c) : 0;
    const int par = (int)(epoch & 1);
    h->n_marks = 0;
    mark_phase(h, st);
    struct Lock {
        glc_moe* h;
        ~Lock() { h->mark_lock = 0; }
    } lock{h};
    h->mark_lock = 1;  // the inner steps record no marks: the phases below do
    if (P > 0) {
        rc = glc_moe_route_dev(h, layer, x, Tl, flags, xin, ids, w, st);
        if (rc) return rc;
    }
    mark_phase(h, st);  // route
    if (peer)  // pack into every destination's window, then its dispatch flag
        CUDA_TRY(glc::ep_pack_peer_launch(xin, ids, Tl, D, k, E, world, rank, cap, h->ep_keys, pl, peers, par, epoch,
                                          win, st));
    else
        CUDA_TRY(glc::ep_pack_launch(xin, ids, Tl, D, k, E, world, cap, h->ep_keys, pl, send, st));
    mark_phase(h, st);  // dispatch into per-rank blocks
    std::vector<size_t> off(world), cnt(world, bb), off_y(world), cnt_y(world, (size_t)cap * row);
    for (int p = 0; p < world; ++p) {
        off[p] = (size_t)p * bb;
        off_y[p] = (size_t)p * cap * row;
    }
    if (peer) {
        CUDA_TRY(glc::ep_wait_launch(win, world, 0, epoch, h->err, st));
        recv = win + glc::ep_win_disp_off(par, world, cap, D);
    } else {
        rc = glc::comm_alltoallv(c, send, off.data(), cnt.data(), recv, off.data(), cnt.data(), st);
        if (rc) return rc;
    }
    mark_phase(h, st);  // exchange out
    CUDA_TRY(glc::ep_unpack_launch(recv, world, cap, D, h->d.expert_begin, El, rows, h->ids, src_off, st));
    // this rank's experts on every row received, the row count on the device
    rc = run_experts_grouped(h, L, rows, world * cap, 1, h->ids, h->ones, nullptr, y, st, false, src_off + world);
    if (rc) return rc;
    if (peer)  // each output row into its home rank's window, then the return flags
        CUDA_TRY(glc::ep_repack_peer_launch(y, src_off, world, rank, cap, D, peers, par, epoch, win, st));
    else
        CUDA_TRY(glc::ep_repack_launch(y, src_off, world, cap, D, y_send, st));
    mark_phase(h, st);  // experts
    if (peer) {
        CUDA_TRY(glc::ep_wait_launch(win, world, 1, epoch, h->err, st));
        y_recv = reinterpret_cast<float*>(win + glc::ep_win_ret_off(par, world, cap, D));
    } else {
        rc = glc::comm_alltoallv(c, y_send, off_y.data(), cnt_y.data(), y_recv, off_y.data(), cnt_y.data(), st);
        if (rc) return rc;
    }
    mark_phase(h, st);  // exchange back
    if (P > 0) {
        CUDA_TRY(glc::ep_unblock_launch(y_recv, P, cap, D, h->ep_keys, pl, y_back, st));
        rc = glc_moe_combine_dev(h, layer, y_back, inv, w, Tl, (flags & GLC_FWD_RESIDUAL) ? x : nullptr, xin, out, st);
        if (rc) return rc;
        if (ids_out) CUDA_TRY(cudaMemcpyAsync(ids_out, ids, sizeof(int32_t) * P, cudaMemcpyDeviceToDevice, st));
        if (w_out) CUDA_TRY(cudaMemcpyAsync(w_out, w, sizeof(float) * P, cudaMemcpyDeviceToDevice, st));
    }
    mark_phase(h, st);  // combine
    return bad;
}

int glc_moe_forward(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags, float* out,
                    int32_t* ids_out, float* w_out) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (T <= 0) return GLC_OK;
    if (!x || !out) return fail(GLC_ERR_INVALID_ARG, "null activation pointer");
    if (T > h->d.max_tokens) return fail(GLC_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, h->d.max_tokens);
    const int D = h->d.hidden_dim, k = h->d.top_k;
    cudaStream_t st = h->stream;
    if (h->d_res_map && !h->profiling && fused_applies(h, T, flags)) {
        LayerDev* L = layer_of(h, layer);
        if (!L->loaded) return fail(GLC_ERR_STATE, "layer %d has no weights", layer);
        // The kernel writes its outputs into mapped host memory and its last
        // CTA writes the launch's epoch to a mapped word: no copy back and no
        // stream synchronisation.  The input goes through the pinned staging
        // buffer; after the first call of a (layer, T, flags) shape the copy
        // and the launch are replayed from a captured graph, whose one
        // launch call costs the host far less than a copy plus a cooperative
        // launch (both on the critical path of this synchronous call).
        const size_t xbytes = sizeof(float) * (size_t)T * D;
        std::memcpy(h->h_x, x, xbytes);
        const bool debug = h->debug_stall_cta != 0 || h->debug_wait_limit_ns != 0;
        auto host_params = [&]() {
            glc::FusedDecodeParams fp = fused_params(h, L, T, flags);
            fp.x = h->x;
            fp.resid = (flags & GLC_FWD_RESIDUAL) ? h->x : nullptr;
            fp.out = reinterpret_cast<float*>(h->d_res_map + h->res_off_out);
            fp.ids = reinterpret_cast<int*>(h->d_res_map + h->res_off_ids);
            fp.w = reinterpret_cast<float*>(h->d_res_map + h->res_off_w);
            fp.done_ctr = reinterpret_cast<unsigned long long*>(h->err + 4);
            fp.host_done = h->d_sig_map;
            fp.host_err = reinterpret_cast<int*>(h->d_sig_map + 1);
            fp.pdl = h->d_x_map ? 1 : 0;  // behind the copy kernel
            return fp;
        };
        cudaGraphExec_t cached = nullptr;
        if (!debug)
            for (const auto& g : h->fwd_graphs)
                if (g.layer == layer && g.T == T && g.flags == flags) cached = g.exec;
        const bool replay = cached != nullptr;
        if (replay) {
            CUDA_TRY(cudaGraphLaunch(cached, st));
        } else {
            CUDA_TRY(stage_input(h, xbytes, st));
            const cudaError_t e = glc::fused_decode_launch(host_params(), h->num_sms, st);
            if (e == cudaErrorNotSupported) goto separate_launches;
            if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "fused decode launch: %s", cudaGetErrorString(e));
        }
        {
            const unsigned long long epoch = ++h->host_epoch;
            const volatile unsigned long long* done = h->h_sig;
            const auto t0 = std::chrono::steady_clock::now();
            bool finished = true;
            for (uint32_t n = 0; *done != epoch; ++n)
                if ((n & 1023u) == 1023u && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(30)) {
                    finished = false;
                    break;
                }
            std::atomic_thread_fence(std::memory_order_acquire);
            if (!finished || reinterpret_cast<const volatile int*>(h->h_sig + 1)[0] != 0) {
                CUDA_TRY(cudaStreamSynchronize(st));
                rc = check_device_error(h);
                return rc ? rc : fail(GLC_ERR_TIMEOUT, "fused decode launch did not report its completion");
            }
        }
        std::memcpy(out, h->h_res + h->res_off_out, sizeof(float) * (size_t)T * D);
        if (ids_out) std::memcpy(ids_out, h->h_res + h->res_off_ids, sizeof(int) * (size_t)T * k);
        if (w_out) std::memcpy(w_out, h->h_res + h->res_off_w, sizeof(float) * (size_t)T * k);
        if (!replay && !debug) {
            // capture this shape for the next calls (the launch above did the
            // first-use set-up, which is not capturable); on any failure the
            // calls of this shape simply stay eager
            cudaGraph_t g = nullptr;
            cudaGraphExec_t exec = nullptr;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                const glc::FusedDecodeParams fp = host_params();
                const bool ok = stage_input(h, xbytes, st) == cudaSuccess &&
                                glc::fused_decode_launch(fp, h->num_sms, st) == cudaSuccess;
                if (cudaStreamEndCapture(st, &g) != cudaSuccess || !ok || cudaGraphInstantiate(&exec, g, 0) != cudaSuccess)
                    exec = nullptr;
                if (g) cudaGraphDestroy(g);
            }
            cudaGetLastError();
            if (exec) {
                constexpr size_t kMaxFwdGraphs = 64;
                if (h->fwd_graphs.size() < kMaxFwdGraphs) {
                    h->fwd_graphs.push_back({exec, layer, T, flags});
                } else {
                    auto& slot = h->fwd_graphs[h->fwd_next++ % kMaxFwdGraphs];
                    cudaGraphExecDestroy(slot.exec);
                    slot = {exec, layer, T, flags};
                }
            }
        }
        return GLC_OK;
    }
separate_launches:
    CUDA_TRY(cudaMemcpyAsync(h->x, x, sizeof(float) * (size_t)T * D, cudaMemcpyHostToDevice, st));
    rc = glc_moe_forward_dev(h, layer, h->x, T, flags, h->out, nullptr, nullptr, st);
    if (rc) return rc;
    // One copy back: the error word, expert ids, combine weights and output
    // are adjacent in the result block (no separate round trip for the error).
    CUDA_TRY(cudaMemcpyAsync(h->h_res, h->res, h->res_off_out + sizeof(float) * (size_t)T * D,
                             cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (reinterpret_cast<const int*>(h->h_res)[0] != 0) return check_device_error(h);
    std::memcpy(out, h->h_res + h->res_off_out, sizeof(float) * (size_t)T * D);
    if (ids_out) std::memcpy(ids_out, h->h_res + h->res_off_ids, sizeof(int) * (size_t)T * k);
    if (w_out) std::memcpy(w_out, h->h_res + h->res_off_w, sizeof(float) * (size_t)T * k);
    return GLC_OK;
}

int glc_moe_graph_build(glc_moe* h, int32_t layer, const float* x, int32_t T, uint32_t flags, float* out) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!x || !out || T <= 0) return fail(GLC_ERR_INVALID_ARG, "bad graph arguments");
    if (h->slots) return fail(GLC_ERR_UNSUPPORTED, "expert slots page in on the host: not capturable");
    // One eager run first: first-use set-up (shared-memory opt-in) is not capturable.
    rc = glc_moe_forward_dev(h, layer, x, T, flags, out, nullptr, nullptr, h->stream);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    if (h->graph_exec) { cudaGraphExecDestroy(h->graph_exec); h->graph_exec = nullptr; }
    if (h->graph) { cudaGraphDestroy(h->graph); h->graph = nullptr; }
    const int prof = h->profiling;
    h->profiling = 0;
    CUDA_TRY(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    rc = glc_moe_forward_dev(h, layer, x, T, flags, out, nullptr, nullptr, h->stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(h->stream, &g);
    h->profiling = prof;
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "stream capture: %s", cudaGetErrorString(e));
    h->graph = g;
    CUDA_TRY(cudaGraphInstantiate(&h->graph_exec, g, 0));
    return GLC_OK;
}

int glc_moe_graph_launch(glc_moe* h, void* stream) {
    int rc = check_handle(h);
    if (rc) return rc;
    if (!h->graph_exec) return fail(GLC_ERR_STATE, "no graph built");
    CUDA_TRY(cudaGraphLaunch(h->graph_exec, stream ? (cudaStream_t)stream : h->stream));
    return GLC_OK;
}

int glc_attn_workspace_bytes(int32_t n_heads, int32_t n_kv_heads, int32_t max_len, uint64_t* bytes) {
    if (!bytes) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (n_heads <= 0 || n_kv_heads <= 0 || max_len <= 0 || n_heads % n_kv_heads)
        return fail(GLC_ERR_INVALID_ARG, "bad attention shape (%d heads, %d KV heads, max_len %d)", n_heads,
                    n_kv_heads, max_len);
    *bytes = glc::attn_workspace_bytes(n_heads, n_kv_heads, max_len);
    return GLC_OK;
}

int glc_attn_decode_dev(const float* q, const float* k_new, const float* v_new, void* k_cache, void* v_cache,
                        int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_len, int32_t pos,
                        float rope_theta, float* out, void* workspace, uint64_t workspace_bytes, void* stream) {
    if (!q || !k_new || !v_new || !k_cache || !v_cache || !out || !workspace)
        return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (head_dim != 128) return fail(GLC_ERR_UNSUPPORTED, "head_dim %d (only 128)", head_dim);
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > glc::kAttnMaxGroup)
        return fail(GLC_ERR_UNSUPPORTED, "%d heads over %d KV heads (a multiple, at most %d per KV head)", n_heads,
                    n_kv_heads, glc::kAttnMaxGroup);
    if (max_len <= 0 || pos < 0 || pos >= max_len)
        return fail(GLC_ERR_INVALID_ARG, "position %d outside the cache (max_len %d)", pos, max_len);
    if (max_len > glc::kAttnMaxLen) return fail(GLC_ERR_UNSUPPORTED, "max_len %d (at most %d)", max_len, glc::kAttnMaxLen);
    if (!(rope_theta > 0.f)) return fail(GLC_ERR_INVALID_ARG, "rope_theta must be positive");
    if (((uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)workspace) & 15u)
        return fail(GLC_ERR_INVALID_ARG, "caches and workspace must be 16-byte aligned");
    if (workspace_bytes < glc::attn_workspace_bytes(n_heads, n_kv_heads, max_len))
        return fail(GLC_ERR_INVALID_ARG, "workspace of %llu bytes is too small", (unsigned long long)workspace_bytes);
    glc::AttnParams p{};
    p.q = q;
    p.k_new = k_new;
    p.v_new = v_new;
    p.k_cache = static_cast<uint16_t*>(k_cache);
    p.v_cache = static_cast<uint16_t*>(v_cache);
    p.out = out;
    p.work = static_cast<float*>(workspace);
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.head_dim = head_dim;
    p.max_len = max_len;
    p.pos = pos;
    p.theta = rope_theta;
    CUDA_TRY(glc::attn_decode_launch(p, (cudaStream_t)stream));
    return GLC_OK;
}

// Per-device state of the raw GEMV entry points: the device error word of
// their bounded waits and the chain kernel's grid-barrier counter.
struct GemvDeviceState {
    int* err = nullptr;
    unsigned long long* bar = nullptr;
    int num_sms = 0;
};

static int gemv_state(GemvDeviceState** out) {
    static GemvDeviceState st[glc::kMaxDevices];
    static std::mutex mu;
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= glc::kMaxDevices) return fail(GLC_ERR_INVALID_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(mu);
    GemvDeviceState& s = st[dev];
    if (!s.err) {
        CUDA_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
        int* e = nullptr;
        unsigned long long* b = nullptr;
        CUDA_TRY(cudaMalloc(&e, sizeof(int)));
        if (cudaMalloc(&b, sizeof(unsigned long long)) != cudaSuccess) {
            cudaFree(e);
            return fail(GLC_ERR_OOM, "GEMV device state");
        }
        CUDA_TRY(cudaMemset(e, 0, sizeof(int)));
        CUDA_TRY(cudaMemset(b, 0, sizeof(unsigned long long)));
        s.bar = b;
        s.err = e;
    }
    *out = &s;
    return GLC_OK;
}

int glc_gemv_q4k_dev(const void* W, const float* x, float* y, int32_t K, int32_t N, void* stream) {
    if (!W || !x || !y) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (N <= 0 || K <= 0) return fail(GLC_ERR_INVALID_ARG, "K and N must be positive");
    if (K % 256) return fail(GLC_ERR_UNSUPPORTED, "Dimension %d is not a multiple of 256 for quantization Q4_K.", K);
    if (((uintptr_t)W | (uintptr_t)x) & 15u) return fail(GLC_ERR_INVALID_ARG, "W and x must be 16-byte aligned");
    GemvDeviceState* st = nullptr;
    if (int rc = gemv_state(&st)) return rc;
    glc::GemvParams p{};
    p.mode = glc::kGemvPlain;
    p.K = K;
    p.rows = N;
    p.nseg = 1;
    p.kslots = 1;
    p.num_experts = 1;
    p.A = (const uint8_t*)W;
    p.x = x;
    p.y = y;
    p.err = st->err;
    CUDA_TRY(glc::gemv_launch(p, st->num_sms, (cudaStream_t)stream));
    return GLC_OK;
}

static_assert(GLC_GEMV_SET == glc::kChainSet && GLC_GEMV_ADD == glc::kChainAdd &&
                  GLC_GEMV_GATE_UP == glc::kChainGateUp,
              "the chain ops of the C ABI and of the kernel share their values");

int glc_gemv_q4k_chain_dev(const glc_gemv_job* jobs, int32_t n, void* stream) {
    if (!jobs) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (n <= 0 || n > glc::kMaxChainJobs) return fail(GLC_ERR_INVALID_ARG, "%d jobs (1..%d)", n, glc::kMaxChainJobs);
    GemvDeviceState* st = nullptr;
    if (int rc = gemv_state(&st)) return rc;
    glc::GemvChainParams p{};
    for (int j = 0; j < n; ++j) {
        const glc_gemv_job& a = jobs[j];
        if (!a.W || !a.x || !a.y) return fail(GLC_ERR_INVALID_ARG, "job %d: null pointer", j);
        if (a.K <= 0 || a.N <= 0) return fail(GLC_ERR_INVALID_ARG, "job %d: K and N must be positive", j);
        if (a.K % 256)
            return fail(GLC_ERR_UNSUPPORTED, "job %d: dimension %d is not a multiple of 256 for quantization Q4_K.", j,
                        a.K);
        if (a.op != GLC_GEMV_SET && a.op != GLC_GEMV_ADD && a.op != GLC_GEMV_GATE_UP)
            return fail(GLC_ERR_INVALID_ARG, "job %d: unknown op %d", j, a.op);
        if (a.op == GLC_GEMV_GATE_UP && !a.W_up) return fail(GLC_ERR_INVALID_ARG, "job %d: GATE_UP needs W_up", j);
        if (((uintptr_t)a.W | (uintptr_t)a.W_up | (uintptr_t)a.x | (uintptr_t)a.norm_w) & 15u)
            return fail(GLC_ERR_INVALID_ARG, "job %d: W, W_up, x and norm_w must be 16-byte aligned", j);
        if (a.norm_w && !(a.norm_eps >= 0.f)) return fail(GLC_ERR_INVALID_ARG, "job %d: bad norm_eps", j);
        glc::GemvJob& b = p.jobs[j];
        b.A = (const uint8_t*)a.W;
        b.B = (const uint8_t*)a.W_up;
        b.x = a.x;
        b.y = a.y;
        b.norm_w = a.norm_w;
        b.norm_eps = a.norm_eps;
        b.K = a.K;
        b.N = a.N;
        b.op = (unsigned short)a.op;  // GLC_GEMV_* and glc::GemvChainOp share their values
        b.after_previous = a.after_previous ? 1 : 0;
    }
    p.njobs = n;
    p.bar = st->bar;
    p.err = st->err;
    CUDA_TRY(glc::gemv_chain_launch(p, st->num_sms, (cudaStream_t)stream));
    return GLC_OK;
}

int glc_gemv_poll_error(void) {
    GemvDeviceState* st = nullptr;
    if (int rc = gemv_state(&st)) return rc;
    CUDA_TRY(cudaDeviceSynchronize());
    int code = 0;
    CUDA_TRY(cudaMemcpy(&code, st->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code == 0) return GLC_OK;
    // a wait that gave up leaves the barrier counter short of a whole instance
    CUDA_TRY(cudaMemset(st->err, 0, sizeof(int)));
    CUDA_TRY(cudaMemset(st->bar, 0, sizeof(unsigned long long)));
    return fail(GLC_ERR_TIMEOUT, "device-side wait of a GEMV gave up (code %d)", code);
}

int glc_router_topk_dev(const float* x, const float* router_w, int32_t T, int32_t D, int32_t E, int32_t k,
                        int32_t renormalize, int32_t rmsnorm, float* xin_out, float* logits_out,
                        int32_t* ids_out, float* w_out, void* stream) {
    if (!x || !router_w || !ids_out || !w_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (T < 0 || D <= 0 || E <= 0 || E > 64 || k <= 0 || k > E || k > 16)
        return fail(GLC_ERR_INVALID_ARG, "router shape out of range (T=%d D=%d E=%d k=%d)", T, D, E, k);
    glc::RouterParams rp{};
    rp.x = x;
    rp.Wr = router_w;
    rp.T = T;
    rp.D = D;
    rp.E = E;
    rp.k = k;
    rp.renorm = renormalize;
    rp.rmsnorm = rmsnorm;
    rp.xin = xin_out;
    rp.logits = logits_out;
    rp.ids = ids_out;
    rp.w = w_out;
    CUDA_TRY(glc::router_launch(rp, (cudaStream_t)stream));
    return GLC_OK;
}

int glc_dispatch_plan_dev(const int32_t* ids, int32_t P, int32_t E, int32_t* counts, int32_t* offsets,
                          int32_t* perm, int32_t* inv, void* stream) {
    if (!ids || !counts || !offsets || !perm || !inv) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (P < 0 || E <= 0 || E > 64) return fail(GLC_ERR_INVALID_ARG, "P=%d E=%d out of range", P, E);
    const int gmax = glc::plan_max_groups(P, E);
    // The group table (not returned) comes from the stream-ordered pool and
    // goes back to it behind the kernel: no device-wide synchronisation, and
    // the call returns without waiting for the stream.
    cudaStream_t st = (cudaStream_t)stream;
    int* scratch = nullptr;
    CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), sizeof(int) * (size_t)(6 * gmax + E + 2), st));
    glc::DispatchPlan plan{};
    plan.counts = counts;
    plan.offsets = offsets;
    plan.perm = perm;
    plan.inv = inv;
    plan.grp_e = scratch;
    plan.grp_ntok = scratch + gmax;
    plan.grp_N = scratch + 2 * gmax;
    plan.grp_pos0 = scratch + 3 * gmax;
    plan.grp_units = scratch + 4 * gmax;
    plan.grp_first = scratch + 5 * gmax;
    plan.meta = scratch + 5 * gmax + E;
    const cudaError_t e = glc::dispatch_plan_launch(ids, P, E, plan, st);
    const cudaError_t f = cudaFreeAsync(scratch, st);
    if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "dispatch plan: %s", cudaGetErrorString(e));
    if (f != cudaSuccess) return fail(GLC_ERR_CUDA, "dispatch plan scratch: %s", cudaGetErrorString(f));
    return GLC_OK;
}

int32_t glc_wire_token_bytes(int32_t mode, int32_t dim) {
    switch (mode) {
        case GLC_WIRE_FP32: return dim * 4;
        case GLC_WIRE_FP16: return dim * 2;
        case GLC_WIRE_INT8: return dim + 4;
        case GLC_WIRE_FP8_E4M3: return dim + 4;
        default: return dim * 2;
    }
}

int glc_wire_quantize_dev(int32_t mode, const float* x, int32_t T, int32_t D, uint8_t* out, void* stream) {
    if (T < 0 || D < 0) return fail(GLC_ERR_INVALID_ARG, "negative shape");
    if (T == 0 || D == 0) return GLC_OK;
    if (!x || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    CUDA_TRY(glc::wire_quantize_launch(mode, x, T, D, out, (cudaStream_t)stream));
    return GLC_OK;
}

int glc_wire_dequantize_dev(int32_t mode, const uint8_t* in, int32_t T, int32_t D, float* out, void* stream) {
    if (T < 0 || D < 0) return fail(GLC_ERR_INVALID_ARG, "negative shape");
    if (T == 0 || D == 0) return GLC_OK;
    if (!in || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    CUDA_TRY(glc::wire_dequantize_launch(mode, in, T, D, out, (cudaStream_t)stream));
    return GLC_OK;
}

int glc_wire_quantize(int32_t mode, const float* x, int32_t T, int32_t D, uint8_t* out, size_t out_bytes) {
    if (T < 0 || D < 0) return fail(GLC_ERR_INVALID_ARG, "negative shape");
    const size_t need = (size_t)glc_wire_token_bytes(mode, D) * (size_t)T;
    if (out_bytes < need)  // QuantizeBatch: destination too small (QuantizationKernels.cs:89-90)
        return fail(GLC_ERR_INVALID_ARG, "Destination buffer too small (%zu < %zu)", out_bytes, need);
    if (need == 0) return GLC_OK;
    if (!x || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    // device buffers from the stream-ordered pool (no device-wide
    // synchronisation); the host copies make the call synchronous
    const cudaStream_t st = cudaStreamLegacy;
    float* dx = nullptr;
    uint8_t* dq = nullptr;
    CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&dx), sizeof(float) * (size_t)T * D, st));
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&dq), need, st);
    if (e != cudaSuccess) { cudaFreeAsync(dx, st); return fail(GLC_ERR_OOM, "device buffer: %s", cudaGetErrorString(e)); }
    e = cudaMemcpyAsync(dx, x, sizeof(float) * (size_t)T * D, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = glc::wire_quantize_launch(mode, dx, T, D, dq, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dq, need, cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(dx, st);
    cudaFreeAsync(dq, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "wire quantize: %s", cudaGetErrorString(e));
    return GLC_OK;
}

int glc_wire_dequantize(int32_t mode, const uint8_t* in, size_t in_bytes, int32_t T, int32_t D, float* out) {
    if (T < 0 || D < 0) return fail(GLC_ERR_INVALID_ARG, "negative shape");
    const size_t need = (size_t)glc_wire_token_bytes(mode, D) * (size_t)T;
    if (in_bytes < need) return fail(GLC_ERR_INVALID_ARG, "Source buffer too small (%zu < %zu)", in_bytes, need);
    if (need == 0) return GLC_OK;
    if (!in || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const cudaStream_t st = cudaStreamLegacy;
    float* dx = nullptr;
    uint8_t* dq = nullptr;
    CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&dq), need, st));
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&dx), sizeof(float) * (size_t)T * D, st);
    if (e != cudaSuccess) { cudaFreeAsync(dq, st); return fail(GLC_ERR_OOM, "device buffer: %s", cudaGetErrorString(e)); }
    e = cudaMemcpyAsync(dq, in, need, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = glc::wire_dequantize_launch(mode, dq, T, D, dx, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dx, sizeof(float) * (size_t)T * D, cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(dx, st);
    cudaFreeAsync(dq, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail(GLC_ERR_CUDA, "wire dequantize: %s", cudaGetErrorString(e));
    return GLC_OK;
}

static void put_u32(uint8_t* p, uint32_t v) { for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(v >> (8 * i)); }
static uint32_t get_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int glc_fused_header_write(const glc_fused_header* h, uint8_t* o) {
    if (!h || !o) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    put_u32(o, 0x47414354u);  // "GACT"
    put_u32(o + 4, (uint32_t)h->sequence_id);
    put_u32(o + 8, (uint32_t)(h->sequence_id >> 32));
    put_u32(o + 12, (uint32_t)h->token_index);
    put_u32(o + 16, (uint32_t)h->layer_index);
    put_u32(o + 20, (uint32_t)h->hidden_dim);
    o[24] = h->precision_mode;
    o[25] = h->flags;
    o[26] = (uint8_t)h->batch_tokens;
    o[27] = (uint8_t)(h->batch_tokens >> 8);
    uint32_t s;
    std::memcpy(&s, &h->scale, 4);
    put_u32(o + 28, s);
    return GLC_OK;
}

int glc_fused_header_read(const uint8_t* in, glc_fused_header* h) {
    if (!in || !h) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const uint32_t magic = get_u32(in);
    if (magic != 0x47414354u)  // ReadFrom throws InvalidOperationException (FusedActivationHeader.cs:158-159)
        return fail(GLC_ERR_INVALID_ARG, "Invalid FusedActivationHeader magic: 0x%08X, expected 0x47414354", magic);
    h->sequence_id = (uint64_t)get_u32(in + 4) | ((uint64_t)get_u32(in + 8) << 32);
    h->token_index = (int32_t)get_u32(in + 12);
    h->layer_index = (int32_t)get_u32(in + 16);
    h->hidden_dim = (int32_t)get_u32(in + 20);
    h->precision_mode = in[24];
    h->flags = in[25];
    h->batch_tokens = (uint16_t)(in[26] | (in[27] << 8));
    const uint32_t s = get_u32(in + 28);
    std::memcpy(&h->scale, &s, 4);
    return GLC_OK;
}

int32_t glc_fused_header_payload_bytes(const glc_fused_header* h) {
    if (!h) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const int tokens = h->batch_tokens > 0 ? h->batch_tokens : 1;
    if (h->flags & 0x10) return tokens * 4;  // Stage0TokenInput: token ids
    switch (h->precision_mode) {
        case GLC_WIRE_FP32: return h->hidden_dim * tokens * 4;
        case GLC_WIRE_FP16: return h->hidden_dim * tokens * 2;
        case GLC_WIRE_INT8: return (h->hidden_dim + 4) * tokens;
        case GLC_WIRE_FP8_E4M3: return (h->hidden_dim + 4) * tokens;
        default: return h->hidden_dim * tokens * 2;
    }
}

}  // extern "C"
