// stage.cu -- a dense decoder pipeline stage on sm_100a: one token through a
// range of transformer layers with its KV cache, the counterpart of
// IClusterStageModel.ForwardStage (Pipeline/IClusterStageModel.cs:19; the
// reference's stage bodies are its external model package, Program.cs:41-110,
// 1382-1390) for the Qwen2-style dense layers of a pipeline-parallel model
// (the reference splits the layer range over LAN nodes, DistributedClusterSession.cs:
// 775-830, and quantises the activations at every stage boundary, Program.cs:743).
//
// Per layer, on the stage's stream:
//   qkv = [Wq; Wk; Wv] (RMSNorm(x) * w_attn)      (one Q4_K GEMV over the stacked
//         rows; the weighted RMSNorm is folded in: the lanes take x * w_attn
//         and the epilogue scales by the norm's 1 / rms, which every CTA forms)
//   o   = attention(q + bq, k + bk, v + bv; the layer's fp16 KV cache at pos)
//         (attention.cu; the biases are added as it reads its inputs)
//   x   = x + Wo o                                (GEMV, residual in the epilogue)
//   a   = SiLU(Wgate h) * (Wup h), h = RMSNorm(x) * w_ffn   (gate/up GEMV, the
//         norm folded in the same way, SwiGLU epilogue)
//   x   = x + Wdown a                             (GEMV, residual in the epilogue)
// with, on a first stage, x = dequantised row `token` of the Q4_K embedding
// table and, on a last stage asked for logits, logits = Wlm RMSNorm(x) * w_final
// and the arg-max token.  A mixture-of-experts stage (Mixtral-style layers)
// replaces the feed-forward by the router (the weighted RMSNorm folded in,
// softmax top-k), the routed experts' gate/up GEMV with SwiGLU and their down
// GEMV with the k-ordered weighted combine and the residual in its epilogue
// (GpuFirstExpertStageWorker.ProcessRoutedTopK, GpuFirstExpertStageWorker.cs:
// 416-583), between the attention's O projection and the next layer's QKV:
// one launch of the fused decode kernel (decode_fused.cu, its router split
// over a thread-block cluster when the router rows do not fit one CTA).
// Dense stages use two launches per layer: the attention, then ONE GEMV
// chain (gemv_chain.cu) holding the O projection, gate/up, down and the next
// layer's QKV projection (or the LM head), whose weights stream back to back
// while only its consumer warps wait grid-wide between the dependent jobs.
// The position lives in device memory, so the whole stage step is one CUDA
// graph replayed for every token (the attention's launch shape does not depend
// on the position); the chains and the attention are programmatically
// serialised, so each starts (streaming weights, or loading cache rows) as the
// kernel before it leaves each SM.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../../../include/glacier_b200.h"
#include "common.cuh"
#include "kernels.h"
#include "synth.h"

namespace glc {
int set_last_error(int code, const char* msg);
}

namespace {

using glc::grid_dep_launch_dependents;
using glc::grid_dep_wait;

constexpr int kHeadDim = 128;

// x[0..D) = dequantised row *token of a Q4_K table [rows][D/256*144]
// ((d*sc)*q - dmin*m, the GGUF Q4_K values), one thread per weight.
__global__ void __launch_bounds__(256) q4k_row_kernel(const uint8_t* __restrict__ table, const int* __restrict__ token,
                                                      int rows, int D, float* __restrict__ x) {
    grid_dep_wait();
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i >= D) return;
    int t = *token;
    t = t < 0 ? 0 : (t >= rows ? rows - 1 : t);
    const uint8_t* blk = table + (size_t)t * (D / 256) * 144 + (size_t)(i / 256) * 144;
    const int w = i & 255, c = w >> 6, l = w & 63, j = 2 * c + (l >> 5);
    const uint8_t* sc = blk + 4;
    int s, m;
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const uint8_t qb = blk[16 + 32 * c + (l & 31)];
    const int q = (l < 32) ? (qb & 0xF) : (qb >> 4);
    const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
    // each product rounded, as the GGUF dequantisation does (no contraction)
    x[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
}

// Arg-max of n logits (NaN as -inf, the lower index on ties) into *out.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ v, int n, int* __restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    grid_dep_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += 1024) {
        const float x = isnan(v[i]) ? -INFINITY : v[i];
        if (x > best || (x == best && i < bi)) { best = x; bi = i; }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < 32; ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
        *out = bi == 0x7fffffff ? 0 : bi;
    }
}

__global__ void fill_int_kernel(int* p, int v) { *p = v; }

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return glc::set_last_error(code, buf);
}

#define CUDA_TRY(call)                                                                          \
    do {                                                                                        \
        const cudaError_t e_ = (call);                                                          \
        if (e_ != cudaSuccess) return fail(GLC_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

size_t rowbytes(int k) { return (size_t)(k / 256) * 144; }

struct StageLayer {
    float* attn_norm = nullptr;
    uint8_t* wqkv = nullptr;  // [(Hq + 2 Hkv) * 128][rowbytes(D)]
    float* bqkv = nullptr;
    uint8_t* wo = nullptr;    // [D][rowbytes(Hq * 128)]
    float* ffn_norm = nullptr;
    uint8_t* wgate = nullptr;  // [FF][rowbytes(D)]
    uint8_t* wup = nullptr;
    uint8_t* wdown = nullptr;  // [D][rowbytes(FF)]
    uint16_t* kc = nullptr;    // fp16 [Hkv][max_len][128]
    uint16_t* vc = nullptr;
    // mixture-of-experts layers
    float* router = nullptr;   // fp32 [D][E]
    uint8_t* egate = nullptr;  // [E][F][rowbytes(D)]
    uint8_t* eup = nullptr;
    uint8_t* edown = nullptr;  // [E][D][rowbytes(F)]
    bool loaded = false;
};

// host-side bytes of each tensor of a layer
struct Sizes {
    size_t qkv_rows, wqkv, wo, wgu, wdown, cache;
    size_t egu, edown;  // one expert's gate (= up) and down bytes
};

}  // namespace

struct glc_stage {
    glc_stage_desc d{};
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    Sizes sz{};
    std::vector<StageLayer> layers;
    uint8_t* embed = nullptr;     // Q4_K [vocab][rowbytes(D)] (first stage)
    float* final_norm = nullptr;  // [D] (last stage)
    uint8_t* lm_head = nullptr;   // Q4_K [vocab][rowbytes(D)] (last stage)
    // device workspace
    float* x = nullptr;      // [D] the stage's residual stream
    float* qkv = nullptr;    // [(Hq + 2 Hkv) * 128]
    float* attn = nullptr;   // [Hq * 128]
    float* act = nullptr;    // [FF]
    float* logits = nullptr; // [vocab]
    float* attn_work = nullptr;
    float* xin = nullptr;    // [D] RMSNorm(x) * w_ffn (mixture of experts)
    int* ids = nullptr;      // [k] routed experts
    float* rw = nullptr;     // [k] their weights
    int* pos = nullptr;      // the position the next step uses
    int* token = nullptr;    // input token (first stage) / arg-max token (last stage)
    int* err = nullptr;
    unsigned long long* bar = nullptr;  // the GEMV chains' grid-barrier counter
    // the captured stage step per (embed, logits) variant
    cudaGraphExec_t graphs[4] = {};
};

namespace {

int check(glc_stage* h) {
    if (!h) return fail(GLC_ERR_INVALID_ARG, "null stage handle");
    return GLC_OK;
}

glc::GemvJob job(const uint8_t* A, const float* x, float* y, int K, int N, int op, bool after_previous,
               const float* norm_w = nullptr, float eps = 0.f, const uint8_t* B = nullptr);

int next_layer_qkv(glc_stage* h, int l, bool logits, cudaStream_t st);

// A mixture-of-experts layer after its attention: x += Wo o (a chain of one
// job), then the feed-forward: the router on RMSNorm(x) * w_ffn, the routed
// gate/up GEMVs with SwiGLU and the routed down GEMVs combining into x in k
// order, as one fused launch (decode_fused.cu) or, when the layer does not
// fit it, as three launches; then the next layer's QKV projection (or the LM
// head after the last layer).
int moe_layer_ffn(glc_stage* h, const StageLayer& L, int l, bool logits, cudaStream_t st) {
    const glc_stage_desc& d = h->d;
    const int D = d.hidden_dim, F = d.expert_ffn_dim, E = d.num_experts, k = d.top_k;
    const int Hq = d.n_heads;
    glc::GemvChainParams c{};
    c.bar = h->bar;
    c.err = h->err;
    c.jobs[0] = job(L.wo, h->attn, h->x, Hq * kHeadDim, D, glc::kChainAdd, false);
    c.njobs = 1;
    CUDA_TRY(glc::gemv_chain_launch(c, h->num_sms, st));
    // The feed-forward in one launch (router on RMSNorm(x) * w_ffn, routed
    // gate/up + SwiGLU, down + k-ordered combine into x); the residual is
    // updated in place (every CTA stages x before the kernel's grid barrier
    // and writes its own rows of x after it).
    glc::FusedDecodeParams fp{};
    fp.x = h->x;
    fp.resid = h->x;
    fp.out = h->x;
    fp.Wr = L.router;
    fp.gate = L.egate;
    fp.up = L.eup;
    fp.down = L.edown;
    fp.gu_expert_bytes = (long long)h->sz.egu;
    fp.dn_expert_bytes = (long long)h->sz.edown;
    fp.act = h->act;
    fp.ids = h->ids;
    fp.w = h->rw;
    fp.bar = h->bar;
    fp.err = h->err;
    fp.T = 1;
    fp.D = D;
    fp.F = F;
    fp.E = E;
    fp.k = k;
    fp.renorm = d.moe_renormalize;
    fp.rmsnorm = 1;
    fp.norm_w = L.ffn_norm;
    fp.norm_eps = d.rms_eps;
    const cudaError_t fe = glc::fused_decode_launch(fp, h->num_sms, st);
    if (fe == cudaSuccess) return next_layer_qkv(h, l, logits, st);
    if (fe != cudaErrorNotSupported) return fail(GLC_ERR_CUDA, "fused feed-forward: %s", cudaGetErrorString(fe));
    (void)cudaGetLastError();
    // does not fit the fused kernel: router, gate/up and down as three launches
    glc::RouterParams rp{};
    rp.x = h->x;
    rp.Wr = L.router;
    rp.T = 1;
    rp.D = D;
    rp.E = E;
    rp.k = k;
    rp.renorm = d.moe_renormalize;
    rp.rmsnorm = 1;
    rp.norm_w = L.ffn_norm;
    rp.norm_eps = d.rms_eps;
    rp.xin = h->xin;
    rp.ids = h->ids;
    rp.w = h->rw;
    CUDA_TRY(glc::router_launch(rp, st));
    glc::GemvParams gu{};  // act[j] = SiLU(Gate_ids[j] h) * (Up_ids[j] h)
    gu.mode = glc::kGemvGateUp;
    gu.K = D;
    gu.rows = F;
    gu.nseg = k;
    gu.kslots = k;
    gu.num_experts = E;
    gu.A = L.egate;
    gu.B = L.eup;
    gu.expert_bytes = (long long)h->sz.egu;
    gu.ids = h->ids;
    gu.x = h->xin;
    gu.y = h->act;
    gu.err = h->err;
    CUDA_TRY(glc::gemv_launch(gu, h->num_sms, st));
    glc::GemvParams dn{};  // x = x + sum_j w_j Down_ids[j] act[j], in k order
    dn.mode = glc::kGemvDownCombine;
    dn.K = F;
    dn.rows = D;
    dn.nseg = 1;
    dn.kslots = k;
    dn.num_experts = E;
    dn.A = L.edown;
    dn.expert_bytes = (long long)h->sz.edown;
    dn.ids = h->ids;
    dn.cw = h->rw;
    dn.x = h->act;
    dn.y = h->x;
    dn.accumulate = 1;
    dn.err = h->err;
    CUDA_TRY(glc::gemv_launch(dn, h->num_sms, st));
    return next_layer_qkv(h, l, logits, st);
}

// After a mixture-of-experts layer: the next layer's QKV (or the LM head) as a chain launch.
int next_layer_qkv(glc_stage* h, int l, bool logits, cudaStream_t st) {
    const glc_stage_desc& d = h->d;
    const int D = d.hidden_dim, qrows = (d.n_heads + 2 * d.n_kv_heads) * kHeadDim;
    glc::GemvChainParams c{};
    c.bar = h->bar;
    c.err = h->err;
    if (l + 1 < d.layer_count) {
        const StageLayer& N = h->layers[l + 1];
        c.jobs[c.njobs++] = job(N.wqkv, h->x, h->qkv, D, qrows, glc::kChainSet, false, N.attn_norm, d.rms_eps);
    } else if (logits) {
        c.jobs[c.njobs++] = job(h->lm_head, h->x, h->logits, D, d.vocab, glc::kChainSet, false, h->final_norm,
                                d.rms_eps);
    }
    if (c.njobs) CUDA_TRY(glc::gemv_chain_launch(c, h->num_sms, st));
    return GLC_OK;
}

glc::GemvJob job(const uint8_t* A, const float* x, float* y, int K, int N, int op, bool after_previous,
               const float* norm_w, float eps, const uint8_t* B) {
    glc::GemvJob j{};
    j.A = A;
    j.B = B;
    j.x = x;
    j.y = y;
    j.norm_w = norm_w;
    j.norm_eps = eps;
    j.K = K;
    j.N = N;
    j.op = op;
    j.after_previous = after_previous ? 1 : 0;
    return j;
}

// One token through the stage's layers on `st` (position from h->pos): the
// QKV projection of the first layer, then per layer the attention and ONE
// GEMV chain [x += Wo o; a = SwiGLU(Wg, Wu; RMSNorm(x) w_ffn); x += Wd a;
// the next layer's QKV (or the LM head)], each job after the first waiting
// grid-wide for the one before while the weights keep streaming.
int stage_step(glc_stage* h, bool embed, bool logits, cudaStream_t st) {
    const glc_stage_desc& d = h->d;
    const int D = d.hidden_dim, FF = d.ffn_dim, Hq = d.n_heads, Hkv = d.n_kv_heads;
    const int qrows = (Hq + 2 * Hkv) * kHeadDim;
    if (embed) {
        q4k_row_kernel<<<(D + 255) / 256, 256, 0, st>>>(h->embed, h->token, d.vocab, D, h->x);
        CUDA_TRY(cudaGetLastError());
    }
    glc::GemvChainParams c{};
    c.bar = h->bar;
    c.err = h->err;
    // qkv = [Wq; Wk; Wv] (RMSNorm(x) * w_attn) of the first layer
    c.jobs[0] = job(h->layers[0].wqkv, h->x, h->qkv, D, qrows, glc::kChainSet, false, h->layers[0].attn_norm,
                    d.rms_eps);
    c.njobs = 1;
    CUDA_TRY(glc::gemv_chain_launch(c, h->num_sms, st));
    for (int l = 0; l < d.layer_count; ++l) {
        StageLayer& L = h->layers[l];
        glc::AttnParams ap{};  // the biases are added as the attention reads q, k and v
        ap.q = h->qkv;
        ap.k_new = h->qkv + (size_t)Hq * kHeadDim;
        ap.v_new = h->qkv + (size_t)(Hq + Hkv) * kHeadDim;
        ap.k_cache = L.kc;
        ap.v_cache = L.vc;
        ap.out = h->attn;
        ap.work = h->attn_work;
        ap.n_heads = Hq;
        ap.n_kv_heads = Hkv;
        ap.head_dim = kHeadDim;
        ap.max_len = d.max_len;
        ap.pos = 0;
        ap.pos_dev = h->pos;  // written by the step's first kernel, which has no early trigger
        ap.theta = d.rope_theta;
        ap.bq = L.bqkv;
        ap.bk = L.bqkv + (size_t)Hq * kHeadDim;
        ap.bv = L.bqkv + (size_t)(Hq + Hkv) * kHeadDim;
        CUDA_TRY(glc::attn_decode_launch(ap, st));
        if (d.num_experts > 0) {
            const int rc = moe_layer_ffn(h, L, l, logits, st);
            if (rc) return rc;
            continue;
        }
        c.njobs = 0;
        c.jobs[c.njobs++] = job(L.wo, h->attn, h->x, Hq * kHeadDim, D, glc::kChainAdd, false);
        c.jobs[c.njobs++] = job(L.wgate, h->x, h->act, D, FF, glc::kChainGateUp, true, L.ffn_norm, d.rms_eps, L.wup);
        c.jobs[c.njobs++] = job(L.wdown, h->act, h->x, FF, D, glc::kChainAdd, true);
        if (l + 1 < d.layer_count) {
            const StageLayer& N = h->layers[l + 1];
            c.jobs[c.njobs++] = job(N.wqkv, h->x, h->qkv, D, qrows, glc::kChainSet, true, N.attn_norm, d.rms_eps);
        } else if (logits) {  // logits = W_lm (RMSNorm(x) * w_final)
            c.jobs[c.njobs++] = job(h->lm_head, h->x, h->logits, D, d.vocab, glc::kChainSet, true, h->final_norm,
                                    d.rms_eps);
        }
        CUDA_TRY(glc::gemv_chain_launch(c, h->num_sms, st));
    }
    if (logits) {
        argmax_kernel<<<1, 1024, 0, st>>>(h->logits, d.vocab, h->token);
        CUDA_TRY(cudaGetLastError());
    }
    return GLC_OK;
}

void free_stage(glc_stage* h) {
    for (auto& L : h->layers) {
        cudaFree(L.attn_norm); cudaFree(L.wqkv); cudaFree(L.bqkv); cudaFree(L.wo); cudaFree(L.ffn_norm);
        cudaFree(L.wgate); cudaFree(L.wup); cudaFree(L.wdown); cudaFree(L.kc); cudaFree(L.vc);
        cudaFree(L.router); cudaFree(L.egate); cudaFree(L.eup); cudaFree(L.edown);
    }
    cudaFree(h->embed); cudaFree(h->final_norm); cudaFree(h->lm_head);
    cudaFree(h->x); cudaFree(h->qkv); cudaFree(h->attn); cudaFree(h->act); cudaFree(h->logits);
    cudaFree(h->attn_work); cudaFree(h->xin); cudaFree(h->ids); cudaFree(h->rw); cudaFree(h->pos); cudaFree(h->token);
    cudaFree(h->err);
    cudaFree(h->bar);
    for (auto& g : h->graphs)
        if (g) cudaGraphExecDestroy(g);
    if (h->stream) cudaStreamDestroy(h->stream);
}

}  // namespace

extern "C" {

int glc_stage_create(const glc_stage_desc* desc, glc_stage** out) {
    if (!desc || !out) return fail(GLC_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const glc_stage_desc& d = *desc;
    const bool moe = d.num_experts > 0;
    if (d.hidden_dim <= 0 || (!moe && d.ffn_dim <= 0) || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.layer_count <= 0)
        return fail(GLC_ERR_INVALID_ARG, "dimensions and layer count must be positive");
    if (d.num_experts < 0 || (moe && (d.num_experts < 2 || d.num_experts > 8)))
        return fail(GLC_ERR_UNSUPPORTED, "num_experts %d: 0 (dense) or 2..8", d.num_experts);
    if (moe && (d.top_k < 1 || d.top_k > d.num_experts))
        return fail(GLC_ERR_INVALID_ARG, "top_k %d outside 1..%d", d.top_k, d.num_experts);
    if (moe && (d.expert_ffn_dim <= 0 || d.expert_ffn_dim % 256))
        return fail(GLC_ERR_UNSUPPORTED, "expert_ffn_dim %d: a positive multiple of 256", d.expert_ffn_dim);
    if (d.head_dim != kHeadDim) return fail(GLC_ERR_UNSUPPORTED, "head_dim %d: 128 supported", d.head_dim);
    if (d.hidden_dim % 256 || (!moe && d.ffn_dim % 256) || (d.n_heads * kHeadDim) % 256)
        return fail(GLC_ERR_UNSUPPORTED, "Q4_K needs hidden, ffn and head widths that are multiples of 256");
    if (d.n_heads % d.n_kv_heads || d.n_heads / d.n_kv_heads > glc::kAttnMaxGroup)
        return fail(GLC_ERR_UNSUPPORTED, "at most %d query heads per KV head", glc::kAttnMaxGroup);
    if (d.max_len <= 0 || d.max_len > glc::kAttnMaxLen) return fail(GLC_ERR_INVALID_ARG, "max_len 1..%d", glc::kAttnMaxLen);
    if ((d.has_embedding || d.has_lm_head) && d.vocab <= 0) return fail(GLC_ERR_INVALID_ARG, "vocab must be positive");
    CUDA_TRY(cudaSetDevice(d.device));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, d.device));
    if (prop.major < 10) return fail(GLC_ERR_UNSUPPORTED, "sm_100a required");
    glc_stage* h = new glc_stage();
    h->d = d;
    h->num_sms = prop.multiProcessorCount;
    const int D = d.hidden_dim, FF = moe ? 0 : d.ffn_dim, Hq = d.n_heads, Hkv = d.n_kv_heads;
    const int F = moe ? d.expert_ffn_dim : 0, E = moe ? d.num_experts : 0;
    h->sz.qkv_rows = (size_t)(Hq + 2 * Hkv) * kHeadDim;
    h->sz.wqkv = h->sz.qkv_rows * rowbytes(D);
    h->sz.wo = (size_t)D * rowbytes(Hq * kHeadDim);
    h->sz.wgu = (size_t)FF * rowbytes(D);
    h->sz.wdown = (size_t)D * rowbytes(FF);
    h->sz.cache = (size_t)Hkv * d.max_len * kHeadDim * sizeof(uint16_t);
    h->sz.egu = (size_t)F * rowbytes(D);
    h->sz.edown = (size_t)D * rowbytes(F);
    h->layers.resize(d.layer_count);
    auto bad = [&](const char* what) {
        free_stage(h);
        delete h;
        return fail(GLC_ERR_OOM, "cudaMalloc: %s", what);
    };
#define SALLOC(ptr, bytes) \
    if (cudaMalloc(reinterpret_cast<void**>(&(ptr)), (bytes)) != cudaSuccess) return bad(#ptr)
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return bad("stream");
    for (auto& L : h->layers) {
        SALLOC(L.attn_norm, sizeof(float) * D);
        SALLOC(L.wqkv, h->sz.wqkv);
        SALLOC(L.bqkv, sizeof(float) * h->sz.qkv_rows);
        SALLOC(L.wo, h->sz.wo);
        SALLOC(L.ffn_norm, sizeof(float) * D);
        if (moe) {
            SALLOC(L.router, sizeof(float) * D * E);
            SALLOC(L.egate, h->sz.egu * E);
            SALLOC(L.eup, h->sz.egu * E);
            SALLOC(L.edown, h->sz.edown * E);
        } else {
            SALLOC(L.wgate, h->sz.wgu);
            SALLOC(L.wup, h->sz.wgu);
            SALLOC(L.wdown, h->sz.wdown);
        }
        SALLOC(L.kc, h->sz.cache);
        SALLOC(L.vc, h->sz.cache);
        cudaMemset(L.kc, 0, h->sz.cache);
        cudaMemset(L.vc, 0, h->sz.cache);
    }
    if (d.has_embedding) SALLOC(h->embed, (size_t)d.vocab * rowbytes(D));
    if (d.has_lm_head) {
        SALLOC(h->final_norm, sizeof(float) * D);
        SALLOC(h->lm_head, (size_t)d.vocab * rowbytes(D));
        SALLOC(h->logits, sizeof(float) * d.vocab);
    }
    SALLOC(h->x, sizeof(float) * D);
    SALLOC(h->qkv, sizeof(float) * h->sz.qkv_rows);
    SALLOC(h->attn, sizeof(float) * Hq * kHeadDim);
    SALLOC(h->act, sizeof(float) * std::max(FF, d.top_k * F));
    if (moe) {
        SALLOC(h->xin, sizeof(float) * D);
        SALLOC(h->ids, sizeof(int) * d.top_k);
        SALLOC(h->rw, sizeof(float) * d.top_k);
    }
    SALLOC(h->attn_work, glc::attn_workspace_bytes(Hq, Hkv, d.max_len));
    SALLOC(h->pos, sizeof(int));
    SALLOC(h->token, sizeof(int));
    SALLOC(h->err, sizeof(int) * 8);
    SALLOC(h->bar, sizeof(unsigned long long));
#undef SALLOC
    cudaMemset(h->bar, 0, sizeof(unsigned long long));
    cudaMemset(h->pos, 0, sizeof(int));
    cudaMemset(h->token, 0, sizeof(int));
    cudaMemset(h->err, 0, sizeof(int) * 8);
    if (cudaDeviceSynchronize() != cudaSuccess) return bad("initialisation");
    *out = h;
    return GLC_OK;
}

int glc_stage_destroy(glc_stage* h) {
    if (!h) return GLC_OK;
    cudaSetDevice(h->d.device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    free_stage(h);
    delete h;
    return GLC_OK;
}

}  // extern "C"

namespace {

// The attention weights and norms of w into layer L (biases NULL = zero).
int load_attention(glc_stage* h, StageLayer& L, const glc_dense_layer_weights* w) {
    const int D = h->d.hidden_dim, Hq = h->d.n_heads, Hkv = h->d.n_kv_heads;
    const size_t rq = (size_t)Hq * kHeadDim * rowbytes(D), rk = (size_t)Hkv * kHeadDim * rowbytes(D);
    CUDA_TRY(cudaMemcpy(L.attn_norm, w->attn_norm, sizeof(float) * D, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.wqkv, w->wq, rq, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.wqkv + rq, w->wk, rk, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.wqkv + rq + rk, w->wv, rk, cudaMemcpyHostToDevice));
    const size_t nq = (size_t)Hq * kHeadDim, nk = (size_t)Hkv * kHeadDim;
    if (w->bq) CUDA_TRY(cudaMemcpy(L.bqkv, w->bq, sizeof(float) * nq, cudaMemcpyHostToDevice));
    else CUDA_TRY(cudaMemset(L.bqkv, 0, sizeof(float) * nq));
    if (w->bk) CUDA_TRY(cudaMemcpy(L.bqkv + nq, w->bk, sizeof(float) * nk, cudaMemcpyHostToDevice));
    else CUDA_TRY(cudaMemset(L.bqkv + nq, 0, sizeof(float) * nk));
    if (w->bv) CUDA_TRY(cudaMemcpy(L.bqkv + nq + nk, w->bv, sizeof(float) * nk, cudaMemcpyHostToDevice));
    else CUDA_TRY(cudaMemset(L.bqkv + nq + nk, 0, sizeof(float) * nk));
    CUDA_TRY(cudaMemcpy(L.wo, w->wo, h->sz.wo, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.ffn_norm, w->ffn_norm, sizeof(float) * D, cudaMemcpyHostToDevice));
    return GLC_OK;
}

}  // namespace

extern "C" {

int glc_stage_load_layer(glc_stage* h, int32_t layer, const glc_dense_layer_weights* w) {
    int rc = check(h);
    if (rc) return rc;
    if (h->d.num_experts > 0) return fail(GLC_ERR_STATE, "a mixture-of-experts stage loads layers with glc_stage_load_moe_layer");
    if (!w || !w->attn_norm || !w->wq || !w->wk || !w->wv || !w->wo || !w->ffn_norm || !w->w_gate || !w->w_up ||
        !w->w_down)
        return fail(GLC_ERR_INVALID_ARG, "null weight pointer");
    if (layer < 0 || layer >= h->d.layer_count) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    CUDA_TRY(cudaSetDevice(h->d.device));
    StageLayer& L = h->layers[layer];
    if ((rc = load_attention(h, L, w))) return rc;
    CUDA_TRY(cudaMemcpy(L.wgate, w->w_gate, h->sz.wgu, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.wup, w->w_up, h->sz.wgu, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.wdown, w->w_down, h->sz.wdown, cudaMemcpyHostToDevice));
    L.loaded = true;
    return GLC_OK;
}

int glc_stage_load_moe_layer(glc_stage* h, int32_t layer, const glc_dense_layer_weights* w, const float* router,
                             const void* gate_exps, const void* up_exps, const void* down_exps) {
    int rc = check(h);
    if (rc) return rc;
    if (h->d.num_experts <= 0) return fail(GLC_ERR_STATE, "a dense stage loads layers with glc_stage_load_layer");
    if (!w || !w->attn_norm || !w->wq || !w->wk || !w->wv || !w->wo || !w->ffn_norm || !router || !gate_exps ||
        !up_exps || !down_exps)
        return fail(GLC_ERR_INVALID_ARG, "null weight pointer");
    if (layer < 0 || layer >= h->d.layer_count) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    CUDA_TRY(cudaSetDevice(h->d.device));
    StageLayer& L = h->layers[layer];
    if ((rc = load_attention(h, L, w))) return rc;
    const int E = h->d.num_experts;
    CUDA_TRY(cudaMemcpy(L.router, router, sizeof(float) * h->d.hidden_dim * E, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.egate, gate_exps, h->sz.egu * E, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.eup, up_exps, h->sz.egu * E, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(L.edown, down_exps, h->sz.edown * E, cudaMemcpyHostToDevice));
    L.loaded = true;
    return GLC_OK;
}

int glc_stage_load_io(glc_stage* h, const void* embedding, const float* final_norm, const void* lm_head) {
    int rc = check(h);
    if (rc) return rc;
    CUDA_TRY(cudaSetDevice(h->d.device));
    const size_t tb = (size_t)h->d.vocab * rowbytes(h->d.hidden_dim);
    if (h->d.has_embedding) {
        if (!embedding) return fail(GLC_ERR_INVALID_ARG, "the first stage needs the embedding table");
        CUDA_TRY(cudaMemcpy(h->embed, embedding, tb, cudaMemcpyHostToDevice));
    }
    if (h->d.has_lm_head) {
        if (!final_norm || !lm_head) return fail(GLC_ERR_INVALID_ARG, "the last stage needs the final norm and LM head");
        CUDA_TRY(cudaMemcpy(h->final_norm, final_norm, sizeof(float) * h->d.hidden_dim, cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy(h->lm_head, lm_head, tb, cudaMemcpyHostToDevice));
    }
    return GLC_OK;
}

// The documented synthetic weights of global layer `layer_begin + layer`:
// Q4_K matrices from the seeded generator (sigma_d 0.001; tags
// 200000 + 16 * global_layer + m, m = 0 q, 1 k, 2 v, 3 o, 4 gate, 5 up, 6 down),
// norms 1 + N(0, 0.02) (tags 200007/200008 + 16 * global_layer), biases N(0, 0.02)
// (tag 200009 + 16 * global_layer over the stacked q, k, v rows).
int glc_stage_synth_layer(glc_stage* h, int32_t layer, uint64_t seed) {
    int rc = check(h);
    if (rc) return rc;
    if (layer < 0 || layer >= h->d.layer_count) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    CUDA_TRY(cudaSetDevice(h->d.device));
    StageLayer& L = h->layers[layer];
    const int D = h->d.hidden_dim, FF = h->d.ffn_dim;
    const uint64_t base = 200000ull + 16ull * (uint64_t)(h->d.layer_begin + layer);
    const int nt = 16;
    std::vector<uint8_t> buf(std::max({h->sz.wqkv, h->sz.wo, h->sz.wgu, h->sz.wdown}));  // dense matrices
    const size_t rq = (size_t)h->d.n_heads * kHeadDim, rk = (size_t)h->d.n_kv_heads * kHeadDim;
    glc::synth_q4k(seed, base + 0, 0.001f, buf.data(), rq * rowbytes(D) / 144, nt);
    glc::synth_q4k(seed, base + 1, 0.001f, buf.data() + rq * rowbytes(D), rk * rowbytes(D) / 144, nt);
    glc::synth_q4k(seed, base + 2, 0.001f, buf.data() + (rq + rk) * rowbytes(D), rk * rowbytes(D) / 144, nt);
    CUDA_TRY(cudaMemcpy(L.wqkv, buf.data(), h->sz.wqkv, cudaMemcpyHostToDevice));
    glc::synth_q4k(seed, base + 3, 0.001f, buf.data(), h->sz.wo / 144, nt);
    CUDA_TRY(cudaMemcpy(L.wo, buf.data(), h->sz.wo, cudaMemcpyHostToDevice));
    std::vector<float> v(std::max({(size_t)D, h->sz.qkv_rows, (size_t)D * std::max(h->d.num_experts, 1)}));
    glc::synth_normal(seed, base + 7, 0.02f, v.data(), D, 1);
    for (int i = 0; i < D; ++i) v[i] = 1.0f + v[i];
    CUDA_TRY(cudaMemcpy(L.attn_norm, v.data(), sizeof(float) * D, cudaMemcpyHostToDevice));
    glc::synth_normal(seed, base + 8, 0.02f, v.data(), D, 1);
    for (int i = 0; i < D; ++i) v[i] = 1.0f + v[i];
    CUDA_TRY(cudaMemcpy(L.ffn_norm, v.data(), sizeof(float) * D, cudaMemcpyHostToDevice));
    if (h->d.num_experts > 0) {
        // no q/k/v biases; the router N(0, 0.02) (tag base + 10); expert e's
        // gate / up / down Q4_K (tags 1000000 + 64 global_layer + 3 e + m)
        const int E = h->d.num_experts;
        const uint64_t gl = (uint64_t)(h->d.layer_begin + layer);
        CUDA_TRY(cudaMemset(L.bqkv, 0, sizeof(float) * h->sz.qkv_rows));
        glc::synth_normal(seed, base + 10, 0.02f, v.data(), (size_t)D * E, 1);
        CUDA_TRY(cudaMemcpy(L.router, v.data(), sizeof(float) * D * E, cudaMemcpyHostToDevice));
        std::vector<uint8_t> eb(std::max(h->sz.egu, h->sz.edown));
        for (int e = 0; e < E; ++e) {
            const uint64_t t = 1000000ull + 64ull * gl + 3ull * (uint64_t)e;
            glc::synth_q4k(seed, t + 0, 0.001f, eb.data(), h->sz.egu / 144, nt);
            CUDA_TRY(cudaMemcpy(L.egate + (size_t)e * h->sz.egu, eb.data(), h->sz.egu, cudaMemcpyHostToDevice));
            glc::synth_q4k(seed, t + 1, 0.001f, eb.data(), h->sz.egu / 144, nt);
            CUDA_TRY(cudaMemcpy(L.eup + (size_t)e * h->sz.egu, eb.data(), h->sz.egu, cudaMemcpyHostToDevice));
            glc::synth_q4k(seed, t + 2, 0.001f, eb.data(), h->sz.edown / 144, nt);
            CUDA_TRY(cudaMemcpy(L.edown + (size_t)e * h->sz.edown, eb.data(), h->sz.edown, cudaMemcpyHostToDevice));
        }
        L.loaded = true;
        return GLC_OK;
    }
    glc::synth_q4k(seed, base + 4, 0.001f, buf.data(), h->sz.wgu / 144, nt);
    CUDA_TRY(cudaMemcpy(L.wgate, buf.data(), h->sz.wgu, cudaMemcpyHostToDevice));
    glc::synth_q4k(seed, base + 5, 0.001f, buf.data(), h->sz.wgu / 144, nt);
    CUDA_TRY(cudaMemcpy(L.wup, buf.data(), h->sz.wgu, cudaMemcpyHostToDevice));
    glc::synth_q4k(seed, base + 6, 0.001f, buf.data(), h->sz.wdown / 144, nt);
    CUDA_TRY(cudaMemcpy(L.wdown, buf.data(), h->sz.wdown, cudaMemcpyHostToDevice));
    glc::synth_normal(seed, base + 9, 0.02f, v.data(), h->sz.qkv_rows, 1);
    CUDA_TRY(cudaMemcpy(L.bqkv, v.data(), sizeof(float) * h->sz.qkv_rows, cudaMemcpyHostToDevice));
    (void)FF;
    L.loaded = true;
    return GLC_OK;
}

// Embedding table (tag 300000), final norm 1 + N(0, 0.02) (tag 300001) and
// LM head (tag 300002): Q4_K [vocab][D] with sigma_d 0.001.
int glc_stage_synth_io(glc_stage* h, uint64_t seed) {
    int rc = check(h);
    if (rc) return rc;
    CUDA_TRY(cudaSetDevice(h->d.device));
    const int D = h->d.hidden_dim;
    const size_t tb = (size_t)h->d.vocab * rowbytes(D);
    if (h->d.has_embedding || h->d.has_lm_head) {
        std::vector<uint8_t> buf(tb);
        if (h->d.has_embedding) {
            glc::synth_q4k(seed, 300000, 0.001f, buf.data(), tb / 144, 16);
            CUDA_TRY(cudaMemcpy(h->embed, buf.data(), tb, cudaMemcpyHostToDevice));
        }
        if (h->d.has_lm_head) {
            glc::synth_q4k(seed, 300002, 0.001f, buf.data(), tb / 144, 16);
            CUDA_TRY(cudaMemcpy(h->lm_head, buf.data(), tb, cudaMemcpyHostToDevice));
            std::vector<float> v(D);
            glc::synth_normal(seed, 300001, 0.02f, v.data(), D, 1);
            for (int i = 0; i < D; ++i) v[i] = 1.0f + v[i];
            CUDA_TRY(cudaMemcpy(h->final_norm, v.data(), sizeof(float) * D, cudaMemcpyHostToDevice));
        }
    }
    return GLC_OK;
}

int glc_stage_reset(glc_stage* h) {
    int rc = check(h);
    if (rc) return rc;
    CUDA_TRY(cudaSetDevice(h->d.device));
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    for (auto& L : h->layers) {
        CUDA_TRY(cudaMemset(L.kc, 0, h->sz.cache));
        CUDA_TRY(cudaMemset(L.vc, 0, h->sz.cache));
    }
    return GLC_OK;
}

int glc_stage_forward_dev(glc_stage* h, int32_t pos, const int32_t* token, const float* x_in, float* x_out,
                          float* logits, int32_t* token_out, void* stream) {
    int rc = check(h);
    if (rc) return rc;
    const glc_stage_desc& d = h->d;
    if (pos < 0 || pos >= d.max_len) return fail(GLC_ERR_INVALID_ARG, "pos %d outside [0, %d)", pos, d.max_len);
    for (const auto& L : h->layers)
        if (!L.loaded) return fail(GLC_ERR_STATE, "a layer of the stage has no weights");
    const bool embed = d.has_embedding && !x_in;
    const bool head = d.has_lm_head && (logits || token_out);
    if (!embed && !x_in) return fail(GLC_ERR_INVALID_ARG, "x_in is needed (the stage has no embedding)");
    if (embed && !token) return fail(GLC_ERR_INVALID_ARG, "token is needed (no x_in)");
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    const size_t xb = sizeof(float) * d.hidden_dim;
    // the step's inputs: position, token or activation
    fill_int_kernel<<<1, 1, 0, st>>>(h->pos, pos);
    CUDA_TRY(cudaGetLastError());
    if (embed) CUDA_TRY(cudaMemcpyAsync(h->token, token, sizeof(int), cudaMemcpyDeviceToDevice, st));
    else CUDA_TRY(cudaMemcpyAsync(h->x, x_in, xb, cudaMemcpyDeviceToDevice, st));
    // the layers: one captured graph per (embed, head) variant, replayed
    cudaGraphExec_t& g = h->graphs[(embed ? 1 : 0) | (head ? 2 : 0)];
    if (!g) {
        // first use of the variant: eager once (function attributes, opt-in
        // shared memory), then capture it for the next calls
        rc = stage_step(h, embed, head, st);
        if (rc) return rc;
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int crc = stage_step(h, embed, head, st);
            if (cudaStreamEndCapture(st, &graph) != cudaSuccess || crc != GLC_OK ||
                cudaGraphInstantiate(&g, graph, 0) != cudaSuccess)
                g = nullptr;
            if (graph) cudaGraphDestroy(graph);
        }
        cudaGetLastError();
        // the eager step above already produced this call's outputs
    } else {
        CUDA_TRY(cudaGraphLaunch(g, st));
    }
    if (x_out) CUDA_TRY(cudaMemcpyAsync(x_out, h->x, xb, cudaMemcpyDeviceToDevice, st));
    if (head && logits) CUDA_TRY(cudaMemcpyAsync(logits, h->logits, sizeof(float) * d.vocab, cudaMemcpyDeviceToDevice, st));
    if (head && token_out) CUDA_TRY(cudaMemcpyAsync(token_out, h->token, sizeof(int), cudaMemcpyDeviceToDevice, st));
    return GLC_OK;
}

int glc_stage_read_kv_cache(glc_stage* h, int32_t layer, int32_t rows, void* k_out, void* v_out) {
    int rc = check(h);
    if (rc) return rc;
    if (!k_out || !v_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (layer < 0 || layer >= h->d.layer_count) return fail(GLC_ERR_INVALID_ARG, "layer %d out of range", layer);
    if (rows < 0 || rows > h->d.max_len) return fail(GLC_ERR_INVALID_ARG, "rows %d outside 0..%d", rows, h->d.max_len);
    if (rows == 0) return GLC_OK;
    CUDA_TRY(cudaSetDevice(h->d.device));
    CUDA_TRY(cudaStreamSynchronize(h->stream));
    const size_t rowb = (size_t)kHeadDim * sizeof(uint16_t);
    const StageLayer& L = h->layers[layer];
    CUDA_TRY(cudaMemcpy2D(k_out, rows * rowb, L.kc, (size_t)h->d.max_len * rowb, rows * rowb, h->d.n_kv_heads,
                          cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy2D(v_out, rows * rowb, L.vc, (size_t)h->d.max_len * rowb, rows * rowb, h->d.n_kv_heads,
                          cudaMemcpyDeviceToHost));
    return GLC_OK;
}

int glc_stage_poll_error(glc_stage* h) {
    int rc = check(h);
    if (rc) return rc;
    int code = 0;
    CUDA_TRY(cudaMemcpy(&code, h->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code) {
        // a wait that gave up leaves the chains' barrier counter short of a whole instance
        cudaDeviceSynchronize();
        cudaMemset(h->err, 0, sizeof(int) * 8);
        cudaMemset(h->bar, 0, sizeof(unsigned long long));
        return fail(code == glc::kDevBadArg ? GLC_ERR_INVALID_ARG : GLC_ERR_TIMEOUT, "device code %d", code);
    }
    return GLC_OK;
}

}  // extern "C"
