/*
 * glc_oracle.c -- CPU oracle for the quantized MoE feed-forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see glc_oracle.h).  Built with -ffp-contract=off
 * so that every multiply and add below is rounded exactly where it is written;
 * fmaf() is used only where the canonical order calls for a fused step.
 *
 * Parity status:
 *   - wire codecs and header: pinned by the reference's own tests
 *     (DynamicMultiPrecisionWireTests.cs, PhaseBDistributedRemediationTests.cs,
 *     FusedZeroAllocationTransportTests.cs; fixtures in tests/golden/).
 *   - RMSNorm and combine: pinned by DistributedPipelineTests.cs:76-139.
 *   - Q4_K dequant / GEMV: the reference's implementation is in the missing
 *     Glacier.Inference 1.3.2 package and no reference test covers Q4_K, so it
 *     is pinned by known-answer super-blocks built from the published format
 *     (tests/golden/q4k_known_answers.json), not by reference outputs.
 *   - Router: no reference code or test; canonical order defined here and by
 *     the product's router kernel.
 */
#include "glc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define GAMMA 0x9E3779B97F4A7C15ULL

/* ------------------------------------------------------------------------ */
/* Seeded generator: SplitMix64 output function, random access by index.     */
/* ------------------------------------------------------------------------ */
uint64_t oc_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
uint64_t oc_stream_seed(uint64_t seed, uint64_t tag) { return oc_mix64(seed + GAMMA * (tag + 1)); }
uint64_t oc_draw(uint64_t stream, uint64_t i) { return oc_mix64(stream + GAMMA * (i + 1)); }
float oc_uniform(uint64_t stream, uint64_t i) {
    return ((float)(oc_draw(stream, i) >> 40) + 0.5f) * 5.9604644775390625e-8f;
}
float oc_normal(uint64_t stream, uint64_t i) {
    float u1 = oc_uniform(stream, 2 * i);
    float u2 = oc_uniform(stream, 2 * i + 1);
    double r = sqrt(-2.0 * log((double)u1));
    double th = 6.283185307179586 * (double)u2;
    return (float)(r * cos(th));
}
void oc_fill_normal(uint64_t seed, uint64_t tag, float sigma, float* out, size_t n) {
    uint64_t s = oc_stream_seed(seed, tag);
    for (size_t i = 0; i < n; i++) out[i] = sigma * oc_normal(s, i);
}
uint64_t oc_expert_tag(int expert, int matrix) { return 1000ULL + 4ULL * (uint64_t)expert + (uint64_t)matrix; }

/* Q4_K super-block b of a matrix stream: d, dmin = fp16(|sigma_d * N(0,1)|);
 * the 140 bytes of scales[12] and qs[128] are uniform random bytes, which makes
 * every 6-bit sub-scale / sub-min uniform on 0..63 and every quant uniform on
 * 0..15 (all 96 scale bits and all 1024 quant bits are used by the format). */
void oc_synth_q4k(uint64_t seed, uint64_t tag, float sigma_d, uint8_t* out, size_t n_blocks) {
    uint64_t s = oc_stream_seed(seed, tag);
    uint64_t sbytes = oc_mix64(s ^ 0xD1B54A32D192ED03ULL);
    for (size_t b = 0; b < n_blocks; b++) {
        uint8_t* blk = out + b * 144;
        uint16_t d = oc_f32_to_f16(fabsf(sigma_d * oc_normal(s, 2 * b)));
        uint16_t dm = oc_f32_to_f16(fabsf(sigma_d * oc_normal(s, 2 * b + 1)));
        blk[0] = (uint8_t)d; blk[1] = (uint8_t)(d >> 8);
        blk[2] = (uint8_t)dm; blk[3] = (uint8_t)(dm >> 8);
        uint8_t tmp[144];
        for (int j = 0; j < 18; j++) {
            uint64_t v = oc_draw(sbytes, 18 * b + j);
            for (int t = 0; t < 8; t++) tmp[8 * j + t] = (uint8_t)(v >> (8 * t));
        }
        memcpy(blk + 4, tmp, 140);
    }
}

/* ------------------------------------------------------------------------ */
/* IEEE binary16, round to nearest even (own implementation of the format).  */
/* ------------------------------------------------------------------------ */
uint16_t oc_f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(man ? (sign | 0x7E00u | (man >> 13)) : (sign | 0x7C00u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}
float oc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) x = sign;
        else {
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        x = sign | 0x7F800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f; memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------ */
/* Q4_K (GGUF): 256 weights per 144-byte super-block:                        */
/*   [0:2) d fp16, [2:4) dmin fp16, [4:16) scales (8 x 6-bit sc, 8 x 6-bit m),*/
/*   [16:144) qs: 4 chunks of 32 bytes; chunk c low nibbles = weights         */
/*   64c..64c+31 (sub-block 2c), high nibbles = 64c+32..64c+63 (2c+1).        */
/*   weight = (d*sc_j)*q - (dmin*m_j).                                         */
/* ------------------------------------------------------------------------ */
void oc_q4k_get_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static void q4k_dequant_block(const uint8_t* blk, float* y) {
    float d = oc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
    float dmin = oc_f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
    const uint8_t* scales = blk + 4;
    const uint8_t* q = blk + 16;
    for (int c = 0; c < 4; c++) {
        uint8_t s1, m1, s2, m2;
        oc_q4k_get_scale_min(2 * c, scales, &s1, &m1);
        oc_q4k_get_scale_min(2 * c + 1, scales, &s2, &m2);
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        float d2 = d * (float)s2, mm2 = dmin * (float)m2;
        for (int l = 0; l < 32; l++) {
            y[64 * c + l] = d1 * (float)(q[32 * c + l] & 0xF) - mm1;
            y[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - mm2;
        }
    }
}

void oc_q4k_dequant(const uint8_t* blocks, size_t n_weights, float* out) {
    for (size_t b = 0; b < n_weights / 256; b++) q4k_dequant_block(blocks + 144 * b, out + 256 * b);
}

/* ------------------------------------------------------------------------ */
/* parallel-for over rows (results do not depend on the thread count: every  */
/* row is computed by one thread in a fixed order).                          */
/* ------------------------------------------------------------------------ */
static int g_threads = 1;
void oc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

typedef void (*row_fn)(void* ctx, int r0, int r1);
typedef struct { row_fn fn; void* ctx; int r0, r1; } par_job;
static void* par_entry(void* p) { par_job* j = (par_job*)p; j->fn(j->ctx, j->r0, j->r1); return NULL; }
static void parallel_rows(row_fn fn, void* ctx, int n, int nthreads) {
    if (nthreads <= 1 || n < 2 * nthreads) { fn(ctx, 0, n); return; }
    pthread_t th[256];
    par_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].r0 = (int)((long long)n * t / nthreads);
        jobs[t].r1 = (int)((long long)n * (t + 1) / nthreads);
        if (t > 0) pthread_create(&th[t], NULL, par_entry, &jobs[t]);
    }
    par_entry(&jobs[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* Parity GEMV: the reference test's scalar oracle shape
 * (Qwen38FlashNextDistributedLoadTests.cs:71-75): fp32 dequantized weight,
 * fp32 product, double accumulation, one rounding to fp32 at the end. */
typedef struct { const uint8_t* W; const float* x; float* y; int K; } gemv_ctx;
static void gemv_rows(void* p, int r0, int r1) {
    gemv_ctx* c = (gemv_ctx*)p;
    size_t rb = (size_t)(c->K / 256) * 144;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)c->K);
    for (int r = r0; r < r1; r++) {
        oc_q4k_dequant(c->W + rb * (size_t)r, (size_t)c->K, tmp);
        double dot = 0.0;
        for (int k = 0; k < c->K; k++) dot += (double)(tmp[k] * c->x[k]);
        c->y[r] = (float)dot;
    }
    free(tmp);
}
void oc_q4k_gemv(const uint8_t* W, const float* x, float* y, int K, int N) {
    gemv_ctx c = {W, x, y, K};
    parallel_rows(gemv_rows, &c, N, g_threads);
}

/* SwiGLU: act = silu(gate) * up = gate / (1 + e^-gate) * up   (QuantKernels.SwiGLU,
 * CpuWarmExpertPoolWorker.cs:325). */
void oc_swiglu(const float* g, const float* u, float* act, int n) {
    for (int i = 0; i < n; i++) act[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

/* ExecuteExpertSwiGlu (CpuWarmExpertPoolWorker.cs:281-344): gate, up, SwiGLU, down. */
void oc_expert_forward(const uint8_t* w1, const uint8_t* w3, const uint8_t* w2, int D, int F,
                       const float* x, float* y) {
    float* g = (float*)malloc(sizeof(float) * (size_t)F);
    float* u = (float*)malloc(sizeof(float) * (size_t)F);
    float* a = (float*)malloc(sizeof(float) * (size_t)F);
    oc_q4k_gemv(w1, x, g, D, F);
    oc_q4k_gemv(w3, x, u, D, F);
    oc_swiglu(g, u, a, F);
    oc_q4k_gemv(w2, a, y, F, D);
    free(g); free(u); free(a);
}

/* ------------------------------------------------------------------------ */
/* Canonical fp32 reduction shared with the product's kernels: 256 strided   */
/* partials p[t] = fmaf(x[d], w[d*stride], p[t]) for d = t, t+256, ..., then */
/* a xor-butterfly inside each warp of 32 (16,8,4,2,1) and a pairwise tree   */
/* over the 8 warp sums: ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).                */
/* ------------------------------------------------------------------------ */
static float reduce256(float* p) {
    float s[8];
    for (int w = 0; w < 8; w++) {
        float v[32];
        for (int i = 0; i < 32; i++) v[i] = p[32 * w + i];
        for (int off = 16; off >= 1; off >>= 1) {
            float nv[32];
            for (int i = 0; i < 32; i++) nv[i] = v[i] + v[i ^ off];
            memcpy(v, nv, sizeof(v));
        }
        s[w] = v[0];
    }
    return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}
float oc_dot_canonical(const float* x, const float* w, int D, int stride) {
    float p[256];
    for (int t = 0; t < 256; t++) {
        float acc = 0.0f;
        for (int d = t; d < D; d += 256) acc = fmaf(x[d], w[(size_t)d * stride], acc);
        p[t] = acc;
    }
    return reduce256(p);
}

/* RMSNorm without learned weight, eps 1e-5 (StageWorkers.cs:89-91):
 * rms = 1 / sqrt(sumSq / D + 1e-5); y = x * rms.  sumSq uses the canonical
 * reduction (x_d * x_d fused into the partials). */
void oc_rmsnorm(const float* x, float* y, int D) {
    float p[256];
    for (int t = 0; t < 256; t++) {
        float acc = 0.0f;
        for (int d = t; d < D; d += 256) acc = fmaf(x[d], x[d], acc);
        p[t] = acc;
    }
    float ss = reduce256(p);
    float rms = 1.0f / sqrtf(ss / (float)D + 1e-5f);
    for (int d = 0; d < D; d++) y[d] = x[d] * rms;
}

/* Router gate GEMV: logits[e] = sum_d x[d] * Wr[d][e] (Wr row-major D x E). */
void oc_router_logits(const float* x, const float* Wr, int D, int E, float* logits) {
    for (int e = 0; e < E; e++) logits[e] = oc_dot_canonical(x, Wr + e, D, E);
}

/* top-k on logits (descending; ties -> lower expert index; NaN ranks as -inf),
 * then softmax weights: renorm=1 -> softmax over the k selected logits
 * (softmax -> top-k -> renormalise), renorm=0 -> full softmax probabilities. */
void oc_router_topk(const float* logits, int E, int k, int renorm, int32_t* ids, float* w) {
    unsigned char taken[4096];
    memset(taken, 0, (size_t)E);
    for (int j = 0; j < k; j++) {
        int best = -1; float bv = 0.0f;
        for (int e = 0; e < E; e++) {
            if (taken[e]) continue;
            float v = isnan(logits[e]) ? -INFINITY : logits[e];
            if (best < 0 || v > bv) { best = e; bv = v; }
        }
        taken[best] = 1;
        ids[j] = best;
    }
    float mx = isnan(logits[ids[0]]) ? -INFINITY : logits[ids[0]];
    float den = 0.0f;
    if (renorm) {
        for (int j = 0; j < k; j++) den += expf(logits[ids[j]] - mx);
    } else {
        for (int e = 0; e < E; e++) den += expf(logits[e] - mx);
    }
    for (int j = 0; j < k; j++) w[j] = expf(logits[ids[j]] - mx) / den;
}

/* token->expert dispatch plan over P = T*k (token, slot) pairs: counts per
 * expert, exclusive offsets (E+1), and a stable permutation grouping pairs by
 * expert in ascending pair order; inv[p] = position of pair p. */
void oc_dispatch_plan(const int32_t* ids, int P, int E, int32_t* counts, int32_t* offsets,
                      int32_t* perm, int32_t* inv) {
    for (int e = 0; e < E; e++) counts[e] = 0;
    for (int p = 0; p < P; p++) counts[ids[p]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; e++) offsets[e + 1] = offsets[e] + counts[e];
    int32_t* run = (int32_t*)calloc((size_t)E, sizeof(int32_t));
    for (int p = 0; p < P; p++) {
        int e = ids[p];
        int pos = offsets[e] + run[e]++;
        perm[pos] = p;
        inv[p] = pos;
    }
    free(run);
}

/* combine step acc = (y * w) + acc, unfused, as TensorPrimitives.MultiplyAdd
 * (StageWorkers.cs:159). */
static void axpy_unfused(float* acc, const float* y, float w, int n) {
    for (int i = 0; i < n; i++) { float t = y[i] * w; acc[i] = t + acc[i]; }
}

/* ProcessRoutedTopK (GpuFirstExpertStageWorker.cs:416-583): output cleared,
 * then accumulated in k order; expert ids clamped to [0, E); no residual,
 * no RMSNorm; empty selection -> zeros. */
void oc_routed_topk(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    int D, int F, int E, const float* x, const int32_t* ids, const float* w,
                    int k, float* out) {
    size_t gsl = (size_t)F * (size_t)(D / 256) * 144, dsl = (size_t)D * (size_t)(F / 256) * 144;
    float* y = (float*)malloc(sizeof(float) * (size_t)D);
    memset(out, 0, sizeof(float) * (size_t)D);
    for (int j = 0; j < k; j++) {
        int e = ids[j] < 0 ? 0 : (ids[j] >= E ? E - 1 : ids[j]);
        oc_expert_forward(gate_exps + gsl * e, up_exps + gsl * e, down_exps + dsl * e, D, F, x, y);
        axpy_unfused(out, y, w[j], D);
    }
    free(y);
}

/* Full MoE layer over T tokens:
 *   flags bit0 (RMSNORM): xin = RMSNorm(x) (AttentionRootStageWorker) else xin = x
 *   logits = xin . Wr, top-k + softmax weights
 *   acc = flags bit1 (RESIDUAL) ? x : 0       (DistributedPipelineCoordinator.cs:104-113)
 *   acc = (y_j * w_j) + acc for j = 0..k-1      (:116-134)
 *   shared expert (Fs > 0): acc = (ys * sigmoid(xin . g)) + acc
 */
void oc_moe_forward(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    const float* router_w, const uint8_t* sh_gate, const uint8_t* sh_up,
                    const uint8_t* sh_down, const float* sh_gate_vec, int D, int F, int E, int k,
                    int Fs, int renorm, int flags, const float* x, int T, float* out,
                    int32_t* ids_out, float* w_out) {
    size_t gsl = (size_t)F * (size_t)(D / 256) * 144, dsl = (size_t)D * (size_t)(F / 256) * 144;
    float* xin = (float*)malloc(sizeof(float) * (size_t)D);
    float* y = (float*)malloc(sizeof(float) * (size_t)D);
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * D;
        float* ot = out + (size_t)t * D;
        if (flags & 1) oc_rmsnorm(xt, xin, D); else memcpy(xin, xt, sizeof(float) * (size_t)D);
        oc_router_logits(xin, router_w, D, E, logits);
        int32_t* ids = ids_out + (size_t)t * k;
        float* w = w_out + (size_t)t * k;
        oc_router_topk(logits, E, k, renorm, ids, w);
        if (flags & 2) memcpy(ot, xt, sizeof(float) * (size_t)D); else memset(ot, 0, sizeof(float) * (size_t)D);
        for (int j = 0; j < k; j++) {
            int e = ids[j];
            oc_expert_forward(gate_exps + gsl * e, up_exps + gsl * e, down_exps + dsl * e, D, F, xin, y);
            axpy_unfused(ot, y, w[j], D);
        }
        if (Fs > 0) {
            float s = oc_dot_canonical(xin, sh_gate_vec, D, 1);
            float sg = 1.0f / (1.0f + expf(-s));
            oc_expert_forward(sh_gate, sh_up, sh_down, D, Fs, xin, y);
            axpy_unfused(ot, y, sg, D);
        }
    }
    free(xin); free(y); free(logits);
}

/* ------------------------------------------------------------------------ */
/* Timed CPU port: the reference CPU path's shape (one expert at a time:     */
/* gate GEMV, up GEMV, SwiGLU, down GEMV; k-ordered combine), with the       */
/* mat-vec written the way a SIMD CPU kernel does it: one super-block is     */
/* dequantized to fp32 and dotted with 8 independent fp32 accumulators,      */
/* rows split over nthreads threads (CpuWarmExpertPoolWorker multithreaded). */
/* ------------------------------------------------------------------------ */
typedef struct { const uint8_t* W; const float* x; float* y; int K; } fgemv_ctx;
static void fgemv_rows(void* p, int r0, int r1) {
    fgemv_ctx* c = (fgemv_ctx*)p;
    int nsb = c->K / 256;
    size_t rb = (size_t)nsb * 144;
    float tmp[256];
    for (int r = r0; r < r1; r++) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const uint8_t* row = c->W + rb * (size_t)r;
        for (int b = 0; b < nsb; b++) {
            q4k_dequant_block(row + 144 * b, tmp);
            const float* xb = c->x + 256 * b;
            for (int i = 0; i < 256; i += 8)
                for (int l = 0; l < 8; l++) acc[l] += tmp[i + l] * xb[i + l];
        }
        c->y[r] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    }
}
static void fgemv(const uint8_t* W, const float* x, float* y, int K, int N, int nthreads) {
    fgemv_ctx c = {W, x, y, K};
    parallel_rows(fgemv_rows, &c, N, nthreads);
}
void oc_cpu_expert_forward_fast(const uint8_t* w1, const uint8_t* w3, const uint8_t* w2, int D,
                                int F, const float* x, float* y, int nthreads) {
    float* g = (float*)malloc(sizeof(float) * (size_t)F);
    float* u = (float*)malloc(sizeof(float) * (size_t)F);
    float* a = (float*)malloc(sizeof(float) * (size_t)F);
    fgemv(w1, x, g, D, F, nthreads);
    fgemv(w3, x, u, D, F, nthreads);
    oc_swiglu(g, u, a, F);
    fgemv(w2, a, y, F, D, nthreads);
    free(g); free(u); free(a);
}
void oc_cpu_moe_token_fast(const uint8_t* gate_exps, const uint8_t* up_exps,
                           const uint8_t* down_exps, const float* router_w, int D, int F, int E,
                           int k, int renorm, int flags, const float* x, float* out, int nthreads) {
    size_t gsl = (size_t)F * (size_t)(D / 256) * 144, dsl = (size_t)D * (size_t)(F / 256) * 144;
    float* xin = (float*)malloc(sizeof(float) * (size_t)D);
    float* y = (float*)malloc(sizeof(float) * (size_t)D);
    float logits[256];
    int32_t ids[64];
    float w[64];
    if (flags & 1) oc_rmsnorm(x, xin, D); else memcpy(xin, x, sizeof(float) * (size_t)D);
    oc_router_logits(xin, router_w, D, E, logits);
    oc_router_topk(logits, E, k, renorm, ids, w);
    if (flags & 2) memcpy(out, x, sizeof(float) * (size_t)D); else memset(out, 0, sizeof(float) * (size_t)D);
    for (int j = 0; j < k; j++) {
        int e = ids[j];
        oc_cpu_expert_forward_fast(gate_exps + gsl * e, up_exps + gsl * e, down_exps + dsl * e, D, F,
                                   xin, y, nthreads);
        axpy_unfused(out, y, w[j], D);
    }
    free(xin); free(y);
}
/* The same token with a Qwen2-MoE shared expert (Fs rows, sigmoid gate over
 * the normalised input) after the routed experts: out += sigmoid(xin.g) * y_s,
 * the routed part as above (CPU port, rows split over nthreads). */
void oc_cpu_moe_token_shared_fast(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                                  const float* router_w, const uint8_t* sh_gate, const uint8_t* sh_up,
                                  const uint8_t* sh_down, const float* sh_gate_vec, int D, int F, int E, int k,
                                  int Fs, int renorm, int flags, const float* x, float* out, int nthreads) {
    oc_cpu_moe_token_fast(gate_exps, up_exps, down_exps, router_w, D, F, E, k, renorm, flags, x, out, nthreads);
    float* xin = (float*)malloc(sizeof(float) * (size_t)D);
    float* y = (float*)malloc(sizeof(float) * (size_t)D);
    if (flags & 1) oc_rmsnorm(x, xin, D); else memcpy(xin, x, sizeof(float) * (size_t)D);
    const float s = oc_dot_canonical(xin, sh_gate_vec, D, 1);
    const float sg = 1.0f / (1.0f + expf(-s));
    oc_cpu_expert_forward_fast(sh_gate, sh_up, sh_down, D, Fs, xin, y, nthreads);
    axpy_unfused(out, y, sg, D);
    free(xin); free(y);
}

/* ------------------------------------------------------------------------ */
/* Wire codecs (QuantizationKernels.cs).                                     */
/* ------------------------------------------------------------------------ */
int oc_wire_token_bytes(int mode, int dim) {
    switch (mode) {  /* GetPackedTokenBytes, QuantizationKernels.cs:57-67 */
        case 0: return dim * 4;
        case 1: return dim * 2;
        case 2: return dim + 4;
        case 3: return dim + 4;
        default: return dim * 2;
    }
}
static void put_f32(uint8_t* p, float f) { uint32_t u; memcpy(&u, &f, 4); for (int i = 0; i < 4; i++) p[i] = (uint8_t)(u >> (8 * i)); }
static float get_f32(const uint8_t* p) { uint32_t u = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); float f; memcpy(&f, &u, 4); return f; }

/* FindMaxAbsolute (:212-216): |MaxMagnitude(x)|, NaN propagates, empty -> 0. */
static float max_abs(const float* x, int n) {
    float m = 0.0f; int nan = 0;
    for (int i = 0; i < n; i++) { float a = fabsf(x[i]); if (isnan(a)) nan = 1; else if (a > m) m = a; }
    return nan ? NAN : m;
}
/* QuantizeInt8Symmetric (:222-474): [f32 scale LE][n x int8]. */
float oc_quantize_int8(const float* x, int n, uint8_t* dst) {
    float mx = max_abs(x, n);
    int8_t* q = (int8_t*)(dst + 4);
    if (!isfinite(mx) || mx < 1e-10f) { memset(q, 0, (size_t)n); put_f32(dst, 1.0f); return 1.0f; }
    float scale = mx / 127.0f;
    float inv = 127.0f / mx;
    if (!isfinite(scale) || !isfinite(inv) || scale <= 0.0f) { memset(q, 0, (size_t)n); put_f32(dst, 1.0f); return 1.0f; }
    for (int i = 0; i < n; i++) {
        float v = x[i] * inv;
        float r = rintf(v);              /* round half to even (default rounding mode) */
        if (r > 127.0f) r = 127.0f;
        if (r < -127.0f) r = -127.0f;
        q[i] = (int8_t)r;
    }
    put_f32(dst, scale);
    return scale;
}
/* DequantizeInt8Symmetric (:479-586): x = q * scale, non-finite scale -> zeros. */
void oc_dequantize_int8(const uint8_t* src, int n, float* out) {
    float scale = get_f32(src);
    const int8_t* q = (const int8_t*)(src + 4);
    if (!isfinite(scale)) { memset(out, 0, sizeof(float) * (size_t)n); return; }
    for (int i = 0; i < n; i++) out[i] = (float)q[i] * scale;
}
/* FloatToFp8E4M3 (:688-736). */
uint8_t oc_float_to_fp8_e4m3(float val) {
    uint32_t bits; memcpy(&bits, &val, 4);
    uint8_t sign = (uint8_t)((bits >> 24) & 0x80u);
    uint32_t ab = bits & 0x7FFFFFFFu;
    if (ab == 0 || ab > 0x7F800000u) return 0x00;
    if (ab >= 0x43E00000u) return (uint8_t)(sign | 0x7E);
    if (ab < 0x3C800000u) {
        float av; memcpy(&av, &ab, 4);
        int sub = (int)rintf(av * 512.0f);
        if (sub <= 0) return sign;
        if (sub >= 8) return (uint8_t)(sign | 0x08);
        return (uint8_t)(sign | sub);
    }
    int e4 = (int)(ab >> 23) - (127 - 7);
    uint32_t m23 = ab & 0x7FFFFFu;
    uint32_t m3 = m23 >> 20;
    uint32_t rem = m23 & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (m3 & 1u))) {
        m3++;
        if (m3 >= 8u) { m3 = 0; e4++; }
    }
    if (e4 >= 15 && m3 >= 7u) { e4 = 15; m3 = 6u; }
    return (uint8_t)(sign | (e4 << 3) | (int)m3);
}
/* E4M3FN decode table entry (:23-51): NaN (0x7F/0xFF) -> 0. */
float oc_fp8_e4m3_to_float(uint8_t b) {
    float sign = (b & 0x80) ? -1.0f : 1.0f;
    int exp = (b >> 3) & 0x0F, mant = b & 0x07;
    if (exp == 15 && mant == 7) return 0.0f;
    if (exp == 0) return sign * ((float)mant / 512.0f);
    return sign * (ldexpf(1.0f, exp - 7) * (1.0f + (float)mant / 8.0f));
}
float oc_quantize_fp8(const float* x, int n, uint8_t* dst) {
    float mx = max_abs(x, n);
    uint8_t* q = dst + 4;
    if (!isfinite(mx) || mx < 1e-10f) { memset(q, 0, (size_t)n); put_f32(dst, 1.0f); return 1.0f; }
    float scale = mx / 448.0f;
    float inv = 448.0f / mx;
    if (!isfinite(scale) || !isfinite(inv) || scale <= 0.0f) { memset(q, 0, (size_t)n); put_f32(dst, 1.0f); return 1.0f; }
    for (int i = 0; i < n; i++) q[i] = oc_float_to_fp8_e4m3(x[i] * inv);
    put_f32(dst, scale);
    return scale;
}
void oc_dequantize_fp8(const uint8_t* src, int n, float* out) {
    float scale = get_f32(src);
    if (!isfinite(scale)) { memset(out, 0, sizeof(float) * (size_t)n); return; }
    for (int i = 0; i < n; i++) out[i] = oc_fp8_e4m3_to_float(src[4 + i]) * scale;
}
int oc_wire_quantize(int mode, const float* x, int T, int D, uint8_t* out) {
    int tb = oc_wire_token_bytes(mode, D);
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * D;
        uint8_t* o = out + (size_t)t * tb;
        switch (mode) {
            case 0: memcpy(o, xt, sizeof(float) * (size_t)D); break;
            case 2: oc_quantize_int8(xt, D, o); break;
            case 3: oc_quantize_fp8(xt, D, o); break;
            default:
                for (int i = 0; i < D; i++) { uint16_t h = oc_f32_to_f16(xt[i]); o[2 * i] = (uint8_t)h; o[2 * i + 1] = (uint8_t)(h >> 8); }
        }
    }
    return T * tb;
}
int oc_wire_dequantize(int mode, const uint8_t* in, int T, int D, float* out) {
    int tb = oc_wire_token_bytes(mode, D);
    for (int t = 0; t < T; t++) {
        const uint8_t* s = in + (size_t)t * tb;
        float* o = out + (size_t)t * D;
        switch (mode) {
            case 0: memcpy(o, s, sizeof(float) * (size_t)D); break;
            case 2: oc_dequantize_int8(s, D, o); break;
            case 3: oc_dequantize_fp8(s, D, o); break;
            default:
                for (int i = 0; i < D; i++) o[i] = oc_f16_to_f32((uint16_t)(s[2 * i] | (s[2 * i + 1] << 8)));
        }
    }
    return T * tb;
}

/* ------------------------------------------------------------------------ */
/* FusedActivationHeader (FusedActivationHeader.cs:41-171), 32 bytes LE.     */
/* ------------------------------------------------------------------------ */
void oc_header_write(uint64_t seq, int32_t token, int32_t layer, int32_t dim, uint8_t prec,
                     uint8_t flags, uint16_t batch, float scale, uint8_t* o) {
    uint32_t magic = 0x47414354u;
    for (int i = 0; i < 4; i++) o[i] = (uint8_t)(magic >> (8 * i));
    for (int i = 0; i < 8; i++) o[4 + i] = (uint8_t)(seq >> (8 * i));
    for (int i = 0; i < 4; i++) o[12 + i] = (uint8_t)((uint32_t)token >> (8 * i));
    for (int i = 0; i < 4; i++) o[16 + i] = (uint8_t)((uint32_t)layer >> (8 * i));
    for (int i = 0; i < 4; i++) o[20 + i] = (uint8_t)((uint32_t)dim >> (8 * i));
    o[24] = prec;
    o[25] = flags;
    o[26] = (uint8_t)batch; o[27] = (uint8_t)(batch >> 8);
    put_f32(o + 28, scale);
}
static uint32_t get_u32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
int oc_header_read(const uint8_t* in, uint64_t* seq, int32_t* token, int32_t* layer, int32_t* dim,
                   uint8_t* prec, uint8_t* flags, uint16_t* batch, float* scale) {
    if (get_u32(in) != 0x47414354u) return -1;
    *seq = (uint64_t)get_u32(in + 4) | ((uint64_t)get_u32(in + 8) << 32);
    *token = (int32_t)get_u32(in + 12);
    *layer = (int32_t)get_u32(in + 16);
    *dim = (int32_t)get_u32(in + 20);
    *prec = in[24];
    *flags = in[25];
    *batch = (uint16_t)(in[26] | (in[27] << 8));
    *scale = get_f32(in + 28);
    return 0;
}
/* GetPayloadByteCount (:109-125). */
int oc_header_payload_bytes(const uint8_t* in) {
    int dim = (int32_t)get_u32(in + 20);
    uint16_t batch = (uint16_t)(in[26] | (in[27] << 8));
    int tokens = batch > 0 ? batch : 1;
    if (in[25] & 0x10) return tokens * 4;
    switch (in[24]) {
        case 0: return dim * tokens * 4;
        case 1: return dim * tokens * 2;
        case 2: return (dim + 4) * tokens;
        case 3: return (dim + 4) * tokens;
        default: return dim * tokens * 2;
    }
}
