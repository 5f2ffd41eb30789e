/*
 * glc_oracle.h -- CPU oracle for the quantized MoE feed-forward hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library and its
 * host bindings) links, loads or calls this code.  It is used by tests/ as the
 * CPU reference of the parity tests, by __graft_entry__.smoke() to verify one
 * small GPU run, and by bench.py's CPU-baseline leg as the timed CPU port of
 * the reference's CPU path.
 *
 * The reference (Glacier.Inference.Distributed, C# / .NET 10) cannot be built
 * or run here (no .NET SDK; its Q4_K mat-vec, SwiGLU and router live in the
 * un-vendored NuGet package Glacier.Inference 1.3.2).  This file restates:
 *   - CpuWarmExpertPoolWorker.ExecuteExpertSwiGlu   (CpuWarmExpertPoolWorker.cs:281-344)
 *   - DistributedPipelineCoordinator.ExecuteStep    (DistributedPipelineCoordinator.cs:72-137)
 *   - AttentionRootStageWorker RMSNorm              (StageWorkers.cs:86-91)
 *   - AccumulatorStageWorker combine / residual     (StageWorkers.cs:152-173)
 *   - GpuFirstExpertStageWorker.ProcessRoutedTopK   (GpuFirstExpertStageWorker.cs:416-583)
 *   - QuantizationKernels wire codecs (bit-exact)   (Protocol/QuantizationKernels.cs:57-736)
 *   - FusedActivationHeader byte layout             (Protocol/FusedActivationHeader.cs:41-218)
 * and the published GGUF Q4_K super-block format (the external
 * QuantKernels.MatVecMul called at CpuWarmExpertPoolWorker.cs:379).
 */
#ifndef GLC_ORACLE_H
#define GLC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (same documented generator as the product) ---- */
uint64_t oc_mix64(uint64_t z);
uint64_t oc_stream_seed(uint64_t seed, uint64_t tag);
uint64_t oc_draw(uint64_t stream, uint64_t i);
float oc_uniform(uint64_t stream, uint64_t i);
float oc_normal(uint64_t stream, uint64_t i);
void oc_fill_normal(uint64_t seed, uint64_t tag, float sigma, float* out, size_t n);
void oc_synth_q4k(uint64_t seed, uint64_t tag, float sigma_d, uint8_t* out, size_t n_blocks);
uint64_t oc_expert_tag(int expert, int matrix);

/* ---- IEEE binary16 ---- */
uint16_t oc_f32_to_f16(float f);
float oc_f16_to_f32(uint16_t h);

/* ---- Q4_K ---- */
void oc_q4k_get_scale_min(int j, const uint8_t* scales, uint8_t* sc, uint8_t* m);
void oc_q4k_dequant(const uint8_t* blocks, size_t n_weights, float* out);
void oc_q4k_gemv(const uint8_t* W, const float* x, float* y, int K, int N);

/* ---- expert / layer math ---- */
void oc_set_threads(int n);
void oc_swiglu(const float* g, const float* u, float* act, int n);
void oc_expert_forward(const uint8_t* w1, const uint8_t* w3, const uint8_t* w2, int D, int F,
                       const float* x, float* y);
void oc_rmsnorm(const float* x, float* y, int D);
float oc_dot_canonical(const float* x, const float* w, int D, int stride);
void oc_router_logits(const float* x, const float* Wr, int D, int E, float* logits);
void oc_router_topk(const float* logits, int E, int k, int renorm, int32_t* ids, float* w);
void oc_dispatch_plan(const int32_t* ids, int P, int E, int32_t* counts, int32_t* offsets,
                      int32_t* perm, int32_t* inv);
void oc_routed_topk(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    int D, int F, int E, const float* x, const int32_t* ids, const float* w,
                    int k, float* out);
void oc_moe_forward(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                    const float* router_w, const uint8_t* sh_gate, const uint8_t* sh_up,
                    const uint8_t* sh_down, const float* sh_gate_vec, int D, int F, int E, int k,
                    int Fs, int renorm, int flags, const float* x, int T, float* out,
                    int32_t* ids_out, float* w_out);

/* ---- timed CPU port (fp32 accumulation, rows split over threads) ---- */
void oc_cpu_expert_forward_fast(const uint8_t* w1, const uint8_t* w3, const uint8_t* w2, int D,
                                int F, const float* x, float* y, int nthreads);
void oc_cpu_moe_token_fast(const uint8_t* gate_exps, const uint8_t* up_exps,
                           const uint8_t* down_exps, const float* router_w, int D, int F, int E,
                           int k, int renorm, int flags, const float* x, float* out,
                           int nthreads);
void oc_cpu_moe_token_shared_fast(const uint8_t* gate_exps, const uint8_t* up_exps, const uint8_t* down_exps,
                                  const float* router_w, const uint8_t* sh_gate, const uint8_t* sh_up,
                                  const uint8_t* sh_down, const float* sh_gate_vec, int D, int F, int E, int k,
                                  int Fs, int renorm, int flags, const float* x, float* out, int nthreads);

/* ---- wire codecs (QuantizationKernels) ---- */
int oc_wire_token_bytes(int mode, int dim);
float oc_quantize_int8(const float* x, int n, uint8_t* dst);
void oc_dequantize_int8(const uint8_t* src, int n, float* out);
float oc_quantize_fp8(const float* x, int n, uint8_t* dst);
void oc_dequantize_fp8(const uint8_t* src, int n, float* out);
uint8_t oc_float_to_fp8_e4m3(float v);
float oc_fp8_e4m3_to_float(uint8_t b);
int oc_wire_quantize(int mode, const float* x, int T, int D, uint8_t* out);
int oc_wire_dequantize(int mode, const uint8_t* in, int T, int D, float* out);

/* ---- FusedActivationHeader ---- */
void oc_header_write(uint64_t seq, int32_t token, int32_t layer, int32_t dim, uint8_t prec,
                     uint8_t flags, uint16_t batch, float scale, uint8_t* out32);
int oc_header_read(const uint8_t* in32, uint64_t* seq, int32_t* token, int32_t* layer,
                   int32_t* dim, uint8_t* prec, uint8_t* flags, uint16_t* batch, float* scale);
int oc_header_payload_bytes(const uint8_t* in32);

#ifdef __cplusplus
}
#endif
#endif
