// kernels.h -- host-visible launch interfaces of the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace glc {

constexpr int kMaxDevices = 64;
constexpr int kGemvMaxThreads = 17 * 32;  // 16 consumer warps + 1 producer warp

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
    // filled by gemv_configure
    int nsegw, nw, stage_rows, stages;
};

int gemv_configure(GemvParams& p, int num_sms, size_t smem_limit, size_t* smem_bytes, int* grid);
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
};
cudaError_t router_launch(const RouterParams& p, cudaStream_t stream);

// Wire codec (QuantizationKernels), one CTA per token.
cudaError_t wire_quantize_launch(int mode, const float* x, int T, int D, uint8_t* out,
                                 cudaStream_t stream);
cudaError_t wire_dequantize_launch(int mode, const uint8_t* in, int T, int D, float* out,
                                   cudaStream_t stream);

}  // namespace glc
