"""Small single-kernel workloads of the hot path, for kernel profiles.

    python -m glacier.inference.distributed_b200.cases <case> [--reps N]

Each case builds its inputs on cuda:0 (weights by the library's seeded
synthetic generator, the shapes of the Mixtral-8x7B, Qwen2-57B-A14B,
Qwen2.5-14B and Mixtral-8x22B layers), runs three warm-up calls and then ``reps`` calls of the
one kernel family it names, and exits 0.  Inputs that a kernel streams are
larger than the 126 MB L2 (rotating copies where one copy is smaller), so the
DRAM counters of a capture describe HBM traffic.  A capture names the kernel
with ``-k`` and skips the warm-up launches with ``-s``; the launches each case
makes per call are listed in CASES.
"""
from __future__ import annotations

import argparse
import sys

import numpy as np

MIXTRAL = dict(D=4096, F=14336, E=8, k=2, seed=20241201)
QWEN = dict(D=3584, F=2560, E=64, k=8, Fs=20480, seed=20241202)
QWEN14B = dict(D=5120, FF=13824, Hq=40, Hkv=8, max_len=2048, seed=20241203)
MIXTRAL22B = dict(D=6144, F=16384, E=8, k=2, Hq=48, Hkv=8, max_len=4096, seed=20241204)

# case -> (kernels launched per call, one line of what it runs)
CASES = {
    "gemv_k4096": ("q4k_gemv_kernel x1", "y = W x, K=4096, N=28672 (gate+up rows of one expert pair), 4 rotating 66 MB copies"),
    "gemv_k14336": ("q4k_gemv_kernel x1", "y = W x, K=14336, N=8192 (down rows of two experts), 4 rotating 66 MB copies"),
    "gemv_chain": ("q4k_gemv_chain_kernel x1",
                   "64 GEMVs K=4096, N=28672 in one launch, each behind a grid-wide wait, 4 rotating 66 MB copies"),
    "router": ("router_kernel x1", "Mixtral router: T=64, D=4096, E=8, top-2 renormalised, RMSNorm"),
    "router_wide": ("router_wide_kernel x1", "Qwen2-57B router: T=16, D=3584, E=64, top-8, RMSNorm"),
    "wire": ("wire_quantize_kernel x1 + wire_dequantize_kernel x1",
             "symmetric INT8 per token, T=4096, D=4096 (64 MB fp32 in)"),
    "dispatch": ("dispatch_plan_kernel x1", "histogram / scan / stable permute of P=8192 slot ids over E=64"),
    "attention": ("attn_decode_kernel x1 (a 16- or 8-CTA cluster per KV head)",
                  "40 query / 8 KV heads x 128, position 2047 of a 2048-row fp16 cache, 16 rotating layer caches"),
    "decode_fused": ("moe_decode_fused_kernel x1", "Mixtral-8x7B layer decode, T=1 (one launch)"),
    "decode_wide": ("moe_decode_wide_kernel x1", "Qwen2-57B-A14B layer decode with its shared expert, T=1 (one launch)"),
    "stage": ("per layer: attn_decode_kernel x1, q4k_gemv_chain_kernel x1",
              "Qwen2.5-14B dense stage of 2 layers, one token at position 2040"),
    "moe_stage": ("per layer: attn_decode_kernel x1, q4k_gemv_chain_kernel x2, moe_decode_fused_kernel x1",
                  "Mixtral-8x22B mixture-of-experts stage of 2 layers, one token at position 4090"),
}


def _stream(torch):
    from .api import torch_stream_handle
    s = torch.cuda.Stream()
    return s, torch_stream_handle(s)


def case_gemv(torch, glc, K, N, reps):
    w = MIXTRAL
    worker = glc.GpuExpertStageWorker(w["D"], w["F"], w["E"], w["k"], max_tokens=1)
    worker.synth_layer(0, w["seed"])
    g, _u, d, _r = worker.layer_device_ptrs(0)
    base, step = (g, 2 * w["F"] * glc.q4k_row_bytes(w["D"])) if K == w["D"] else \
        (d, 2 * w["D"] * glc.q4k_row_bytes(w["F"]))
    x = torch.from_numpy(np.random.default_rng(7).standard_normal(K).astype(np.float32)).cuda()
    y = torch.empty(N, device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for i in range(3 + reps):
            glc.gemv_q4k_dev(base + (i % 4) * step, x.data_ptr(), y.data_ptr(), K, N, s)
    torch.cuda.synchronize()
    worker.dispose()


def case_gemv_chain(torch, glc, reps):
    w = MIXTRAL
    K, N = w["D"], 2 * w["F"]
    worker = glc.GpuExpertStageWorker(w["D"], w["F"], w["E"], w["k"], max_tokens=1)
    worker.synth_layer(0, w["seed"])
    g = worker.layer_device_ptrs(0)[0]
    step = N * glc.q4k_row_bytes(K)
    x = torch.from_numpy(np.random.default_rng(7).standard_normal(K).astype(np.float32)).cuda()
    y = torch.empty(N, device="cuda")
    jobs = [dict(W=g + (i % 4) * step, x=x.data_ptr(), y=y.data_ptr(), K=K, N=N, after_previous=i > 0)
            for i in range(64)]
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for _ in range(3 + reps):
            glc.gemv_q4k_chain_dev(jobs, s)
    torch.cuda.synchronize()
    glc.gemv_poll_error()
    worker.dispose()


def case_router(torch, glc, wide, reps):
    w = QWEN if wide else MIXTRAL
    T = 16 if wide else 64
    D, E, k = w["D"], w["E"], w["k"]
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).cuda()
    r = torch.from_numpy((rng.standard_normal((D, E)) * 0.02).astype(np.float32)).cuda()
    xin = torch.empty(T, D, device="cuda")
    lg = torch.empty(T, E, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wt = torch.empty(T, k, device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for _ in range(3 + reps):
            glc.router_topk_dev(x.data_ptr(), r.data_ptr(), T, D, E, k, not wide, True, xin.data_ptr(),
                                lg.data_ptr(), ids.data_ptr(), wt.data_ptr(), s)
    torch.cuda.synchronize()


def case_wire(torch, glc, reps):
    T, D, mode = 4096, 4096, 2  # INT8
    x = torch.randn(T, D, device="cuda")
    nb = glc.QuantizationKernels.GetPackedBatchBytes(mode, D, T)
    buf = torch.empty(nb, dtype=torch.uint8, device="cuda")
    y = torch.empty(T, D, device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for _ in range(3 + reps):
            glc.QuantizationKernels.quantize_dev(mode, x.data_ptr(), T, D, buf.data_ptr(), s)
            glc.QuantizationKernels.dequantize_dev(mode, buf.data_ptr(), T, D, y.data_ptr(), s)
    torch.cuda.synchronize()


def case_dispatch(torch, glc, reps):
    P, E = 8192, 64
    ids = torch.from_numpy(np.random.default_rng(5).integers(0, E, P).astype(np.int32)).cuda()
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    offs = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(P, dtype=torch.int32, device="cuda")
    inv = torch.empty(P, dtype=torch.int32, device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for _ in range(3 + reps):
            glc.dispatch_plan_dev(ids.data_ptr(), P, E, counts.data_ptr(), offs.data_ptr(), perm.data_ptr(),
                                  inv.data_ptr(), s)
    torch.cuda.synchronize()


def case_attention(torch, glc, reps):
    q = QWEN14B
    Hq, Hkv, L = q["Hq"], q["Hkv"], q["max_len"]
    ncache = 16  # 16 x 2 x 4 MB: the caches of 16 layers, more than L2
    kc = [(torch.randn(Hkv, L, 128, device="cuda") * 0.5).half() for _ in range(ncache)]
    vc = [(torch.randn(Hkv, L, 128, device="cuda") * 0.5).half() for _ in range(ncache)]
    qv = torch.randn(Hq * 128, device="cuda")
    kn = torch.randn(Hkv * 128, device="cuda")
    vn = torch.randn(Hkv * 128, device="cuda")
    out = torch.empty(Hq * 128, device="cuda")
    wb = glc.attn_workspace_bytes(Hq, Hkv, L)
    work = torch.empty(wb // 4 + 1, device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for i in range(3 + reps):
            c = i % ncache
            glc.attn_decode_dev(qv.data_ptr(), kn.data_ptr(), vn.data_ptr(), kc[c].data_ptr(), vc[c].data_ptr(),
                                Hq, Hkv, L, L - 1, 1e6, out.data_ptr(), work.data_ptr(), wb, stream=s)
    torch.cuda.synchronize()


def case_decode(torch, glc, wide, reps):
    w = QWEN if wide else MIXTRAL
    worker = glc.GpuExpertStageWorker(w["D"], w["F"], w["E"], w["k"], shared_ffn_dim=w.get("Fs", 0),
                                      renormalize=not wide, max_tokens=1)
    worker.synth_layer(0, w["seed"])
    xs = [torch.randn(1, w["D"], device="cuda") for _ in range(4)]
    out = torch.empty(1, w["D"], device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for i in range(3 + reps):
            worker.forward_dev(0, xs[i % 4].data_ptr(), 1, 3, out.data_ptr(), stream=s)  # RMSNorm | residual
    torch.cuda.synchronize()
    worker.poll_error()
    worker.dispose()


def case_stage(torch, glc, reps):
    q = QWEN14B
    st_ = glc.DenseStage(q["D"], q["FF"], q["Hq"], q["Hkv"], 0, 2, q["max_len"], 1e6, 1e-6)
    for l in range(2):
        st_.synth_layer(l, q["seed"])
    x = torch.randn(q["D"], device="cuda")
    y = torch.empty(q["D"], device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for i in range(3 + reps):
            st_.forward_dev(2040 + i % 4, x_in_ptr=x.data_ptr(), x_out_ptr=y.data_ptr(), stream=s)
    torch.cuda.synchronize()
    st_.poll_error()
    st_.dispose()


def case_moe_stage(torch, glc, reps):
    q = MIXTRAL22B
    st_ = glc.DenseStage(q["D"], 0, q["Hq"], q["Hkv"], 0, 2, q["max_len"], 1e6, 1e-5, num_experts=q["E"],
                         top_k=q["k"], expert_ffn_dim=q["F"], moe_renormalize=True)
    for l in range(2):
        st_.synth_layer(l, q["seed"])
    x = torch.randn(q["D"], device="cuda")
    y = torch.empty(q["D"], device="cuda")
    st, s = _stream(torch)
    with torch.cuda.stream(st):
        for i in range(3 + reps):
            st_.forward_dev(4090 + i % 4, x_in_ptr=x.data_ptr(), x_out_ptr=y.data_ptr(), stream=s)
    torch.cuda.synchronize()
    st_.poll_error()
    st_.dispose()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args(argv)
    import torch

    from . import api as glc
    if not torch.cuda.is_available():
        print("a CUDA device is required", file=sys.stderr)
        return 2
    torch.cuda.set_device(0)
    c, n = a.case, a.reps
    if c == "gemv_k4096":
        case_gemv(torch, glc, 4096, 28672, n)
    elif c == "gemv_k14336":
        case_gemv(torch, glc, 14336, 8192, n)
    elif c == "gemv_chain":
        case_gemv_chain(torch, glc, n)
    elif c in ("router", "router_wide"):
        case_router(torch, glc, c == "router_wide", n)
    elif c == "wire":
        case_wire(torch, glc, n)
    elif c == "dispatch":
        case_dispatch(torch, glc, n)
    elif c == "attention":
        case_attention(torch, glc, n)
    elif c in ("decode_fused", "decode_wide"):
        case_decode(torch, glc, c == "decode_wide", n)
    elif c == "stage":
        case_stage(torch, glc, n)
    elif c == "moe_stage":
        case_moe_stage(torch, glc, n)
    print(f"{c}: {CASES[c][0]} per call, {3 + n} calls: ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
