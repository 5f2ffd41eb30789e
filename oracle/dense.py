"""CPU restatement of one token through a dense decoder stage (Qwen2-style).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the CPU reference for the
stage entry points (glc_stage_*); the product package never imports it.

Parity unpinned: the reference's stage bodies live in its external model
package (caller side IClusterStageModel.ForwardStage, Pipeline/IClusterStageModel.cs:19;
bodies Program.cs:41-110, 1382-1390), so there is no reference code, test or
golden vector for this path.  This module states the semantics the stage
implements, per layer:

    h   = x / sqrt(mean(x^2) + eps) * w_attn
    q, k, v = Wq h + bq, Wk h + bk, Wv h + bv
    o   = attention (oracle/attention.py: rotate-half RoPE, fp16 KV cache, GQA)
    x   = x + Wo o
    h   = x / sqrt(mean(x^2) + eps) * w_ffn
    x   = x + Wdown (SiLU(Wgate h) * (Wup h))

with the embedding row of the token on a first stage and logits = Wlm (RMSNorm(x)
* w_final) on a last stage.  A mixture-of-experts layer (Mixtral-style: no
q/k/v biases) replaces the feed-forward by

    h   = x / sqrt(mean(x^2) + eps) * w_ffn
    p   = softmax(Wr^T h) (fp32 router [D][E]); the top-k experts (ties to the
          lower index), their weights renormalised to sum 1
    x   = x + sum_j p_j Wdown_j (SiLU(Wgate_j h) * (Wup_j h))   (in k order)

Matrix-vector products use the oracle's Q4_K GEMV
(fp32 dequantised weights, fp32 products, double accumulation); everything
else is float64.  The synthetic weights are those of glc_stage_synth_layer /
glc_stage_synth_io (the documented generator, tags below).
"""
from __future__ import annotations

import numpy as np

from . import oracle as o
from .attention import attn_decode

SIGMA_D = 0.001


def layer_tags(global_layer: int) -> int:
    return 200000 + 16 * global_layer


def synth_layer(seed: int, global_layer: int, D: int, FF: int, Hq: int, Hkv: int) -> dict:
    """The synthetic weights of one layer (bytes and floats as the stage makes them)."""
    b = layer_tags(global_layer)
    hd = 128
    L = {
        "wq": o.synth_q4k(seed, b + 0, Hq * hd, D, SIGMA_D),
        "wk": o.synth_q4k(seed, b + 1, Hkv * hd, D, SIGMA_D),
        "wv": o.synth_q4k(seed, b + 2, Hkv * hd, D, SIGMA_D),
        "wo": o.synth_q4k(seed, b + 3, D, Hq * hd, SIGMA_D),
        "w_gate": o.synth_q4k(seed, b + 4, FF, D, SIGMA_D),
        "w_up": o.synth_q4k(seed, b + 5, FF, D, SIGMA_D),
        "w_down": o.synth_q4k(seed, b + 6, D, FF, SIGMA_D),
        "attn_norm": (np.float32(1.0) + o.fill_normal(seed, b + 7, 0.02, D)).astype(np.float32),
        "ffn_norm": (np.float32(1.0) + o.fill_normal(seed, b + 8, 0.02, D)).astype(np.float32),
    }
    bias = o.fill_normal(seed, b + 9, 0.02, (Hq + 2 * Hkv) * hd)
    L["bq"], L["bk"], L["bv"] = bias[:Hq * hd], bias[Hq * hd:(Hq + Hkv) * hd], bias[(Hq + Hkv) * hd:]
    return L


def expert_tag(global_layer: int, e: int, m: int) -> int:
    """Tag of expert e's matrix m (0 gate, 1 up, 2 down) in a mixture-of-experts layer."""
    return 1000000 + 64 * global_layer + 3 * e + m


def synth_moe_layer(seed: int, global_layer: int, D: int, F: int, E: int, Hq: int, Hkv: int) -> dict:
    """The synthetic weights of one mixture-of-experts layer: the attention
    part and norms as synth_layer (no biases), the fp32 router N(0, 0.02)
    [D][E] (tag layer_tags + 10) and E experts of gate / up [F][D] and
    down [D][F] Q4_K."""
    b = layer_tags(global_layer)
    hd = 128
    L = {
        "wq": o.synth_q4k(seed, b + 0, Hq * hd, D, SIGMA_D),
        "wk": o.synth_q4k(seed, b + 1, Hkv * hd, D, SIGMA_D),
        "wv": o.synth_q4k(seed, b + 2, Hkv * hd, D, SIGMA_D),
        "wo": o.synth_q4k(seed, b + 3, D, Hq * hd, SIGMA_D),
        "attn_norm": (np.float32(1.0) + o.fill_normal(seed, b + 7, 0.02, D)).astype(np.float32),
        "ffn_norm": (np.float32(1.0) + o.fill_normal(seed, b + 8, 0.02, D)).astype(np.float32),
        "router": o.fill_normal(seed, b + 10, 0.02, D * E).reshape(D, E),
        "gate": [o.synth_q4k(seed, expert_tag(global_layer, e, 0), F, D, SIGMA_D) for e in range(E)],
        "up": [o.synth_q4k(seed, expert_tag(global_layer, e, 1), F, D, SIGMA_D) for e in range(E)],
        "down": [o.synth_q4k(seed, expert_tag(global_layer, e, 2), D, F, SIGMA_D) for e in range(E)],
    }
    zero = np.zeros(Hq * hd, np.float64)
    L["bq"], L["bk"], L["bv"] = zero, zero[:Hkv * hd], zero[:Hkv * hd]
    return L


def moe_ffn(L: dict, x, D: int, F: int, k: int, eps: float):
    """x + the routed experts' SwiGLU feed-forward of RMSNorm(x) * w_ffn; also returns the ids."""
    x = np.asarray(x, np.float64)
    h = rmsnorm_w(x, L["ffn_norm"], eps)
    lg = h @ np.asarray(L["router"], np.float64)
    p = np.exp(lg - lg.max())
    p = p / p.sum()
    ids = sorted(range(len(p)), key=lambda e: (-p[e], e))[:k]
    w = np.array([p[e] for e in ids])
    w = w / w.sum()
    for j, e in enumerate(ids):
        g = gemv(L["gate"][e], h, D, F)
        u = gemv(L["up"][e], h, D, F)
        x = x + w[j] * gemv(L["down"][e], g / (1.0 + np.exp(-g)) * u, F, D)
    return x, ids


def moe_layer_forward(L: dict, x, pos: int, kc, vc, D: int, F: int, k: int, Hq: int, Hkv: int, theta: float,
                      eps: float, stored_rows=None):
    """One mixture-of-experts layer at position pos; returns (x', kc', vc', ids).
    stored_rows: optional fp16 (k, v) rows for position pos (see attn_decode)."""
    hd = 128
    x = np.asarray(x, np.float64)
    h = rmsnorm_w(x, L["attn_norm"], eps)
    q = gemv(L["wq"], h, D, Hq * hd)
    kk = gemv(L["wk"], h, D, Hkv * hd)
    v = gemv(L["wv"], h, D, Hkv * hd)
    att, kc, vc = attn_decode(q.astype(np.float32).reshape(Hq, hd), kk.astype(np.float32).reshape(Hkv, hd),
                              v.astype(np.float32).reshape(Hkv, hd), kc, vc, pos, theta, stored_rows)
    x = x + gemv(L["wo"], att.reshape(-1), Hq * hd, D)
    x, ids = moe_ffn(L, x, D, F, k, eps)
    return x, kc, vc, ids


def synth_io(seed: int, vocab: int, D: int) -> dict:
    return {"embedding": o.synth_q4k(seed, 300000, vocab, D, SIGMA_D),
            "final_norm": (np.float32(1.0) + o.fill_normal(seed, 300001, 0.02, D)).astype(np.float32),
            "lm_head": o.synth_q4k(seed, 300002, vocab, D, SIGMA_D)}


def rmsnorm_w(x, w, eps):
    x = np.asarray(x, np.float64)
    r = x / np.sqrt(np.mean(x * x) + eps)
    return r if w is None else r * np.asarray(w, np.float64)


def gemv(W, x, K, N):
    return o.gemv(W, np.asarray(x, np.float32), K, N).astype(np.float64)


def embed(table, token: int, D: int):
    rb = (D // 256) * 144
    return o.dequant(np.ascontiguousarray(table[token * rb:(token + 1) * rb]), D).astype(np.float64)


def layer_forward(L: dict, x, pos: int, kc, vc, D: int, FF: int, Hq: int, Hkv: int, theta: float, eps: float):
    """One layer at position pos; returns (x', kc', vc')."""
    hd = 128
    x = np.asarray(x, np.float64)
    h = rmsnorm_w(x, L["attn_norm"], eps)
    q = gemv(L["wq"], h, D, Hq * hd) + L["bq"]
    k = gemv(L["wk"], h, D, Hkv * hd) + L["bk"]
    v = gemv(L["wv"], h, D, Hkv * hd) + L["bv"]
    att, kc, vc = attn_decode(q.astype(np.float32).reshape(Hq, hd), k.astype(np.float32).reshape(Hkv, hd),
                              v.astype(np.float32).reshape(Hkv, hd), kc, vc, pos, theta)
    x = x + gemv(L["wo"], att.reshape(-1), Hq * hd, D)
    h = rmsnorm_w(x, L["ffn_norm"], eps)
    g = gemv(L["w_gate"], h, D, FF)
    u = gemv(L["w_up"], h, D, FF)
    a = g / (1.0 + np.exp(-g)) * u
    x = x + gemv(L["w_down"], a, FF, D)
    return x, kc, vc


def logits(io: dict, x, D: int, vocab: int, eps: float):
    return gemv(io["lm_head"], rmsnorm_w(x, io["final_norm"], eps), D, vocab)
