"""CPU restatement of decode attention over an fp16 KV cache (float64 numpy).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the CPU reference for
glc_attn_decode_dev; the product package never imports it.

Parity unpinned: the reference's attention body lives in its external model
package (caller side IClusterStageModel.ForwardStage, IClusterStageModel.cs:19;
body Program.cs:1390), so there is no reference code, test or golden vector
for this path.  This module states the semantics the kernel implements:
rotate-half RoPE (pairs (i, i + d/2), frequencies theta^(-2i/d)) at position
pos on q and the new key; the rotated key and the value stored as fp16 in row
pos of the caches; softmax(q.K^T / sqrt(d)) V over positions 0..pos, query
head h reading KV head h // (n_heads // n_kv_heads).
"""
from __future__ import annotations

import numpy as np


def rope(x: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """Rotate-half RoPE of the last axis of x (float64) at position pos."""
    x = np.asarray(x, np.float64)
    d = x.shape[-1]
    half = d // 2
    i = np.arange(half, dtype=np.float64)
    ang = pos * np.exp(-(2.0 * i / d) * np.log(theta))
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def attn_decode(q, k_new, v_new, k_cache, v_cache, pos: int, theta: float, stored_rows=None):
    """Returns (out [n_heads][d] float64, k_cache', v_cache' (fp16 copies with row pos written)).
    stored_rows: optional (k_row, v_row) [n_kv][d] fp16 to use as row pos instead of this
    function's own rounding (to compare a kernel's later arithmetic on the rows it stored)."""
    q = np.asarray(q, np.float32)
    n_heads, d = q.shape
    n_kv = k_new.shape[0]
    G = n_heads // n_kv
    kc = np.array(k_cache, np.float16, copy=True)
    vc = np.array(v_cache, np.float16, copy=True)
    kc[:, pos] = rope(np.asarray(k_new, np.float32), pos, theta).astype(np.float16)
    vc[:, pos] = np.asarray(v_new, np.float32).astype(np.float16)
    if stored_rows is not None:
        kc[:, pos], vc[:, pos] = stored_rows[0], stored_rows[1]
    qr = rope(q, pos, theta)
    out = np.empty((n_heads, d), np.float64)
    for h in range(n_heads):
        g = h // G
        K = kc[g, :pos + 1].astype(np.float64)
        V = vc[g, :pos + 1].astype(np.float64)
        s = K @ qr[h] / np.sqrt(d)
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ V
    return out, kc, vc
