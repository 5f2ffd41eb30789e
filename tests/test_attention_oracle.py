"""CPU checks of the decode-attention oracle (oracle/attention.py).

The reference holds no attention code or vectors (its body is external), so
the oracle is pinned by closed-form cases instead: RoPE at position 0 is the
identity and preserves norms elsewhere; one cached position returns its value
row exactly; equal keys give the mean of the values; GQA maps query head h to
KV head h // G.
"""
import numpy as np

from oracle import attention as att


def test_rope_identity_at_zero_and_norm_preserving():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 128))
    assert np.array_equal(att.rope(x, 0, 1e6), x)
    for pos in (1, 17, 2047, 4095):
        y = att.rope(x, pos, 1e6)
        assert np.allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-12)
    # pair (i, i + 64) of frequency 1 (i = 0) turns by exactly pos radians
    e = np.zeros(128); e[0] = 1.0
    y = att.rope(e, 3, 1e6)
    assert np.isclose(y[0], np.cos(3.0)) and np.isclose(y[64], np.sin(3.0))


def test_single_position_returns_its_value_row():
    rng = np.random.default_rng(1)
    Hq, Hkv, L = 8, 2, 4
    q = rng.standard_normal((Hq, 128)).astype(np.float32)
    k = rng.standard_normal((Hkv, 128)).astype(np.float32)
    v = rng.standard_normal((Hkv, 128)).astype(np.float32)
    kc = np.zeros((Hkv, L, 128), np.float16)
    vc = np.zeros((Hkv, L, 128), np.float16)
    out, kc2, vc2 = att.attn_decode(q, k, v, kc, vc, 0, 1e6)
    for h in range(Hq):
        assert np.array_equal(out[h], v[h // 4].astype(np.float16).astype(np.float64))
    assert np.array_equal(vc2[:, 0], v.astype(np.float16))
    assert np.array_equal(kc2[:, 0], k.astype(np.float16))  # RoPE at 0 is the identity


def test_equal_keys_average_the_values_and_gqa_mapping():
    rng = np.random.default_rng(2)
    Hq, Hkv, L = 6, 3, 8
    pos = 5
    kc = np.zeros((Hkv, L, 128), np.float16)
    vc = rng.standard_normal((Hkv, L, 128)).astype(np.float16)
    q = rng.standard_normal((Hq, 128)).astype(np.float32)
    # the new key rotates to zero only if it is zero: all scores equal
    out, _, vc2 = att.attn_decode(q, np.zeros((Hkv, 128), np.float32), rng.standard_normal((Hkv, 128)),
                                  kc, vc, pos, 1e6)
    for h in range(Hq):
        g = h // 2
        assert np.allclose(out[h], vc2[g, :pos + 1].astype(np.float64).mean(axis=0), rtol=1e-12, atol=1e-12)
