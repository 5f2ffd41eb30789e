"""The dense-stage oracle (oracle/dense.py) on closed-form cases, on the CPU.

* RMSNorm of a constant vector is the weight (the reference's RMSNorm test
  shape, DistributedPipelineTests.cs:76-97, with a weight);
* the embedding row is the Q4_K dequantisation of the token's row;
* the synthetic weights are deterministic and distinct per layer;
* a layer whose projections are all zero returns its input.
"""
import numpy as np


def test_rmsnorm_weighted_constant(oracle):
    from oracle import dense as dn
    w = np.linspace(0.5, 1.5, 512).astype(np.float32)
    y = dn.rmsnorm_w(np.full(512, 2.0, np.float32), w, 1e-6)
    np.testing.assert_allclose(y, w, rtol=1e-6)


def test_embedding_row_is_its_dequantisation(oracle):
    from oracle import dense as dn
    io = dn.synth_io(3, 10, 512)
    rb = 2 * 144
    for t in (0, 4, 9):
        want = oracle.dequant(np.ascontiguousarray(io["embedding"][t * rb:(t + 1) * rb]), 512)
        assert np.array_equal(dn.embed(io["embedding"], t, 512), want.astype(np.float64))


def test_synthetic_layers_deterministic_and_distinct(oracle):
    from oracle import dense as dn
    a = dn.synth_layer(9, 0, 512, 1024, 4, 2)
    b = dn.synth_layer(9, 0, 512, 1024, 4, 2)
    c = dn.synth_layer(9, 1, 512, 1024, 4, 2)
    for key in a:
        assert np.array_equal(a[key], b[key]), key
        assert not np.array_equal(a[key], c[key]), key


def test_layer_with_zero_projections_returns_input(oracle):
    from oracle import dense as dn
    D, FF, Hq, Hkv = 512, 1024, 4, 2
    L = dn.synth_layer(1, 0, D, FF, Hq, Hkv)
    for key in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
        L[key] = np.zeros_like(L[key])  # d = dmin = 0: every weight is 0
    for key in ("bq", "bk", "bv"):
        L[key] = np.zeros_like(L[key])
    x = np.random.default_rng(2).standard_normal(D).astype(np.float32)
    kc = np.zeros((Hkv, 8, 128), np.float16)
    y, kc2, vc2 = dn.layer_forward(L, x, 3, kc, kc.copy(), D, FF, Hq, Hkv, 1e6, 1e-6)
    assert np.array_equal(y, x.astype(np.float64))
    assert not kc2.any() and not vc2.any()
