"""Batched (T > 1) MoE path on the GPU against the CPU oracle: dispatch plan
(bit-exact), grouped tcgen05 expert GEMMs with the SwiGLU / combine epilogues
(rel-L2 <= 1e-3 of the layer output), expert ids bit-exact."""
import numpy as np
import pytest

from test_gpu_parity import LAYER_TOL, dev, make_layer, rel_l2, stream, worker_for

pytestmark = pytest.mark.gpu

BATCHED, DECODE = 8, 4


@pytest.mark.parametrize("P,E", [(128, 8), (2048, 64), (3000, 64), (5, 3), (1, 8)])
def test_dispatch_plan_matches_oracle(cuda, glc, oracle, P, E):
    torch = cuda
    rng = np.random.default_rng(P + E)
    ids = rng.integers(0, E, size=P).astype(np.int32)
    if P > 100:
        ids[: P // 3] = 1  # a heavy expert
    d_ids = dev(torch, ids)
    counts = torch.empty(E, dtype=torch.int32, device="cuda")
    offsets = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(P, dtype=torch.int32, device="cuda")
    inv = torch.empty(P, dtype=torch.int32, device="cuda")
    glc.dispatch_plan_dev(d_ids.data_ptr(), P, E, counts.data_ptr(), offsets.data_ptr(),
                          perm.data_ptr(), inv.data_ptr(), stream(torch))
    torch.cuda.synchronize()
    rc, ro, rp, ri = oracle.dispatch_plan(ids, E)
    assert np.array_equal(counts.cpu().numpy(), rc)
    assert np.array_equal(offsets.cpu().numpy(), ro)
    assert np.array_equal(perm.cpu().numpy(), rp)
    assert np.array_equal(inv.cpu().numpy(), ri)


@pytest.mark.parametrize("T,flags", [(4, 0), (2, 3), (17, 1), (40, 2)])
def test_batched_small_matches_oracle(cuda, glc, oracle, T, flags):
    D, F, E, k = 512, 1024, 8, 2
    L = make_layer(oracle, 71 + T, D, F, E, k)
    w = worker_for(glc, L, max_tokens=64)
    x = oracle.fill_normal(71 + T, 1, 1.0, T * D).reshape(T, D)
    out, ids, wt = w.forward(0, x, flags | BATCHED)
    ro, rids, rw = oracle.moe_forward(L, x, flags)
    assert np.array_equal(ids, rids)
    assert rel_l2(out, ro) <= LAYER_TOL
    out2, _, _ = w.forward(0, x, flags | DECODE)
    assert rel_l2(out2, ro) <= LAYER_TOL
    w.dispose()


def test_batched_many_tokens_one_expert(cuda, glc, oracle):
    """More than one MMA group per expert (>32 tokens routed to it)."""
    D, F, E, k = 512, 768, 2, 1
    L = make_layer(oracle, 81, D, F, E, k)
    w = worker_for(glc, L, max_tokens=96)
    x = oracle.fill_normal(81, 1, 1.0, 96 * D).reshape(96, D)
    out, ids, _ = w.forward(0, x, BATCHED)
    ro, rids, _ = oracle.moe_forward(L, x, 0)
    assert np.array_equal(ids, rids)
    assert np.bincount(ids.ravel(), minlength=E).max() > 32
    assert rel_l2(out, ro) <= LAYER_TOL
    w.dispose()


def test_batched_mixtral_prefill_64_tokens(cuda, glc, oracle):
    """Mixtral-8x7B layer, a 64-token batch (D=4096, F=14336, E=8, k=2): all
    expert ids against the oracle router, outputs of 6 tokens against the full
    oracle layer."""
    D, F, E, k, T = 4096, 14336, 8, 2, 64
    L = make_layer(oracle, 4242, D, F, E, k)
    w = worker_for(glc, L, max_tokens=T, synth_seed=4242)
    x = oracle.fill_normal(4242, 1, 1.0, T * D).reshape(T, D)
    out, ids, wt = w.forward(0, x, 1)
    xin = np.stack([oracle.rmsnorm(x[t]) for t in range(T)])
    for t in range(T):
        _, rid, rwt = oracle.router(xin[t], L["router"], E, k, True)
        assert np.array_equal(ids[t], rid)
        np.testing.assert_allclose(wt[t], rwt, rtol=2e-6, atol=1e-7)
    sel = [0, 1, 17, 33, 48, 63]
    ro, rids, _ = oracle.moe_forward(L, x[sel], 1)
    assert np.array_equal(ids[sel], rids)
    assert rel_l2(out[sel], ro) <= LAYER_TOL
    w.dispose()


def test_batched_qwen_shapes_with_shared_expert(cuda, glc, oracle):
    """Qwen2-57B-A14B-shaped routed experts (D=3584, F=2560, E=64, k=8, no
    renormalisation) with a sigmoid-gated shared expert, 16-token batch."""
    D, F, E, k, Fs, T = 3584, 2560, 64, 8, 1024, 16
    L = make_layer(oracle, 5151, D, F, E, k, renorm=False, Fs=Fs)
    w = worker_for(glc, L, max_tokens=T)
    x = oracle.fill_normal(5151, 1, 1.0, T * D).reshape(T, D)
    out, ids, _ = w.forward(0, x, 0)
    sel = [0, 5, 15]
    ro, rids, _ = oracle.moe_forward(L, x[sel], 0)
    assert np.array_equal(ids[sel], rids)
    assert rel_l2(out[sel], ro) <= LAYER_TOL
    w.dispose()


@pytest.mark.parametrize("D,F,E,k,T,Fs", [(512, 1024, 2, 1, 150, 0), (512, 768, 8, 2, 200, 2048)])
def test_wide_groups_equal_narrow_groups(cuda, glc, oracle, monkeypatch, D, F, E, k, T, Fs):
    """The grouped GEMMs' wide layout (groups of up to 64 tokens, MMA N up to
    128) against the narrow one (32 tokens, N up to 64) on batches where
    experts hold 33..64 and more than 64 tokens (74 and 76 routed; the
    shared expert's 200, whose down projection is K-sliced by the same count
    in both layouts): identical outputs, and the oracle's within the layer
    tolerance.  GLC_GROUPED_WIDE forces the layout; the default choice (wide
    groups here, the wide down projection always) gives the same bits."""
    L = make_layer(oracle, 6100 + T, D, F, E, k, Fs=Fs)
    w = worker_for(glc, L, max_tokens=T)
    x = oracle.fill_normal(6100 + T, 1, 1.0, T * D).reshape(T, D)
    outs = {}
    for wide in ("0", "1", ""):  # narrow, wide, the default choice
        monkeypatch.setenv("GLC_GROUPED_WIDE", wide)
        outs[wide] = w.forward(0, x, 1 | BATCHED)
    monkeypatch.delenv("GLC_GROUPED_WIDE")
    (on, idn, wn), (ow, idw, ww) = outs["0"], outs["1"]
    assert np.bincount(idw.ravel(), minlength=E).max() > 32
    assert np.array_equal(idn, idw) and np.array_equal(wn, ww)
    assert np.array_equal(on, ow), float(np.abs(on - ow).max())
    assert np.array_equal(outs[""][0], ow)
    ro, rids, _ = oracle.moe_forward(L, x, 1)
    assert np.array_equal(idw, rids)
    assert rel_l2(ow, ro) <= LAYER_TOL
    w.poll_error()
    w.dispose()
