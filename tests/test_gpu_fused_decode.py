"""The fused decode-layer launch against the three-launch decode path and the oracle.

The fused kernel (router + gate/up/SwiGLU + grid barrier + down/combine in one
persistent launch) uses the same lane math and per-row reduction order as the
separate router and GEMV launches, so its outputs, expert ids and combine
weights must match them bit for bit; against the CPU oracle the bound is the
layer tolerance rel-L2 <= 1e-3 with bit-exact expert ids.
"""
import numpy as np
import pytest

from test_gpu_parity import LAYER_TOL, make_layer, rel_l2, worker_for

pytestmark = pytest.mark.gpu

DECODE, UNFUSED = 4, 16


def _run(w, x, flags):
    w.set_profiling(True)
    out, ids, wt = w.forward(0, x, flags)
    n = len(w.kernel_times_ms())
    w.set_profiling(False)
    return out, ids, wt, n


@pytest.mark.parametrize("D,F,E,k,T,flags,renorm", [
    (512, 1024, 8, 2, 1, 3, True),     # Mixtral-like routing, RMSNorm + residual
    (512, 1024, 8, 2, 4, 1, True),     # four tokens: eight (token, slot) pairs
    (768, 512, 16, 4, 2, 2, True),     # K = 768: one lane segment per row
    (1024, 512, 32, 4, 3, 3, False),   # softmax over all experts, 32-expert router
    (256, 2560, 8, 1, 1, 0, True),     # top-1, K of the down rows = 2560
    (6144, 512, 8, 2, 1, 3, True),     # 196 KB router: staged split over a 2-CTA cluster
    (4096, 512, 16, 4, 2, 3, True),    # 256 KB router, two tokens: split over a 2-CTA cluster
])
def test_fused_matches_separate_launches_bit_exact(cuda, glc, oracle, D, F, E, k, T, flags, renorm):
    L = make_layer(oracle, 7000 + D + T, D, F, E, k, renorm=renorm)
    w = worker_for(glc, L, max_tokens=4)
    x = oracle.fill_normal(7000 + T, 1, 1.0, T * D).reshape(T, D)
    fo, fids, fw, nf = _run(w, x, flags | DECODE)
    so, sids, sw, ns = _run(w, x, flags | DECODE | UNFUSED)
    assert nf == 1 and ns == 3, (nf, ns)  # one fused launch vs router + gate/up + down
    assert np.array_equal(fids, sids) and np.array_equal(fw, sw)
    assert np.array_equal(fo, so)
    ro, rids, rw = oracle.moe_forward(L, x, flags)
    assert np.array_equal(fids, rids)
    np.testing.assert_allclose(fw, rw, rtol=2e-6, atol=1e-7)
    assert rel_l2(fo, ro) <= LAYER_TOL
    w.dispose()


def test_fused_mixtral_full_size_repeat_and_graph(cuda, glc, oracle):
    """Mixtral-8x7B layer (D=4096, F=14336, E=8, k=2), one token, RMSNorm + residual:
    fused == separate launches bit for bit, on repeated calls (the grid-barrier
    words are reused) and under CUDA-graph replay; oracle within tolerance."""
    torch = cuda
    D, F, E, k = 4096, 14336, 8, 2
    L = make_layer(oracle, 4321, D, F, E, k)
    w = worker_for(glc, L, max_tokens=1, synth_seed=4321)
    xs = [oracle.fill_normal(4321 + i, 1, 1.0, D)[None, :] for i in range(3)]
    for x in xs:
        fo, fids, fw, nf = _run(w, x, 3)
        so, sids, sw, ns = _run(w, x, 3 | UNFUSED)
        assert nf == 1 and ns == 3
        assert np.array_equal(fids, sids) and np.array_equal(fo, so)
    ro, rids, _ = oracle.moe_forward(L, xs[-1], 3)
    assert np.array_equal(fids, rids)
    assert rel_l2(fo, ro) <= LAYER_TOL

    xd = torch.from_numpy(xs[0]).cuda()
    od = torch.empty(1, D, device="cuda")
    w.graph_build(0, xd.data_ptr(), 1, 3, od.data_ptr())
    for x in xs:
        xd.copy_(torch.from_numpy(x))
        od.zero_()
        from glacier.inference.distributed_b200.api import torch_stream_handle
        w.graph_launch(torch_stream_handle())
        torch.cuda.synchronize()
        so, _, _, _ = _run(w, x, 3 | UNFUSED)
        assert np.array_equal(od.cpu().numpy(), so)
    w.poll_error()
    w.dispose()


def test_fused_falls_back_when_router_does_not_fit(cuda, glc, oracle):
    """A 64-expert router at D=3584 (917 KB) does not fit the shared-memory
    staging; the forward then runs the separate launches."""
    D, F, E, k = 3584, 512, 64, 8
    L = make_layer(oracle, 99, D, F, E, k, renorm=False)
    w = worker_for(glc, L, max_tokens=1)
    x = oracle.fill_normal(99, 1, 1.0, D)[None, :]
    out, ids, _, n = _run(w, x, 0)
    assert n == 3
    ro, rids, _ = oracle.moe_forward(L, x, 0)
    assert np.array_equal(ids, rids)
    assert rel_l2(out, ro) <= LAYER_TOL
    w.dispose()
