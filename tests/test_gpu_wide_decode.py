"""The wide fused decode launch (decode_wide.cu) against the oracle and the
separate launches.

A layer with a Qwen2-MoE shared expert, or whose router is too large to stage
in shared memory, decodes in one persistent launch: router warps spread over
the CTAs (one logit each, canonical order), the shared expert's weight stream
starting before the routing is known, then the routed experts, a grid barrier
and the down projection of k routed slots + the shared row per output row.
Expert ids are bit-exact against the oracle router and the separate router
launch; layer outputs are within rel-L2 1e-3 of the oracle and agree with the
separate launches to fp32 summation order (1e-5).
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


@pytest.mark.parametrize("D,F,E,k,Fs,T,flags,renorm", [
    (512, 2048, 16, 4, 2048, 1, 3, False),    # shared expert, RMSNorm + residual
    (512, 2048, 16, 4, 2048, 4, 1, True),     # four tokens
    (768, 2048, 64, 8, 0, 2, 3, False),       # 64-expert router that does not fit the staging, no shared expert
    (1024, 4096, 32, 2, 4096, 3, 2, True),    # two warps per routed slot
    (3584, 2560, 64, 8, 2560, 1, 3, False),   # Qwen2-57B routing and down slots, smaller shared expert
])
def test_wide_decode_matches_oracle_and_separate_launches(cuda, glc, oracle, D, F, E, k, Fs, T, flags, renorm):
    L = make_layer(oracle, 9100 + D + T, D, F, E, k, renorm=renorm, Fs=Fs)
    w = worker_for(glc, L, max_tokens=4)
    x = oracle.fill_normal(9100 + T, 1, 1.0, T * D).reshape(T, D)
    fo, fids, fw, nf = _run(w, x, flags | DECODE)
    assert nf == 1, nf  # one launch for the whole layer
    so, sids, sw, ns = _run(w, x, flags | DECODE | UNFUSED)
    assert ns >= 3
    assert np.array_equal(fids, sids) and np.array_equal(fw, sw)
    assert rel_l2(fo, so) <= 1e-5
    ro, rids, rw = oracle.moe_forward(L, x, flags)
    assert np.array_equal(fids, rids)
    np.testing.assert_allclose(fw, rw, rtol=2e-6, atol=1e-7)
    assert rel_l2(fo, ro) <= LAYER_TOL
    # repeated calls reuse both grid-wide counters; results are identical
    for _ in range(3):
        o2, i2, _, _ = _run(w, x, flags | DECODE)
        assert np.array_equal(i2, fids) and np.array_equal(o2, fo)
    w.dispose()


def test_wide_decode_graph_replay_and_device_path(cuda, glc, oracle):
    """forward_dev captured in a CUDA graph and replayed over changing inputs
    equals the eager call on each input."""
    torch = cuda
    D, F, E, k, Fs = 512, 2048, 16, 4, 2048
    L = make_layer(oracle, 9300, D, F, E, k, renorm=False, Fs=Fs)
    w = worker_for(glc, L, max_tokens=1)
    xs = [oracle.fill_normal(9300 + i, 1, 1.0, D)[None, :] for i in range(3)]
    want = [w.forward(0, x, 3 | DECODE)[0] for x in xs]
    xd = torch.from_numpy(xs[0]).cuda()
    od = torch.empty(1, D, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        w.forward_dev(0, xd.data_ptr(), 1, 3 | DECODE, od.data_ptr(), stream=s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        w.forward_dev(0, xd.data_ptr(), 1, 3 | DECODE, od.data_ptr(), stream=s.cuda_stream)
    for x, ref in zip(xs, want):
        xd.copy_(torch.from_numpy(x))
        torch.cuda.synchronize()
        with torch.cuda.stream(s):
            g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(od.cpu().numpy(), ref)
    w.poll_error()
    del g
    w.dispose()
