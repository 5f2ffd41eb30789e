"""The GEMV chain (glc_gemv_q4k_chain_dev) on the GPU.

* every job of a chain of independent SET jobs is bit-identical to the
  stand-alone GEMV (glc_gemv_q4k_dev) on the same inputs (the same lane
  layout and reduction order), at the Mixtral gate/up and down shapes and at
  the Qwen2.5-14B shapes (K = 5120, 13824: a partly idle last warp);
* a dependent chain (RMSNorm'd QKV-like SET, ADD residual, RMSNorm'd GATE_UP,
  ADD down projection reading the GATE_UP output) against the oracle's float64
  chain within rel-L2 1e-4 per output (GEMV tolerance);
* N smaller than the CTA count (CTAs with no rows) and argument checks.
"""
import numpy as np
import pytest

from test_gpu_parity import GEMV_TOL, rel_l2, stream

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("shapes", [[(4096, 2048), (14336, 1024), (4096, 777)],
                                    [(5120, 7168), (13824, 5120), (5120, 100)]])
def test_independent_jobs_bit_identical_to_single_gemv(cuda, glc, oracle, shapes):
    torch = cuda
    jobs, singles, keep = [], [], []
    for i, (K, N) in enumerate(shapes):
        W = _dev(torch, oracle.synth_q4k(70 + i, 3, N, K))
        x = _dev(torch, oracle.fill_normal(80 + i, 1, 1.0, K))
        y = torch.empty(N, device="cuda")
        y1 = torch.empty(N, device="cuda")
        keep += [W, x]
        jobs.append(dict(W=W.data_ptr(), x=x.data_ptr(), y=y.data_ptr(), K=K, N=N))
        glc.gemv_q4k_dev(W.data_ptr(), x.data_ptr(), y1.data_ptr(), K, N, stream(torch))
        singles.append((y, y1))
    glc.gemv_q4k_chain_dev(jobs, stream(torch))
    torch.cuda.synchronize()
    glc.gemv_poll_error()
    for y, y1 in singles:
        assert torch.equal(y, y1)


def _rms(x, w, eps):
    x = np.asarray(x, np.float64)
    return x / np.sqrt(np.mean(x * x) + eps) * np.asarray(w, np.float64)


def test_dependent_chain_matches_oracle(cuda, glc, oracle):
    """x1 = x0 + Wo (RMSNorm(x0) w_a)      (SET into t, ADD into x1; as a layer's O path)
       a  = SiLU(Wg h) * (Wu h), h = RMSNorm(x1) w_f
       x2 = x1 + Wd a"""
    torch = cuda
    D, FF, eps = 1024, 2816, 1e-6
    rng = np.random.default_rng(5)
    x0 = rng.standard_normal(D).astype(np.float32)
    wa = (1.0 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    wf = (1.0 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    Wq = oracle.synth_q4k(91, 1, D, D)
    Wo = oracle.synth_q4k(91, 2, D, D)
    Wg = oracle.synth_q4k(91, 3, FF, D)
    Wu = oracle.synth_q4k(91, 4, FF, D)
    Wd = oracle.synth_q4k(91, 5, D, FF)
    d = {k: _dev(torch, v) for k, v in dict(x0=x0, wa=wa, wf=wf, Wq=Wq, Wo=Wo, Wg=Wg, Wu=Wu, Wd=Wd).items()}
    x = d["x0"].clone()
    t = torch.empty(D, device="cuda")
    a = torch.empty(FF, device="cuda")
    jobs = [
        dict(W=d["Wq"].data_ptr(), x=x.data_ptr(), y=t.data_ptr(), K=D, N=D, norm_w=d["wa"].data_ptr(), norm_eps=eps),
        dict(W=d["Wo"].data_ptr(), x=t.data_ptr(), y=x.data_ptr(), K=D, N=D, op="add", after_previous=True),
        dict(W=d["Wg"].data_ptr(), W_up=d["Wu"].data_ptr(), x=x.data_ptr(), y=a.data_ptr(), K=D, N=FF, op="gate_up",
             norm_w=d["wf"].data_ptr(), norm_eps=eps, after_previous=True),
        dict(W=d["Wd"].data_ptr(), x=a.data_ptr(), y=x.data_ptr(), K=FF, N=D, op="add", after_previous=True),
    ]
    glc.gemv_q4k_chain_dev(jobs, stream(torch))
    torch.cuda.synchronize()
    glc.gemv_poll_error()

    def mv(W, v, K, N):
        return oracle.dequant(W, N * K).reshape(N, K).astype(np.float64) @ np.asarray(v, np.float64)

    want_t = mv(Wq, _rms(x0, wa, eps), D, D)
    want_x1 = x0.astype(np.float64) + mv(Wo, want_t, D, D)
    h = _rms(want_x1, wf, eps)
    g, u = mv(Wg, h, D, FF), mv(Wu, h, D, FF)
    want_a = g / (1.0 + np.exp(-g)) * u
    want_x2 = want_x1 + mv(Wd, want_a, FF, D)
    assert rel_l2(t.cpu().numpy(), want_t) <= GEMV_TOL
    assert rel_l2(a.cpu().numpy(), want_a) <= GEMV_TOL
    assert rel_l2(x.cpu().numpy(), want_x2) <= GEMV_TOL


def test_repeated_chains_keep_the_barrier_consistent(cuda, glc, oracle):
    """Many launches of a 3-job dependent chain in a row (the barrier counter
    only grows; each launch adds whole instances): outputs stay identical."""
    torch = cuda
    K = N = 512
    W = _dev(torch, oracle.synth_q4k(17, 1, N, K))
    x = _dev(torch, oracle.fill_normal(18, 1, 0.1, K))
    y1, y2, y3 = (torch.empty(N, device="cuda") for _ in range(3))
    jobs = [dict(W=W.data_ptr(), x=x.data_ptr(), y=y1.data_ptr(), K=K, N=N),
            dict(W=W.data_ptr(), x=y1.data_ptr(), y=y2.data_ptr(), K=K, N=N, after_previous=True),
            dict(W=W.data_ptr(), x=y2.data_ptr(), y=y3.data_ptr(), K=K, N=N, after_previous=True)]
    glc.gemv_q4k_chain_dev(jobs, stream(torch))
    torch.cuda.synchronize()
    ref = y3.clone()
    for _ in range(50):
        glc.gemv_q4k_chain_dev(jobs, stream(torch))
    torch.cuda.synchronize()
    glc.gemv_poll_error()
    assert torch.equal(y3, ref)
    # and the chain equals three single GEMVs in a row
    z1, z2, z3 = (torch.empty(N, device="cuda") for _ in range(3))
    glc.gemv_q4k_dev(W.data_ptr(), x.data_ptr(), z1.data_ptr(), K, N, stream(torch))
    glc.gemv_q4k_dev(W.data_ptr(), z1.data_ptr(), z2.data_ptr(), K, N, stream(torch))
    glc.gemv_q4k_dev(W.data_ptr(), z2.data_ptr(), z3.data_ptr(), K, N, stream(torch))
    torch.cuda.synchronize()
    assert torch.equal(z3, ref)


def test_chain_rejects_bad_arguments(cuda, glc):
    torch = cuda
    buf = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(glc.GlcError, match="multiple of 256"):
        glc.gemv_q4k_chain_dev([dict(W=p, x=p, y=p, K=300, N=4)])
    with pytest.raises(glc.GlcError):  # GATE_UP without its up rows
        glc.gemv_q4k_chain_dev([dict(W=p, x=p, y=p, K=256, N=4, op="gate_up")])
    with pytest.raises(glc.GlcError):  # misaligned input
        glc.gemv_q4k_chain_dev([dict(W=p, x=p + 4, y=p, K=256, N=4)])
    with pytest.raises(glc.GlcError):  # too many jobs
        glc.gemv_q4k_chain_dev([dict(W=p, x=p, y=p, K=256, N=4)] * 65)
