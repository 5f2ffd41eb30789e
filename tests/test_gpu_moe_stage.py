"""The mixture-of-experts decoder stage (glc_stage_* with num_experts > 0,
Mixtral-style layers) on the GPU against the float64 stage oracle
(oracle/dense.py): attention as in the dense stage (no q/k/v biases), then
the router on RMSNorm(x) * w_ffn (softmax top-k renormalised), the routed
experts' SwiGLU and the k-ordered weighted combine into the residual.

Outputs (the residual stream and the logits) within rel-L2 1e-3 of the
oracle at every position; the arg-max token is the oracle's (or, at a near
tie, a logit within the tolerance of the oracle's maximum).
"""
import numpy as np
import pytest

from test_gpu_parity import LAYER_TOL, rel_l2

pytestmark = pytest.mark.gpu


def _stage(glc, D, F, E, k, Hq, Hkv, begin, count, max_len, vocab=0, emb=False, head=False, eps=1e-5):
    return glc.DenseStage(D, 0, Hq, Hkv, begin, count, max_len, 1e6, eps, vocab, emb, head,
                          num_experts=E, top_k=k, expert_ffn_dim=F, moe_renormalize=True)


def test_small_moe_stage_with_embedding_and_head_over_positions(cuda, glc, oracle):
    from oracle import dense as dn
    torch = cuda
    D, F, E, k, Hq, Hkv, layers, max_len, vocab, seed = 1024, 512, 8, 2, 8, 2, 2, 96, 700, 61
    st = _stage(glc, D, F, E, k, Hq, Hkv, 0, layers, max_len, vocab, True, True)
    for l in range(layers):
        st.synth_layer(l, seed)
    st.synth_io(seed)
    Ls = [dn.synth_moe_layer(seed, l, D, F, E, Hq, Hkv) for l in range(layers)]
    io = dn.synth_io(seed, vocab, D)
    caches = [(np.zeros((Hkv, max_len, 128), np.float16), np.zeros((Hkv, max_len, 128), np.float16))
              for _ in range(layers)]
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    x_out = torch.empty(D, device="cuda")
    lg = torch.empty(vocab, device="cuda")
    token = 11
    seen = set()
    for pos in range(70):  # crosses the attention's 64-position boundary
        tok.fill_(token)
        st.forward_dev(pos, token_ptr=tok.data_ptr(), x_out_ptr=x_out.data_ptr(), logits_ptr=lg.data_ptr(),
                       token_out_ptr=tok_out.data_ptr())
        torch.cuda.synchronize()
        x = dn.embed(io["embedding"], token, D)
        for l in range(layers):
            x, kc, vc, ids = dn.moe_layer_forward(Ls[l], x, pos, caches[l][0], caches[l][1], D, F, k, Hq, Hkv,
                                                  1e6, 1e-5)
            caches[l] = (kc, vc)
            seen.update(ids)
        want = dn.logits(io, x, D, vocab, 1e-5)
        assert rel_l2(x_out.cpu().numpy(), x) <= LAYER_TOL, pos
        got = lg.cpu().numpy()
        assert rel_l2(got, want) <= LAYER_TOL, pos
        g = int(tok_out.item())
        assert g == int(np.argmax(got))
        assert g == int(np.argmax(want)) or want[g] >= want.max() - LAYER_TOL * np.abs(want).max(), pos
        token = g
    assert len(seen) >= 4  # the positions route to several experts
    st.poll_error()
    st.dispose()


def test_mixtral_8x22b_layer_shape(cuda, glc, oracle):
    """One layer of the Mixtral-8x22B geometry (hidden 6144, 8 experts of FFN
    16384, top-2, 48 query / 8 KV heads, a 4096-position cache), input x given,
    at positions 0, 1, 64 and 4095.

    The stored fp16 K / V rows of each position are checked against the
    oracle's within one fp16 ulp plus 3e-4 of the row's rms: the GEMV stages
    its input as int16 codes per 32-block (error about max/32767/sqrt(12)
    per element, ~2e-5 of the rms for normal inputs), so the projection
    feeding a row carries ~2.5e-5 of its norm, ~1e-4 at the largest element
    of a 1024-value row.  The layer output is then compared with the oracle
    run on the rows the stage stored: with these synthetic weights (Q4_K
    fields with a positive mean) the residual becomes a nearly constant
    vector that SwiGLU amplifies quadratically, so a one-ulp fp16 rounding
    difference of a value row alone moves the output by ~1e-3."""
    from oracle import dense as dn
    torch = cuda
    D, F, E, k, Hq, Hkv, max_len, seed = 6144, 16384, 8, 2, 48, 8, 4096, 67
    st = _stage(glc, D, F, E, k, Hq, Hkv, 3, 1, max_len)
    st.synth_layer(0, seed)
    L = dn.synth_moe_layer(seed, 3, D, F, E, Hq, Hkv)
    kc = np.zeros((Hkv, max_len, 128), np.float16)
    vc = np.zeros((Hkv, max_len, 128), np.float16)
    rng = np.random.default_rng(9)
    x_out = torch.empty(D, device="cuda")
    for pos in (0, 1, 64, 4095):
        x = rng.standard_normal(D).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        st.forward_dev(pos, x_in_ptr=xd.data_ptr(), x_out_ptr=x_out.data_ptr())
        torch.cuda.synchronize()
        gk, gv = st.read_kv_cache(0, pos + 1)
        _, ok_, ov_, _ = dn.moe_layer_forward(L, x, pos, kc, vc, D, F, k, Hq, Hkv, 1e6, 1e-5)
        for got_row, want_row in ((gk[:, pos], ok_[:, pos]), (gv[:, pos], ov_[:, pos])):
            # one fp16 ulp of each value plus 3e-4 of the row's rms (the int16-staged projection's error)
            g64, w64 = got_row.astype(np.float64), want_row.astype(np.float64)
            ulp = np.spacing(np.abs(want_row)).astype(np.float64)
            rms = np.sqrt(np.mean(w64 * w64))
            assert np.all(np.abs(g64 - w64) <= ulp + 3e-4 * rms), (pos, float(np.abs(g64 - w64).max()), rms)
            assert rel_l2(g64, w64) <= 3e-4, pos
        want, kc, vc, _ = dn.moe_layer_forward(L, x, pos, kc, vc, D, F, k, Hq, Hkv, 1e6, 1e-5,
                                               stored_rows=(gk[:, pos], gv[:, pos]))
        r = rel_l2(x_out.cpu().numpy(), want)
        assert r <= LAYER_TOL, (pos, r)
    st.poll_error()
    st.dispose()


def test_moe_stage_rejects_bad_arguments(cuda, glc):
    with pytest.raises(glc.GlcError):
        _stage(glc, 512, 512, 9, 2, 4, 2, 0, 1, 64)  # more experts than the router takes
    with pytest.raises(glc.GlcError):
        _stage(glc, 512, 512, 2, 3, 4, 2, 0, 1, 64)  # top-k above the experts
    with pytest.raises(glc.GlcError):
        _stage(glc, 512, 500, 8, 2, 4, 2, 0, 1, 64)  # expert width not a multiple of 256
    st = _stage(glc, 512, 512, 8, 2, 4, 2, 0, 1, 64)
    z = np.zeros(1 << 16, np.uint8)
    with pytest.raises(glc.GlcError):  # a dense layer into a mixture-of-experts stage
        st.load_layer(0, np.ones(512, np.float32), z, z, z, None, None, None, z, np.ones(512, np.float32), z, z, z)
    st.dispose()
