"""The dense decoder stage (glc_stage_*) on the GPU against the float64 stage
oracle (oracle/dense.py): weighted RMSNorm, the stacked QKV GEMV with biases,
decode attention over the fp16 KV cache, the O projection and the SwiGLU
feed-forward with residuals, the embedding row and the LM head.

Outputs (the stage's residual stream and the logits) within rel-L2 1e-3 of
the oracle at every position; the KV cache rows the stage writes equal the
oracle's fp16 rows to one fp16 ulp; the arg-max token is the oracle's (or,
at a near tie, a logit within the tolerance of the oracle's maximum).  The
first call of a variant runs eagerly and later calls replay the captured
graph, so a multi-position run covers both.
"""
import numpy as np
import pytest

from test_gpu_parity import LAYER_TOL, rel_l2

pytestmark = pytest.mark.gpu


def _stage(glc, D, FF, Hq, Hkv, begin, count, max_len, vocab=0, emb=False, head=False, eps=1e-6):
    return glc.DenseStage(D, FF, Hq, Hkv, begin, count, max_len, 1e6, eps, vocab, emb, head)


def _oracle_kv(Hkv, max_len):
    return np.zeros((Hkv, max_len, 128), np.float16), np.zeros((Hkv, max_len, 128), np.float16)


def test_small_stage_with_embedding_and_head_over_positions(cuda, glc, oracle):
    from oracle import dense as dn
    torch = cuda
    D, FF, Hq, Hkv, layers, max_len, vocab, seed = 512, 1024, 4, 2, 3, 160, 1000, 31
    st = _stage(glc, D, FF, Hq, Hkv, 0, layers, max_len, vocab, True, True)
    for l in range(layers):
        st.synth_layer(l, seed)
    st.synth_io(seed)
    Ls = [dn.synth_layer(seed, l, D, FF, Hq, Hkv) for l in range(layers)]
    io = dn.synth_io(seed, vocab, D)
    caches = [_oracle_kv(Hkv, max_len) for _ in range(layers)]
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    x_out = torch.empty(D, device="cuda")
    lg = torch.empty(vocab, device="cuda")
    token = 7
    for pos in range(70):  # crosses the attention's 64-position chunk boundary
        tok.fill_(token)
        st.forward_dev(pos, token_ptr=tok.data_ptr(), x_out_ptr=x_out.data_ptr(), logits_ptr=lg.data_ptr(),
                       token_out_ptr=tok_out.data_ptr())
        torch.cuda.synchronize()
        x = dn.embed(io["embedding"], token, D)
        for l in range(layers):
            x, kc, vc = dn.layer_forward(Ls[l], x, pos, caches[l][0], caches[l][1], D, FF, Hq, Hkv, 1e6, 1e-6)
            caches[l] = (kc, vc)
        want = dn.logits(io, x, D, vocab, 1e-6)
        assert rel_l2(x_out.cpu().numpy(), x) <= LAYER_TOL, pos
        got = lg.cpu().numpy()
        assert rel_l2(got, want) <= LAYER_TOL, pos
        g = int(tok_out.item())
        assert g == int(np.argmax(got))
        assert g == int(np.argmax(want)) or want[g] >= want.max() - LAYER_TOL * np.abs(want).max(), pos
        token = g  # greedy decoding feeds the arg-max back
    st.poll_error()
    st.dispose()


def test_qwen25_14b_layer_shape(cuda, glc, oracle):
    """One layer of the Qwen2.5-14B geometry (hidden 5120, FFN 13824, 40 query /
    8 KV heads, head dim 128, RoPE theta 1e6, 2048-position cache), input x
    given, at positions 0, 1, 63, 64, 200 and 2047 (caches filled in that
    order; unwritten rows are zero on both sides)."""
    from oracle import dense as dn
    torch = cuda
    D, FF, Hq, Hkv, max_len, seed = 5120, 13824, 40, 8, 2048, 47
    st = _stage(glc, D, FF, Hq, Hkv, 5, 1, max_len)
    st.synth_layer(0, seed)
    L = dn.synth_layer(seed, 5, D, FF, Hq, Hkv)
    kc, vc = _oracle_kv(Hkv, max_len)
    rng = np.random.default_rng(5)
    x_out = torch.empty(D, device="cuda")
    for pos in (0, 1, 63, 64, 200, 2047):
        x = rng.standard_normal(D).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        st.forward_dev(pos, x_in_ptr=xd.data_ptr(), x_out_ptr=x_out.data_ptr())
        torch.cuda.synchronize()
        want, kc, vc = dn.layer_forward(L, x, pos, kc, vc, D, FF, Hq, Hkv, 1e6, 1e-6)
        r = rel_l2(x_out.cpu().numpy(), want)
        assert r <= LAYER_TOL, (pos, r)
    st.poll_error()
    st.dispose()


def test_stage_rejects_bad_arguments(cuda, glc):
    with pytest.raises(glc.GlcError):
        _stage(glc, 500, 1024, 4, 2, 0, 1, 64)  # hidden not a multiple of 256
    with pytest.raises(glc.GlcError):
        _stage(glc, 512, 1024, 4, 3, 0, 1, 64)  # query heads not a multiple of KV heads
    st = _stage(glc, 512, 1024, 4, 2, 0, 1, 64)
    st.synth_layer(0, 1)
    with pytest.raises(glc.GlcError):
        st.forward_dev(64, x_in_ptr=1, x_out_ptr=1)  # pos beyond the cache
    with pytest.raises(glc.GlcError):
        st.forward_dev(0)  # no input and no embedding
    st.dispose()
