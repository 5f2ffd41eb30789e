"""Decode attention on the GPU (glc_attn_decode_dev) against the float64 oracle.

Tolerances: output rel-L2 <= 1e-3 against the oracle evaluated on the same
fp16 caches (the kernel accumulates in fp32 and rotates in fp32 with
double-precision angles); cache rows: the stored value row is bit-exact (one
fp32 -> fp16 rounding), the stored rotated key within one fp16 ulp (fp32 vs
float64 rotation before the same rounding), every other row untouched.
"""
import numpy as np
import pytest

from oracle import attention as att

pytestmark = pytest.mark.gpu

TOL = 1e-3
THETA = 1e6


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def run(torch, glc, q, k, v, kc, vc, pos):
    Hq, Hkv, L = q.shape[0], k.shape[0], kc.shape[1]
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dkc = torch.from_numpy(kc.view(np.uint16).copy()).cuda()
    dvc = torch.from_numpy(vc.view(np.uint16).copy()).cuda()
    out = torch.empty(Hq, 128, device="cuda")
    nb = glc.attn_workspace_bytes(Hq, Hkv, L)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    glc.attn_decode_dev(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), Hq, Hkv, L,
                        pos, THETA, out.data_ptr(), ws.data_ptr(), nb, stream=1)
    torch.cuda.synchronize()
    return (out.cpu().numpy(), dkc.cpu().numpy().view(np.float16), dvc.cpu().numpy().view(np.float16))


@pytest.mark.parametrize("Hq,Hkv,L,pos", [(40, 8, 2048, 0), (40, 8, 2048, 1), (40, 8, 2048, 63),
                                          (40, 8, 2048, 64), (40, 8, 2048, 2047), (48, 8, 4096, 4095),
                                          (8, 8, 256, 100), (64, 8, 512, 300), (5, 1, 130, 129)])
def test_attention_matches_oracle(cuda, glc, Hq, Hkv, L, pos):
    torch = cuda
    rng = np.random.default_rng(1000 + pos + Hq)
    q = rng.standard_normal((Hq, 128)).astype(np.float32)
    k = rng.standard_normal((Hkv, 128)).astype(np.float32)
    v = rng.standard_normal((Hkv, 128)).astype(np.float32)
    kc = rng.standard_normal((Hkv, L, 128)).astype(np.float16)  # rows > pos hold garbage on purpose
    vc = rng.standard_normal((Hkv, L, 128)).astype(np.float16)
    out, gk, gv = run(torch, glc, q, k, v, kc, vc, pos)
    ref, rk, rv = att.attn_decode(q, k, v, kc, vc, pos, THETA)
    assert rel_l2(out, ref) <= TOL
    assert np.array_equal(gv, rv)
    ulp = np.abs(gk[:, pos].view(np.int16).astype(np.int32) - rk[:, pos].view(np.int16).astype(np.int32))
    assert ulp.max() <= 1
    mask = np.ones(L, bool)
    mask[pos] = False
    assert np.array_equal(gk[:, mask], kc[:, mask])


def test_sequential_decode_steps(cuda, glc):
    """Positions 0..69 one after another on the same caches (crosses a chunk
    boundary); each step is checked against the oracle on the GPU's caches."""
    torch = cuda
    Hq, Hkv, L = 8, 2, 128
    rng = np.random.default_rng(7)
    dkc = torch.zeros(Hkv, L, 128, dtype=torch.int16, device="cuda")
    dvc = torch.zeros(Hkv, L, 128, dtype=torch.int16, device="cuda")
    nb = glc.attn_workspace_bytes(Hq, Hkv, L)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    out = torch.empty(Hq, 128, device="cuda")
    for pos in range(70):
        q = rng.standard_normal((Hq, 128)).astype(np.float32)
        k = rng.standard_normal((Hkv, 128)).astype(np.float32)
        v = rng.standard_normal((Hkv, 128)).astype(np.float32)
        kc = dkc.cpu().numpy().view(np.float16)
        vc = dvc.cpu().numpy().view(np.float16)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        glc.attn_decode_dev(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dkc.data_ptr(), dvc.data_ptr(), Hq, Hkv, L,
                            pos, THETA, out.data_ptr(), ws.data_ptr(), nb, stream=1)
        torch.cuda.synchronize()
        ref, _, _ = att.attn_decode(q, k, v, kc, vc, pos, THETA)
        assert rel_l2(out.cpu().numpy(), ref) <= TOL, pos


def test_attention_rejects_bad_arguments(cuda, glc):
    torch = cuda
    buf = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(glc.GlcError):  # head_dim 64
        glc.attn_decode_dev(p, p, p, p, p, 8, 8, 16, 0, THETA, p, p, 1 << 20, head_dim=64, stream=1)
    with pytest.raises(glc.GlcError):  # 16 query heads per KV head
        glc.attn_decode_dev(p, p, p, p, p, 16, 1, 16, 0, THETA, p, p, 1 << 20, stream=1)
    with pytest.raises(glc.GlcError):  # position outside the cache
        glc.attn_decode_dev(p, p, p, p, p, 8, 8, 16, 16, THETA, p, p, 1 << 20, stream=1)
    with pytest.raises(glc.GlcError):  # cache longer than the kernel takes (rejected before any launch)
        glc.attn_decode_dev(p, p, p, p, p, 8, 8, 65536, 3, THETA, p, p, 1 << 20, stream=1)
    with pytest.raises(glc.GlcError):  # workspace too small
        glc.attn_decode_dev(p, p, p, p, p, 8, 8, 16, 3, THETA, p, p, 16, stream=1)
