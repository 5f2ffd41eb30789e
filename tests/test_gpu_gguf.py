"""A MoE layer loaded from a GGUF file (gguf.load_moe_layer) computes exactly
what the same tensors loaded directly compute, and matches the oracle."""
import numpy as np
import pytest

from glacier.inference.distributed_b200 import gguf as G
from test_gguf import META, moe_tensors, write_gguf
from test_gpu_parity import LAYER_TOL, rel_l2

pytestmark = pytest.mark.gpu


def test_gguf_layer_matches_direct_load_and_oracle(cuda, glc, oracle, tmp_path):
    D, F, E, k = 512, 1024, 8, 2
    t, (gate, up, down, rt) = moe_tensors(oracle, 1, D, F, E, 31)
    p = tmp_path / "layer.gguf"
    write_gguf(p, META, t)
    f = G.GgufFile(str(p))
    a = glc.GpuExpertStageWorker(D, F, E, k, renormalize=True, max_tokens=4)
    G.load_moe_layer(a, f, 0, file_layer=1)
    b = glc.GpuExpertStageWorker(D, F, E, k, renormalize=True, max_tokens=4)
    b.load_layer(0, gate, up, down, np.ascontiguousarray(rt.T))
    x = oracle.fill_normal(55, 1, 1.0, 3 * D).reshape(3, D)
    oa, ia, wa = a.forward(0, x, 3)
    ob, ib, wb = b.forward(0, x, 3)
    assert np.array_equal(oa, ob) and np.array_equal(ia, ib) and np.array_equal(wa, wb)
    L = {"D": D, "F": F, "E": E, "k": k, "renorm": True, "Fs": 0, "gate": gate, "up": up, "down": down,
         "router": np.ascontiguousarray(rt.T).reshape(-1)}
    ro, rids, _ = oracle.moe_forward(L, x, 3)
    assert np.array_equal(ia, rids)
    assert rel_l2(oa, ro) <= LAYER_TOL
    a.dispose()
    b.dispose()
