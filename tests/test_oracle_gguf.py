"""Q4_K and GGUF parity pinned against the format's published implementation.

The reference's Q4_K mat-vec lives in the un-vendored ``Glacier.Inference``
1.3.2 package (call site CpuWarmExpertPoolWorker.cs:379, external
``QuantKernels.MatVecMul``), so no reference code or test pins the Q4_K math.
The GGUF project's own Python package, ``gguf`` (gguf-py 0.19.0 on this
image), carries the published Q4_K dequantiser (``gguf.quants.Q4_K``) and the
GGUF file writer and reader.  These tests pin, on the CPU:

* the oracle's Q4_K dequantisation against ``gguf.quants.dequantize`` bit for
  bit (both compute ``(d*sc)*q - dmin*m`` in fp32), on the seeded generator's
  blocks at every K the configs use and on every known-answer block;
* the oracle's GEMV against a float64 dot over gguf's dequantised rows;
* the repo's GGUF reader against files written by ``gguf.GGUFWriter``, and the
  repo's test writer's files against ``gguf.GGUFReader``.
"""
import json
import os
import types

import numpy as np
import pytest

gguf = pytest.importorskip("gguf", reason="gguf-py (the GGUF project's Python package) is not installed")
from gguf import GGMLQuantizationType as QT  # noqa: E402

from glacier.inference.distributed_b200 import gguf as G  # noqa: E402

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
Q4K = json.load(open(os.path.join(REPO, "tests", "golden", "q4k_known_answers.json")))


def _gguf_dequant(blocks: np.ndarray) -> np.ndarray:
    return gguf.quants.dequantize(np.ascontiguousarray(blocks, np.uint8).reshape(-1, 144), QT.Q4_K).reshape(-1)


@pytest.mark.parametrize("K,rows", [(256, 64), (4096, 8), (14336, 3), (20480, 2), (3584, 5), (2560, 7)])
def test_dequant_equals_gguf_py_bitwise(oracle, K, rows):
    blocks = oracle.synth_q4k(20241201, oracle.expert_tag(3, 1), rows, K)
    mine = oracle.dequant(blocks, rows * K)
    ref = _gguf_dequant(blocks).astype(np.float32)
    assert mine.shape == ref.shape
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


def test_known_answer_blocks_equal_gguf_py(oracle):
    for case in Q4K["cases"]:
        blk = np.array(case["block"], np.uint8)
        ref = _gguf_dequant(blk).astype(np.float32)
        mine = oracle.dequant(blk, 256)
        assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32)), case["name"]
        # and the committed closed-form answers agree with gguf-py too
        assert np.array_equal(np.array(case["dequant"], np.float32), ref), case["name"]


def test_extreme_fields_equal_gguf_py(oracle):
    """Every 6-bit scale/min value, both nibbles, and d / dmin at fp16 extremes
    (largest normal, subnormal, negative, zero)."""
    rng = np.random.default_rng(11)
    blocks = rng.integers(0, 256, size=(64, 144), dtype=np.uint8)
    specials = np.array([0x7BFF, 0x0001, 0x8400, 0x0000, 0x3C00, 0xFBFF, 0x03FF, 0x1400], np.uint16)
    for i in range(64):
        blocks[i, 0:2] = np.frombuffer(specials[i % 8].tobytes(), np.uint8)
        blocks[i, 2:4] = np.frombuffer(specials[(i // 8) % 8].tobytes(), np.uint8)
    mine = oracle.dequant(blocks.reshape(-1), 64 * 256)
    ref = _gguf_dequant(blocks).astype(np.float32)
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("K,N", [(4096, 96), (14336, 32), (3584, 64), (20480, 16)])
def test_gemv_matches_float64_dot_over_gguf_rows(oracle, K, N):
    W = oracle.synth_q4k(7, oracle.expert_tag(0, 2), N, K)
    x = oracle.fill_normal(7, 1, 1.0, K)
    y = oracle.gemv(W, x, K, N)
    Wd = _gguf_dequant(W).astype(np.float64).reshape(N, K)
    ref = Wd @ x.astype(np.float64)
    rel = np.linalg.norm(y.astype(np.float64) - ref) / np.linalg.norm(ref)
    assert rel <= 1e-6, rel


# ------------------------------------------------------------------ GGUF files
def _moe_arrays(oracle, D, F, E, Fs, seed):
    gate = np.stack([oracle.synth_q4k(seed, oracle.expert_tag(e, 0), F, D).reshape(F, -1) for e in range(E)])
    up = np.stack([oracle.synth_q4k(seed, oracle.expert_tag(e, 1), F, D).reshape(F, -1) for e in range(E)])
    down = np.stack([oracle.synth_q4k(seed, oracle.expert_tag(e, 2), D, F).reshape(D, -1) for e in range(E)])
    router_ed = oracle.fill_normal(seed, 2, 0.02, E * D).reshape(E, D)
    sh = dict(gate=oracle.synth_q4k(seed, 101, Fs, D).reshape(Fs, -1),
              up=oracle.synth_q4k(seed, 102, Fs, D).reshape(Fs, -1),
              down=oracle.synth_q4k(seed, 103, D, Fs).reshape(D, -1),
              gvec=oracle.fill_normal(seed, 104, 0.02, D).reshape(1, D))
    return gate, up, down, router_ed, sh


def test_gguf_writer_file_loads_through_repo_reader(tmp_path, oracle):
    """A Qwen2-MoE-shaped block written by gguf.GGUFWriter (Q4_K experts and
    shared expert as raw blocks, F32 router and shared gate) loads through the
    repo's reader to the same bytes, in the layouts load_moe_layer hands on."""
    D, F, E, Fs, L = 512, 256, 8, 768, 2
    gate, up, down, router_ed, sh = _moe_arrays(oracle, D, F, E, Fs, 31)
    path = str(tmp_path / "w.gguf")
    w = gguf.GGUFWriter(path, "qwen2moe")
    w.add_block_count(L + 1)
    w.add_expert_count(E)
    w.add_uint32("qwen2moe.expert_used_count", 8)
    w.add_float32("qwen2moe.rope.freq_base", 1e6)
    w.add_tensor(f"blk.{L}.ffn_gate_exps.weight", gate, raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_up_exps.weight", up, raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_down_exps.weight", down, raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_gate_inp.weight", router_ed)
    w.add_tensor(f"blk.{L}.ffn_gate_shexp.weight", sh["gate"], raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_up_shexp.weight", sh["up"], raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_down_shexp.weight", sh["down"], raw_dtype=QT.Q4_K)
    w.add_tensor(f"blk.{L}.ffn_gate_inp_shexp.weight", sh["gvec"])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    f = G.GgufFile(path)
    assert f.metadata["general.architecture"] == "qwen2moe"
    assert f.metadata["qwen2moe.expert_count"] == E
    assert f.metadata["qwen2moe.expert_used_count"] == 8
    assert f.tensors[f"blk.{L}.ffn_gate_exps.weight"].dims == (D, F, E)
    assert f.tensors[f"blk.{L}.ffn_down_exps.weight"].dims == (F, D, E)
    assert f.tensors[f"blk.{L}.ffn_gate_exps.weight"].ggml_type == G.GGML_TYPE_Q4_K
    assert np.array_equal(f.raw(f"blk.{L}.ffn_up_exps.weight"), up.reshape(-1))

    got = {}
    worker = types.SimpleNamespace(hidden_dim=D, expert_ffn_dim=F, num_experts=E,
                                   desc=types.SimpleNamespace(expert_begin=2, expert_count=4, shared_ffn_dim=Fs))
    worker.load_layer = lambda layer, *arrays: got.update(layer=layer, arrays=arrays)
    G.load_moe_layer(worker, f, 0, file_layer=L)
    a = got["arrays"]
    assert np.array_equal(a[0], gate[2:6].reshape(-1))  # the shard's experts 2..5
    assert np.array_equal(a[1], up[2:6].reshape(-1))
    assert np.array_equal(a[2], down[2:6].reshape(-1))
    assert np.array_equal(a[3], router_ed.T)  # [D][E]
    assert np.array_equal(a[4], sh["gate"].reshape(-1))
    assert np.array_equal(a[5], sh["up"].reshape(-1))
    assert np.array_equal(a[6], sh["down"].reshape(-1))
    assert np.array_equal(a[7], sh["gvec"].reshape(-1))
    # and the expert bytes dequantise identically through gguf-py and the oracle
    e3 = f.raw(f"blk.{L}.ffn_gate_exps.weight")[3 * F * (D // 256) * 144:4 * F * (D // 256) * 144]
    assert np.array_equal(oracle.dequant(np.ascontiguousarray(e3), F * D), _gguf_dequant(e3).astype(np.float32))


def test_repo_written_file_reads_through_gguf_reader(tmp_path, oracle):
    """The files the repo's tests write (tests/test_gguf.py writer) parse with
    gguf.GGUFReader to the same tensors, shapes and metadata."""
    from test_gguf import META, moe_tensors, write_gguf
    D, F, E = 256, 512, 4
    t, (gate, up, down, rt) = moe_tensors(oracle, 5, D, F, E, 13)
    p = str(tmp_path / "r.gguf")
    write_gguf(p, META, t, align=32)
    r = gguf.GGUFReader(p)
    names = {tt.name: tt for tt in r.tensors}
    ge = names["blk.5.ffn_gate_exps.weight"]
    assert ge.tensor_type == QT.Q4_K
    assert [int(v) for v in ge.shape] == [D, F, E]
    assert np.array_equal(np.asarray(ge.data).reshape(-1), gate)
    dn = names["blk.5.ffn_down_exps.weight"]
    assert np.array_equal(np.asarray(dn.data).reshape(-1), down)
    ri = names["blk.5.ffn_gate_inp.weight"]
    assert ri.tensor_type == QT.F32
    assert np.array_equal(np.asarray(ri.data).reshape(E, D), rt)
    arch = r.fields["general.architecture"]
    assert bytes(arch.parts[arch.data[0]]).decode() == "mixtral"
    # gguf-py's dequantisation of the file's expert bytes equals the oracle's
    blocks = np.asarray(ge.data).reshape(-1)[:F * (D // 256) * 144]
    assert np.array_equal(oracle.dequant(np.ascontiguousarray(blocks), F * D), _gguf_dequant(blocks).astype(np.float32))
