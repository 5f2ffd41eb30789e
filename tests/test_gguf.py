"""GGUF reader (glacier.inference.distributed_b200.gguf) on files written here.

The writer below follows the GGUF v3 layout (header, typed metadata, tensor
infos, data section at the alignment).  No real GGUF checkpoint exists
offline, so the files are synthetic: Q4_K expert tensors from the oracle's
seeded generator and an F32 router.
"""
import struct
import types

import numpy as np
import pytest

from glacier.inference.distributed_b200 import gguf as G


def _s(b: bytearray, text: str):
    raw = text.encode()
    b += struct.pack("<Q", len(raw)) + raw


def write_gguf(path, metadata, tensors, align=32, version=3):
    """metadata: {key: (type, value)}; tensors: [(name, dims, ggml_type, bytes)]."""
    b = bytearray(struct.pack("<IIQQ", G.GGUF_MAGIC, version, len(tensors), len(metadata)))
    for k, (t, v) in metadata.items():
        _s(b, k)
        b += struct.pack("<I", t)
        if t == 8:
            _s(b, v)
        elif t == 9:
            et, items = v
            b += struct.pack("<IQ", et, len(items))
            for it in items:
                b += struct.pack(G._SCALAR[et], it)
        else:
            b += struct.pack(G._SCALAR[t], v)
    off, offs = 0, []
    for name, dims, t, data in tensors:
        offs.append(off)
        off = (off + len(data) + align - 1) // align * align
    for (name, dims, t, data), o in zip(tensors, offs):
        _s(b, name)
        b += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", t, o)
    b += b"\0" * ((-len(b)) % align)
    base = len(b)
    for (name, dims, t, data), o in zip(tensors, offs):
        b += b"\0" * (base + o - len(b))
        b += bytes(data)
    open(path, "wb").write(b)


def moe_tensors(oracle, L, D, F, E, seed):
    gate = np.concatenate([oracle.synth_q4k(seed, oracle.expert_tag(e, 0), F, D) for e in range(E)])
    up = np.concatenate([oracle.synth_q4k(seed, oracle.expert_tag(e, 1), F, D) for e in range(E)])
    down = np.concatenate([oracle.synth_q4k(seed, oracle.expert_tag(e, 2), D, F) for e in range(E)])
    router_ed = oracle.fill_normal(seed, 2, 0.02, E * D).reshape(E, D)  # GGUF: [E][D]
    t = [(f"blk.{L}.ffn_gate_exps.weight", (D, F, E), G.GGML_TYPE_Q4_K, gate),
         (f"blk.{L}.ffn_up_exps.weight", (D, F, E), G.GGML_TYPE_Q4_K, up),
         (f"blk.{L}.ffn_down_exps.weight", (F, D, E), G.GGML_TYPE_Q4_K, down),
         (f"blk.{L}.ffn_gate_inp.weight", (D, E), G.GGML_TYPE_F32, router_ed.tobytes())]
    return t, (gate, up, down, router_ed)


META = {"general.architecture": (8, "mixtral"), "mixtral.expert_count": (4, 4),
        "mixtral.rope.freq_base": (6, 1e6), "general.flags": (9, (4, [1, 2, 3])), "x.ok": (7, True)}


def test_round_trip_metadata_and_tensors(tmp_path, oracle):
    D, F, E = 256, 512, 4
    t, (gate, up, down, rt) = moe_tensors(oracle, 3, D, F, E, 5)
    p = tmp_path / "m.gguf"
    write_gguf(p, META, t, align=64)
    f = G.GgufFile(str(p))
    assert f.version == 3
    assert f.metadata["general.architecture"] == "mixtral" and f.metadata["mixtral.expert_count"] == 4
    assert f.metadata["general.flags"] == [1, 2, 3] and f.metadata["x.ok"] is True
    assert abs(f.metadata["mixtral.rope.freq_base"] - 1e6) < 1
    assert f.tensors["blk.3.ffn_down_exps.weight"].dims == (F, D, E)
    assert np.array_equal(f.raw("blk.3.ffn_gate_exps.weight"), gate)
    assert np.array_equal(f.raw("blk.3.ffn_down_exps.weight"), down)
    assert np.array_equal(f.f32("blk.3.ffn_gate_inp.weight"), rt)


def _fake_worker(D, F, E, begin=0, count=0, Fs=0):
    got = {}
    w = types.SimpleNamespace(hidden_dim=D, expert_ffn_dim=F, num_experts=E,
                              desc=types.SimpleNamespace(expert_begin=begin, expert_count=count, shared_ffn_dim=Fs))
    w.load_layer = lambda layer, *arrays: got.update(layer=layer, arrays=arrays)
    return w, got


def test_load_moe_layer_layouts_and_shard(tmp_path, oracle):
    D, F, E = 256, 512, 4
    t, (gate, up, down, rt) = moe_tensors(oracle, 7, D, F, E, 9)
    p = tmp_path / "m.gguf"
    write_gguf(p, META, t)
    f = G.GgufFile(str(p))
    w, got = _fake_worker(D, F, E)
    G.load_moe_layer(w, f, 0, file_layer=7)
    a = got["arrays"]
    assert got["layer"] == 0
    assert np.array_equal(a[0], gate) and np.array_equal(a[1], up) and np.array_equal(a[2], down)
    assert np.array_equal(a[3], rt.T)  # router to [D][E]
    # an expert-parallel shard takes experts [1, 3)
    w, got = _fake_worker(D, F, E, begin=1, count=2)
    G.load_moe_layer(w, f, 0, file_layer=7)
    per_gu, per_dn = F * (D // 256) * 144, D * (F // 256) * 144
    assert np.array_equal(got["arrays"][0], gate[per_gu:3 * per_gu])
    assert np.array_equal(got["arrays"][2], down[per_dn:3 * per_dn])


def test_rejects_bad_files_and_shapes(tmp_path, oracle):
    D, F, E = 256, 512, 4
    t, _ = moe_tensors(oracle, 0, D, F, E, 1)
    p = tmp_path / "m.gguf"
    write_gguf(p, META, t)
    raw = p.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + raw[4:])
    with pytest.raises(G.GgufError):
        G.GgufFile(str(bad))
    bad.write_bytes(raw[:len(raw) // 2])  # data cut short
    with pytest.raises(G.GgufError):
        G.GgufFile(str(bad))
    f = G.GgufFile(str(p))
    w, _ = _fake_worker(D, 2 * F, E)  # the layer wants another F
    with pytest.raises(G.GgufError):
        G.load_moe_layer(w, f, 0)
    w, _ = _fake_worker(D, F, E)
    with pytest.raises(G.GgufError):  # no block 5
        G.load_moe_layer(w, f, 0, file_layer=5)
