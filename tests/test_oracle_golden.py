"""The CPU oracle pinned against the reference's own known-answer tests and the
Q4_K format known answers (tests/golden/)."""
import json
import math
import os
import struct

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REF = json.load(open(os.path.join(GOLDEN, "reference_vectors.json")))
Q4K = json.load(open(os.path.join(GOLDEN, "q4k_known_answers.json")))


def _cos(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    return 1.0 if na == 0 or nb == 0 else float(a @ b / (na * nb))


def test_int8_round_half_even(oracle):
    c = REF["int8_round_half_even"]
    x = np.array(c["input"], np.float32)
    buf = oracle.wire_quantize(2, x)
    codes = buf[4:].view(np.int8)
    for i, v in c["expect_codes"].items():
        assert codes[int(i)] == v
    deq = oracle.wire_dequantize(2, buf, 1, x.size)[0]
    for i, v in c["expect_dequant"].items():
        assert round(float(deq[int(i)]) - v, c["dequant_precision_decimals"]) == 0


def test_int8_scale_first4(oracle):
    c = REF["int8_scale_first4"]
    x = np.zeros(c["dim"], np.float32)
    for i, v in c["nonzero"].items():
        x[int(i)] = v
    buf = oracle.wire_quantize(2, x)
    scale = struct.unpack("<f", bytes(buf[:4]))[0]
    assert round(scale - c["expect_scale"], c["scale_decimals"]) == 0
    codes = buf[4:].view(np.int8)
    for i, v in c["expect_codes"].items():
        assert codes[int(i)] == v
    assert buf.size == 5124


def test_int8_zero_and_extreme_and_nan(oracle):
    z = REF["int8_zero_vector"]
    buf = oracle.wire_quantize(2, np.zeros(z["dim"], np.float32))
    assert struct.unpack("<f", bytes(buf[:4]))[0] == z["expect_scale"]
    assert not buf[4:].any()
    e = REF["int8_extreme"]
    x = np.zeros(e["dim"], np.float32)
    for i, v in e["nonzero"].items():
        x[int(i)] = v
    s = struct.unpack("<f", bytes(oracle.wire_quantize(2, x)[:4]))[0]
    assert math.isfinite(s) and s > 0
    n = np.array([1.0, np.nan, 5.0], np.float32)
    buf = oracle.wire_quantize(2, n)
    assert struct.unpack("<f", bytes(buf[:4]))[0] == 1.0 and not buf[4:].any()


def test_fp8_edges(oracle):
    c = REF["fp8_edges"]
    x = np.array(c["input"], np.float32)
    buf = oracle.wire_quantize(3, x)
    out = oracle.wire_dequantize(3, buf, 1, x.size)[0]
    assert out[0] == c["expect_out0"]
    assert _cos(x, out) > c["expect_cosine_gt"]


def test_payload_sizes(oracle):
    c = REF["payload_sizes"]
    for mode, size in c["expect"].items():
        assert oracle.lib().oc_wire_token_bytes(int(mode), c["dim"]) == size


def test_header_bytes(oracle):
    for key in ("header_roundtrip_a", "header_roundtrip_b"):
        c = REF[key]
        f = c["fields"]
        out = np.zeros(32, np.uint8)
        oracle.lib().oc_header_write(f["sequence_id"], f["token_index"], f["layer_index"],
                                     f["hidden_dim"], f["precision_mode"], f["flags"],
                                     f["batch_tokens"], f["scale"], out)
        assert out.tolist() == c["expect_bytes"]
        assert oracle.lib().oc_header_payload_bytes(out) == c["expect_payload_bytes"]
    assert REF["header_roundtrip_b"]["expect_bytes"][:4] == REF["header_roundtrip_b"]["expect_magic_bytes"]


def test_rmsnorm_and_combine(oracle):
    c = REF["rmsnorm_constant"]
    y = oracle.rmsnorm(np.full(c["dim"], c["value"], np.float32))
    assert np.all((y >= c["expect_range"][0]) & (y <= c["expect_range"][1]))
    c = REF["combine_exact"]
    acc = np.full(c["dim"], c["residual"], np.float32)
    seen = [float(acc[0])]
    for val, w in c["experts"]:
        y = np.full(c["dim"], val, np.float32)
        acc = (y * np.float32(w)) + acc
        seen.append(float(acc[0]))
    assert seen == c["expect_after"]


def test_q4k_known_answers(oracle):
    for case in Q4K["cases"]:
        blk = np.array(case["block"], np.uint8)
        got = oracle.dequant(blk, 256).astype(np.float64)
        want = np.array(case["dequant"], np.float64)
        # fp32 evaluation of (d*sc)*q - dmin*m: a few ulp of the largest term
        tol = 4 * np.finfo(np.float32).eps * (np.abs(want).max() + 1e-30)
        assert np.max(np.abs(got - want)) <= tol, case["name"]
        for j in range(8):
            sc = np.zeros(1, np.uint8)
            m = np.zeros(1, np.uint8)
            import ctypes as C
            s_ = C.c_uint8()
            m_ = C.c_uint8()
            oracle.lib().oc_q4k_get_scale_min.argtypes = [C.c_int, C.c_void_p, C.POINTER(C.c_uint8),
                                                          C.POINTER(C.c_uint8)]
            oracle.lib().oc_q4k_get_scale_min(j, blk[4:].ctypes.data, C.byref(s_), C.byref(m_))
            assert (s_.value, m_.value) == (case["sc"][j], case["m"][j]), (case["name"], j)
            del sc, m


def test_fp16_matches_numpy(oracle):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-2, 1.0, 3e3, 6e4)])
    mine = np.array([oracle.lib().oc_f32_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(mine, x.astype(np.float16).view(np.uint16))


def test_synth_q4k_distribution(oracle):
    blk = oracle.synth_q4k(7, oracle.expert_tag(0, 0), rows=64, k=1024)
    b = blk.reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and 0.004 < float(np.mean(d)) < 0.012  # E|N(0,0.01)| = 0.008
    q = np.concatenate([b[:, 16:] & 0xF, b[:, 16:] >> 4]).ravel()
    hist = np.bincount(q, minlength=16) / q.size
    assert np.all(np.abs(hist - 1 / 16) < 0.01)
    again = oracle.synth_q4k(7, oracle.expert_tag(0, 0), rows=64, k=1024)
    assert np.array_equal(blk, again)


def test_dispatch_plan_stable(oracle):
    rng = np.random.default_rng(1)
    E = 8
    ids = rng.integers(0, E, size=(64, 2)).astype(np.int32)
    counts, offsets, perm, inv = oracle.dispatch_plan(ids, E)
    flat = ids.reshape(-1)
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(counts)]))
    assert np.array_equal(perm, np.argsort(flat, kind="stable"))
    assert np.array_equal(inv[perm], np.arange(flat.size))


def test_router_ties_lower_index(oracle):
    logits = np.array([1.0, 3.0, 3.0, 2.0, np.nan, 3.0], np.float32)
    ids = np.empty(3, np.int32)
    w = np.empty(3, np.float32)
    oracle.lib().oc_router_topk(logits, 6, 3, 1, ids, w)
    assert ids.tolist() == [1, 2, 5]
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_routed_topk_empty_is_zero_and_matches_layer(oracle):
    D, F, E = 256, 512, 4
    g = np.concatenate([oracle.synth_q4k(3, oracle.expert_tag(e, 0), F, D) for e in range(E)])
    u = np.concatenate([oracle.synth_q4k(3, oracle.expert_tag(e, 1), F, D) for e in range(E)])
    dn = np.concatenate([oracle.synth_q4k(3, oracle.expert_tag(e, 2), D, F) for e in range(E)])
    x = oracle.fill_normal(3, 1, 1.0, D)
    y = oracle.routed_topk(g, u, dn, D, F, E, x, np.array([2, 9], np.int32), np.array([0.75, 0.25], np.float32))
    y2 = oracle.expert_forward(g[2 * F * 144:3 * F * 144], u[2 * F * 144:3 * F * 144],
                               dn[2 * D * 2 * 144:3 * D * 2 * 144], D, F, x)
    y3 = oracle.expert_forward(g[3 * F * 144:], u[3 * F * 144:], dn[3 * D * 2 * 144:], D, F, x)
    want = (y3 * np.float32(0.25)) + ((y2 * np.float32(0.75)) + np.zeros(D, np.float32))
    assert np.array_equal(y, want)  # id 9 is clamped to E-1 = 3
