"""Writes the golden fixtures under tests/golden/.

reference_vectors.json -- the known-answer cases of the reference's own tests
  for this path, restated from the test sources (file:line cited per case):
  inputs are rebuilt the way the C# test builds them (float32 arithmetic), the
  expected values are the reference tests' assertions.
q4k_known_answers.json -- hand-built Q4_K super-blocks with chosen d, dmin,
  6-bit sub-scales/mins and quants, packed by an independent Python
  implementation of the published GGUF Q4_K layout, with the closed-form
  dequantised values d*sc_j*q - dmin*m_j.  The reference has no Q4_K test (its
  Q4_K code is in the un-vendored Glacier.Inference package), so these pin the
  format, not reference outputs.

Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def header_bytes(seq, tok, layer, dim, prec, flags, batch, scale) -> list[int]:
    # FusedActivationHeader.WriteTo (src/.../Protocol/FusedActivationHeader.cs:135-149)
    return list(struct.pack("<IQiiiBBHf", 0x47414354, seq, tok, layer, dim, prec, flags, batch,
                            scale))


def reference_vectors() -> dict:
    cases = {}
    # PhaseBDistributedRemediationTests.cs:503-521 -- ToEven rounding, SIMD body + scalar tail.
    x = np.array([f32(i - 33) * (f32(127.0) / f32(66.0)) for i in range(67)], np.float32)
    x[0], x[66] = -127.0, 127.0
    x[1], x[2], x[3], x[64], x[65] = 0.5, 1.5, 2.5, -0.5, -1.5
    cases["int8_round_half_even"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/PhaseBDistributedRemediationTests.cs:503-525",
        "input": x.tolist(),
        "expect_codes": {"1": 0, "2": 2, "3": 2, "64": 0, "65": -2},
        "expect_dequant": {"2": 2.0, "65": -2.0},
        "dequant_precision_decimals": 4,
    }
    # DynamicMultiPrecisionWireTests.cs:124-142 -- scale in bytes 0..3, codes +-127.
    cases["int8_scale_first4"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DynamicMultiPrecisionWireTests.cs:124-142",
        "dim": 5120, "nonzero": {"0": 12.7, "100": -12.7},
        "expect_scale": float(f32(12.7) / f32(127.0)), "scale_decimals": 5,
        "expect_codes": {"0": 127, "100": -127},
    }
    # DynamicMultiPrecisionWireTests.cs:171-187 -- zero vector.
    cases["int8_zero_vector"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DynamicMultiPrecisionWireTests.cs:171-187",
        "dim": 5120, "expect_scale": 1.0, "expect_all_codes": 0,
    }
    # DynamicMultiPrecisionWireTests.cs:190-204 -- extreme and subnormal inputs.
    cases["int8_extreme"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DynamicMultiPrecisionWireTests.cs:190-204",
        "dim": 5120, "nonzero": {"0": 1e-35, "1": -1e-35, "2": 1e15, "3": -1e15},
        "expect": "scale finite and > 0",
    }
    # PhaseBDistributedRemediationTests.cs:500-501 -- NaN propagates through FindMaxAbsolute.
    cases["maxabs_nan"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/PhaseBDistributedRemediationTests.cs:497-501",
        "input": [1.0, "nan", 5.0], "expect": "token quantises to zero codes with scale 1.0",
    }
    # PhaseBDistributedRemediationTests.cs:528-538 -- FP8 edge cases.
    cases["fp8_edges"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/PhaseBDistributedRemediationTests.cs:528-538",
        "input": [0.0, -0.0, 1.0, -1.5, 0.00390625, 448.0, -500.0],
        "expect_out0": 0.0, "expect_cosine_gt": 0.99,
    }
    # DynamicMultiPrecisionWireTests.cs:62-72, 116-121, 210-215 -- payload sizes at D=5120.
    cases["payload_sizes"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DynamicMultiPrecisionWireTests.cs:62-72",
        "dim": 5120, "expect": {"0": 20480, "1": 10240, "2": 5124, "3": 5124},
    }
    # DynamicMultiPrecisionWireTests.cs:35-60 -- header round trip.
    cases["header_roundtrip_a"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DynamicMultiPrecisionWireTests.cs:35-60",
        "fields": {"sequence_id": 0x1234567890ABCDEF, "token_index": 42, "layer_index": 17,
                   "hidden_dim": 5120, "precision_mode": 2, "flags": 4 | 2,
                   "scale": float(f32(0.0357)), "batch_tokens": 64},
        "expect_bytes": header_bytes(0x1234567890ABCDEF, 42, 17, 5120, 2, 6, 64, f32(0.0357)),
        "expect_payload_bytes": (5120 + 4) * 64,
    }
    # FusedZeroAllocationTransportTests.cs:43-100 -- LE byte pattern, magic "TCAG".
    cases["header_roundtrip_b"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/FusedZeroAllocationTransportTests.cs:43-100",
        "fields": {"sequence_id": 0xAABBCCDDEEFF0011, "token_index": 105, "layer_index": 19,
                   "hidden_dim": 5120, "precision_mode": 1, "flags": 8 | 2, "scale": 1.25,
                   "batch_tokens": 256},
        "expect_bytes": header_bytes(0xAABBCCDDEEFF0011, 105, 19, 5120, 1, 10, 256, 1.25),
        "expect_magic_bytes": [0x54, 0x43, 0x41, 0x47],
        "expect_offsets": {"Magic": 0, "SequenceId": 4, "TokenIndex": 12, "LayerIndex": 16,
                           "HiddenDim": 20, "PrecisionMode": 24, "Flags": 25, "BatchTokens": 26,
                           "Scale": 28},
        "expect_payload_bytes": 5120 * 256 * 2,
    }
    # DistributedPipelineTests.cs:76-97 -- RMSNorm of a constant 2.0 vector.
    cases["rmsnorm_constant"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DistributedPipelineTests.cs:76-97",
        "dim": 64, "value": 2.0, "expect_range": [0.99, 1.01],
    }
    # DistributedPipelineTests.cs:100-139 -- residual + weighted accumulate.
    cases["combine_exact"] = {
        "source": "tests/Glacier.Inference.Distributed.Tests/DistributedPipelineTests.cs:100-139",
        "dim": 64, "residual": 10.0, "experts": [[2.0, 0.5], [4.0, 0.25]],
        "expect_after": [10.0, 11.0, 12.0],
    }
    return cases


def pack_scales(sc: list[int], m: list[int]) -> list[int]:
    """Inverse of the Q4_K 6-bit scale/min unpacking (GGUF layout)."""
    s = [0] * 12
    for j in range(8):
        if j < 4:
            s[j] |= sc[j] & 63
            s[j + 4] |= m[j] & 63
        else:
            s[j + 4] |= (sc[j] & 0xF) | ((m[j] & 0xF) << 4)
            s[j - 4] |= (sc[j] >> 4) << 6
            s[j] |= (m[j] >> 4) << 6
    return s


def q4k_block(d: float, dmin: float, sc, m, q) -> tuple[bytes, list[float]]:
    qs = bytearray(128)
    for c in range(4):
        for l in range(32):
            lo = q[64 * c + l]
            hi = q[64 * c + 32 + l]
            qs[32 * c + l] = (lo & 0xF) | ((hi & 0xF) << 4)
    raw = struct.pack("<ee", d, dmin) + bytes(pack_scales(sc, m)) + bytes(qs)
    dd, dm = (float(np.float16(d)), float(np.float16(dmin)))
    vals = [dd * sc[i // 32] * q[i] - dm * m[i // 32] for i in range(256)]
    return raw, vals


def q4k_known_answers() -> dict:
    cases = []
    specs = [
        ("ramp", 1.0, 0.5, [j + 1 for j in range(8)], [2 * j for j in range(8)],
         [i % 16 for i in range(256)]),
        ("max_fields", 0.0078125, 0.00390625, [63] * 8, [63] * 8, [15] * 256),
        ("high_bits_only", 0.25, 0.125, [48, 32, 16, 63, 47, 31, 17, 60],
         [33, 49, 63, 1, 62, 18, 34, 50], [(7 * i + 3) % 16 for i in range(256)]),
        ("zero_scale", 2.0, 1.0, [0] * 8, [5] * 8, [(i * 5) % 16 for i in range(256)]),
        ("negative_d", -0.5, -0.25, [3, 9, 27, 63, 1, 2, 4, 8], [1, 3, 9, 27, 63, 0, 5, 11],
         [(i * i) % 16 for i in range(256)]),
    ]
    for name, d, dm, sc, m, q in specs:
        raw, vals = q4k_block(d, dm, sc, m, q)
        cases.append({"name": name, "d": d, "dmin": dm, "sc": sc, "m": m, "block": list(raw),
                      "dequant": vals})
    return {"format": "GGUF Q4_K: [d f16][dmin f16][scales 12B][qs 128B]; "
                      "weight = d*sc_j*q - dmin*m_j", "cases": cases}


def main() -> None:
    with open(os.path.join(HERE, "reference_vectors.json"), "w") as f:
        json.dump(reference_vectors(), f, indent=1)
    with open(os.path.join(HERE, "q4k_known_answers.json"), "w") as f:
        json.dump(q4k_known_answers(), f, indent=1)


if __name__ == "__main__":
    main()
