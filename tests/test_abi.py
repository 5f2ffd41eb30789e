"""The C ABI library loads, exports every symbol include/glacier_b200.h
declares, and its host-only entry points (no GPU needed) match the reference
layouts.  No compute call is made here."""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = json.load(open(os.path.join(REPO, "tests", "golden", "reference_vectors.json")))


def declared_functions():
    src = open(os.path.join(REPO, "include", "glacier_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(glc_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol(glc):
    names = declared_functions()
    assert len(names) >= 20
    raw = C.CDLL(glc.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), n
    from glacier.inference.distributed_b200 import _lib
    assert set(names) <= set(_lib.exported_symbols()) | set(names)
    missing = set(names) - set(_lib.exported_symbols())
    assert not missing, f"binding lacks {sorted(missing)}"


def test_abi_version_and_row_bytes(glc):
    assert glc.lib().glc_abi_version() == 1
    assert glc.q4k_row_bytes(4096) == 2304
    assert glc.q4k_row_bytes(14336) == 8064
    assert glc.q4k_row_bytes(100) == -1


def test_wire_token_bytes(glc):
    c = REF["payload_sizes"]
    for mode, size in c["expect"].items():
        assert glc.QuantizationKernels.GetPackedTokenBytes(int(mode), c["dim"]) == size
    assert glc.QuantizationKernels.GetPackedTokenBytes(2, 4096) == 4100
    assert glc.QuantizationKernels.GetPackedTokenBytes(2, 3584) == 3588
    assert glc.QuantizationKernels.GetPackedTokenBytes(9, 10) == 20  # unknown mode -> FP16 size


@pytest.mark.parametrize("key", ["header_roundtrip_a", "header_roundtrip_b"])
def test_fused_header_layout(glc, key):
    c = REF[key]
    f = c["fields"]
    h = glc.FusedActivationHeader(f["sequence_id"], f["token_index"], f["layer_index"],
                                  f["hidden_dim"], f["precision_mode"], f["flags"], f["scale"],
                                  f["batch_tokens"])
    b = h.write_to()
    assert list(b) == c["expect_bytes"]
    back = glc.FusedActivationHeader.read_from(b)
    assert back == h
    assert h.get_payload_byte_count() == c["expect_payload_bytes"]


def test_fused_header_bad_magic_raises(glc):
    b = bytearray(glc.FusedActivationHeader(1, 0, 0, 5120, 2).write_to())
    b[0] ^= 0xFF
    with pytest.raises(glc.GlcError, match="magic"):
        glc.FusedActivationHeader.read_from(bytes(b))
    with pytest.raises(glc.GlcError):
        glc.FusedActivationHeader.read_from(b"\x00" * 8)


def test_header_payload_stage0_token_input(glc):
    h = glc.FusedActivationHeader(1, 0, 0, 5120, 2, flags=0x10, batch_tokens=7)
    assert h.get_payload_byte_count() == 28


def test_wire_host_api_rejects_small_destination(glc):
    x = np.zeros(16, np.float32)
    out = np.zeros(10, np.uint8)
    with pytest.raises(glc.GlcError, match="too small"):
        glc.QuantizationKernels.QuantizeBatch(x, out, 16, 1, 2)


def test_create_without_gpu_fails_loudly(glc):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(glc.GlcError):
        glc.GpuExpertStageWorker(256, 256, 4, 2)
