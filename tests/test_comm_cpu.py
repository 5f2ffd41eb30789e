"""The communicator entry points of the C ABI without a GPU: the NCCL id is
made on the host (NCCL is loaded at first use), and joining a communicator
with no device fails cleanly with a status instead of crashing."""
import pytest

from glacier.inference.distributed_b200 import Communicator, GlcError
from glacier.inference.distributed_b200 import _lib


def test_unique_id_is_128_fresh_bytes():
    a, b = Communicator.unique_id(), Communicator.unique_id()
    assert len(a) == len(b) == _lib.GLC_COMM_ID_BYTES
    assert a != b


def test_create_rejects_bad_arguments():
    uid = Communicator.unique_id()
    with pytest.raises(GlcError) as e:
        Communicator(uid, 0, 0, 0)
    assert e.value.status == -1  # GLC_ERR_INVALID_ARG
    with pytest.raises(GlcError):
        Communicator(uid[:100], 2, 0, 0)


def test_create_without_device_reports_cuda_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(GlcError) as e:
        Communicator(Communicator.unique_id(), 1, 0, 0)
    assert e.value.status == -2  # GLC_ERR_CUDA
