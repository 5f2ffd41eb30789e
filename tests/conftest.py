import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    o.set_threads(os.cpu_count() or 1)
    return o


@pytest.fixture(scope="session")
def glc():
    from glacier.inference import distributed_b200 as g
    g.lib()  # raises if the library was not built
    return g


@pytest.fixture(scope="session")
def cuda(glc):
    """A GPU test must run on the GPU: no device is an error, not a skip."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for a gpu-marked test")
    torch.cuda.init()
    return torch
