"""The allocation-free dispatch plan (glc_dispatch_plan_noalloc_dev).

Callers that cannot allocate device memory on their hot path -- a decode loop
that must not let cudaMalloc/cudaFree synchronise the device and stall other
streams, or a host that budgets device memory itself -- use this entry point
instead of glc_dispatch_plan_dev.  Its scratch lives in a fixed device array
inside the library.  This file checks, through the C ABI, that it returns the
same plan as the allocating entry point on two calls in a row, and that it
rejects sizes beyond its stated limits.  It is collected last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _plan(torch, fn, ids, E):
    P = ids.numel()
    counts = torch.full((E,), -1, dtype=torch.int32, device="cuda")
    offsets = torch.full((E + 1,), -1, dtype=torch.int32, device="cuda")
    perm = torch.full((P,), -1, dtype=torch.int32, device="cuda")
    inv = torch.full((P,), -1, dtype=torch.int32, device="cuda")
    st = fn(ids.data_ptr(), P, E, counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
            inv.data_ptr(), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return st, [t.cpu().numpy() for t in (counts, offsets, perm, inv)]


@pytest.mark.parametrize("P,E", [(3000, 64), (128, 8)])
def test_noalloc_plan_matches_allocating_entry_point(cuda, glc, P, E):
    torch = cuda
    L = glc.lib()
    rng = np.random.default_rng(P)
    for call in range(2):  # two calls in a row: the shared scratch must not leak state
        ids = torch.from_numpy(rng.integers(0, E, size=P).astype(np.int32)).cuda()
        st_ref, ref = _plan(torch, L.glc_dispatch_plan_dev, ids, E)
        st_new, new = _plan(torch, L.glc_dispatch_plan_noalloc_dev, ids, E)
        assert st_ref == 0 and st_new == 0, glc.lib().glc_last_error()
        for a, b in zip(new, ref):  # integer outputs: identical
            assert np.array_equal(a, b), f"call {call}"


def test_noalloc_plan_rejects_sizes_beyond_limit(cuda, glc):
    L = glc.lib()
    st = L.glc_dispatch_plan_noalloc_dev(1, 65537, 8, 1, 1, 1, 1, None)
    assert st == -1 and b"65536" in L.glc_last_error()
    st = L.glc_dispatch_plan_noalloc_dev(1, 16, 65, 1, 1, 1, 1, None)
    assert st == -1 and b"64 experts" in L.glc_last_error()
