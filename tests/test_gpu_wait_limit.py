"""Failure detection on the GPU without a fault.

Every device-side wait of the fused decode kernel is bounded: a wait that runs
out records an error code in the handle's device error word, the kernel
returns, and the host reports GLC_ERR_TIMEOUT and clears the device words.
Here one launch leaves one CTA out of the grid barrier (glc_moe_debug_stall)
with a 10 ms limit, so the other CTAs' wait at the barrier runs out.  Nothing
faults, traps or hangs: the test checks the reported status, then that the
very next launch of the same handle gives the result of a launch made before
the failure, bit for bit (the context and the handle are still usable).
"""
import numpy as np
import pytest

from test_gpu_parity import LAYER_TOL, make_layer, rel_l2, worker_for

pytestmark = pytest.mark.gpu

GLC_ERR_TIMEOUT = -7
LIMIT_NS = 10_000_000  # 10 ms


def test_wait_that_runs_out_is_reported_and_the_handle_recovers(cuda, glc, oracle):
    torch = cuda
    D, F, E, k = 512, 1024, 8, 2
    L = make_layer(oracle, 4242, D, F, E, k)
    w = worker_for(glc, L, max_tokens=4)
    x = oracle.fill_normal(4242, 1, 1.0, D)[None, :]
    good, gids, gw = w.forward(0, x, 3)
    ro, rids, _ = oracle.moe_forward(L, x, 3)
    assert np.array_equal(gids, rids) and rel_l2(good, ro) <= LAYER_TOL

    # host-buffer forward: the error word comes back with the completion words
    for cta in (7, 0):
        w.debug_stall(cta, LIMIT_NS)
        with pytest.raises(glc.GlcError) as e:
            w.forward(0, x, 3)
        assert e.value.status == GLC_ERR_TIMEOUT
        out, ids, wt = w.forward(0, x, 3)
        assert np.array_equal(out, good) and np.array_equal(ids, gids) and np.array_equal(wt, gw)

    # device-pointer forward on the handle's stream: glc_moe_poll_error reports it
    xd = torch.from_numpy(x).cuda()
    od = torch.empty(1, D, device="cuda")
    torch.cuda.synchronize()
    w.debug_stall(3, LIMIT_NS)
    w.forward_dev(0, xd.data_ptr(), 1, 3, od.data_ptr())
    with pytest.raises(glc.GlcError) as e:
        w.poll_error()
    assert e.value.status == GLC_ERR_TIMEOUT
    w.forward_dev(0, xd.data_ptr(), 1, 3, od.data_ptr())
    w.poll_error()
    torch.cuda.synchronize()
    assert np.array_equal(od.cpu().numpy(), good)
    w.dispose()


def test_stall_hook_rejects_bad_arguments(cuda, glc, oracle):
    L = make_layer(oracle, 11, 256, 512, 4, 2)
    w = worker_for(glc, L, max_tokens=1)
    with pytest.raises(glc.GlcError):
        w.debug_stall(-1, LIMIT_NS)
    with pytest.raises(glc.GlcError):
        w.debug_stall(100000, LIMIT_NS)
    with pytest.raises(glc.GlcError):
        w.debug_stall(0, 0)
    w.dispose()
