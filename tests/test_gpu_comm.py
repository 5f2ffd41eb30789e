"""Two GPUs through the C ABI's own communicator (NCCL inside the library, no
torch.distributed): the entry points a host without torch (the reference's C#
process) uses for multi-GPU work.  Skipped with fewer than two GPUs.

* Stage boundary: rank 0 glc_pp_send's activations in every wire mode, rank 1
  glc_pp_recv's them; header fields and the dequantised values equal the
  oracle codec's bit for bit.
* Expert parallelism: glc_moe_ep_forward over 2 ranks (experts 0..3 and 4..7)
  equals a full single-GPU layer on the same tokens bit for bit, for the
  per-row GEMV experts and for the grouped tensor-core experts.
"""
import os
import sys
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECODE, BATCHED = 4, 8


def _need_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _run(rank, world, uid, fn, errq):
    import faulthandler
    # No NVLink multicast objects: a rank that the watchdog below ends must not
    # leave memory bound to one (NCCL reads this when the communicator opens).
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    faulthandler.dump_traceback_later(180, exit=True)
    try:
        sys.path.insert(0, REPO)
        sys.path.insert(0, os.path.join(REPO, "tests"))
        import torch
        torch.cuda.set_device(rank)
        from glacier.inference.distributed_b200 import Communicator
        comm = Communicator(uid, world, rank, rank)
        try:
            fn(rank, world, comm)
        finally:
            torch.cuda.synchronize()
            comm.dispose()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _spawn(fn, world=2):
    import torch.multiprocessing as mp
    from glacier.inference.distributed_b200 import Communicator
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    uid = Communicator.unique_id()
    procs = [ctx.Process(target=_run, args=(r, world, uid, fn, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(c == 0 for c in codes) and not errs, "\n".join(errs) or f"exit codes {codes}"


def _pp_case(rank, world, comm):
    import torch
    from oracle import oracle as o
    from glacier.inference.distributed_b200 import FusedActivationHeader
    o.build()
    for mode, (T, D) in [(2, (3, 5120)), (3, (2, 4096)), (1, (1, 3584)), (0, (2, 64))]:
        x = o.fill_normal(31 + mode, 1, 1.0, T * D).reshape(T, D)
        if rank == 0:
            hdr = FusedActivationHeader(40 + mode, 2, 27, D, mode, 0, 1.0, T)
            comm.pp_send(1, hdr, torch.from_numpy(x).cuda().data_ptr())
            torch.cuda.synchronize()
        else:
            back = torch.empty(4, D, device="cuda")
            hdr = comm.pp_recv(0, back.data_ptr(), 4, D)
            torch.cuda.synchronize()
            assert (hdr.sequence_id, hdr.layer_index, hdr.hidden_dim, hdr.precision_mode, hdr.batch_tokens) == \
                (40 + mode, 27, D, mode, T)
            want = o.wire_dequantize(mode, np.asarray(o.wire_quantize(mode, x)), T, D)
            assert np.array_equal(back[:T].cpu().numpy(), want)


def test_stage_boundary_through_c_abi(cuda, oracle):
    _need_two_gpus()
    _spawn(_pp_case)


def _ep_case(rank, world, comm):
    import torch
    from oracle import oracle as o
    from glacier.inference import distributed_b200 as glc
    from test_gpu_parity import LAYER_TOL, make_layer, rel_l2
    o.build()
    D, F, E, k, seed = 512, 1024, 8, 2, 777
    L = make_layer(o, seed, D, F, E, k)
    epr = E // world
    T = 3 + rank
    shard = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=world * 4, expert_begin=rank * epr,
                                     expert_count=epr, device=rank)
    shard.synth_layer(0, seed)
    full = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=8, device=rank)
    full.synth_layer(0, seed)
    x = o.fill_normal(900 + rank, 1, 1.0, T * D).reshape(T, D)
    xd = torch.from_numpy(x).cuda()
    for mode in (DECODE, BATCHED):
        flags = 3 | mode
        out = torch.empty(T, D, device="cuda")
        ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
        w = torch.empty(T, k, device="cuda")
        torch.cuda.synchronize()
        shard.ep_forward_dev(comm, 0, xd.data_ptr(), T, flags, out.data_ptr(), ids.data_ptr(), w.data_ptr())
        torch.cuda.synchronize()
        fo, fids, fw = full.forward(0, x, flags)
        assert np.array_equal(ids.cpu().numpy(), fids)
        assert np.array_equal(w.cpu().numpy(), fw)
        assert np.array_equal(out.cpu().numpy(), fo), (mode, float(np.abs(out.cpu().numpy() - fo).max()))
        ro, rids, _ = o.moe_forward(L, x, flags)
        assert np.array_equal(fids, rids)
        assert rel_l2(fo, ro) <= LAYER_TOL
    shard.poll_error()
    shard.dispose()
    full.dispose()


def test_expert_parallel_through_c_abi_matches_single_gpu(cuda, oracle):
    _need_two_gpus()
    _spawn(_ep_case)
