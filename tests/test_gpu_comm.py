"""Two GPUs through the C ABI's own communicator (NCCL inside the library, no
torch.distributed): the entry points a host without torch (the reference's C#
process) uses for multi-GPU work.  Skipped with fewer than two GPUs.

* Stage boundary: rank 0 glc_pp_send's activations in every wire mode, rank 1
  glc_pp_recv's them; header fields and the dequantised values equal the
  oracle codec's bit for bit.
* Expert parallelism: glc_moe_ep_forward over 2 ranks (experts 0..3 and 4..7)
  equals a full single-GPU layer on the same tokens bit for bit (the rows a
  rank receives are a batch: the grouped tensor-core experts, whatever the
  decode/batched flag), with the exchanges over NVLink peer memory and
  through NCCL.
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
    # over peer memory (three calls: both parities of the window's areas), then through NCCL
    for peer, mode in ((True, DECODE), (True, BATCHED), (True, BATCHED), (False, DECODE), (False, BATCHED)):
        comm.set_peer_exchange(peer)
        flags = 3 | mode
        out = torch.empty(T, D, device="cuda")
        ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
        w = torch.empty(T, k, device="cuda")
        torch.cuda.synchronize()
        shard.ep_forward_dev(comm, 0, xd.data_ptr(), T, flags, out.data_ptr(), ids.data_ptr(), w.data_ptr())
        torch.cuda.synchronize()
        fo, fids, fw = full.forward(0, x, 3 | BATCHED)
        assert np.array_equal(ids.cpu().numpy(), fids)
        assert np.array_equal(w.cpu().numpy(), fw)
        assert np.array_equal(out.cpu().numpy(), fo), (peer, mode, float(np.abs(out.cpu().numpy() - fo).max()))
        ro, rids, _ = o.moe_forward(L, x, flags)
        assert np.array_equal(fids, rids)
        assert rel_l2(fo, ro) <= LAYER_TOL
    shard.poll_error()
    shard.dispose()
    full.dispose()


def test_expert_parallel_through_c_abi_matches_single_gpu(cuda, oracle):
    _need_two_gpus()
    _spawn(_ep_case)


def _ep_bad_t_case(rank, world, comm):
    """A rank whose batch exceeds the handle's per-rank capacity gets
    GLC_ERR_INVALID_ARG; it still takes part in the exchanges with no pairs,
    so the other rank completes with the right result."""
    import torch
    from oracle import oracle as o
    from glacier.inference import distributed_b200 as glc
    o.build()
    D, F, E, k, seed = 512, 1024, 8, 2, 778
    epr = E // world
    shard = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=world * 2, expert_begin=rank * epr,
                                     expert_count=epr, device=rank)
    shard.synth_layer(0, seed)
    T = 3 if rank == 1 else 2  # capacity is max_tokens / world = 2 tokens
    x = o.fill_normal(950 + rank, 1, 1.0, T * D).reshape(T, D)
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(T, D, device="cuda")
    torch.cuda.synchronize()
    if rank == 1:
        with pytest.raises(glc.GlcError) as e:
            shard.ep_forward_dev(comm, 0, xd.data_ptr(), T, 3 | BATCHED, out.data_ptr())
        assert e.value.status == -1
        torch.cuda.synchronize()
    else:
        shard.ep_forward_dev(comm, 0, xd.data_ptr(), T, 3 | BATCHED, out.data_ptr())
        torch.cuda.synchronize()
        full = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=8, device=rank)
        full.synth_layer(0, seed)
        fo, _, _ = full.forward(0, x, 3 | BATCHED)
        assert np.array_equal(out.cpu().numpy(), fo)
        full.dispose()
    shard.dispose()


def test_expert_parallel_rank_over_capacity_does_not_stall_peers(cuda):
    _need_two_gpus()
    _spawn(_ep_bad_t_case)


def test_expert_parallel_one_rank_equals_single_gpu_layer(cuda, glc, oracle):
    """The whole expert-parallel call on a one-rank communicator (one GPU):
    route, fixed-size dispatch blocks, the exchange to itself (through its own
    peer window, then through NCCL), the experts on the rows sized on the
    device, the exchange back and the combine give the single-GPU layer bit
    for bit, on repeated calls with changing batch sizes and either flag; the
    phase marks are the six of the call."""
    import torch
    from test_gpu_parity import LAYER_TOL, make_layer, rel_l2
    D, F, E, k, seed = 512, 1024, 8, 2, 779
    L = make_layer(oracle, seed, D, F, E, k)
    comm = glc.Communicator(glc.Communicator.unique_id(), 1, 0, 0)
    shard = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=6, expert_begin=0, expert_count=E)
    shard.synth_layer(0, seed)
    full = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=6)
    full.synth_layer(0, seed)
    # over the (self-mapped) peer window, then through NCCL
    for peer, T, mode in [(p, T, m) for p in (True, False)
                          for T, m in ((6, BATCHED), (1, BATCHED), (4, DECODE), (0, BATCHED), (5, BATCHED))]:
        comm.set_peer_exchange(peer)
        x = oracle.fill_normal(990 + T, 1, 1.0, max(T, 1) * D).reshape(max(T, 1), D)[:T]
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda() if T else torch.empty(1, D, device="cuda")
        out = torch.empty(max(T, 1), D, device="cuda")
        ids = torch.empty(max(T, 1), k, dtype=torch.int32, device="cuda")
        w = torch.empty(max(T, 1), k, device="cuda")
        torch.cuda.synchronize()
        shard.ep_forward_dev(comm, 0, xd.data_ptr(), T, 3 | mode, out.data_ptr(), ids.data_ptr(), w.data_ptr())
        torch.cuda.synchronize()
        if T == 0:
            continue
        fo, fids, fw = full.forward(0, x, 3 | BATCHED)  # the received rows always run as a batch
        assert np.array_equal(ids.cpu().numpy()[:T], fids)
        assert np.array_equal(w.cpu().numpy()[:T], fw)
        assert np.array_equal(out.cpu().numpy()[:T], fo), T
        ro, rids, _ = oracle.moe_forward(L, x, 3)
        assert np.array_equal(fids, rids) and rel_l2(fo, ro) <= LAYER_TOL
    shard.set_profiling(True)
    x = oracle.fill_normal(991, 1, 1.0, 3 * D).reshape(3, D)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(3, D, device="cuda")
    shard.ep_forward_dev(comm, 0, xd.data_ptr(), 3, 3 | BATCHED, out.data_ptr())
    torch.cuda.synchronize()
    phases = shard.kernel_times_ms()
    shard.set_profiling(False)
    assert len(phases) == 6 and all(p >= 0 for p in phases), phases
    shard.poll_error()
    shard.dispose()
    full.dispose()
    comm.dispose()
