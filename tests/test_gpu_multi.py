"""Two GPUs, NCCL: expert parallelism and the pipeline-stage boundary on the
CUDA kernels (skipped when fewer than two GPUs are visible).

* EP: experts 0..3 on rank 0, 4..7 on rank 1 (Mixtral-like routing, top-2);
  every rank's layer output, ids and weights must equal a full single-GPU
  layer on the same tokens bit for bit (each pair's expert output is computed
  the same way; the combine applies the same fp32 operations in the same
  order), for the per-row GEMV experts and for the grouped tensor-core
  experts; and match the CPU oracle within the layer tolerance.
* PP: rank 0 quantises on its GPU and sends header + payload; rank 1 receives
  and dequantises on its GPU; the result equals the oracle codec bit for bit.
"""
import os
import socket
import sys
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECODE, BATCHED, UNFUSED = 4, 8, 16


def _need_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, fn, errq):
    import faulthandler
    import torch
    import torch.distributed as dist
    # a rank that is still running after 180 s prints every thread's stack and
    # exits, so a stuck collective or wait shows where it is instead of hanging
    faulthandler.dump_traceback_later(180, exit=True)
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        sys.path.insert(0, REPO)
        sys.path.insert(0, os.path.join(REPO, "tests"))
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        fn(rank, world)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _spawn(fn, world=2):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, errq)) for r in range(world)]
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


def _ep_case(rank, world):
    import torch
    from oracle import oracle as o
    from glacier.inference import distributed_b200 as glc
    from glacier.inference.distributed_b200.ep import CudaExpertShard, ExpertParallelStageWorker
    from test_gpu_parity import LAYER_TOL, make_layer, rel_l2
    o.build()
    D, F, E, k, seed = 512, 1024, 8, 2, 777
    L = make_layer(o, seed, D, F, E, k)
    epr = E // world
    T = 3 + rank
    cap = world * 4  # rows a rank can receive: every token of every rank
    shard = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=cap, expert_begin=rank * epr, expert_count=epr,
                                     device=rank)
    shard.synth_layer(0, seed)
    full = glc.GpuExpertStageWorker(D, F, E, k, max_tokens=8, device=rank)
    full.synth_layer(0, seed)
    ep = ExpertParallelStageWorker(CudaExpertShard(shard))
    x = o.fill_normal(900 + rank, 1, 1.0, T * D).reshape(T, D)
    xd = torch.from_numpy(x).cuda()
    for mode in (DECODE, BATCHED):
        flags = 3 | mode
        out, ids, w = ep.forward(0, xd, flags)
        torch.cuda.synchronize()
        fo, fids, fw = full.forward(0, x, flags)
        assert np.array_equal(ids.cpu().numpy(), fids)
        assert np.array_equal(w.cpu().numpy(), fw)
        assert np.array_equal(out.cpu().numpy(), fo), (mode, float(np.abs(out.cpu().numpy() - fo).max()))
        ro, rids, _ = o.moe_forward(L, x, 3)
        assert np.array_equal(fids, rids)
        assert rel_l2(fo, ro) <= LAYER_TOL
    shard.poll_error()
    shard.dispose()
    full.dispose()


def test_expert_parallel_two_gpus_matches_single_gpu(cuda, oracle):
    _need_two_gpus()
    _spawn(_ep_case)


def _pp_case(rank, world):
    import torch
    from oracle import oracle as o
    from glacier.inference.distributed_b200.pp import StageBoundaryLink
    o.build()
    link = StageBoundaryLink()
    for mode, (T, D) in [(2, (3, 5120)), (3, (2, 4096)), (1, (1, 3584)), (0, (2, 64))]:
        x = o.fill_normal(31 + mode, 1, 1.0, T * D).reshape(T, D)
        if rank == 0:
            link.send(torch.from_numpy(x).cuda(), 1, mode, sequence_id=mode, token_index=2, layer_index=27)
            torch.cuda.synchronize()
        else:
            hdr, back = link.recv(0, "cuda")
            torch.cuda.synchronize()
            assert (hdr.hidden_dim, hdr.precision_mode, hdr.batch_tokens, hdr.layer_index) == (D, mode, T, 27)
            want = o.wire_dequantize(mode, np.asarray(o.wire_quantize(mode, x)), T, D)
            assert np.array_equal(back.cpu().numpy(), want)


def test_stage_boundary_two_gpus(cuda, oracle):
    _need_two_gpus()
    _spawn(_pp_case)
