"""Multi-rank host logic on CPU: world_size-2 process groups over gloo.

* Expert parallelism: ``ExpertParallelStageWorker`` (the product's
  orchestration: route, group pairs by destination rank, all-to-all of counts,
  rows and expert ids, experts, reverse all-to-all, k-ordered combine) drives a
  CPU stand-in for the per-rank compute built from the oracle.  Every rank's
  output, expert ids and weights must equal the oracle's single-process layer
  on that rank's tokens exactly: the exchange only moves rows.
* Pipeline boundary: ``StageBoundaryLink`` sends a FusedActivationHeader and
  the wire payload from rank 0 to rank 1 with an oracle codec; the receiver
  must get the header fields and the payload bytes the codec produced.

The GPU versions of both (NCCL, the CUDA kernels) are in test_gpu_multi.py.
"""
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(o, seed, D, F, E, k, renorm):
    L = {"D": D, "F": F, "E": E, "k": k, "renorm": renorm, "Fs": 0}
    L["gate"] = np.concatenate([o.synth_q4k(seed, o.expert_tag(e, 0), F, D) for e in range(E)])
    L["up"] = np.concatenate([o.synth_q4k(seed, o.expert_tag(e, 1), F, D) for e in range(E)])
    L["down"] = np.concatenate([o.synth_q4k(seed, o.expert_tag(e, 2), D, F) for e in range(E)])
    L["router"] = o.fill_normal(seed, 2, 0.02, D * E)
    return L


class OracleShard:
    """CPU stand-in for CudaExpertShard: the same five steps on the oracle,
    holding only this rank's experts (and the full router)."""

    def __init__(self, o, L, rank, world):
        self.o, self.L = o, L
        self.hidden_dim, self.top_k, self.num_experts = L["D"], L["k"], L["E"]
        self.epr = L["E"] // world
        self.begin = rank * self.epr
        D, F = L["D"], L["F"]
        self.gsl = F * (D // 256) * 144
        self.dsl = D * (F // 256) * 144

    def route(self, layer, x, flags):
        o, L = self.o, self.L
        xs = x.numpy()
        xin = np.stack([o.rmsnorm(r) for r in xs]) if flags & 1 else xs.copy()
        ids = np.empty((xs.shape[0], L["k"]), np.int32)
        w = np.empty((xs.shape[0], L["k"]), np.float32)
        for t in range(xs.shape[0]):
            _, ids[t], w[t] = o.router(xin[t], L["router"], L["E"], L["k"], L["renorm"])
        return torch.from_numpy(xin), torch.from_numpy(ids), torch.from_numpy(w)

    def dispatch(self, xin, ids, world):
        k = self.top_k
        flat = ids.numpy().reshape(-1)
        keys = np.minimum(flat // self.epr, world - 1)
        perm = np.argsort(keys, kind="stable").astype(np.int32)
        inv = np.empty_like(perm)
        inv[perm] = np.arange(perm.size, dtype=np.int32)
        counts = np.bincount(keys, minlength=world).astype(np.int32)
        rows = xin.numpy()[perm // k]
        return (torch.from_numpy(counts), torch.from_numpy(inv), torch.from_numpy(np.ascontiguousarray(rows)),
                torch.from_numpy(flat[perm].astype(np.int32)))

    def experts(self, layer, rows, row_ids, flags):
        o, L = self.o, self.L
        D, F = L["D"], L["F"]
        y = np.empty((rows.shape[0], D), np.float32)
        for r in range(rows.shape[0]):
            e = int(row_ids[r])
            assert self.begin <= e < self.begin + self.epr, "row routed to the wrong rank"
            y[r] = o.expert_forward(L["gate"][e * self.gsl:(e + 1) * self.gsl],
                                    L["up"][e * self.gsl:(e + 1) * self.gsl],
                                    L["down"][e * self.dsl:(e + 1) * self.dsl], D, F, rows[r].numpy())
        return torch.from_numpy(y)

    def combine(self, layer, y_back, inv, w, resid, xin):
        T, k = w.shape
        out = resid.numpy().copy() if resid is not None else np.zeros((T, self.hidden_dim), np.float32)
        yb, iv, wn = y_back.numpy(), inv.numpy(), w.numpy()
        for t in range(T):
            for j in range(k):
                out[t] = (yb[iv[t * k + j]] * wn[t, j]).astype(np.float32) + out[t]
        return torch.from_numpy(out)


def _run(rank, world, port, fn, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        sys.path.insert(0, REPO)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        fn(rank, world)
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        errq.put(f"rank {rank}: {traceback.format_exc()}")
        raise


def _spawn(fn, world=2):
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
    from oracle import oracle as o
    from glacier.inference.distributed_b200.ep import ExpertParallelStageWorker
    o.build()
    for (D, F, E, k, renorm, flags) in [(256, 512, 4, 2, True, 3), (512, 256, 8, 3, False, 1)]:
        L = _layer(o, 4242 + E, D, F, E, k, renorm)
        T = 3 + rank  # different token counts per rank
        x = o.fill_normal(100 + rank, 1, 1.0, T * D).reshape(T, D)
        ep = ExpertParallelStageWorker(OracleShard(o, L, rank, world))
        out, ids, w = ep.forward(0, torch.from_numpy(x), flags)
        ro, rids, rw = o.moe_forward(L, x, flags)
        assert np.array_equal(ids.numpy(), rids), (ids, rids)
        assert np.array_equal(w.numpy(), rw)
        assert np.array_equal(out.numpy(), ro), float(np.abs(out.numpy() - ro).max())


def test_expert_parallel_two_ranks_matches_single_process():
    _spawn(_ep_case)


class OracleCodec:
    def __init__(self, o):
        self.o = o

    def quantize(self, mode, x):
        return torch.from_numpy(np.asarray(self.o.wire_quantize(mode, x.numpy())))

    def dequantize(self, mode, payload, T, D):
        return torch.from_numpy(self.o.wire_dequantize(mode, payload.numpy(), T, D))


def _pp_case(rank, world):
    from oracle import oracle as o
    from glacier.inference.distributed_b200.pp import StageBoundaryLink
    o.build()
    link = StageBoundaryLink(OracleCodec(o))
    for mode, (T, D) in [(2, (3, 5120)), (3, (2, 256)), (1, (1, 64)), (0, (2, 32))]:
        x = o.fill_normal(7 + mode, 1, 1.0, T * D).reshape(T, D)
        if rank == 0:
            link.send(torch.from_numpy(x), 1, mode, sequence_id=11 + mode, token_index=5, layer_index=27)
        else:
            hdr, back = link.recv(0, "cpu")
            assert (hdr.sequence_id, hdr.token_index, hdr.layer_index) == (11 + mode, 5, 27)
            assert (hdr.hidden_dim, hdr.precision_mode, hdr.batch_tokens) == (D, mode, T)
            want = o.wire_dequantize(mode, np.asarray(o.wire_quantize(mode, x)), T, D)
            assert np.array_equal(back.numpy(), want)


def test_stage_boundary_link_two_ranks():
    _spawn(_pp_case)


def _pp_switcher_case(rank, world):
    from oracle import oracle as o
    from glacier.inference.distributed_b200 import DynamicPrecisionSwitcher, WirePrecisionMode
    from glacier.inference.distributed_b200.pp import StageBoundaryLink
    o.build()
    sw = DynamicPrecisionSwitcher()
    link = StageBoundaryLink(OracleCodec(o), switcher=sw)
    # (tokens, decode?, round-trip ms) -> the mode the switcher picks and the header carries
    cases = [(1, True, 0.4, WirePrecisionMode.FP16), (64, False, 0.4, WirePrecisionMode.INT8_Symmetric),
             (8, False, 0.4, WirePrecisionMode.FP16), (1, True, 9.0, WirePrecisionMode.INT8_Symmetric)]
    for i, (T, decode, rtt, want_mode) in enumerate(cases):
        x = o.fill_normal(90 + i, 1, 1.0, T * 256).reshape(T, 256)
        if rank == 0:
            sw.update_measured_latency(rtt) if i < 3 else [sw.update_measured_latency(rtt) for _ in range(30)]
            link.send(torch.from_numpy(x), 1, None, sequence_position=100, is_decode=decode)
        else:
            hdr, back = link.recv(0, "cpu")
            assert hdr.precision_mode == want_mode and hdr.batch_tokens == T
            want = o.wire_dequantize(want_mode, np.asarray(o.wire_quantize(want_mode, x)), T, 256)
            assert np.array_equal(back.numpy(), want)


def test_stage_boundary_link_picks_modes_with_the_switcher():
    _spawn(_pp_switcher_case)
