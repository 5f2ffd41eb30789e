"""Expert parallelism over a torch.distributed process group (one process per GPU).

The reference runs every selected expert of a token on one worker, one after
another (DistributedPipelineCoordinator.ExecuteStep, DistributedPipelineCoordinator.cs:
143-207), and scales out only by moving whole activations between LAN nodes.
Here the experts of a layer are split into contiguous shards, one per rank
(expert e lives on rank e // (E // world)); the router is replicated and every
rank routes its own batch of tokens.  One step is

    route -> group (token, slot) pairs by destination rank and gather their rows
          -> all-to-all of the pair counts, rows and expert ids
          -> each rank runs its experts on the rows it received
          -> reverse all-to-all of the expert outputs
          -> k-ordered weighted combine (+ residual, + shared expert) at home.

Each pair's expert output is computed exactly as on one GPU and the combine
applies the same fp32 operations in the same order, so the expert-parallel
layer returns the single-GPU result bit for bit.

The compute steps come from a *shard* object (``CudaExpertShard`` here: the
sm_100a kernels behind the C ABI, device tensors); the exchange is plain
``torch.distributed`` (NCCL on GPUs), so the orchestration is independent of
where the compute runs.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .api import GpuExpertStageWorker, torch_stream_handle


class CudaExpertShard:
    """The compute steps of one rank, on a ``GpuExpertStageWorker`` that holds
    this rank's expert shard (``expert_begin``/``expert_count``) and the full
    router.  All tensors live on the worker's GPU; calls are asynchronous on
    the current torch stream."""

    def __init__(self, worker: GpuExpertStageWorker):
        self.worker = worker
        self.hidden_dim = worker.hidden_dim
        self.top_k = worker.top_k
        self.num_experts = worker.num_experts

    @staticmethod
    def _stream() -> int:
        return torch_stream_handle()

    def route(self, layer: int, x: torch.Tensor, flags: int):
        T, D = x.shape
        xin = torch.empty(T, D, dtype=torch.float32, device=x.device)
        ids = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        self.worker.route_dev(layer, x.data_ptr(), T, flags, xin.data_ptr(), ids.data_ptr(),
                              w.data_ptr(), self._stream())
        return xin, ids, w

    def dispatch(self, xin: torch.Tensor, ids: torch.Tensor, world: int):
        T, D = xin.shape
        P = T * self.top_k
        dev = xin.device
        counts = torch.empty(world, dtype=torch.int32, device=dev)
        offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
        perm = torch.empty(P, dtype=torch.int32, device=dev)
        inv = torch.empty(P, dtype=torch.int32, device=dev)
        rows = torch.empty(P, D, dtype=torch.float32, device=dev)
        row_ids = torch.empty(P, dtype=torch.int32, device=dev)
        self.worker.ep_dispatch_dev(xin.data_ptr(), ids.data_ptr(), T, world, counts.data_ptr(),
                                    offsets.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                    rows.data_ptr(), row_ids.data_ptr(), self._stream())
        return counts, inv, rows, row_ids

    def experts(self, layer: int, rows: torch.Tensor, row_ids: torch.Tensor, flags: int):
        R, D = rows.shape
        y = torch.empty(R, D, dtype=torch.float32, device=rows.device)
        if R:
            self.worker.experts_dev(layer, rows.data_ptr(), row_ids.data_ptr(), R, flags,
                                    y.data_ptr(), self._stream())
        return y

    def combine(self, layer: int, y_back: torch.Tensor, inv: torch.Tensor, w: torch.Tensor,
                resid: torch.Tensor | None, xin: torch.Tensor):
        T = w.shape[0]
        out = torch.empty(T, self.hidden_dim, dtype=torch.float32, device=w.device)
        self.worker.combine_dev(layer, y_back.data_ptr(), inv.data_ptr(), w.data_ptr(), T,
                                resid.data_ptr() if resid is not None else None, xin.data_ptr(),
                                out.data_ptr(), self._stream())
        return out


class ExpertParallelStageWorker:
    """An MoE layer whose experts are sharded over the ranks of ``group``.

    ``forward(layer, x, flags)`` takes this rank's tokens ``x`` [T, D] and
    returns ``(out [T, D], ids [T, k], weights [T, k])`` for them, with the
    flags of ``glc_moe_forward`` (RMSNorm ingress, residual; DECODE / BATCHED
    select the expert kernels).  Every rank must call ``forward`` the same
    number of times (the exchange is collective); T may differ per rank.
    """

    def __init__(self, shard, group=None):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if shard.num_experts % self.world:
            raise ValueError(f"{shard.num_experts} experts do not split over {self.world} ranks")

    def forward(self, layer: int, x: torch.Tensor, flags: int = 0):
        s, g = self.shard, self.group
        xin, ids, w = s.route(layer, x, flags)
        counts, inv, rows, row_ids = s.dispatch(xin, ids, self.world)
        # pair counts per destination rank -> per source rank
        send_counts = counts.to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=g)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        R = sum(rc)
        D = x.shape[1]
        recv_rows = torch.empty(R, D, dtype=rows.dtype, device=rows.device)
        recv_ids = torch.empty(R, dtype=row_ids.dtype, device=row_ids.device)
        dist.all_to_all_single(recv_rows, rows, output_split_sizes=rc, input_split_sizes=sc, group=g)
        dist.all_to_all_single(recv_ids, row_ids, output_split_sizes=rc, input_split_sizes=sc, group=g)
        y = s.experts(layer, recv_rows, recv_ids, flags)
        y_back = torch.empty(rows.shape[0], D, dtype=y.dtype, device=y.device)
        dist.all_to_all_single(y_back, y, output_split_sizes=sc, input_split_sizes=rc, group=g)
        resid = x if flags & _lib.GLC_FWD_RESIDUAL else None
        out = s.combine(layer, y_back, inv, w, resid, xin)
        return out, ids, w
