"""Host-side mirror of the reference's operator API for the MoE FFN hot path.

Names follow the reference so that callers (and tests) read like the
reference's own code:

* ``GpuExpertStageWorker.process_activation``  -> IInferenceStageWorker.ProcessActivation
  (IInferenceStageWorker.cs:43; CpuWarmExpertPoolWorker.cs:203-278)
* ``GpuExpertStageWorker.process_routed_topk`` -> GpuFirstExpertStageWorker.ProcessRoutedTopK
  (GpuFirstExpertStageWorker.cs:416-583)
* ``GpuExpertStageWorker.forward``             -> router + DistributedPipelineCoordinator.ExecuteStep
  (DistributedPipelineCoordinator.cs:72-137) for T tokens
* ``QuantizationKernels``                       -> Protocol/QuantizationKernels.cs:57-163
* ``FusedActivationHeader``                     -> Protocol/FusedActivationHeader.cs:41-218

Every call goes through the C ABI of libglacier_b200.so; nothing here computes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import GlcError, check, lib

WirePrecisionMode = type("WirePrecisionMode", (), {
    "FP32": 0, "FP16": 1, "INT8_Symmetric": 2, "FP8_E4M3": 3})


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


def torch_stream_handle(stream=None) -> int:
    """cudaStream_t of a torch stream (default: the current one) for the C ABI.

    torch's default stream has the handle 0, which the handle-based *_dev entry
    points read as "the handle's own stream" (a non-blocking stream that does
    not order with the default stream); it is passed as cudaStreamLegacy
    instead, so work stays ordered with torch's own operations."""
    import torch
    s = (stream if stream is not None else torch.cuda.current_stream()).cuda_stream
    return s if s != 0 else CUDA_STREAM_LEGACY


def q4k_row_bytes(k: int) -> int:
    return int(lib().glc_q4k_row_bytes(int(k)))


def device_count() -> int:
    n = C.c_int32(0)
    st = lib().glc_device_count(C.byref(n))
    return int(n.value) if st == 0 else 0


class GpuExpertStageWorker:
    """One MoE layer family resident in HBM on one device (GGUF Q4_K experts)."""

    def __init__(self, hidden_dim: int, expert_ffn_dim: int, num_experts: int, top_k: int, *,
                 shared_ffn_dim: int = 0, renormalize: bool = True, device: int = 0,
                 num_layers: int = 1, max_tokens: int = 1, expert_begin: int = 0,
                 expert_count: int = 0, expert_slots: int = 0):
        """expert_slots > 0: expert residency (glc_moe_set_expert_slots) -- the
        routed experts stay in pinned host memory and that many of them at a
        time in HBM, paged in as the routing selects them."""
        self.desc = _lib.MoeDesc(hidden_dim, expert_ffn_dim, num_experts, top_k, shared_ffn_dim,
                                 int(renormalize), _lib.GLC_GGUF_Q4_K, device, num_layers,
                                 max_tokens, expert_begin, expert_count)
        h = C.c_void_p()
        check(lib().glc_moe_create(C.byref(self.desc), C.byref(h)))
        self._h = h
        if expert_slots:
            try:
                check(lib().glc_moe_set_expert_slots(h, expert_slots))
            except GlcError:
                self.dispose()
                raise
        self.hidden_dim, self.expert_ffn_dim = hidden_dim, expert_ffn_dim
        self.num_experts, self.top_k = num_experts, top_k
        self.max_tokens = max_tokens

    # -- lifecycle --------------------------------------------------------
    def dispose(self) -> None:
        if self._h:
            check(lib().glc_moe_destroy(self._h))
            self._h = None

    close = dispose

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def _handle(self):
        if not self._h:
            raise GlcError(-5, "handle was disposed")
        return self._h

    # -- expert residency --------------------------------------------------
    def prefetch_experts(self, layer: int, expert_ids) -> None:
        """Stage these experts of ``layer`` into HBM slots (router lookahead)."""
        ids = np.ascontiguousarray(np.asarray(expert_ids, dtype=np.int32))
        check(lib().glc_moe_prefetch_experts(self._handle(), layer,
                                             ids.ctypes.data_as(C.POINTER(C.c_int32)), len(ids)))

    def expert_residency(self) -> dict:
        """Slot capacity and the VRAM-hit / transfer / prefetch counters."""
        out = (C.c_int64 * 4)()
        check(lib().glc_moe_expert_residency(self._handle(), out))
        return {"slots": out[0], "hits": out[1], "transfers": out[2], "prefetches": out[3]}

    # -- weights ----------------------------------------------------------
    def load_layer(self, layer: int, gate_exps: np.ndarray, up_exps: np.ndarray,
                   down_exps: np.ndarray, router: np.ndarray | None = None,
                   shared_gate=None, shared_up=None, shared_down=None, shared_gate_vec=None):
        keep = [np.ascontiguousarray(a) if a is not None else None for a in
                (gate_exps, up_exps, down_exps, router, shared_gate, shared_up, shared_down,
                 shared_gate_vec)]
        w = _lib.LayerWeights(*[_ptr(a) for a in keep])
        check(lib().glc_moe_load_layer(self._handle(), layer, C.byref(w)))

    def synth_layer(self, layer: int, seed: int) -> None:
        check(lib().glc_moe_synth_layer(self._handle(), layer, C.c_uint64(seed)))

    def layer_device_ptrs(self, layer: int = 0):
        g, u, d, r = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
        check(lib().glc_moe_layer_device_ptrs(self._handle(), layer, C.byref(g), C.byref(u),
                                              C.byref(d), C.byref(r)))
        return g.value, u.value, d.value, r.value

    # -- telemetry --------------------------------------------------------
    def set_profiling(self, enable: bool) -> None:
        check(lib().glc_moe_set_profiling(self._handle(), int(enable)))

    def kernel_times_ms(self) -> list[float]:
        buf = (C.c_float * 16)()
        n = C.c_int32(0)
        check(lib().glc_moe_kernel_times(self._handle(), buf, 16, C.byref(n)))
        return [float(buf[i]) for i in range(min(n.value, 16))]

    def poll_error(self) -> None:
        check(lib().glc_moe_poll_error(self._handle()))

    def debug_stall(self, cta: int, wait_limit_ns: int) -> None:
        """Failure-detection test hook: the next fused decode launch leaves CTA
        ``cta`` out of its grid barrier with every wait limited to
        ``wait_limit_ns``; that launch reports GLC_ERR_TIMEOUT."""
        check(lib().glc_moe_debug_stall(self._handle(), cta, wait_limit_ns))

    # -- operator API -----------------------------------------------------
    def process_activation(self, layer: int, expert_id: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        if x.size < self.hidden_dim:
            raise GlcError(-1, f"Input activation size ({x.nbytes} bytes) is smaller than required "
                               f"hidden dimension ({4 * self.hidden_dim} bytes for D={self.hidden_dim}).")
        y = np.empty(self.hidden_dim, np.float32)
        check(lib().glc_expert_forward(self._handle(), layer, expert_id, _ptr(x), _ptr(y)))
        return y

    def process_routed_topk(self, layer: int, x: np.ndarray, ids, weights) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        weights = np.ascontiguousarray(weights, np.float32)
        k = min(ids.size, weights.size)
        out = np.empty(self.hidden_dim, np.float32)
        check(lib().glc_routed_topk(self._handle(), layer, _ptr(x), _ptr(ids), _ptr(weights), k,
                                    _ptr(out)))
        return out

    def forward(self, layer: int, x: np.ndarray, flags: int = 0):
        """The MoE layer on host buffers (glc_moe_forward): returns (out [T][D],
        expert ids [T][k], combine weights [T][k])."""
        x = np.ascontiguousarray(x, np.float32)
        if x.ndim == 1:
            x = x[None, :]
        T = x.shape[0]
        out = np.empty_like(x)
        ids = np.empty((T, self.top_k), np.int32)
        w = np.empty((T, self.top_k), np.float32)
        check(lib().glc_moe_forward(self._handle(), layer, _ptr(x), T, flags, _ptr(out), _ptr(ids),
                                    _ptr(w)))
        return out, ids, w

    def forward_dev(self, layer: int, x_ptr: int, T: int, flags: int, out_ptr: int,
                    ids_ptr: int | None = None, w_ptr: int | None = None, stream: int | None = None):
        check(lib().glc_moe_forward_dev(self._handle(), layer, x_ptr, T, flags, out_ptr, ids_ptr,
                                        w_ptr, stream))

    def ep_forward_dev(self, comm: "Communicator", layer: int, x_ptr: int, T: int, flags: int, out_ptr: int,
                       ids_ptr: int | None = None, w_ptr: int | None = None, stream: int | None = None) -> None:
        """The expert-parallel layer over ``comm`` (glc_moe_ep_forward): this worker
        holds expert shard comm.rank of comm.nranks; device pointers."""
        check(lib().glc_moe_ep_forward(self._handle(), comm._handle(), layer, x_ptr, T, flags, out_ptr,
                                       ids_ptr, w_ptr, stream))

    def graph_build(self, layer: int, x_ptr: int, T: int, flags: int, out_ptr: int) -> None:
        check(lib().glc_moe_graph_build(self._handle(), layer, x_ptr, T, flags, out_ptr))

    def graph_launch(self, stream: int | None = None) -> None:
        check(lib().glc_moe_graph_launch(self._handle(), stream))

    def process_activation_dev(self, layer: int, expert_id: int, x_ptr: int, y_ptr: int,
                               stream: int | None = None):
        check(lib().glc_expert_forward_dev(self._handle(), layer, expert_id, x_ptr, y_ptr, stream))

    # -- expert-parallel steps (device pointers, asynchronous on `stream`) --
    def route_dev(self, layer: int, x_ptr: int, T: int, flags: int, xin_ptr: int, ids_ptr: int,
                  w_ptr: int, stream: int | None = None) -> None:
        check(lib().glc_moe_route_dev(self._handle(), layer, x_ptr, T, flags, xin_ptr, ids_ptr,
                                      w_ptr, stream))

    def ep_dispatch_dev(self, xin_ptr: int, ids_ptr: int, T: int, world: int, counts_ptr: int,
                        offsets_ptr: int, perm_ptr: int, inv_ptr: int, rows_ptr: int,
                        row_ids_ptr: int, stream: int | None = None) -> None:
        check(lib().glc_moe_ep_dispatch_dev(self._handle(), xin_ptr, ids_ptr, T, world, counts_ptr,
                                            offsets_ptr, perm_ptr, inv_ptr, rows_ptr, row_ids_ptr,
                                            stream))

    def experts_dev(self, layer: int, rows_ptr: int, ids_ptr: int, R: int, flags: int, y_ptr: int,
                    stream: int | None = None) -> None:
        check(lib().glc_moe_experts_dev(self._handle(), layer, rows_ptr, ids_ptr, R, flags, y_ptr,
                                        stream))

    def combine_dev(self, layer: int, y_ptr: int, inv_ptr: int, w_ptr: int, T: int,
                    resid_ptr: int | None, xin_ptr: int | None, out_ptr: int,
                    stream: int | None = None) -> None:
        check(lib().glc_moe_combine_dev(self._handle(), layer, y_ptr, inv_ptr, w_ptr, T, resid_ptr,
                                        xin_ptr, out_ptr, stream))


def gemv_q4k_dev(W_ptr: int, x_ptr: int, y_ptr: int, K: int, N: int, stream: int | None = None):
    """QuantKernels.MatVecMul(Q4_K, W, x, y, nCols=K, nRows=N) on device pointers."""
    check(lib().glc_gemv_q4k_dev(W_ptr, x_ptr, y_ptr, K, N, stream))


def gemv_q4k_chain_dev(jobs, stream: int | None = None) -> None:
    """A chain of MatVecMul calls in one launch (glc_gemv_q4k_chain_dev).
    ``jobs``: dicts with W, x, y (device pointers), K, N and optionally op
    ("set" | "add" | "gate_up"), W_up, norm_w, norm_eps, after_previous."""
    ops = {"set": _lib.GLC_GEMV_SET, "add": _lib.GLC_GEMV_ADD, "gate_up": _lib.GLC_GEMV_GATE_UP}
    arr = (_lib.GemvJob * len(jobs))()
    for a, j in zip(arr, jobs):
        a.W, a.W_up, a.x, a.y = j["W"], j.get("W_up"), j["x"], j["y"]
        a.norm_w, a.norm_eps = j.get("norm_w"), float(j.get("norm_eps", 0.0))
        a.K, a.N, a.op = int(j["K"]), int(j["N"]), ops[j.get("op", "set")]
        a.after_previous = int(bool(j.get("after_previous", False)))
    check(lib().glc_gemv_q4k_chain_dev(arr, len(jobs), stream))


def gemv_poll_error() -> None:
    """Raises GlcError when a bounded device-side wait of a GEMV gave up."""
    check(lib().glc_gemv_poll_error())


def attn_workspace_bytes(n_heads: int, n_kv_heads: int, max_len: int) -> int:
    n = C.c_uint64(0)
    check(lib().glc_attn_workspace_bytes(n_heads, n_kv_heads, max_len, C.byref(n)))
    return int(n.value)


def attn_decode_dev(q_ptr: int, k_new_ptr: int, v_new_ptr: int, k_cache_ptr: int, v_cache_ptr: int,
                    n_heads: int, n_kv_heads: int, max_len: int, pos: int, rope_theta: float, out_ptr: int,
                    work_ptr: int, work_bytes: int, head_dim: int = 128, stream: int | None = None) -> None:
    """Decode attention of one token at position ``pos`` (glc_attn_decode_dev):
    RoPE on q and the new key, the new key and value stored as fp16 in row
    ``pos`` of the caches, grouped-query attention over positions 0..pos."""
    check(lib().glc_attn_decode_dev(q_ptr, k_new_ptr, v_new_ptr, k_cache_ptr, v_cache_ptr, n_heads, n_kv_heads,
                                    head_dim, max_len, pos, rope_theta, out_ptr, work_ptr, work_bytes, stream))


def dispatch_plan_dev(ids_ptr, P, E, counts_ptr, offsets_ptr, perm_ptr, inv_ptr, stream=None):
    check(lib().glc_dispatch_plan_dev(ids_ptr, P, E, counts_ptr, offsets_ptr, perm_ptr, inv_ptr, stream))


def router_topk_dev(x_ptr, router_ptr, T, D, E, k, renormalize, rmsnorm, xin_ptr, logits_ptr,
                    ids_ptr, w_ptr, stream=None):
    check(lib().glc_router_topk_dev(x_ptr, router_ptr, T, D, E, k, int(renormalize), int(rmsnorm),
                                    xin_ptr, logits_ptr, ids_ptr, w_ptr, stream))


class QuantizationKernels:
    """GPU implementation of the wire codec, same names and byte layout as the reference."""

    @staticmethod
    def GetPackedTokenBytes(mode: int, dim: int) -> int:
        return int(lib().glc_wire_token_bytes(mode, dim))

    @staticmethod
    def GetPackedBatchBytes(mode: int, dim: int, token_count: int) -> int:
        return QuantizationKernels.GetPackedTokenBytes(mode, dim) * token_count

    @staticmethod
    def QuantizeBatch(x: np.ndarray, destination: np.ndarray, dim: int, token_count: int,
                      mode: int) -> None:
        x = np.ascontiguousarray(x, np.float32)
        if x.size < dim * token_count:
            raise GlcError(-1, "Input float span smaller than dim * tokenCount")
        check(lib().glc_wire_quantize(mode, _ptr(x), token_count, dim, _ptr(destination),
                                      destination.nbytes))

    @staticmethod
    def DequantizeBatch(source: np.ndarray, destination: np.ndarray, dim: int, token_count: int,
                        mode: int) -> None:
        if destination.size < dim * token_count:
            raise GlcError(-1, "Destination float span smaller than dim * tokenCount")
        src = np.ascontiguousarray(source, np.uint8)
        check(lib().glc_wire_dequantize(mode, _ptr(src), src.nbytes, token_count, dim,
                                        _ptr(destination)))

    @staticmethod
    def QuantizeToken(x: np.ndarray, destination: np.ndarray, mode: int) -> float:
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        QuantizationKernels.QuantizeBatch(x, destination, x.size, 1, mode)
        if mode in (2, 3):
            return float(np.frombuffer(destination[:4].tobytes(), "<f4")[0])
        return 1.0

    @staticmethod
    def DequantizeToken(source: np.ndarray, destination: np.ndarray, mode: int) -> None:
        QuantizationKernels.DequantizeBatch(source, destination, destination.size, 1, mode)

    @staticmethod
    def quantize_dev(mode: int, x_ptr: int, T: int, D: int, out_ptr: int, stream=None) -> None:
        check(lib().glc_wire_quantize_dev(mode, x_ptr, T, D, out_ptr, stream))

    @staticmethod
    def dequantize_dev(mode: int, in_ptr: int, T: int, D: int, out_ptr: int, stream=None) -> None:
        check(lib().glc_wire_dequantize_dev(mode, in_ptr, T, D, out_ptr, stream))


@dataclass
class FusedActivationHeader:
    sequence_id: int
    token_index: int
    layer_index: int
    hidden_dim: int
    precision_mode: int
    flags: int = 0
    scale: float = 1.0
    batch_tokens: int = 0
    HeaderSize = 32
    FusedMagic = 0x47414354

    def _c(self) -> _lib.FusedHeader:
        return _lib.FusedHeader(self.sequence_id, self.token_index, self.layer_index,
                                self.hidden_dim, self.precision_mode, self.flags,
                                self.batch_tokens, self.scale)

    def write_to(self) -> bytes:
        buf = (C.c_uint8 * 32)()
        check(lib().glc_fused_header_write(C.byref(self._c()), buf))
        return bytes(buf)

    @staticmethod
    def read_from(data: bytes) -> "FusedActivationHeader":
        if len(data) < 32:
            raise GlcError(-1, "Source too small for FusedActivationHeader")
        buf = (C.c_uint8 * 32).from_buffer_copy(bytes(data[:32]))
        h = _lib.FusedHeader()
        check(lib().glc_fused_header_read(buf, C.byref(h)))
        return FusedActivationHeader(h.sequence_id, h.token_index, h.layer_index, h.hidden_dim,
                                     h.precision_mode, h.flags, h.scale, h.batch_tokens)

    def get_payload_byte_count(self) -> int:
        return int(lib().glc_fused_header_payload_bytes(C.byref(self._c())))


def _load_torch_nccl_first() -> None:
    """The library loads NCCL by soname ("libnccl.so.2") at its first
    communicator call, and a process holds one library per soname: if torch is
    installed, it is imported first so that its own NCCL is the one loaded
    (loading the system one first would leave torch without the newer NCCL
    symbols it needs)."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


class DynamicPrecisionSwitcher:
    """Wire precision of a stage-boundary send, chosen per message
    (DynamicPrecisionSwitcher, DynamicPrecisionSwitcher.cs:10-178): a forced
    mode wins; decode keeps FP16, except under link congestion (smoothed
    round-trip time above ``congestion_latency_threshold_ms``) where it backs
    off to INT8, unless the sequence is deeper than ``deep_context_threshold``
    (FP16 protects the attention logits there); prefill batches of at least
    ``prefill_batch_threshold`` tokens, or any batch under congestion, use
    INT8, smaller ones FP16.  The round-trip time is an exponential moving
    average (factor ``ema_alpha``) whose first sample sets it directly; before
    any sample it reads 0.5 ms.  Every change of the selected mode counts as
    a switch.  On NVLink the round trip is the host-measured time of a
    send/recv pair; the thresholds keep the reference's defaults."""

    def __init__(self, forced_precision: int | None = None):
        self.forced_precision = forced_precision
        self.prefill_batch_threshold = 32
        self.congestion_latency_threshold_ms = 2.5
        self.deep_context_threshold = 16384
        self.ema_alpha = 0.2
        self._ema_ms = -1.0
        self._last = forced_precision if forced_precision is not None else WirePrecisionMode.FP16
        self._switches = 0

    @property
    def current_ema_latency_ms(self) -> float:
        return self._ema_ms if self._ema_ms > 0.0 else 0.5

    @property
    def last_selected_precision(self) -> int:
        return self._last

    @property
    def total_switches(self) -> int:
        return self._switches

    def update_measured_latency(self, rtt_ms: float) -> None:
        if rtt_ms <= 0.0:
            return
        if self._ema_ms <= 0.0:
            self._ema_ms = rtt_ms
        else:
            self._ema_ms = (1.0 - self.ema_alpha) * self._ema_ms + self.ema_alpha * rtt_ms

    record_rtt = update_measured_latency

    def select_precision(self, batch_size: int, sequence_position: int = 0, is_decode: bool = False,
                         override_rtt_ms: float | None = None) -> int:
        if self.forced_precision is not None:
            self._last = self.forced_precision
            return self.forced_precision
        rtt = override_rtt_ms if override_rtt_ms is not None else self.current_ema_latency_ms
        congested = rtt > self.congestion_latency_threshold_ms
        if is_decode:
            if sequence_position > self.deep_context_threshold:
                mode = WirePrecisionMode.FP16
            else:
                mode = WirePrecisionMode.INT8_Symmetric if congested else WirePrecisionMode.FP16
        elif batch_size >= self.prefill_batch_threshold or congested:
            mode = WirePrecisionMode.INT8_Symmetric
        else:
            mode = WirePrecisionMode.FP16
        if mode != self._last:
            self._switches += 1
            self._last = mode
        return mode

    @staticmethod
    def select_optimal_wire_precision(batch_size: int, is_decode: bool, lan_latency_ms: float,
                                      forced_override: int | None = None) -> int:
        """The static form (DynamicPrecisionSwitcher.cs:153-164)."""
        if forced_override is not None:
            return forced_override
        if is_decode:
            return WirePrecisionMode.FP16
        if lan_latency_ms > 2.5:
            return WirePrecisionMode.INT8_Symmetric
        return WirePrecisionMode.INT8_Symmetric if batch_size >= 32 else WirePrecisionMode.FP16

    def reset(self) -> None:
        self._ema_ms = -1.0
        self._switches = 0
        self._last = self.forced_precision if self.forced_precision is not None else WirePrecisionMode.FP16


class Communicator:
    """The NCCL communicator of the C ABI (``glc_comm_*``), for hosts that have
    no ``torch.distributed``: one process per GPU; rank 0 makes the id with
    ``unique_id()``, the host hands the bytes to every rank, and each rank
    constructs ``Communicator(uid, nranks, rank, device)`` (collective)."""

    @staticmethod
    def unique_id() -> bytes:
        _load_torch_nccl_first()
        buf = (C.c_uint8 * _lib.GLC_COMM_ID_BYTES)()
        check(lib().glc_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        self._h = None
        if len(uid) != _lib.GLC_COMM_ID_BYTES:
            raise GlcError(-1, "communicator id must be 128 bytes")
        _load_torch_nccl_first()
        buf = (C.c_uint8 * _lib.GLC_COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        check(lib().glc_comm_create(buf, nranks, rank, device, C.byref(h)))
        self._h = h
        self.nranks, self.rank, self.device = nranks, rank, device

    def _handle(self) -> C.c_void_p:
        if self._h is None:
            raise GlcError(-5, "communicator was destroyed")
        return self._h

    def set_peer_exchange(self, enable: bool) -> None:
        """Expert-parallel exchanges over NVLink peer memory (default) or
        through NCCL (glc_comm_peer_exchange); every rank alike."""
        check(lib().glc_comm_peer_exchange(self._handle(), 1 if enable else 0))

    def peer_exchange_active(self) -> bool:
        """Whether the expert-parallel exchanges go over peer memory (the
        window mapped on every rank, the option on)."""
        r = lib().glc_comm_peer_exchange(self._handle(), -1)
        check(r if r < 0 else 0)
        return r == 1

    def pp_send(self, peer: int, header: "FusedActivationHeader", x_ptr: int, stream=None) -> None:
        """Stage boundary: quantise x [T][D] (from the header) on the GPU and send
        the header and the payload to ``peer``."""
        check(lib().glc_pp_send(self._handle(), peer, C.byref(header._c()), x_ptr, stream))

    def send(self, peer: int, ptr: int, nbytes: int, stream=None) -> None:
        """Raw bytes of device memory to ``peer`` (glc_comm_send), e.g. a token id."""
        check(lib().glc_comm_send(self._handle(), peer, ptr, nbytes, stream))

    def recv(self, peer: int, ptr: int, nbytes: int, stream=None) -> None:
        check(lib().glc_comm_recv(self._handle(), peer, ptr, nbytes, stream))

    def pp_recv(self, peer: int, x_ptr: int, max_tokens: int, hidden_dim: int,
                stream=None) -> "FusedActivationHeader":
        """Receive a header and its payload from ``peer`` and dequantise into x [T][hidden_dim]."""
        h = _lib.FusedHeader()
        check(lib().glc_pp_recv(self._handle(), peer, C.byref(h), x_ptr, max_tokens, hidden_dim, stream))
        return FusedActivationHeader(h.sequence_id, h.token_index, h.layer_index, h.hidden_dim,
                                     h.precision_mode, h.flags, h.scale, h.batch_tokens)

    def dispose(self) -> None:
        if self._h is not None:
            lib().glc_comm_destroy(self._h)
            self._h = None


class DenseStage:
    """A decoder pipeline stage on one GPU, the counterpart of the reference's
    IClusterStageModel (Pipeline/IClusterStageModel.cs:9-36): layers
    [layer_begin, layer_begin + layer_count) of a Qwen2-style (dense) or
    Mixtral-style (``num_experts`` > 0: routed SwiGLU experts) model with
    their fp16 KV caches, plus the embedding table on a first stage and the
    final norm and LM head on a last stage (glc_stage_*)."""

    def __init__(self, hidden_dim: int, ffn_dim: int, n_heads: int, n_kv_heads: int, layer_begin: int,
                 layer_count: int, max_len: int, rope_theta: float = 1e6, rms_eps: float = 1e-6,
                 vocab: int = 0, has_embedding: bool = False, has_lm_head: bool = False, device: int = 0,
                 num_experts: int = 0, top_k: int = 0, expert_ffn_dim: int = 0, moe_renormalize: bool = True):
        self._h = None
        self.desc = _lib.StageDesc(hidden_dim, ffn_dim, n_heads, n_kv_heads, 128, layer_begin, layer_count,
                                   max_len, rope_theta, rms_eps, vocab, int(has_embedding), int(has_lm_head),
                                   device, num_experts, top_k, expert_ffn_dim, int(moe_renormalize))
        h = C.c_void_p()
        check(lib().glc_stage_create(C.byref(self.desc), C.byref(h)))
        self._h = h
        self.hidden_dim, self.vocab = hidden_dim, vocab

    def _handle(self) -> C.c_void_p:
        if self._h is None:
            raise GlcError(-5, "stage was disposed")
        return self._h

    def load_layer(self, layer: int, attn_norm, wq, wk, wv, bq, bk, bv, wo, ffn_norm, w_gate, w_up, w_down) -> None:
        arrays = [attn_norm, wq, wk, wv, bq, bk, bv, wo, ffn_norm, w_gate, w_up, w_down]
        arrays = [None if a is None else np.ascontiguousarray(a) for a in arrays]
        w = _lib.DenseLayerWeights(*[None if a is None else a.ctypes.data for a in arrays])
        check(lib().glc_stage_load_layer(self._handle(), layer, C.byref(w)))

    def load_moe_layer(self, layer: int, attn_norm, wq, wk, wv, wo, ffn_norm, router, gate_exps, up_exps,
                       down_exps) -> None:
        """A mixture-of-experts layer: attention weights and norms, fp32 router
        [D][E], experts' Q4_K gate / up [E][F][D] and down [E][D][F]."""
        arrays = [np.ascontiguousarray(a) for a in (attn_norm, wq, wk, wv, wo, ffn_norm)]
        w = _lib.DenseLayerWeights(arrays[0].ctypes.data, arrays[1].ctypes.data, arrays[2].ctypes.data,
                                   arrays[3].ctypes.data, None, None, None, arrays[4].ctypes.data,
                                   arrays[5].ctypes.data, None, None, None)
        moe = [np.ascontiguousarray(a) for a in (np.asarray(router, np.float32), gate_exps, up_exps, down_exps)]
        check(lib().glc_stage_load_moe_layer(self._handle(), layer, C.byref(w), *[a.ctypes.data for a in moe]))

    def load_io(self, embedding=None, final_norm=None, lm_head=None) -> None:
        arrays = [None if a is None else np.ascontiguousarray(a) for a in (embedding, final_norm, lm_head)]
        check(lib().glc_stage_load_io(self._handle(), *[None if a is None else a.ctypes.data for a in arrays]))

    def synth_layer(self, layer: int, seed: int) -> None:
        check(lib().glc_stage_synth_layer(self._handle(), layer, seed))

    def synth_io(self, seed: int) -> None:
        check(lib().glc_stage_synth_io(self._handle(), seed))

    def reset_kv_cache(self) -> None:
        """ResetKvCache (IClusterStageModel.cs:35)."""
        check(lib().glc_stage_reset(self._handle()))

    def forward_dev(self, pos: int, token_ptr=None, x_in_ptr=None, x_out_ptr=None, logits_ptr=None,
                    token_out_ptr=None, stream=None) -> None:
        """ForwardStage (IClusterStageModel.cs:19) on device pointers."""
        check(lib().glc_stage_forward_dev(self._handle(), pos, token_ptr, x_in_ptr, x_out_ptr, logits_ptr,
                                          token_out_ptr, stream))

    def poll_error(self) -> None:
        check(lib().glc_stage_poll_error(self._handle()))

    def read_kv_cache(self, layer: int, rows: int):
        """Rows [0, rows) of a layer's fp16 K and V caches, each [n_kv_heads][rows][128]."""
        hkv = self.desc.n_kv_heads
        k = np.empty((hkv, rows, 128), np.float16)
        v = np.empty((hkv, rows, 128), np.float16)
        check(lib().glc_stage_read_kv_cache(self._handle(), layer, rows, k.ctypes.data, v.ctypes.data))
        return k, v

    def dispose(self) -> None:
        if self._h is not None:
            lib().glc_stage_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass
