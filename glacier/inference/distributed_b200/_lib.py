"""ctypes binding of libglacier_b200.so (include/glacier_b200.h).

The library is built in-tree (``build.py``) and loaded from this directory.
There is no fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libglacier_b200.so")

GLC_OK = 0
STATUS_NAMES = {
    -1: "GLC_ERR_INVALID_ARG", -2: "GLC_ERR_CUDA", -3: "GLC_ERR_OOM", -4: "GLC_ERR_UNSUPPORTED",
    -5: "GLC_ERR_DISPOSED", -6: "GLC_ERR_NCCL", -7: "GLC_ERR_TIMEOUT", -8: "GLC_ERR_STATE",
}
GLC_GGUF_Q4_K = 12
GLC_WIRE_FP32, GLC_WIRE_FP16, GLC_WIRE_INT8, GLC_WIRE_FP8_E4M3 = 0, 1, 2, 3
GLC_FWD_RMSNORM, GLC_FWD_RESIDUAL, GLC_FWD_DECODE, GLC_FWD_BATCHED, GLC_FWD_UNFUSED = 1, 2, 4, 8, 16


class GlcError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class MoeDesc(C.Structure):
    _fields_ = [
        ("hidden_dim", C.c_int32), ("expert_ffn_dim", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("shared_ffn_dim", C.c_int32), ("renormalize", C.c_int32),
        ("weight_type", C.c_int32), ("device", C.c_int32), ("num_layers", C.c_int32),
        ("max_tokens", C.c_int32), ("expert_begin", C.c_int32), ("expert_count", C.c_int32),
    ]


class LayerWeights(C.Structure):
    _fields_ = [
        ("gate_exps", C.c_void_p), ("up_exps", C.c_void_p), ("down_exps", C.c_void_p),
        ("router", C.c_void_p), ("shared_gate", C.c_void_p), ("shared_up", C.c_void_p),
        ("shared_down", C.c_void_p), ("shared_gate_vec", C.c_void_p),
    ]


class StageDesc(C.Structure):
    _fields_ = [
        ("hidden_dim", C.c_int32), ("ffn_dim", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32), ("layer_begin", C.c_int32), ("layer_count", C.c_int32), ("max_len", C.c_int32),
        ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("vocab", C.c_int32), ("has_embedding", C.c_int32),
        ("has_lm_head", C.c_int32), ("device", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
        ("expert_ffn_dim", C.c_int32), ("moe_renormalize", C.c_int32),
    ]


class DenseLayerWeights(C.Structure):
    _fields_ = [
        ("attn_norm", C.c_void_p), ("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p),
        ("bq", C.c_void_p), ("bk", C.c_void_p), ("bv", C.c_void_p), ("wo", C.c_void_p),
        ("ffn_norm", C.c_void_p), ("w_gate", C.c_void_p), ("w_up", C.c_void_p), ("w_down", C.c_void_p),
    ]


class GemvJob(C.Structure):
    _fields_ = [
        ("W", C.c_void_p), ("W_up", C.c_void_p), ("x", C.c_void_p), ("y", C.c_void_p), ("norm_w", C.c_void_p),
        ("norm_eps", C.c_float), ("K", C.c_int32), ("N", C.c_int32), ("op", C.c_int32),
        ("after_previous", C.c_int32),
    ]


GLC_GEMV_SET, GLC_GEMV_ADD, GLC_GEMV_GATE_UP = 0, 1, 2


class FusedHeader(C.Structure):
    _fields_ = [
        ("sequence_id", C.c_uint64), ("token_index", C.c_int32), ("layer_index", C.c_int32),
        ("hidden_dim", C.c_int32), ("precision_mode", C.c_uint8), ("flags", C.c_uint8),
        ("batch_tokens", C.c_uint16), ("scale", C.c_float),
    ]


vp = C.c_void_p
i32 = C.c_int32
_SIGNATURES = {
    "glc_abi_version": (C.c_int, []),
    "glc_last_error": (C.c_char_p, []),
    "glc_device_count": (C.c_int, [C.POINTER(C.c_int32)]),
    "glc_q4k_row_bytes": (C.c_int64, [i32]),
    "glc_moe_create": (C.c_int, [C.POINTER(MoeDesc), C.POINTER(vp)]),
    "glc_moe_destroy": (C.c_int, [vp]),
    "glc_moe_load_layer": (C.c_int, [vp, i32, C.POINTER(LayerWeights)]),
    "glc_moe_synth_layer": (C.c_int, [vp, i32, C.c_uint64]),
    "glc_moe_layer_device_ptrs": (C.c_int, [vp, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                                            C.POINTER(vp)]),
    "glc_moe_set_profiling": (C.c_int, [vp, i32]),
    "glc_moe_kernel_times": (C.c_int, [vp, C.POINTER(C.c_float), i32, C.POINTER(C.c_int32)]),
    "glc_moe_poll_error": (C.c_int, [vp]),
    "glc_moe_debug_stall": (C.c_int, [vp, i32, C.c_int64]),
    "glc_expert_forward": (C.c_int, [vp, i32, i32, vp, vp]),
    "glc_expert_forward_dev": (C.c_int, [vp, i32, i32, vp, vp, vp]),
    "glc_routed_topk": (C.c_int, [vp, i32, vp, vp, vp, i32, vp]),
    "glc_moe_forward": (C.c_int, [vp, i32, vp, i32, C.c_uint32, vp, vp, vp]),
    "glc_moe_forward_dev": (C.c_int, [vp, i32, vp, i32, C.c_uint32, vp, vp, vp, vp]),
    "glc_moe_graph_build": (C.c_int, [vp, i32, vp, i32, C.c_uint32, vp]),
    "glc_moe_graph_launch": (C.c_int, [vp, vp]),
    "glc_gemv_q4k_dev": (C.c_int, [vp, vp, vp, i32, i32, vp]),
    "glc_gemv_q4k_chain_dev": (C.c_int, [C.POINTER(GemvJob), i32, vp]),
    "glc_gemv_poll_error": (C.c_int, []),
    "glc_attn_workspace_bytes": (C.c_int, [i32, i32, i32, C.POINTER(C.c_uint64)]),
    "glc_attn_decode_dev": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, C.c_float, vp, vp,
                                      C.c_uint64, vp]),
    "glc_router_topk_dev": (C.c_int, [vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
    "glc_dispatch_plan_dev": (C.c_int, [vp, i32, i32, vp, vp, vp, vp, vp]),
    "glc_dispatch_plan_noalloc_dev": (C.c_int, [vp, i32, i32, vp, vp, vp, vp, vp]),
    "glc_moe_route_dev": (C.c_int, [vp, i32, vp, i32, C.c_uint32, vp, vp, vp, vp]),
    "glc_moe_ep_dispatch_dev": (C.c_int, [vp, vp, vp, i32, i32, vp, vp, vp, vp, vp, vp, vp]),
    "glc_moe_experts_dev": (C.c_int, [vp, i32, vp, vp, i32, C.c_uint32, vp, vp]),
    "glc_moe_combine_dev": (C.c_int, [vp, i32, vp, vp, vp, i32, vp, vp, vp, vp]),
    "glc_wire_token_bytes": (i32, [i32, i32]),
    "glc_wire_quantize": (C.c_int, [i32, vp, i32, i32, vp, C.c_size_t]),
    "glc_wire_dequantize": (C.c_int, [i32, vp, C.c_size_t, i32, i32, vp]),
    "glc_wire_quantize_dev": (C.c_int, [i32, vp, i32, i32, vp, vp]),
    "glc_wire_dequantize_dev": (C.c_int, [i32, vp, i32, i32, vp, vp]),
    "glc_fused_header_write": (C.c_int, [C.POINTER(FusedHeader), vp]),
    "glc_fused_header_read": (C.c_int, [vp, C.POINTER(FusedHeader)]),
    "glc_fused_header_payload_bytes": (i32, [C.POINTER(FusedHeader)]),
    "glc_comm_unique_id": (C.c_int, [vp]),
    "glc_comm_create": (C.c_int, [vp, i32, i32, i32, C.POINTER(vp)]),
    "glc_comm_destroy": (C.c_int, [vp]),
    "glc_comm_peer_exchange": (C.c_int, [vp, C.c_int32]),
    "glc_moe_set_expert_slots": (C.c_int, [vp, C.c_int32]),
    "glc_moe_prefetch_experts": (C.c_int, [vp, C.c_int32, C.POINTER(C.c_int32), C.c_int32]),
    "glc_moe_expert_residency": (C.c_int, [vp, C.POINTER(C.c_int64)]),
    "glc_pp_send": (C.c_int, [vp, i32, C.POINTER(FusedHeader), vp, vp]),
    "glc_pp_recv": (C.c_int, [vp, i32, C.POINTER(FusedHeader), vp, i32, i32, vp]),
    "glc_moe_ep_forward": (C.c_int, [vp, vp, i32, vp, i32, C.c_uint32, vp, vp, vp, vp]),
    "glc_comm_send": (C.c_int, [vp, i32, vp, C.c_size_t, vp]),
    "glc_comm_recv": (C.c_int, [vp, i32, vp, C.c_size_t, vp]),
    "glc_stage_create": (C.c_int, [vp, C.POINTER(vp)]),
    "glc_stage_destroy": (C.c_int, [vp]),
    "glc_stage_load_layer": (C.c_int, [vp, i32, vp]),
    "glc_stage_load_io": (C.c_int, [vp, vp, vp, vp]),
    "glc_stage_load_moe_layer": (C.c_int, [vp, i32, vp, vp, vp, vp, vp]),
    "glc_stage_synth_layer": (C.c_int, [vp, i32, C.c_uint64]),
    "glc_stage_synth_io": (C.c_int, [vp, C.c_uint64]),
    "glc_stage_reset": (C.c_int, [vp]),
    "glc_stage_forward_dev": (C.c_int, [vp, i32, vp, vp, vp, vp, vp, vp]),
    "glc_stage_poll_error": (C.c_int, [vp]),
    "glc_stage_read_kv_cache": (C.c_int, [vp, i32, i32, vp, vp]),
}
GLC_COMM_ID_BYTES = 128

_lib = None


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def lib() -> C.CDLL:
    """Load the in-tree shared library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run python -m glacier.inference.distributed_b200.build")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != GLC_OK:
        raise GlcError(status, lib().glc_last_error().decode("utf-8", "replace"))
