"""ctypes view of the CPU oracle (oracle/glc_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
(to verify one small GPU run) and by bench.py's CPU-baseline leg.  The
product package never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libglc_oracle.so")
SRC = os.path.join(HERE, "glc_oracle.c")

CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
          "-std=c11", "-Wall", "-Wno-unused-function"]


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (the recipe is this function)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
            os.path.getmtime(SRC), os.path.getmtime(os.path.join(HERE, "glc_oracle.h"))):
        tmp = LIB_PATH + ".tmp"
        subprocess.check_call(["gcc", *CFLAGS, "-o", tmp, SRC, "-lm", "-lpthread"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None

P = np.ctypeslib.ndpointer
f32p = P(dtype=np.float32, flags="C_CONTIGUOUS")
u8p = P(dtype=np.uint8, flags="C_CONTIGUOUS")
i32p = P(dtype=np.int32, flags="C_CONTIGUOUS")


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        sig = {
            "oc_mix64": (C.c_uint64, [C.c_uint64]),
            "oc_stream_seed": (C.c_uint64, [C.c_uint64, C.c_uint64]),
            "oc_draw": (C.c_uint64, [C.c_uint64, C.c_uint64]),
            "oc_uniform": (C.c_float, [C.c_uint64, C.c_uint64]),
            "oc_normal": (C.c_float, [C.c_uint64, C.c_uint64]),
            "oc_fill_normal": (None, [C.c_uint64, C.c_uint64, C.c_float, f32p, C.c_size_t]),
            "oc_synth_q4k": (None, [C.c_uint64, C.c_uint64, C.c_float, u8p, C.c_size_t]),
            "oc_expert_tag": (C.c_uint64, [C.c_int, C.c_int]),
            "oc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "oc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "oc_q4k_dequant": (None, [u8p, C.c_size_t, f32p]),
            "oc_q4k_gemv": (None, [u8p, f32p, f32p, C.c_int, C.c_int]),
            "oc_set_threads": (None, [C.c_int]),
            "oc_swiglu": (None, [f32p, f32p, f32p, C.c_int]),
            "oc_expert_forward": (None, [u8p, u8p, u8p, C.c_int, C.c_int, f32p, f32p]),
            "oc_rmsnorm": (None, [f32p, f32p, C.c_int]),
            "oc_dot_canonical": (C.c_float, [f32p, f32p, C.c_int, C.c_int]),
            "oc_router_logits": (None, [f32p, f32p, C.c_int, C.c_int, f32p]),
            "oc_router_topk": (None, [f32p, C.c_int, C.c_int, C.c_int, i32p, f32p]),
            "oc_dispatch_plan": (None, [i32p, C.c_int, C.c_int, i32p, i32p, i32p, i32p]),
            "oc_routed_topk": (None, [u8p, u8p, u8p, C.c_int, C.c_int, C.c_int, f32p, i32p, f32p,
                                      C.c_int, f32p]),
            "oc_moe_forward": (None, [u8p, u8p, u8p, f32p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int, f32p, C.c_int, f32p, i32p, f32p]),
            "oc_cpu_expert_forward_fast": (None, [u8p, u8p, u8p, C.c_int, C.c_int, f32p, f32p,
                                                  C.c_int]),
            "oc_cpu_moe_token_fast": (None, [u8p, u8p, u8p, f32p, C.c_int, C.c_int, C.c_int,
                                             C.c_int, C.c_int, C.c_int, f32p, f32p, C.c_int]),
            "oc_cpu_moe_token_shared_fast": (None, [u8p, u8p, u8p, f32p, u8p, u8p, u8p, f32p, C.c_int,
                                                    C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                    f32p, f32p, C.c_int]),
            "oc_wire_token_bytes": (C.c_int, [C.c_int, C.c_int]),
            "oc_quantize_int8": (C.c_float, [f32p, C.c_int, u8p]),
            "oc_dequantize_int8": (None, [u8p, C.c_int, f32p]),
            "oc_float_to_fp8_e4m3": (C.c_uint8, [C.c_float]),
            "oc_fp8_e4m3_to_float": (C.c_float, [C.c_uint8]),
            "oc_wire_quantize": (C.c_int, [C.c_int, f32p, C.c_int, C.c_int, u8p]),
            "oc_wire_dequantize": (C.c_int, [C.c_int, u8p, C.c_int, C.c_int, f32p]),
            "oc_header_write": (None, [C.c_uint64, C.c_int32, C.c_int32, C.c_int32, C.c_uint8,
                                       C.c_uint8, C.c_uint16, C.c_float, u8p]),
            "oc_header_read": (C.c_int, [u8p, C.POINTER(C.c_uint64), C.POINTER(C.c_int32),
                                         C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                         C.POINTER(C.c_uint8), C.POINTER(C.c_uint8),
                                         C.POINTER(C.c_uint16), C.POINTER(C.c_float)]),
            "oc_header_payload_bytes": (C.c_int, [u8p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


# ---------------------------------------------------------------- helpers ---
def row_bytes(k: int) -> int:
    return (k // 256) * 144


def set_threads(n: int) -> None:
    lib().oc_set_threads(int(n))


def fill_normal(seed: int, tag: int, sigma: float, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oc_fill_normal(seed, tag, sigma, out, n)
    return out


def synth_q4k(seed: int, tag: int, rows: int, k: int, sigma_d: float = 0.01) -> np.ndarray:
    nb = rows * (k // 256)
    out = np.empty(nb * 144, np.uint8)
    lib().oc_synth_q4k(seed, tag, sigma_d, out, nb)
    return out


def expert_tag(e: int, m: int) -> int:
    return int(lib().oc_expert_tag(e, m))


def dequant(blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oc_q4k_dequant(np.ascontiguousarray(blocks, np.uint8), n, out)
    return out


def gemv(W: np.ndarray, x: np.ndarray, K: int, N: int) -> np.ndarray:
    y = np.empty(N, np.float32)
    lib().oc_q4k_gemv(np.ascontiguousarray(W, np.uint8), np.ascontiguousarray(x, np.float32), y, K, N)
    return y


def expert_forward(w1, w3, w2, D, F, x):
    y = np.empty(D, np.float32)
    lib().oc_expert_forward(w1, w3, w2, D, F, np.ascontiguousarray(x, np.float32), y)
    return y


def rmsnorm(x: np.ndarray) -> np.ndarray:
    y = np.empty_like(x, dtype=np.float32)
    lib().oc_rmsnorm(np.ascontiguousarray(x, np.float32), y, x.shape[-1])
    return y


def router(x: np.ndarray, Wr: np.ndarray, E: int, k: int, renorm: bool):
    D = x.shape[-1]
    logits = np.empty(E, np.float32)
    lib().oc_router_logits(np.ascontiguousarray(x, np.float32), np.ascontiguousarray(Wr, np.float32),
                           D, E, logits)
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    lib().oc_router_topk(logits, E, k, int(renorm), ids, w)
    return logits, ids, w


def dispatch_plan(ids: np.ndarray, E: int):
    ids = np.ascontiguousarray(ids.reshape(-1), np.int32)
    P_ = ids.size
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    perm = np.empty(P_, np.int32)
    inv = np.empty(P_, np.int32)
    lib().oc_dispatch_plan(ids, P_, E, counts, offsets, perm, inv)
    return counts, offsets, perm, inv


def routed_topk(gate, up, down, D, F, E, x, ids, w):
    out = np.empty(D, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    lib().oc_routed_topk(gate, up, down, D, F, E, np.ascontiguousarray(x, np.float32), ids, w,
                         ids.size, out)
    return out


def _vp(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def moe_forward(layer: dict, x: np.ndarray, flags: int):
    """Full MoE layer on the oracle; ``layer`` holds numpy arrays (see tests)."""
    T, D = x.shape
    k = layer["k"]
    out = np.empty((T, D), np.float32)
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    Fs = layer.get("Fs", 0)
    lib().oc_moe_forward(layer["gate"], layer["up"], layer["down"], layer["router"],
                         _vp(layer.get("sh_gate")), _vp(layer.get("sh_up")),
                         _vp(layer.get("sh_down")), _vp(layer.get("sh_gate_vec")),
                         D, layer["F"], layer["E"], k, Fs, int(layer["renorm"]), flags,
                         np.ascontiguousarray(x, np.float32), T, out, ids, w)
    return out, ids, w


def wire_quantize(mode: int, x: np.ndarray) -> bytes:
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    T, D = x.shape
    out = np.zeros(T * lib().oc_wire_token_bytes(mode, D), np.uint8)
    lib().oc_wire_quantize(mode, x, T, D, out)
    return out


def wire_dequantize(mode: int, buf: np.ndarray, T: int, D: int) -> np.ndarray:
    out = np.empty((T, D), np.float32)
    lib().oc_wire_dequantize(mode, np.ascontiguousarray(buf, np.uint8), T, D, out)
    return out
