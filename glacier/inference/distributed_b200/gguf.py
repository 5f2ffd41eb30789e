"""GGUF reader for the MoE feed-forward tensors of a layer.

Loads ``blk.<L>.ffn_{gate,up,down}_exps.weight`` (Q4_K, one tensor per
matrix holding every expert: GGUF dims (K, rows, E), i.e. memory
[E][rows][K/256 * 144 B], the layout the reference's CPU worker slices
experts from, CpuWarmExpertPoolWorker.cs:241-258), the router
``blk.<L>.ffn_gate_inp.weight`` (F32, dims (D, E): memory [E][D], transposed
here to the [D][E] the library takes) and, when present, the Qwen2-MoE shared
expert ``ffn_{gate,up,down}_shexp`` with its gate vector
``ffn_gate_inp_shexp``, into a GpuExpertStageWorker layer.

The file format is GGUF version 2 or 3 (little-endian): magic "GGUF", version
u32, tensor count u64, metadata count u64; metadata entries (key string,
value type u32, value; arrays carry an element type and a u64 count); tensor
infos (name, n_dims u32, dims u64 x n_dims, ggml type u32, offset u64 from the
data section); the data section starts at the next multiple of
``general.alignment`` (default 32).  Tensors are mapped read-only with numpy
(no copy until the upload).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF"
GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_K = 12
_BLOCK = {GGML_TYPE_F32: (1, 4), GGML_TYPE_F16: (1, 2), GGML_TYPE_Q4_K: (256, 144)}  # (weights, bytes)

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


class GgufError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    dims: tuple       # GGUF order: dims[0] is the innermost (row length)
    ggml_type: int
    offset: int       # absolute file offset of the data

    def nbytes(self) -> int:
        if self.ggml_type not in _BLOCK:
            raise GgufError(f"{self.name}: ggml type {self.ggml_type} is not supported here")
        per, nb = _BLOCK[self.ggml_type]
        if self.dims[0] % per:
            raise GgufError(f"{self.name}: row length {self.dims[0]} is not a multiple of {per}")
        n = 1
        for d in self.dims[1:]:
            n *= d
        return n * (self.dims[0] // per) * nb


class GgufFile:
    def __init__(self, path: str):
        self.path = path
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        buf = self._map
        pos = 0

        def take(fmt):
            nonlocal pos
            size = struct.calcsize(fmt)
            if pos + size > len(buf):
                raise GgufError("truncated GGUF file")
            v = struct.unpack_from(fmt, buf, pos)[0]
            pos += size
            return v

        def string():
            nonlocal pos
            n = take("<Q")
            if pos + n > len(buf):
                raise GgufError("truncated GGUF string")
            s = bytes(buf[pos:pos + n]).decode("utf-8")
            pos += n
            return s

        def value(t):
            if t in _SCALAR:
                return take(_SCALAR[t])
            if t == _STR:
                return string()
            if t == _ARR:
                et, n = take("<I"), take("<Q")
                return [value(et) for _ in range(n)]
            raise GgufError(f"unknown metadata value type {t}")

        if take("<I") != GGUF_MAGIC:
            raise GgufError("not a GGUF file (bad magic)")
        self.version = take("<I")
        if self.version not in (2, 3):
            raise GgufError(f"GGUF version {self.version} is not supported (2 or 3)")
        n_tensors, n_kv = take("<Q"), take("<Q")
        self.metadata = {}
        for _ in range(n_kv):
            k = string()
            self.metadata[k] = value(take("<I"))
        infos = []
        for _ in range(n_tensors):
            name = string()
            nd = take("<I")
            dims = tuple(take("<Q") for _ in range(nd))
            infos.append((name, dims, take("<I"), take("<Q")))
        align = int(self.metadata.get("general.alignment", 32))
        data = (pos + align - 1) // align * align
        self.tensors = {}
        for name, dims, t, off in infos:
            ti = TensorInfo(name, dims, t, data + off)
            if t in _BLOCK and ti.offset + ti.nbytes() > len(buf):
                raise GgufError(f"{name}: data runs past the end of the file")
            self.tensors[name] = ti

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (read-only view)."""
        if name not in self.tensors:
            raise GgufError(f"tensor {name} not in {self.path}")
        ti = self.tensors[name]
        return self._map[ti.offset:ti.offset + ti.nbytes()]

    def f32(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        if ti.ggml_type != GGML_TYPE_F32:
            raise GgufError(f"{name}: expected F32, found ggml type {ti.ggml_type}")
        return self.raw(name).view(np.float32).reshape(tuple(reversed(ti.dims)))


def load_moe_layer(worker, gguf: GgufFile, layer: int, file_layer: int | None = None) -> None:
    """Uploads the MoE tensors of block ``file_layer`` (default ``layer``) of the
    file into layer ``layer`` of ``worker``; an expert-parallel shard takes
    its experts [expert_begin, expert_begin + expert_count)."""
    L = layer if file_layer is None else file_layer
    D, F, E = worker.hidden_dim, worker.expert_ffn_dim, worker.num_experts
    begin = worker.desc.expert_begin
    count = worker.desc.expert_count or E

    def experts(kind, K, rows):
        name = f"blk.{L}.ffn_{kind}_exps.weight"
        if name not in gguf.tensors:
            raise GgufError(f"tensor {name} not in {gguf.path}")
        ti = gguf.tensors[name]
        if ti.ggml_type != GGML_TYPE_Q4_K:
            raise GgufError(f"{name}: ggml type {ti.ggml_type}, only Q4_K ({GGML_TYPE_Q4_K}) is supported")
        if ti.dims != (K, rows, E):
            raise GgufError(f"{name}: dims {ti.dims}, the layer needs {(K, rows, E)}")
        per = rows * (K // 256) * 144
        return gguf.raw(name)[begin * per:(begin + count) * per]

    gate = experts("gate", D, F)
    up = experts("up", D, F)
    down = experts("down", F, D)
    rname = f"blk.{L}.ffn_gate_inp.weight"
    router = None
    if rname in gguf.tensors:
        r = gguf.f32(rname)
        if r.shape != (E, D):
            raise GgufError(f"{rname}: shape {r.shape}, the layer needs {(E, D)}")
        router = np.ascontiguousarray(r.T)  # [D][E]
    shared = [None] * 4
    Fs = worker.desc.shared_ffn_dim
    if Fs:
        def shexp(kind, K, rows):
            name = f"blk.{L}.ffn_{kind}_shexp.weight"
            ti = gguf.tensors.get(name)
            if ti is None or ti.ggml_type != GGML_TYPE_Q4_K or ti.dims != (K, rows):
                raise GgufError(f"{name}: missing, not Q4_K or not {(K, rows)}")
            return gguf.raw(name)
        shared = [shexp("gate", D, Fs), shexp("up", D, Fs), shexp("down", Fs, D), None]
        gname = f"blk.{L}.ffn_gate_inp_shexp.weight"
        if gname in gguf.tensors:
            shared[3] = gguf.f32(gname).reshape(-1)
    worker.load_layer(layer, gate, up, down, router, *shared)
