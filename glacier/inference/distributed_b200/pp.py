"""Pipeline-stage boundary over a torch.distributed process group (one process per GPU).

Replaces the reference's stage-boundary transport -- activations quantised with
QuantizationKernels.QuantizeBatch (Protocol/QuantizationKernels.cs:134-146),
framed with a FusedActivationHeader (Protocol/FusedActivationHeader.cs:41-125)
and written to a TCP socket (DistributedClusterSession.cs:1123, Program.cs:743)
-- with a point-to-point send/recv (NCCL over NVLink on GPUs).  Each message is
the 32-byte FusedActivationHeader followed by the payload of the reference's
wire format (INT8/FP8: per token [f32 scale][D codes]; FP16; FP32), produced
and consumed on the GPU by the wire-codec kernels; the receiver sizes the
payload with the header's GetPayloadByteCount, as the reference does.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .api import FusedActivationHeader, QuantizationKernels, WirePrecisionMode, torch_stream_handle


class CudaWireCodec:
    """The wire codec on device tensors (the sm_100a kernels), asynchronous on the
    current torch stream."""

    @staticmethod
    def quantize(mode: int, x: torch.Tensor) -> torch.Tensor:
        T, D = x.shape
        out = torch.empty(T * QuantizationKernels.GetPackedTokenBytes(mode, D), dtype=torch.uint8,
                          device=x.device)
        QuantizationKernels.quantize_dev(mode, x.data_ptr(), T, D, out.data_ptr(),
                                         torch_stream_handle())
        return out

    @staticmethod
    def dequantize(mode: int, payload: torch.Tensor, T: int, D: int) -> torch.Tensor:
        out = torch.empty(T, D, dtype=torch.float32, device=payload.device)
        QuantizationKernels.dequantize_dev(mode, payload.data_ptr(), T, D, out.data_ptr(),
                                           torch_stream_handle())
        return out


class StageBoundaryLink:
    """Sends activations to the next pipeline stage and receives them from the
    previous one.  ``send``/``recv`` must be paired across the two ranks."""

    def __init__(self, codec=None, group=None, switcher=None):
        self.codec = codec if codec is not None else CudaWireCodec()
        self.group = group
        self.switcher = switcher  # optional DynamicPrecisionSwitcher: picks the mode when send gets none

    def send(self, x: torch.Tensor, dst: int, mode: int | None = WirePrecisionMode.INT8_Symmetric, *,
             sequence_id: int = 0, token_index: int = 0, layer_index: int = 0, flags: int = 0,
             sequence_position: int = 0, is_decode: bool = False) -> None:
        T, D = x.shape
        if mode is None:
            if self.switcher is None:
                raise ValueError("send without a mode needs a DynamicPrecisionSwitcher")
            mode = self.switcher.select_precision(T, sequence_position, is_decode)
        payload = self.codec.quantize(mode, x)
        hdr = FusedActivationHeader(sequence_id, token_index, layer_index, D, mode, flags, 1.0, T)
        raw = torch.frombuffer(bytearray(hdr.write_to()), dtype=torch.uint8).to(x.device)
        dist.send(raw, dst, group=self.group)
        dist.send(payload, dst, group=self.group)

    def recv(self, src: int, device) -> tuple[FusedActivationHeader, torch.Tensor]:
        raw = torch.empty(FusedActivationHeader.HeaderSize, dtype=torch.uint8, device=device)
        dist.recv(raw, src, group=self.group)
        hdr = FusedActivationHeader.read_from(bytes(raw.cpu().tolist()))
        payload = torch.empty(hdr.get_payload_byte_count(), dtype=torch.uint8, device=device)
        dist.recv(payload, src, group=self.group)
        T = hdr.batch_tokens if hdr.batch_tokens > 0 else 1
        return hdr, self.codec.dequantize(hdr.precision_mode, payload, T, hdr.hidden_dim)
