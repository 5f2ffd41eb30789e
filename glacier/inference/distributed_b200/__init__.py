"""B200 (sm_100a) backend for the quantized MoE feed-forward hot path of
Glacier.Inference.Distributed: Q4_K expert GEMV / grouped GEMM, router,
dispatch, SwiGLU, weighted combine, the INT8 stage-boundary wire codec and
decode attention over an fp16 KV cache, behind the C ABI in
include/glacier_b200.h."""
from ._lib import GlcError, LIB_PATH, lib  # noqa: F401
from .api import (Communicator, DenseStage, DynamicPrecisionSwitcher, FusedActivationHeader, GpuExpertStageWorker,  # noqa: F401
                  QuantizationKernels, WirePrecisionMode, attn_decode_dev, attn_workspace_bytes,
                  device_count, dispatch_plan_dev, gemv_poll_error, gemv_q4k_chain_dev, gemv_q4k_dev,
                  q4k_row_bytes, router_topk_dev,
                  torch_stream_handle)
# ep / pp import torch.distributed; they are imported on use:
#   from glacier.inference.distributed_b200.ep import ExpertParallelStageWorker, CudaExpertShard
#   from glacier.inference.distributed_b200.pp import StageBoundaryLink, CudaWireCodec
