"""kolibri_cuda_ops — drop-in for the reference's JIT-built router extension
(kernels/cuda/kolibri_cuda_router.py, bindings kernels/cuda/router_bindings.cpp:60-127).

forward / forward_vA / forward_vB / forward_vFloat4 (logits, bias, topk) -> (ids int32, weights)
all run the same sm_100a kernel (the reference's variants are aliases of one another plus a
float4-load variant; the B200 kernel always uses 128-bit loads).  Differences from the
reference kernel that are deliberate: the weight is sigmoid of the raw logit read back from
memory rather than `biased - bias` (which can be off by one rounding), and expf is the
accurate one rather than __expf.
"""
from __future__ import annotations

import types

import torch

from .. import _root  # noqa: F401
from kolibri_b200 import ops


def _gate_forward(logits: torch.Tensor, bias: torch.Tensor, topk: int):
    if not logits.is_cuda:
        raise RuntimeError("logits must be a CUDA tensor")
    if logits.dim() != 2:
        raise RuntimeError("logits must be 2D [batch_size, n_experts]")
    n_experts = logits.size(1)
    if n_experts not in (256, 384):
        raise RuntimeError(f"n_experts must be 256 or 384 (got {n_experts})")
    if topk != 6:
        raise RuntimeError(f"Currently gate_forward kernel only supports topk=6 (got {topk})")
    logits_f32 = logits if logits.dtype == torch.float32 else logits.to(torch.float32)
    logits_f32 = logits_f32.contiguous()
    bias_f32 = None
    if bias is not None and bias.numel() > 0:
        bias_f32 = (bias if bias.dtype == torch.float32 else bias.to(torch.float32)).contiguous()
    ids, w = ops.router(logits_f32, bias_f32, k=6, renorm=False, w_dtype=torch.float32)
    if logits.dtype != torch.float32:
        return ids, w.to(logits.dtype)
    return ids, w


kolibri_cuda_ops = types.SimpleNamespace(
    forward=_gate_forward,
    forward_vA=_gate_forward,
    forward_vB=_gate_forward,
    forward_vFloat4=_gate_forward,
)
