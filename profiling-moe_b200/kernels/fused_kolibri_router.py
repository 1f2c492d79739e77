"""fused_kolibri_router — same signature and results as the reference's Triton entry point
(kernels/triton/fused_kolibri_router.py:98-146), computed by the sm_100a router kernel.

    scores = x + bias ; ids = top-k of scores (lower expert index wins ties)
    weights = sigmoid(x[ids])  (un-biased logit, unnormalised unless norm_topk_prob)
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _root  # noqa: F401
from kolibri_b200 import ops


def fused_kolibri_router(
    x: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    k: int = 6,
    norm_topk_prob: bool = False,
    output_dtype: Optional[torch.dtype] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Router logits [batch, num_experts] -> (topk_ids int32 [batch, k], topk_weights [batch, k]
    in output_dtype, default x.dtype)."""
    assert x.is_cuda, "Inputs must be on CUDA"
    b, e = x.shape
    assert e <= 512, f"Kernel currently supports up to 512 experts (got {e})"
    if output_dtype is None:
        output_dtype = x.dtype
    logits = x if x.dtype == torch.float32 else x.float()
    logits = logits.contiguous()
    bias32 = None
    if bias is not None:
        bias32 = (bias if bias.dtype == torch.float32 else bias.float()).contiguous()
    direct = output_dtype in (torch.float32, torch.bfloat16, torch.float16)
    ids, w = ops.router(logits, bias32, k=k, renorm=norm_topk_prob,
                        w_dtype=output_dtype if direct else torch.float32)
    if not direct:
        w = w.to(output_dtype)
    return ids, w
