"""fused_sandwich_norm — drop-in for fusions/01_sandwich_norm/fused/fused_sandwich_norm.py:46-72
(binding sandwich_norm_binding.cpp:11-71) on the sm_100a residual-norm-pair kernel.

    post_attn        = RMSNorm(attn_out, gamma1)
    updated_residual = residual_in + post_attn          (rounded to the input dtype)
    moe_in           = RMSNorm(updated_residual, gamma2)

Any hidden size (the reference kernel accepts only 2560); bf16, fp16 and fp32.
"""
from __future__ import annotations

import os
import sys

import torch

_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from kolibri_b200 import ops  # noqa: E402


def fused_sandwich_norm(
    attn_out: torch.Tensor,
    residual_in: torch.Tensor,
    gamma1: torch.Tensor,
    gamma2: torch.Tensor,
    eps: float = 1e-5,
):
    """-> [updated_residual, moe_in]."""
    for t, n in ((attn_out, "attn_out"), (residual_in, "residual_in"), (gamma1, "gamma1"),
                 (gamma2, "gamma2")):
        if not t.is_cuda:
            raise RuntimeError(f"{n} must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")
    if attn_out.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise RuntimeError("Unsupported dtype: only bfloat16, float16, and float32 are supported")
    s, n = ops.residual_norm_pair(attn_out, residual_in, gamma1, gamma2, eps)
    return [s, n]
