"""fused_add_post_moe_norm — drop-in for fusions/02_post_moe_norm/fused/fused_post_moe_norm.py:54-77
(binding post_moe_norm_binding.cpp:6-79), plus fused_post_moe_pre_attn_norm, the post-MoE
norm fused with the next layer's pre-attention norm (no entry point in the reference; its math
is benchmarks/11_profile_2block_e2e.py:269-270 followed by :229-231).
"""
from __future__ import annotations

import os
import sys

import torch

_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from kolibri_b200 import ops  # noqa: E402


def _cuda_contig(*named):
    for t, n in named:
        if not t.is_cuda:
            raise RuntimeError(f"{n} must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")


def fused_add_post_moe_norm(
    routed_out: torch.Tensor,
    shared_out: torch.Tensor,
    gamma: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    """moe_out = RMSNorm(routed_out + shared_out, gamma)."""
    _cuda_contig((routed_out, "routed_out"), (shared_out, "shared_out"), (gamma, "gamma"))
    if routed_out.shape != shared_out.shape:
        raise RuntimeError("routed_out and shared_out must have the same shape")
    if routed_out.dtype != shared_out.dtype:
        raise RuntimeError("routed_out and shared_out must have the same dtype")
    if routed_out.dtype != gamma.dtype:
        raise RuntimeError("routed_out and gamma must have the same dtype")
    if gamma.numel() != routed_out.shape[-1]:
        raise RuntimeError("gamma must have size equal to hidden_dim")
    if routed_out.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise RuntimeError("Unsupported scalar type for fused_add_post_moe_norm. "
                           "Supported: BF16, FP16, FP32.")
    return ops.add_rms_norm(routed_out, shared_out, gamma, eps)


def fused_post_moe_pre_attn_norm(
    moe_out: torch.Tensor,
    h: torch.Tensor,
    gamma_post_moe: torch.Tensor,
    gamma_pre_attn: torch.Tensor,
    eps: float = 1e-6,
):
    """out = h + RMSNorm(moe_out, gamma_post_moe) ; next = RMSNorm(out, gamma_pre_attn).
    -> (out, next)."""
    _cuda_contig((moe_out, "moe_out"), (h, "h"), (gamma_post_moe, "gamma_post_moe"),
                 (gamma_pre_attn, "gamma_pre_attn"))
    return ops.residual_norm_pair(moe_out, h, gamma_post_moe, gamma_pre_attn, eps)
