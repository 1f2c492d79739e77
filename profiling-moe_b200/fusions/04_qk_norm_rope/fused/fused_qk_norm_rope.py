"""fused_qk_norm_rope — per-head Q/K RMSNorm fused with NeoX RoPE on the sm_100a kernel.

The reference has no local entry point for this stage: it calls TensorRT-LLM's
Kolibri1Attention.apply_rope / fusedQKNormRopeKernel (benchmarks/02_benchmark_attention_norm.py:105-112),
whose math is written out in scratch/diag_rope_fusion.py:31-38.  RNoPE (full-attention) layers
pass zero positions in the reference (benchmarks/02_verify_zero_position_rnope.py); here
rnope=True (or position_ids=None) takes the identity rotation without evaluating cos/sin.
"""
from __future__ import annotations

import os
import sys
from typing import Optional

import torch

_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from kolibri_b200 import ops  # noqa: E402


def fused_qk_norm_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    gamma_q: torch.Tensor,
    gamma_k: torch.Tensor,
    position_ids: Optional[torch.Tensor],
    eps: float = 1e-6,
    theta: float = 10000.0,
    rnope: bool = False,
    inplace: bool = False,
):
    """q [T, Hq, D], k [T, Hkv, D] bf16 (heads contiguous; the token stride may be that of a
    fused qkv buffer) -> (q_out, k_out)."""
    return ops.qk_norm_rope(q, k, gamma_q, gamma_k, None if rnope else position_ids, eps=eps,
                            theta=theta, inplace=inplace)


def apply_qk_norm_rope_qkv(qkv: torch.Tensor, num_heads: int, num_kv_heads: int,
                           gamma_q: torch.Tensor, gamma_k: torch.Tensor,
                           position_ids: Optional[torch.Tensor], eps: float = 1e-6,
                           theta: float = 10000.0, rnope: bool = False) -> torch.Tensor:
    """In-place on a fused qkv buffer [T, (Hq + 2*Hkv) * D] (V untouched), as the fused
    apply_rope path modifies qkv.  Returns qkv."""
    T = qkv.shape[0]
    D = qkv.shape[1] // (num_heads + 2 * num_kv_heads)
    q = qkv[:, : num_heads * D].view(T, num_heads, D) if T else qkv.new_empty((0, num_heads, D))
    k = qkv[:, num_heads * D:(num_heads + num_kv_heads) * D].view(T, num_kv_heads, D) \
        if T else qkv.new_empty((0, num_kv_heads, D))
    ops.qk_norm_rope(q, k, gamma_q, gamma_k, None if rnope else position_ids, eps=eps,
                     theta=theta, inplace=True)
    return qkv
