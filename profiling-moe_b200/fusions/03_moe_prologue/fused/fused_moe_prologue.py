"""MoE prologue entry points — drop-in for fusions/03_moe_prologue/fused/fused_moe_prologue.py:55-115
(binding moe_prologue_binding.cpp:7-215), on the sm_100a kernels.

Deliberate difference: the router weights are UNnormalised by default (sigmoid of the raw
logit, Kolibri's norm_topk_prob=false), whereas the reference prologue router always
renormalises; pass norm_topk_prob=True to get the reference prologue's weights.
Rows inside an expert are in (token, slot) order (the reference's atomics leave it open).
"""
from __future__ import annotations

import os
import sys

import torch

_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from kolibri_b200 import ops  # noqa: E402

NUM_EXPERTS = 384
TOP_K = 6
# Token count below which the map build runs in one CTA (reference: HYBRID_TIPPING_POINT=512,
# fusions/03_moe_prologue/fused/custom_moe_prologue.cuh:16); the B200 library picks its own.


def kolibri_router(scores: torch.Tensor, bias: torch.Tensor = None, norm_topk_prob: bool = False):
    """Top-6 router: scores fp32 [T, 384], bias fp32 [384] or None
    -> [routing_weights fp32 [T, 6], selected_experts int32 [T, 6]]."""
    if not scores.is_cuda:
        raise RuntimeError("scores_in must be a CUDA tensor")
    if not scores.is_contiguous():
        raise RuntimeError("scores_in must be contiguous")
    if scores.dtype != torch.float32:
        raise RuntimeError("scores_in must be float32")
    if scores.size(1) != NUM_EXPERTS:
        raise RuntimeError("num_experts must be 384 for Kolibri")
    if bias is not None:
        if not bias.is_cuda:
            raise RuntimeError("bias must be a CUDA tensor")
        if not bias.is_contiguous():
            raise RuntimeError("bias must be contiguous")
        if bias.dtype != torch.float32:
            raise RuntimeError("bias must be float32")
    ids, w = ops.router(scores, bias, k=TOP_K, renorm=norm_topk_prob)
    return [w, ids]


def kolibri_dispatch_map(
    token_selected_experts: torch.Tensor,
    num_experts: int = 384,
    force_single_block: bool = False,
    force_multi_block: bool = False,
):
    """-> [permuted_row_to_unpermuted int32 [T*6], unpermuted_to_permuted int32 [T*6],
    expert_offsets int64 [385]]."""
    ids = token_selected_experts
    if not ids.is_cuda:
        raise RuntimeError("token_selected_experts must be a CUDA tensor")
    if not ids.is_contiguous():
        raise RuntimeError("token_selected_experts must be contiguous")
    if ids.dtype != torch.int32:
        raise RuntimeError("token_selected_experts must be int32")
    if ids.size(1) != TOP_K:
        raise RuntimeError("top_k must be 6 for Kolibri")
    if num_experts != NUM_EXPERTS:
        raise RuntimeError("num_experts must be 384 for Kolibri")
    mode = (ops.KB_MAPS_SINGLE_CTA if force_single_block
            else ops.KB_MAPS_MULTI_CTA if force_multi_block else ops.KB_MAPS_AUTO)
    _, off, p2u, u2p = ops.expert_maps(ids, num_experts, mode=mode, counts=False)
    return [p2u, u2p, off]


def kolibri_activation_expansion(unpermuted_input: torch.Tensor,
                                 permuted_row_to_unpermuted: torch.Tensor):
    """-> permuted_output [T*6, hidden]: row r = unpermuted_input[p2u[r] % T]."""
    if not unpermuted_input.is_cuda:
        raise RuntimeError("unpermuted_input must be a CUDA tensor")
    if not permuted_row_to_unpermuted.is_cuda:
        raise RuntimeError("permuted_row_to_unpermuted must be a CUDA tensor")
    if not unpermuted_input.is_contiguous():
        raise RuntimeError("unpermuted_input must be contiguous")
    if not permuted_row_to_unpermuted.is_contiguous():
        raise RuntimeError("permuted_row_to_unpermuted must be contiguous")
    if unpermuted_input.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("Unsupported dtype for activation expansion. Supported: BF16, FP16.")
    return ops.expand_rows(unpermuted_input, permuted_row_to_unpermuted)


def fused_moe_prologue(
    unpermuted_input: torch.Tensor,
    router_logits: torch.Tensor,
    router_bias: torch.Tensor = None,
    norm_topk_prob: bool = False,
):
    """Router + expert maps (one fused pass over the logits) + activation expansion.
    -> [permuted_output, routing_weights, selected_experts, expert_offsets,
        permuted_row_to_unpermuted, unpermuted_to_permuted]."""
    if not unpermuted_input.is_cuda:
        raise RuntimeError("unpermuted_input must be a CUDA tensor")
    if not router_logits.is_cuda:
        raise RuntimeError("router_logits must be a CUDA tensor")
    if not unpermuted_input.is_contiguous():
        raise RuntimeError("unpermuted_input must be contiguous")
    if not router_logits.is_contiguous():
        raise RuntimeError("router_logits must be contiguous")
    if unpermuted_input.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError("Unsupported dtype for fused_moe_prologue. Supported: BF16, FP16.")
    ids, w, _, off, p2u, u2p = ops.router_maps(router_logits, router_bias, k=TOP_K,
                                               renorm=norm_topk_prob)
    permuted = ops.expand_rows(unpermuted_input, p2u)
    return [permuted, w, ids, off, p2u, u2p]
