"""kolibri_multi_block_build_expert_maps — drop-in for the reference's multi-block builder
(kernels/cuda/multi_block_expert_maps/kolibri_multi_block_build_expert_maps.py, bindings
multi_block_build_expert_maps_bindings.cpp:10-60).

max_blocks < 0 forces the multi-CTA path (the reference's "force multi-block" convention);
max_blocks >= 0 lets the library choose.  The B200 builder sizes its own grid, so the block
count itself is not a tuning knob here.
"""
from __future__ import annotations

import os
import sys

import torch

_ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..", ".."))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
from kolibri_b200 import ops  # noqa: E402


def kolibri_multi_block_build_expert_maps(
    token_selected_experts: torch.Tensor,
    num_experts: int = 384,
    max_blocks: int = 128,
    return_inverse_map: bool = True,
):
    if not token_selected_experts.is_cuda:
        raise RuntimeError("token_selected_experts must be a CUDA tensor")
    if not token_selected_experts.is_contiguous():
        raise RuntimeError("token_selected_experts must be contiguous")
    if token_selected_experts.dtype != torch.int32:
        raise RuntimeError("token_selected_experts must be int32")
    mode = ops.KB_MAPS_MULTI_CTA if max_blocks < 0 else ops.KB_MAPS_AUTO
    _, off, p2u, u2p = ops.expert_maps(token_selected_experts, num_experts, mode=mode,
                                       counts=False, inverse=return_inverse_map)
    if u2p is None:
        u2p = torch.empty((0,), dtype=torch.int32, device=token_selected_experts.device)
    return [p2u, u2p, off]
