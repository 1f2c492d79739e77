"""Expert-map and expansion entry points of the reference's kernels/cuda/kolibri_build_expert_maps.py
(bindings kernels/cuda/build_expert_maps_bindings.cpp:10-151), on the sm_100a kernels.

All map builders return [permuted_row_to_unpermuted_row int32 [T*k],
unpermuted_row_to_permuted_row int32 [T*k], expert_first_token_offset int64 [E+1]].
Rows inside an expert are in (token, slot) order on every path (the reference's atomic
kernels leave that order unspecified; its CUB baseline uses the same order).
"""
from __future__ import annotations

import torch

from .. import _root  # noqa: F401
from kolibri_b200 import ops


def _check_ids(ids: torch.Tensor) -> None:
    if not ids.is_cuda:
        raise RuntimeError("token_selected_experts must be a CUDA tensor")
    if not ids.is_contiguous():
        raise RuntimeError("token_selected_experts must be contiguous")
    if ids.dtype != torch.int32:
        raise RuntimeError("token_selected_experts must be int32")


def kolibri_build_expert_maps(token_selected_experts: torch.Tensor, num_experts: int = 384):
    """Stable expert maps (single-CTA kernel at decode sizes, two-kernel path above)."""
    _check_ids(token_selected_experts)
    _, off, p2u, u2p = ops.expert_maps(token_selected_experts, num_experts, counts=False)
    return [p2u, u2p, off]


def trtllm_build_expert_maps_b32(token_selected_experts: torch.Tensor, num_experts: int = 384):
    """The reference's CUB BlockRadixRank baseline; its (expert, token, slot) order is the
    order every path here produces, so it is the same builder."""
    return kolibri_build_expert_maps(token_selected_experts, num_experts)


def kolibri_activation_expansion(unpermuted_input: torch.Tensor,
                                 permuted_row_to_unpermuted_row: torch.Tensor):
    """out[r] = unpermuted_input[p2u[r] % num_tokens] (16-byte vector copy)."""
    if not unpermuted_input.is_cuda:
        raise RuntimeError("unpermuted_input must be a CUDA tensor")
    if not permuted_row_to_unpermuted_row.is_cuda:
        raise RuntimeError("permuted_row_to_unpermuted_row must be a CUDA tensor")
    if not unpermuted_input.is_contiguous():
        raise RuntimeError("unpermuted_input must be contiguous")
    if not permuted_row_to_unpermuted_row.is_contiguous():
        raise RuntimeError("permuted_row_to_unpermuted_row must be contiguous")
    if unpermuted_input.dtype not in (torch.float16, torch.bfloat16, torch.float8_e4m3fn,
                                      torch.float8_e5m2):
        raise RuntimeError("Unsupported dtype: only float16, bfloat16, float8_e4m3fn, and "
                           "float8_e5m2 are supported")
    return ops.expand_rows(unpermuted_input, permuted_row_to_unpermuted_row)
