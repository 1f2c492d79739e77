"""The fused router + dispatch entry point of the reference's
kernels/cuda/kolibri_router_dispatch.py:49-64 (binding kernels/cuda/router_dispatch_bindings.cpp:
62-126), on the sm_100a kernels: one fused router + expert-map launch (kb_router_maps) and
the activation expansion with the permuted scales (kb_expand_rows_scaled, one pass).

Returns [permuted_output [T*6, H], permuted_scales fp32 [T*6], permuted_row_to_unpermuted_row
int32 [T*6], expert_first_token_offset int64 [385]], as the reference does.  Differences from
the reference, both deliberate: rows inside an expert segment come in (token, slot) order
(the reference scatters them with shared-memory atomics, an order that varies from run to
run), and the routing weights use the accurate expf (the reference builds with
--use_fast_math), so they match the eager router within 1e-6.
"""
from __future__ import annotations

import torch

from .. import _root  # noqa: F401
from kolibri_b200 import ops

TOP_K = 6


def fused_kolibri_router_dispatch(unpermuted_input: torch.Tensor, scores_in: torch.Tensor,
                                  bias: torch.Tensor):
    for t, n in ((unpermuted_input, "unpermuted_input"), (scores_in, "scores_in"), (bias, "bias")):
        if not t.is_cuda:
            raise RuntimeError(f"{n} must be a CUDA tensor")
        if not t.is_contiguous():
            raise RuntimeError(f"{n} must be contiguous")
    T = unpermuted_input.shape[0]
    E = scores_in.shape[1]
    if E != 384:
        raise RuntimeError("Kolibri router requires 384 experts")
    if bias.shape[0] != E:
        raise RuntimeError("bias size must match num_experts")
    if unpermuted_input.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("Unsupported dtype: only float16 and bfloat16 are supported")
    ids, w, _, offsets, p2u, _ = ops.router_maps(scores_in, bias, k=TOP_K, inverse=False)
    permuted_output, permuted_scales = ops.expand_rows_scaled(unpermuted_input, p2u, w)
    return [permuted_output, permuted_scales, p2u, offsets]
