"""Helpers shared by the test modules."""
from __future__ import annotations

import numpy as np
import torch


def assert_bf16_close(out: torch.Tensor, ref: torch.Tensor, what: str = "") -> None:
    """The norm/RoPE bar: within 1 bf16 ulp of the oracle (rtol 2^-7) or atol 1e-2."""
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    torch.testing.assert_close(o, r, atol=1e-2, rtol=2.0 ** -7, msg=lambda m: f"{what}: {m}")


def bf16_ulp_diff(out: torch.Tensor, ref: torch.Tensor) -> int:
    """Largest distance in bf16 ulps (ordered-integer distance) between two bf16 tensors."""
    a = out.detach().cpu().contiguous().view(torch.int16).to(torch.int32)
    b = ref.detach().cpu().contiguous().view(torch.int16).to(torch.int32)
    def ordered(x):
        return torch.where(x < 0, -(x & 0x7FFF), x)
    return int((ordered(a) - ordered(b)).abs().max().item()) if a.numel() else 0


def np_of(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
