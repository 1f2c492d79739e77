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


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    a = x.detach().float().cpu().abs().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(a)) - 7)


def assert_chain_close(out: torch.Tensor, ref: torch.Tensor, inter: torch.Tensor,
                       what: str = "") -> None:
    """Bar for outputs computed through a rounded bf16 intermediate (h = res + bf16(norm(a))):
    within 1 bf16 ulp / atol 1e-2 of the oracle, plus one ulp of the oracle's intermediate.
    A 1-fp32-ulp difference in the rsqrt factor can move the intermediate by one bf16 ulp,
    which survives the residual add when it cancels."""
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    allow = 1e-2 + 2.0 ** -7 * r.abs() + bf16_ulp(inter)
    d = (o - r).abs()
    bad = d > allow
    assert not bool(bad.any()), (
        f"{what}: {int(bad.sum())} of {d.numel()} elements outside the bar; "
        f"worst {float((d - allow).max()):.3g} over at {tuple(torch.nonzero(bad)[0].tolist())}")


def bf16_ulp_dist(out: torch.Tensor, ref: torch.Tensor) -> torch.Tensor:
    """Element-wise distance in bf16 ulps (ordered-integer distance; +0 and -0 are equal)."""
    a = out.detach().to(torch.bfloat16).cpu().contiguous().view(torch.int16).to(torch.int32)
    b = ref.detach().to(torch.bfloat16).cpu().contiguous().view(torch.int16).to(torch.int32)

    def ordered(x):
        return torch.where(x < 0, -(x & 0x7FFF), x)
    return (ordered(a) - ordered(b)).abs()


def assert_bf16_ulp(out: torch.Tensor, ref: torch.Tensor, what: str = "",
                    inter: torch.Tensor = None, atol: float = 0.0,
                    max_frac: float = 1e-3) -> tuple:
    """The strict norm/RoPE bar: every element within 1 bf16 ulp of the oracle, except two
    named, counted cases (each at most max_frac of the elements):
      inter  the oracle's rounded bf16 intermediate (post = bf16(RMSNorm(a)*g) of
             h = bf16(res + post)): |out - ref| <= ulp(ref) + ulp(inter), when a 1-fp32-ulp
             difference in the rsqrt factor moved the intermediate across a rounding boundary;
      atol   cancellation (RoPE's y1*c - y2*s near zero): |out - ref| <= atol.
    Returns (worst ulp distance, elements accepted by the two cases)."""
    d = bf16_ulp_dist(out, ref)
    worst = int(d.max().item()) if d.numel() else 0
    over = d > 1
    n_over = int(over.sum().item())
    if n_over == 0:
        return worst, 0
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    ok = torch.zeros_like(over)
    if inter is not None:
        ok |= (o - r).abs() <= bf16_ulp(r) + bf16_ulp(inter)
    if atol > 0:
        ok |= (o - r).abs() <= atol
    bad = over & ~ok
    assert not bool(bad.any()), (
        f"{what}: {int(bad.sum())} elements beyond 1 bf16 ulp outside the named cases "
        f"(worst {worst} ulp)")
    assert n_over <= max(1, int(max_frac * d.numel())), (
        f"{what}: {n_over} of {d.numel()} elements beyond 1 ulp (worst {worst} ulp)")
    return worst, n_over
