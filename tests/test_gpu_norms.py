"""Residual norm fusions on the GPU against the eager CPU oracle: bf16 within 1 ulp
(atol 1e-2, rtol 2^-7); fp16/fp32 within the reference's own tolerances."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
import torch.nn.functional as F

from kb_testutil import assert_bf16_close, assert_bf16_ulp, assert_chain_close
from kolibri_b200 import ops
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 64, 1024, 16384])
def test_sandwich_and_post_moe_pair_config3(T, api, record_property):
    ni = wl.norm_inputs(T, seed=3)
    c = lambda t: t.cuda()  # noqa: E731
    h, x = api.fused_sandwich_norm(c(ni.attn_out), c(ni.residual), c(ni.g_post_attn),
                                   c(ni.g_pre_moe), eps=wl.EPS)
    rh, rx = orc.sandwich_ref(ni.attn_out, ni.residual, ni.g_post_attn, ni.g_pre_moe, eps=wl.EPS)
    post = F.rms_norm(ni.attn_out, (wl.HIDDEN,), ni.g_post_attn, eps=wl.EPS)
    assert_chain_close(h, rh, post, "sandwich h")
    assert_chain_close(x, rx, post, "sandwich x")
    # Strict bar: <= 1 bf16 ulp, except counted elements explained by the rounded intermediate
    # (the sums); each normalised output against the oracle's norm of the kernel's own sum.
    H = wl.HIDDEN
    rep = {"h": assert_bf16_ulp(h, rh, "sandwich h", inter=post),
           "x": assert_bf16_ulp(x, F.rms_norm(h.cpu(), (H,), ni.g_pre_moe, eps=wl.EPS),
                                "sandwich x on its own h")}
    # second half of config 3 on the oracle's h (so each stage is checked on its own input)
    o, n = api.fused_post_moe_pre_attn_norm(c(ni.moe_out), c(rh), c(ni.g_post_moe),
                                            c(ni.g_pre_attn), eps=wl.EPS)
    ro, rn = orc.post_moe_pre_attn_ref(ni.moe_out, rh, ni.g_post_moe, ni.g_pre_attn, eps=wl.EPS)
    pm = F.rms_norm(ni.moe_out, (wl.HIDDEN,), ni.g_post_moe, eps=wl.EPS)
    assert_chain_close(o, ro, pm, "pair out")
    assert_chain_close(n, rn, pm, "pair next")
    rep["out"] = assert_bf16_ulp(o, ro, "pair out", inter=pm)
    rep["next"] = assert_bf16_ulp(n, F.rms_norm(o.cpu(), (H,), ni.g_pre_attn, eps=wl.EPS),
                                  "pair next on its own out")
    for k, (worst, named) in rep.items():   # worst ulp distance, elements of the named case
        record_property(f"worst_ulp_{k}", worst)
        record_property(f"named_case_{k}", named)
    print(f"T={T} worst bf16 ulp / named-case elements: {rep}")


def test_norms_golden_reference_eager(api):
    g = np.load(GOLDEN / "norms_c3_T2.npz")
    ni = wl.norm_inputs(2, seed=3)
    b = lambda a: torch.from_numpy(a).view(torch.bfloat16)  # noqa: E731
    h, x = api.fused_sandwich_norm(ni.attn_out.cuda(), ni.residual.cuda(), ni.g_post_attn.cuda(),
                                   ni.g_pre_moe.cuda(), eps=wl.EPS)
    assert_bf16_close(h, b(g["sandwich_h"]), "h")
    assert_bf16_close(x, b(g["sandwich_x"]), "x")
    m = api.fused_add_post_moe_norm(ni.attn_out.cuda(), ni.moe_out.cuda(), ni.g_post_moe.cuda(),
                                    eps=wl.EPS)
    assert_bf16_close(m, b(g["add_post_moe"]), "post-moe")


@pytest.mark.parametrize("H", [2560, 6144])
@pytest.mark.parametrize("T", [1, 16, 64, 256, 1152])
@pytest.mark.parametrize("dtype,atol,rtol", [(torch.bfloat16, 1e-2, 2.0 ** -7),
                                             (torch.float16, 1e-3, 1e-3),
                                             (torch.float32, 1e-5, 1e-5)])
def test_add_post_moe_norm_reference_sizes(H, T, dtype, atol, rtol, api):
    # fusions/02_post_moe_norm/benchmark_and_verify.py:32-82 (seed 42+n, gamma |N|+0.1)
    torch.manual_seed(42 + T)
    routed = torch.randn(T, H, dtype=dtype)
    shared = torch.randn(T, H, dtype=dtype)
    gamma = torch.randn(H, dtype=dtype).abs() + 0.1
    out = api.fused_add_post_moe_norm(routed.cuda(), shared.cuda(), gamma.cuda(), eps=1e-5)
    ref = orc.add_post_moe_norm_ref(routed, shared, gamma, eps=1e-5)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H", [1000, 20000, 8, 2560])
def test_residual_pair_generic_widths(dtype, H):
    g = torch.Generator().manual_seed(H)
    a = torch.randn(37, H, generator=g).to(dtype)
    r = torch.randn(37, H, generator=g).to(dtype)
    g1 = (1 + 0.02 * torch.randn(H, generator=g)).to(dtype)
    g2 = (1 + 0.02 * torch.randn(H, generator=g)).to(dtype)
    s, n = ops.residual_norm_pair(a.cuda(), r.cuda(), g1.cuda(), g2.cuda(), 1e-6)
    rs, rn = orc.sandwich_ref(a, r, g1, g2, eps=1e-6)
    tol = dict(atol=1e-2, rtol=2.0 ** -7) if dtype == torch.bfloat16 else \
        dict(atol=2e-3, rtol=1e-3) if dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    if dtype == torch.bfloat16:
        post = F.rms_norm(a, (H,), g1, eps=1e-6)
        assert_chain_close(s, rs, post, "sum")
        assert_chain_close(n, rn, post, "norm")
    else:
        torch.testing.assert_close(s.cpu().float(), rs.float(), **tol)
        torch.testing.assert_close(n.cpu().float(), rn.float(), **tol)
    out, sm = ops.add_rms_norm(a.cuda(), r.cuda(), g1.cuda(), 1e-6, return_sum=True)
    torch.testing.assert_close(sm.cpu().float(), (a + r).float(), atol=0, rtol=0)
    torch.testing.assert_close(out.cpu().float(), orc.add_post_moe_norm_ref(a, r, g1, 1e-6).float(), **tol)


def test_sandwich_reference_verify_case(api):
    # fusions/01_sandwich_norm/benchmark_and_verify.py:21-63: N=64, d=2560, gammas 1+0.05N
    for dtype, atol, rtol in ((torch.bfloat16, 4e-2, 2e-2), (torch.float16, 1e-2, 1e-2)):
        torch.manual_seed(42)
        a = torch.randn(64, 2560, dtype=dtype)
        r = torch.randn(64, 2560, dtype=dtype)
        g1 = torch.ones(2560, dtype=dtype) + 0.05 * torch.randn(2560, dtype=dtype)
        g2 = torch.ones(2560, dtype=dtype) + 0.05 * torch.randn(2560, dtype=dtype)
        h, x = api.fused_sandwich_norm(a.cuda(), r.cuda(), g1.cuda(), g2.cuda(), eps=1e-5)
        rh, rx = orc.sandwich_ref(a, r, g1, g2, eps=1e-5)
        torch.testing.assert_close(h.cpu(), rh, atol=atol, rtol=rtol)
        torch.testing.assert_close(x.cpu(), rx, atol=atol, rtol=rtol)
