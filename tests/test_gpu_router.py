"""Router parity on the GPU: ids bit-exact, fp32 weights within 1e-6 relative of the CPU
oracle, at the benchmark seeds and on adversarial rows."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from kolibri_b200 import ops
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu

W_RTOL = 1e-6  # fp32 sigmoid weights


def run_and_check(logits, bias, k=6, renorm=False, dev="cuda"):
    ids, w = ops.router(logits.to(dev), None if bias is None else bias.to(dev), k=k, renorm=renorm)
    rid, rw = orc.router_ref(logits, bias, k=k, renorm=renorm)
    assert torch.equal(ids.cpu(), rid), f"ids differ at rows {torch.nonzero((ids.cpu() != rid).any(1))[:8].flatten().tolist()}"
    torch.testing.assert_close(w.cpu(), rw, rtol=W_RTOL, atol=0)
    return ids, w


@pytest.mark.parametrize("T", [1, 7, 128, 4096, 65536])
def test_router_config0(T):
    logits, bias = wl.router_inputs(T, seed=0)
    run_and_check(logits, bias)


def test_router_golden_reference_eager():
    g = np.load(GOLDEN / "router_c0.npz")
    logits, bias = wl.router_inputs(128, seed=0)
    ids, w = ops.router(logits.cuda(), bias.cuda())
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    np.testing.assert_allclose(w.cpu().numpy(), g["w"], rtol=W_RTOL, atol=0)


@pytest.mark.parametrize("E,k", [(384, 1), (384, 8), (384, 16), (384, 32), (256, 6), (512, 6),
                                 (128, 6), (100, 6), (33, 6), (8, 8)])
@pytest.mark.parametrize("renorm", [False, True])
def test_router_shapes(E, k, renorm):
    g = torch.Generator().manual_seed(E * 100 + k)
    logits = torch.randn(257, E, generator=g)
    bias = 0.1 * torch.randn(E, generator=g)
    run_and_check(logits, bias, k=k, renorm=renorm)
    run_and_check(logits, None, k=k, renorm=renorm)


def test_router_ties_exact_path():
    g = torch.Generator().manual_seed(5)
    # coarse integer logits: many equal scores inside and across lanes
    logits = torch.randint(-3, 4, (1024, 384), generator=g).float()
    bias = torch.zeros(384)
    run_and_check(logits, bias)
    run_and_check(logits, torch.randint(-1, 2, (384,), generator=g).float())
    run_and_check(torch.zeros(8, 384), None)


def test_router_displaced_ties_keep_index_order():
    # Equal scores at low indices, larger scores at higher indices: the larger picks arrive
    # later and displace the equal ones, which must keep their index order.
    x = torch.zeros(64, 384)
    x[:, :40] = 3.0
    for r in range(64):
        x[r, 100 + r % 200] = 5.0 + (r % 3)
        x[r, 300 + r % 80] = 4.0
    run_and_check(x, None)
    run_and_check(x, torch.zeros(384), k=8)
    g = torch.Generator().manual_seed(5)
    logits = torch.randint(-3, 4, (1024, 384), generator=g).float()
    run_and_check(logits, torch.randint(-1, 2, (384,), generator=g).float())


def test_router_winners_in_one_lane():
    # Lane 0 of the float4 layout holds experts 0-3, 128-131, 256-259: give it the top 6..12.
    x = torch.randn(64, 384) - 10.0
    lane0 = [0, 1, 2, 3, 128, 129, 130, 131, 256, 257, 258, 259]
    for r in range(64):
        vals = torch.randperm(12)[: (r % 12) + 1]
        x[r, [lane0[i] for i in vals]] = 10.0 + torch.arange(len(vals)).float()
    run_and_check(x, torch.zeros(384))
    run_and_check(x, None, k=8)


def test_router_special_values():
    x = torch.randn(16, 384)
    x[0, 100] = float("nan")
    x[0, 7] = float("inf")
    x[1, :] = -float("inf")
    x[2, ::3] = float("nan")
    x[3, :] = 0.0
    x[3, ::2] = -0.0
    x[4, 200:] = float("inf")
    b = torch.zeros(384)
    b[::5] = -0.0
    ids, _ = ops.router(x.cuda(), b.cuda())
    rid, _ = orc.router_ref(x, b)
    assert torch.equal(ids.cpu(), rid)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_router_weight_dtypes(dtype, api):
    logits, bias = wl.router_inputs(300, seed=9)
    ids, w = api.fused_kolibri_router(logits.cuda(), bias.cuda(), k=6, output_dtype=dtype)
    rid, rw = orc.router_ref(logits, bias)
    assert torch.equal(ids.cpu(), rid) and w.dtype == dtype
    torch.testing.assert_close(w.cpu(), rw.to(dtype), rtol=0, atol=0)


def test_router_reference_entry_points(api):
    logits, bias = wl.router_inputs(200, seed=3)
    lc, bc = logits.cuda(), bias.cuda()
    rid, rw = orc.router_ref(logits, bias)
    ids, w = api.fused_kolibri_router(lc, bc)
    assert ids.dtype == torch.int32 and torch.equal(ids.cpu(), rid)
    for name in ("forward", "forward_vA", "forward_vB", "forward_vFloat4"):
        ids, w = getattr(api.kolibri_cuda_ops, name)(lc, bc, 6)
        assert torch.equal(ids.cpu(), rid)
        torch.testing.assert_close(w.cpu(), rw, rtol=W_RTOL, atol=0)
    ids, w = api.kolibri_cuda_ops.forward(lc, torch.empty(0, device="cuda"), 6)
    assert torch.equal(ids.cpu(), orc.router_ref(logits, None)[0])
    w, ids = api.kolibri_router(lc, bc)
    assert torch.equal(ids.cpu(), rid)
    torch.testing.assert_close(w.cpu(), rw, rtol=W_RTOL, atol=0)
    w, ids = api.kolibri_router(lc, bc, norm_topk_prob=True)
    torch.testing.assert_close(w.sum(-1).cpu(), torch.ones(200), rtol=1e-6, atol=1e-6)
    with pytest.raises(RuntimeError, match="n_experts must be 256 or 384"):
        api.kolibri_cuda_ops.forward(torch.randn(4, 100, device="cuda"), bc[:100], 6)
    with pytest.raises(RuntimeError, match="topk=6"):
        api.kolibri_cuda_ops.forward(lc, bc, 4)


@pytest.mark.parametrize("E", [128, 256, 384])
@pytest.mark.parametrize("k", [6, 8])
def test_router_tile_path_adversarial_rows(E, k):
    # T >= 32, fp32 weights, K <= 8: kb_router runs the tile kernel's routing phase.
    from test_gpu_maps import _adversarial_logits
    x = _adversarial_logits(E)
    g = torch.Generator().manual_seed(7 * E + k)
    bias = torch.randint(-1, 2, (E,), generator=g).float()
    bias[::5] = -0.0
    for b in (None, bias):
        for renorm in (False, True):
            ids, w = ops.router(x.cuda(), None if b is None else b.cuda(), k=k, renorm=renorm)
            rid, rw = orc.router_ref(x, b, k=k, renorm=renorm)
            assert torch.equal(ids.cpu(), rid), \
                f"rows {torch.nonzero((ids.cpu() != rid).any(1))[:8].flatten().tolist()}"
            torch.testing.assert_close(w.cpu(), rw, rtol=W_RTOL, atol=0, equal_nan=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_router_tile_path_tails_and_dtypes(dtype, api):
    # Token counts around the 32-row tile and CTA boundaries, weights in each output type.
    for T in (32, 33, 63, 4767, 148 * 32 * 3 + 5):
        logits, bias = wl.router_inputs(T, seed=T + 1)
        ids, w = api.fused_kolibri_router(logits.cuda(), bias.cuda(), k=6, output_dtype=dtype)
        rid, rw = orc.router_ref(logits, bias)
        assert torch.equal(ids.cpu(), rid), T
        if dtype == torch.float32:
            torch.testing.assert_close(w.cpu(), rw, rtol=W_RTOL, atol=0)
        else:
            # The fp32 weight agrees with the oracle to ~1e-6, so one that sits on a rounding
            # boundary of the output type may round to the neighbouring value: 1 ulp.
            ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10  # 1 ulp, relative
            torch.testing.assert_close(w.cpu().float(), rw.to(dtype).float(), rtol=ulp, atol=0)
