"""MoE finalize on the GPU against the eager combine of the reference harness
(benchmarks/11_profile_2block_e2e.py:259-262): bf16 within 1 ulp (atol 1e-2, rtol 2^-7),
fp16 / fp32 within their own rounding."""
from __future__ import annotations

import pytest
import torch

from kb_testutil import assert_bf16_close
from kolibri_b200 import ops
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu


def case(T, K, H, dtype, E=384, seed=0, bad_ids=False):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    if bad_ids:
        ids[::7, 0] = -1
        ids[::5, -1] = E + 3
    _, _, _, u2p = ops.expert_maps(ids.cuda(), E)
    eo = torch.randn(T * K, H, generator=g).to(dtype)
    w = torch.rand(T, K, generator=g)
    return eo, u2p.cpu(), w


@pytest.mark.parametrize("T,K,H", [(1, 6, 6144), (64, 6, 6144), (1024, 6, 6144), (37, 8, 2560),
                                   (300, 1, 1024), (50, 16, 512)])
def test_finalize_bf16(T, K, H):
    eo, u2p, w = case(T, K, H, torch.bfloat16, seed=T + K)
    got = ops.moe_finalize(eo.cuda(), u2p.cuda(), w.cuda())
    assert_bf16_close(got, orc.finalize_ref(eo, u2p, w), f"finalize T={T} K={K} H={H}")


@pytest.mark.parametrize("dtype,atol,rtol", [(torch.float16, 2e-3, 1e-3), (torch.float32, 1e-5, 1e-6)])
def test_finalize_other_dtypes(dtype, atol, rtol):
    eo, u2p, w = case(200, 6, 2048, dtype, seed=7)
    got = ops.moe_finalize(eo.cuda(), u2p.cuda(), w.cuda())
    torch.testing.assert_close(got.cpu(), orc.finalize_ref(eo, u2p, w), atol=atol, rtol=rtol)


def test_finalize_skips_dropped_slots():
    # ids outside [0, E) leave u2p = -1: those slots add nothing
    eo, u2p, w = case(140, 6, 6144, torch.bfloat16, seed=3, bad_ids=True)
    assert (u2p < 0).any()
    got = ops.moe_finalize(eo.cuda(), u2p.cuda(), w.cuda())
    assert_bf16_close(got, orc.finalize_ref(eo, u2p, w), "finalize dropped slots")


def test_finalize_roundtrip_with_expansion():
    # expand -> identity "experts" -> finalize: out = x * sum_k w[t, k] (one token row each)
    T, K, H = 96, 6, 6144
    g = torch.Generator().manual_seed(11)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 384, (T, K), generator=g, dtype=torch.int32)
    w = torch.rand(T, K, generator=g)
    _, _, p2u, u2p = ops.expert_maps(ids.cuda(), 384)
    permuted = ops.expand_rows(x.cuda(), p2u)
    got = ops.moe_finalize(permuted, u2p, w.cuda())
    assert_bf16_close(got, orc.finalize_ref(permuted.cpu(), u2p.cpu(), w), "roundtrip")
