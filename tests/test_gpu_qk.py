"""Q/K RMSNorm + NeoX RoPE on the GPU against the CPU oracle (formula of the reference's
scratch/diag_rope_fusion.py; RNoPE = per-head F.rms_norm): within 1 bf16 ulp / atol 1e-2, and
at the BASELINE shapes the strict bar: every element within 1 bf16 ulp except counted
cancellation elements of the rotation."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from kb_testutil import assert_bf16_close, assert_bf16_ulp
from kolibri_b200 import ops
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 8, 64, 256, 4096])
@pytest.mark.parametrize("rnope", [False, True])
def test_qk_config2(T, rnope, api):
    q, k, gq, gk, pos = wl.qk_inputs(T, seed=2)
    qo, ko = api.fused_qk_norm_rope(q.cuda(), k.cuda(), gq.cuda(), gk.cuda(), pos.cuda(),
                                    eps=wl.EPS, theta=wl.ROPE_THETA, rnope=rnope)
    rq, rk = orc.qk_norm_rope_ref(q, k, gq, gk, None if rnope else pos, eps=wl.EPS,
                                  theta=wl.ROPE_THETA)
    assert_bf16_close(qo, rq, "q")
    assert_bf16_close(ko, rk, "k")
    # strict bar: <= 1 bf16 ulp, the cancellation case of the rotation (|diff| <= 1e-3) counted
    assert_bf16_ulp(qo, rq, "q", atol=1e-3)
    assert_bf16_ulp(ko, rk, "k", atol=1e-3)
    if rnope:  # zero positions through the RoPE path give the same result
        z = torch.zeros(T, dtype=torch.int32, device="cuda")
        qz, kz = ops.qk_norm_rope(q.cuda(), k.cuda(), gq.cuda(), gk.cuda(), z, eps=wl.EPS)
        assert torch.equal(qz, qo) and torch.equal(kz, ko)


def test_qk_golden_reference_formula():
    g = np.load(GOLDEN / "qk_c2_T4.npz")
    q, k, gq, gk, pos = wl.qk_inputs(4, seed=2)
    b = lambda a: torch.from_numpy(a).view(torch.bfloat16)  # noqa: E731
    qo, ko = ops.qk_norm_rope(q.cuda(), k.cuda(), gq.cuda(), gk.cuda(), pos.cuda(), eps=wl.EPS)
    assert_bf16_close(qo, b(g["q_swa"]), "q swa")
    assert_bf16_close(ko, b(g["k_swa"]), "k swa")
    qo, ko = ops.qk_norm_rope(q.cuda(), k.cuda(), gq.cuda(), gk.cuda(), None, eps=wl.EPS)
    assert_bf16_close(qo, b(g["q_rnope"]), "q rnope")
    assert_bf16_close(ko, b(g["k_rnope"]), "k rnope")


def test_qk_inplace_on_fused_qkv_buffer(api):
    T, Hq, Hkv, D = 33, wl.HQ, wl.HKV, wl.HEAD_DIM
    gen = torch.Generator().manual_seed(3)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=gen).to(torch.bfloat16)
    gq = (1 + 0.02 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    gk = (1 + 0.02 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    pos = torch.randint(0, 8192, (T,), generator=gen, dtype=torch.int32)
    dq = qkv.cuda()
    api.apply_qk_norm_rope_qkv(dq, Hq, Hkv, gq.cuda(), gk.cuda(), pos.cuda(), eps=wl.EPS)
    q = qkv[:, : Hq * D].reshape(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    rq, rk = orc.qk_norm_rope_ref(q, k, gq, gk, pos, eps=wl.EPS)
    out = dq.cpu()
    assert_bf16_close(out[:, : Hq * D].reshape(T, Hq, D), rq, "q")
    assert_bf16_close(out[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D), rk, "k")
    assert torch.equal(out[:, (Hq + Hkv) * D:], qkv[:, (Hq + Hkv) * D:]), "V must be untouched"


@pytest.mark.parametrize("D", [64, 256])
def test_qk_other_head_dims(D):
    gen = torch.Generator().manual_seed(D)
    q = torch.randn(17, 12, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(17, 3, D, generator=gen).to(torch.bfloat16)
    gq = (1 + 0.02 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    gk = (1 + 0.02 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    pos = torch.randint(0, 8192, (17,), generator=gen, dtype=torch.int32)
    qo, ko = ops.qk_norm_rope(q.cuda(), k.cuda(), gq.cuda(), gk.cuda(), pos.cuda(), eps=1e-6,
                              theta=1e6)
    rq, rk = orc.qk_norm_rope_ref(q, k, gq, gk, pos, eps=1e-6, theta=1e6)
    assert_bf16_close(qo, rq, "q")
    assert_bf16_close(ko, rk, "k")
