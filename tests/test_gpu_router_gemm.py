"""Router projection on the tensor cores (kb_router_gemm) against the CPU oracle.

The logits are an fp32-accumulated product rounded once to bf16: they are checked against
the exact (fp64) product rounded to bf16, within one bf16 ulp (the accumulation order differs,
so a sum lying within an fp32 rounding of a bf16 tie may round the other way), and nearly all
of them must be equal.  Near zero the bar is absolute, 1e-4: the tensor cores round the
running fp32 sum (|sum| ~ 1.6 here, ulp ~ 2e-7) at each of the 384 K=16 steps, so a logit
that cancels to ~0 keeps an absolute error of a few 1e-5, as any fp32-accumulating GEMM does.  The routing fused into the epilogue is checked bit for bit: ids equal
and fp32 weights within 1e-6 of router_ref applied to the kernel's own logits, the same bar as
the stand-alone router.  Shapes cover every tile width and hidden split, tokens that do not
fill a tile, ties and non-finite logits.
"""
from __future__ import annotations

import os

import pytest
import torch

from kolibri_b200 import _lib
from kolibri_b200 import ops
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu

W_RTOL = 1e-6
H = 6144


def inputs(T, E=384, Hd=H, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, Hd, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(E, Hd, generator=g)).to(torch.bfloat16)
    b = 0.1 * torch.randn(E, generator=g)
    return x, w, b


def check(x, w, b, k=6, renorm=False, logits_rtol=2 ** -7, min_equal=0.99, atol=1e-4):
    dev = "cuda"
    ids, wt, lg = ops.router_gemm(x.to(dev), w.to(dev), None if b is None else b.to(dev), k=k,
                                  renorm=renorm)
    lg = lg.cpu()
    _, _, ref = orc.router_gemm_ref(x, w, b, k=k, renorm=renorm)
    torch.testing.assert_close(lg, ref, rtol=logits_rtol, atol=atol, equal_nan=True)
    fin = torch.isfinite(ref)
    eq = ((lg == ref) | ~fin).float().mean().item()
    assert eq >= min_equal, f"only {eq:.4f} of the logits equal the rounded exact product"
    rid, rw = orc.router_ref(lg, b, k=k, renorm=renorm)
    bad = (ids.cpu() != rid).any(1).nonzero().flatten()
    assert bad.numel() == 0, f"ids differ at rows {bad[:8].tolist()}"
    torch.testing.assert_close(wt.cpu(), rw, rtol=W_RTOL, atol=0, equal_nan=True)
    return ids, wt, lg


def describe(T, E=384, Hd=H, k=6):
    import ctypes
    bn, ks, grid = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(_lib.load().kb_router_gemm_describe(T, Hd, E, k, ctypes.byref(bn),
                                                   ctypes.byref(ks), ctypes.byref(grid)),
               "kb_router_gemm_describe")
    return bn.value, ks.value, grid.value


@pytest.fixture
def forced(monkeypatch):
    def force(bn=0, ks=0):
        monkeypatch.setenv("KB_RGEMM_BN", str(bn))
        monkeypatch.setenv("KB_RGEMM_KS", str(ks))
    return force


@pytest.mark.parametrize("T", [1, 7, 32, 128, 200, 256, 1000, 4096, 8192])
def test_router_gemm_chain_sizes(T):
    x, w, b = inputs(T, seed=T)
    check(x, w, b)


@pytest.mark.parametrize("bn,ks", [(64, 1), (64, 4), (64, 96), (128, 1), (128, 3), (192, 1),
                                   (192, 2), (192, 5)])
@pytest.mark.parametrize("T", [33, 300])
def test_router_gemm_forced_tiles(forced, bn, ks, T):
    forced(bn, ks)
    got = describe(T)
    assert got[0] == bn
    x, w, b = inputs(T, seed=bn + ks)
    check(x, w, b)


@pytest.mark.parametrize("bn", [64, 128, 192])
def test_router_gemm_per_tile_path(forced, monkeypatch, bn):
    # one hidden split, each tile ranked on its own and the tiles merged per token tile (the
    # path of grids larger than the SMs), forced at a small T
    forced(bn, 1)
    monkeypatch.setenv("KB_RGEMM_COOP", "0")
    x, w, b = inputs(300, seed=bn)
    check(x, w, b)
    check(x, w, None, k=8, renorm=True)


def test_router_gemm_more_tiles_than_sms():
    x, w, b = inputs(20000, seed=7)
    check(x, w, b)


@pytest.mark.parametrize("E,k,renorm", [(128, 1, False), (256, 8, True), (512, 6, False),
                                        (448, 4, True), (64, 8, False)])
def test_router_gemm_shapes(E, k, renorm):
    x, w, b = inputs(150, E=E, Hd=1024, seed=E + k)
    check(x, w, b, k=k, renorm=renorm)
    check(x, w, None, k=k, renorm=renorm)


def test_router_gemm_bn256(forced):
    forced(256, 2)
    x, w, b = inputs(130, E=512, Hd=2048, seed=3)
    check(x, w, b)


def test_router_gemm_ties_and_nonfinite():
    x, w, b = inputs(256, seed=11)
    # equal gate rows give equal logits: with equal biases, exact ties across tiles and lanes
    for src, dst in [(5, 200), (5, 383), (64, 65), (0, 191), (0, 192)]:
        w[dst] = w[src]
        b[dst] = b[src]
    w[17] = w[16]
    b[17] = b[16] = 10.0          # a tie that is certainly selected
    # an infinite activation makes its row's logits +-inf, and NaN where the gate weight is 0
    x[3, 10] = float("inf")
    w[7, 10] = 0.0
    x[9, :] = 0.0                  # an all-zero row: every logit 0, ranked by bias alone
    ids, _, lg = check(x, w, b)
    assert torch.isnan(lg[3, 7]) and ids[3, 0].item() == 7
    assert ids[100, 0].item() == 16 and ids[100, 1].item() == 17
    check(x, w, None)


def test_router_gemm_logits_only_and_repeat():
    x, w, b = inputs(256, seed=21)
    dev = "cuda"
    ids, wt, lg = ops.router_gemm(x.to(dev), w.to(dev), b.to(dev), route=False)
    assert ids is None and wt is None
    _, _, ref = orc.router_gemm_ref(x, w, b)
    torch.testing.assert_close(lg.cpu(), ref, rtol=2 ** -7, atol=1e-4)
    # two calls in a row (split partials, tickets reset by each call) give identical results
    a = ops.router_gemm(x.to(dev), w.to(dev), b.to(dev))
    c = ops.router_gemm(x.to(dev), w.to(dev), b.to(dev))
    for u, v in zip(a, c):
        assert torch.equal(u, v)
    assert torch.equal(a[2], lg)


def test_router_gemm_shapes_share_one_workspace():
    # calls of different shapes in a row on one workspace: no call's scratch may overlap
    # another call's counters
    for T in (1000, 4096, 256, 4096, 33, 8192, 1000):
        x, w, b = inputs(T, seed=T + 1)
        check(x, w, b)


def test_router_gemm_workspace_left_clean():
    lib = _lib.load()
    T, E, k = 256, 384, 6
    bn, ks, _ = describe(T)
    zero = 256 * 1024   # the fixed zero zone: error word and tickets
    need = lib.kb_router_gemm_workspace_bytes(T, H, E, k)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    x, w, b = inputs(T, seed=4)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    wt = torch.empty(T, k, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        _lib.check(lib.kb_router_gemm(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), None,
                                      ids.data_ptr(), wt.data_ptr(), ws.data_ptr(), need, T, H, E,
                                      k, 0, st), "kb_router_gemm")
    torch.cuda.synchronize()
    assert int(ws[:zero].count_nonzero()) == 0
    assert ops.workspace_status(ws, _lib.KB_WS_RGEMM) == _lib.KB_WS_CLEAN
    rid, rw, _ = orc.router_gemm_ref(x, w, b)
    # logits were not stored: ids against the exact rounding, allowing the rare 1-ulp flip
    assert (ids.cpu() == rid).all(1).float().mean().item() > 0.98
    # a too-small workspace and unaligned shapes are refused before any launch
    assert lib.kb_router_gemm(xd.data_ptr(), wd.data_ptr(), None, None, ids.data_ptr(),
                              wt.data_ptr(), ws.data_ptr(), need - 256, T, H, E, k, 0,
                              st) == _lib.KB_ERR_WORKSPACE
    assert lib.kb_router_gemm(xd.data_ptr(), wd.data_ptr(), None, None, ids.data_ptr(),
                              wt.data_ptr(), ws.data_ptr(), need, T, H - 32, E, k, 0,
                              st) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_router_gemm(xd.data_ptr(), wd.data_ptr(), None, None, ids.data_ptr(),
                              wt.data_ptr(), ws.data_ptr(), need, T, H, E, 9, 0,
                              st) == _lib.KB_ERR_UNSUPPORTED
