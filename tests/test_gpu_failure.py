"""Failure detection without a GPU fault: the kernels' bounded waits, the workspace error word
and kb_workspace_status.

Two ways to reach the error path, neither of which faults, traps or hangs a GPU:
  * a workspace whose error word is already set (as a wait that gave up leaves it): the call
    must do nothing but write offsets = -1, and the status must read back 1, until the
    workspace is zero-filled again;
  * kb_set_wait_limit(1): every later wait gives up after one poll, so the grid barriers of the
    multi-CTA maps kernel and the decode chain's logit all-gather give up on purpose; the call
    returns (bounded), the host reads the error word, and after a re-zero with the default
    limit the same call is correct again.
The tensor-core router GEMM (kb_router_gemm) is covered the same way: its mbarrier waits and
grid barriers give up under the one-poll limit, and a poisoned workspace makes it do nothing.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kolibri_b200 import _lib, ops
from kolibri_b200 import decode_chain as dc
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu

E, K = wl.NUM_EXPERTS, wl.TOP_K


def _router_maps_call(lib, logits, bias, outs, ws, T):
    ids, w, c, off, p2u, u2p = outs
    return lib.kb_router_maps(logits.data_ptr(), bias.data_ptr(), ids.data_ptr(), w.data_ptr(),
                              c.data_ptr(), off.data_ptr(), p2u.data_ptr(), u2p.data_ptr(),
                              ws.data_ptr(), ws.numel(), T, E, K, 0, _lib.KB_MAPS_AUTO,
                              torch.cuda.current_stream().cuda_stream)


def _outs(T, dev):
    return [torch.empty(T, K, dtype=torch.int32, device=dev), torch.empty(T, K, device=dev),
            torch.empty(E, dtype=torch.int32, device=dev),
            torch.full((E + 1,), 7, dtype=torch.int64, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev)]


def _check_maps(outs, logits, bias):
    rid, rw = orc.router_ref(logits.cpu(), bias.cpu())
    assert torch.equal(outs[0].cpu(), rid)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, E)
    np.testing.assert_array_equal(outs[3].cpu().numpy(), roff)
    np.testing.assert_array_equal(outs[4].cpu().numpy(), rp2u)
    np.testing.assert_array_equal(outs[5].cpu().numpy(), ru2p)


@pytest.mark.parametrize("T", [4096, 65536])
def test_poisoned_maps_workspace_reports_and_recovers(T):
    """Error word set before the call: offsets all -1, status 1; zero-filled: correct again."""
    dev = torch.device("cuda")
    lib = _lib.load()
    logits, bias = wl.router_inputs(T, seed=5)
    logits, bias = logits.to(dev), bias.to(dev)
    ws = torch.zeros(lib.kb_router_maps_workspace_bytes(T, E, K), dtype=torch.uint8, device=dev)
    ws[4:8] = torch.tensor([1, 0, 0, 0], dtype=torch.uint8)   # the error word (offset 4)
    outs = _outs(T, dev)
    assert _router_maps_call(lib, logits, bias, outs, ws, T) == 0
    assert ops.workspace_status(ws, _lib.KB_WS_MAPS) == _lib.KB_WS_TIMEOUT
    assert bool((outs[3] == -1).all())
    ws.zero_()
    assert ops.workspace_status(ws, _lib.KB_WS_MAPS) == _lib.KB_WS_CLEAN
    assert _router_maps_call(lib, logits, bias, outs, ws, T) == 0
    assert ops.workspace_status(ws, _lib.KB_WS_MAPS) == _lib.KB_WS_CLEAN
    _check_maps(outs, logits, bias)


def test_forced_timeout_maps_returns_and_is_reported():
    """A one-poll wait limit makes the multi-CTA kernel's waits give up: the call returns, the
    host sees the error (now or, for a call that happened to finish, never), later calls
    report offsets = -1, and a re-zeroed workspace with the default limit is correct."""
    dev = torch.device("cuda")
    lib = _lib.load()
    T = 65536
    logits, bias = wl.router_inputs(T, seed=6)
    logits, bias = logits.to(dev), bias.to(dev)
    ws = torch.zeros(lib.kb_router_maps_workspace_bytes(T, E, K), dtype=torch.uint8, device=dev)
    outs = _outs(T, dev)
    old = ops.set_wait_limit(1)
    try:
        assert _router_maps_call(lib, logits, bias, outs, ws, T) == 0
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(old)
    status = ops.workspace_status(ws, _lib.KB_WS_MAPS)
    assert status in (_lib.KB_WS_CLEAN, _lib.KB_WS_TIMEOUT)
    if status == _lib.KB_WS_TIMEOUT:
        outs[3].fill_(7)
        assert _router_maps_call(lib, logits, bias, outs, ws, T) == 0
        torch.cuda.synchronize()
        assert bool((outs[3] == -1).all())
    else:
        _check_maps(outs, logits, bias)
    ws.zero_()
    assert _router_maps_call(lib, logits, bias, outs, ws, T) == 0
    assert ops.workspace_status(ws, _lib.KB_WS_MAPS) == _lib.KB_WS_CLEAN
    _check_maps(outs, logits, bias)


def _chain(T=1, n_layers=3):
    dev = torch.device("cuda")
    layers = dc.make_layers(n_layers, dev)
    ch = dc.DecodeChain(T, layers, dev)
    return ch, layers


def test_poisoned_chain_workspace_reports_and_recovers():
    ch, layers = _chain()
    s = torch.cuda.current_stream()
    descs, ws = ch._mega_setup()
    ws[128:132] = torch.tensor([1, 0, 0, 0], dtype=torch.uint8, device=ws.device)  # error word
    ch.offsets.fill_(7)
    ch.run_mega(s)
    assert ops.workspace_status(ws, _lib.KB_WS_CHAIN) == _lib.KB_WS_TIMEOUT
    assert bool((ch.offsets == -1).all())
    ws.zero_()
    ch.run_mega(s)
    assert ops.workspace_status(ws, _lib.KB_WS_CHAIN) == _lib.KB_WS_CLEAN
    rid, _ = orc.router_ref(ch.logits.cpu(), layers[-1].gate_bias.cpu())
    assert torch.equal(ch.ids.cpu(), rid)


def test_forced_timeout_chain_returns_and_is_reported():
    """With a one-poll limit the logit all-gather (and the weight waits) give up: the launch
    returns, the error word reads 1, later calls write offsets = -1; re-zeroed with the default
    limit, the chain is correct again."""
    ch, layers = _chain(n_layers=5)
    s = torch.cuda.current_stream()
    _, ws = ch._mega_setup()
    old = ops.set_wait_limit(1)
    try:
        ch.run_mega(s)
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(old)
    status = ops.workspace_status(ws, _lib.KB_WS_CHAIN)
    assert status in (_lib.KB_WS_CLEAN, _lib.KB_WS_TIMEOUT)
    if status == _lib.KB_WS_TIMEOUT:
        ch.offsets.fill_(7)
        ch.run_mega(s)
        torch.cuda.synchronize()
        assert bool((ch.offsets == -1).all())
    ws.zero_()
    ch.run_mega(s)
    assert ops.workspace_status(ws, _lib.KB_WS_CHAIN) == _lib.KB_WS_CLEAN
    rid, _ = orc.router_ref(ch.logits.cpu(), layers[-1].gate_bias.cpu())
    assert torch.equal(ch.ids.cpu(), rid)


def test_misaligned_chain_weights_reported():
    """A layer descriptor whose gamma pointer is not 16-byte aligned: the kernel checks every
    descriptor before any bulk copy, reports status 2 and writes offsets = -1."""
    dev = torch.device("cuda")
    layers = dc.make_layers(2, dev)
    buf = torch.empty(wl.HIDDEN + 8, dtype=torch.bfloat16, device=dev)
    layers[1].g_pre_moe = buf[1:1 + wl.HIDDEN]          # 2-byte offset: misaligned
    ch = dc.DecodeChain(1, layers, dev)
    ch.offsets.fill_(7)
    ch.run_mega(torch.cuda.current_stream())
    _, ws = ch._mega_setup()
    assert ops.workspace_status(ws, _lib.KB_WS_CHAIN) == _lib.KB_WS_MISALIGNED
    assert bool((ch.offsets == -1).all())


def test_noalloc_status_clean_after_calls():
    dev = torch.device("cuda")
    logits, bias = wl.router_inputs(64, seed=9)
    ids, *_ = ops.router_maps(logits.to(dev), bias.to(dev))
    c = torch.empty(E, dtype=torch.int32, device=dev)
    off = torch.empty(E + 1, dtype=torch.int64, device=dev)
    p2u = torch.empty(64 * K, dtype=torch.int32, device=dev)
    ops.expert_maps_noalloc(ids, c, off, p2u)
    assert ops.workspace_status(None, _lib.KB_WS_NOALLOC, dev) == _lib.KB_WS_CLEAN


def _router_gemm_call(lib, x, w, b, ids, wt, ws, T):
    return lib.kb_router_gemm(x.data_ptr(), w.data_ptr(), b.data_ptr(), None, ids.data_ptr(),
                              wt.data_ptr(), ws.data_ptr(), ws.numel(), T, wl.HIDDEN, E, K, 0,
                              torch.cuda.current_stream().cuda_stream)


def _gate_inputs(T, dev):
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, wl.HIDDEN, generator=g).to(torch.bfloat16).to(dev)
    w = (0.02 * torch.randn(E, wl.HIDDEN, generator=g)).to(torch.bfloat16).to(dev)
    b = (0.1 * torch.randn(E, generator=g)).to(dev)
    return x, w, b


@pytest.mark.parametrize("T", [1, 256, 20000])
def test_router_gemm_poisoned_and_forced_timeout(T):
    dev = torch.device("cuda")
    lib = _lib.load()
    x, w, b = _gate_inputs(T, dev)
    ids = torch.full((T, K), -7, dtype=torch.int32, device=dev)
    wt = torch.empty(T, K, device=dev)
    ws = torch.zeros(lib.kb_router_gemm_workspace_bytes(T, wl.HIDDEN, E, K), dtype=torch.uint8,
                     device=dev)
    # a poisoned workspace: the call does no work and the status reports it
    ws[:4].view(torch.int32)[0] = _lib.KB_WS_TIMEOUT
    assert _router_gemm_call(lib, x, w, b, ids, wt, ws, T) == 0
    assert ops.workspace_status(ws, _lib.KB_WS_RGEMM) == _lib.KB_WS_TIMEOUT
    assert bool((ids == -7).all())
    # every wait gives up after one poll: the call returns and the host sees the error
    ws.zero_()
    old = ops.set_wait_limit(1)
    try:
        assert _router_gemm_call(lib, x, w, b, ids, wt, ws, T) == 0
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(old)
    assert ops.workspace_status(ws, _lib.KB_WS_RGEMM) in (_lib.KB_WS_CLEAN, _lib.KB_WS_TIMEOUT)
    # zero-filled again, with the default limit: correct
    ws.zero_()
    assert _router_gemm_call(lib, x, w, b, ids, wt, ws, T) == 0
    torch.cuda.synchronize()
    assert ops.workspace_status(ws, _lib.KB_WS_RGEMM) == _lib.KB_WS_CLEAN
    _, _, ref = orc.router_gemm_ref(x.cpu(), w.cpu(), b.cpu())
    rid, _ = orc.router_ref(ref, b.cpu())
    assert (ids.cpu() == rid).all(1).float().mean().item() > 0.98
