"""kb_expert_maps_noalloc: expert maps whose workspace is the library's static device
scratch.  Collected last (file name) so that it runs both alone and after every other test;
the GPU cases compare it bit for bit with kb_expert_maps on two calls in a row."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kolibri_b200 import _lib, ops
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

MAX_TOKENS = 1 << 19
SCRATCH_BYTES = 8 << 20


def test_noalloc_host_validation_without_gpu():
    lib = _lib.load()
    dummy = 256  # never dereferenced: every case below is rejected before any launch
    call = lib.kb_expert_maps_noalloc
    assert call(dummy, dummy, dummy, dummy, dummy, MAX_TOKENS + 1, 384, 6, 0, None) == \
        _lib.KB_ERR_SCRATCH_LIMIT
    assert call(dummy, dummy, dummy, dummy, dummy, 64, 384, 6, 2, None) == _lib.KB_ERR_INVALID_ARG
    assert call(dummy, dummy, None, dummy, dummy, 64, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert call(None, dummy, dummy, dummy, dummy, 64, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert call(dummy, dummy, dummy, dummy, dummy, 64, 384, 33, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert b"static scratch" in lib.kb_status_str(_lib.KB_ERR_SCRATCH_LIMIT)


@pytest.mark.parametrize("E,k", [(384, 6), (512, 32), (512, 1), (256, 8), (100, 3)])
def test_noalloc_limit_covers_max_tokens(E, k):
    # The stated limit: at T = 524288 every workspace the maps paths need fits the scratch.
    assert 0 < _lib.load().kb_expert_maps_workspace_bytes(MAX_TOKENS, E, k) <= SCRATCH_BYTES


def _outputs(T, E, k, dev):
    return (torch.full((E,), -7, dtype=torch.int32, device=dev),
            torch.full((E + 1,), -7, dtype=torch.int64, device=dev),
            torch.full((T * k,), -7, dtype=torch.int32, device=dev),
            torch.full((T * k,), -7, dtype=torch.int32, device=dev))


def _same(a, b):
    for x, y in zip(a, b):
        assert torch.equal(x.cpu(), y.cpu())


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,k", [(1, 384, 6), (700, 384, 6), (4096, 384, 6), (65536, 384, 6),
                                   (3000, 512, 8), (999, 100, 3)])
def test_noalloc_matches_expert_maps_twice(T, E, k):
    dev = torch.device("cuda")
    if E == 384 and k == 6:
        ids = orc.router_ref(*wl.router_inputs(T, seed=1))[0].to(dev)
    else:
        g = torch.Generator().manual_seed(T + E)
        ids = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32).to(dev)
    ref = ops.expert_maps(ids, E)
    first, second = _outputs(T, E, k, dev), _outputs(T, E, k, dev)
    ops.expert_maps_noalloc(ids, *first, num_experts=E)
    ops.expert_maps_noalloc(ids, *second, num_experts=E)
    torch.cuda.synchronize()
    _same(ref, first)
    _same(ref, second)


@pytest.mark.gpu
def test_noalloc_allocates_no_device_memory():
    dev = torch.device("cuda")
    T, E, k = 65536, 384, 6
    ids = orc.router_ref(*wl.router_inputs(T, seed=1))[0].to(dev)
    outs = [_outputs(T, E, k, dev) for _ in range(3)]
    ops.expert_maps_noalloc(ids, *outs[0], num_experts=E)  # set-up and module load
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    ops.expert_maps_noalloc(ids, *outs[1], num_experts=E)
    ops.expert_maps_noalloc(ids, *outs[2], num_experts=E)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0
    _same(outs[0], outs[1])
    _same(outs[0], outs[2])


@pytest.mark.gpu
def test_noalloc_rezero_empty_and_interleaved():
    dev = torch.device("cuda")
    # T = 0: set-up only; offsets and counts come back zero.
    c, off, p2u, u2p = _outputs(0, 384, 6, dev)
    ids0 = torch.zeros((0, 6), dtype=torch.int32, device=dev)
    ops.expert_maps_noalloc(ids0, c, off, p2u, u2p)
    assert int(off.abs().sum()) == 0 and int(c.abs().sum()) == 0
    # Alternate sizes (the scratch counters must reset themselves), with one re-zero.
    for i, T in enumerate((70000, 513, 3000, 70000)):
        ids = torch.randint(0, 384, (T, 6), dtype=torch.int32, device=dev)
        got = _outputs(T, 384, 6, dev)
        ops.expert_maps_noalloc(ids, *got, rezero=(i == 2))
        rc, roff, rp2u, ru2p = orc.expert_maps_ref(ids.cpu(), 384)
        np.testing.assert_array_equal(got[0].cpu().numpy(), rc)
        np.testing.assert_array_equal(got[1].cpu().numpy(), roff)
        np.testing.assert_array_equal(got[2].cpu().numpy(), rp2u)
        np.testing.assert_array_equal(got[3].cpu().numpy(), ru2p)
