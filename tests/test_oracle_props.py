"""Oracle self-checks: the expert-map invariants of the reference's multi-block test
(kernels/cuda/multi_block_expert_maps/test_multi_block_build_expert_maps.py:31-73, same sizes
and seed) and the router's tie / special-value semantics."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kolibri_oracle as orc


def check_map_invariants(ids: np.ndarray, counts, offsets, p2u, u2p, E=384):
    T, k = ids.shape
    n = T * k
    flat = ids.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    nv = int(valid.sum())
    assert offsets[0] == 0 and offsets[-1] == nv
    assert np.all(np.diff(offsets) >= 0)
    np.testing.assert_array_equal(np.diff(offsets), np.bincount(flat[valid], minlength=E))
    np.testing.assert_array_equal(counts, np.diff(offsets))
    np.testing.assert_array_equal(np.sort(p2u[:nv]), np.sort((np.nonzero(valid)[0] % k) * T
                                                             + np.nonzero(valid)[0] // k))
    assert np.all(p2u[nv:] == -1)
    np.testing.assert_array_equal(u2p[p2u[:nv]], np.arange(nv))
    tok, slot = p2u[:nv] % T, p2u[:nv] // T
    np.testing.assert_array_equal(ids[tok, slot], np.repeat(np.arange(E), np.diff(offsets)))
    # stable order inside every expert
    e_of = np.repeat(np.arange(E), np.diff(offsets))
    key = e_of.astype(np.int64) * n + tok * k + slot
    assert np.all(np.diff(key) > 0)


@pytest.mark.parametrize("T", [16, 64, 512, 1152, 98304])
def test_maps_invariants_reference_sizes(T):
    torch.manual_seed(42)
    ids = torch.randint(0, 384, (T, 6), dtype=torch.int32).numpy()
    check_map_invariants(ids, *orc.expert_maps_ref(ids, 384))


def test_maps_edge_cases():
    # all tokens on one expert, invalid ids skipped, empty input
    ids = np.full((33, 6), 7, dtype=np.int32)
    check_map_invariants(ids, *orc.expert_maps_ref(ids, 384))
    ids = np.random.default_rng(0).integers(-3, 390, size=(50, 6)).astype(np.int32)
    c, off, p2u, u2p = orc.expert_maps_ref(ids, 384)
    check_map_invariants(ids, c, off, p2u, u2p)
    bad = ((ids < 0) | (ids >= 384))
    tok, slot = np.nonzero(bad)
    assert np.all(u2p[slot * 50 + tok] == -1)
    c, off, p2u, u2p = orc.expert_maps_ref(np.zeros((0, 6), np.int32), 384)
    assert off.shape == (385,) and np.all(off == 0) and p2u.size == 0


def test_router_ties_and_special_values():
    z = torch.zeros(2, 384)
    ids, w = orc.router_ref(z, torch.zeros(384), k=6)
    assert ids.tolist() == [[0, 1, 2, 3, 4, 5]] * 2
    # -0 and +0 tie: the lower index wins
    x = torch.zeros(1, 384)
    x[0, ::2] = -0.0
    ids, _ = orc.router_ref(x, None, k=6)
    assert ids.tolist() == [[0, 1, 2, 3, 4, 5]]
    # NaN ranks first, then +inf
    x = torch.randn(1, 384)
    x[0, 100] = float("nan")
    x[0, 7] = float("inf")
    x[0, 300] = float("nan")
    ids, _ = orc.router_ref(x, None, k=6)
    assert ids[0, :3].tolist() == [100, 300, 7]
    # weight is sigmoid of the raw (un-biased) logit
    x = torch.randn(4, 384)
    b = torch.randn(384)
    ids, w = orc.router_ref(x, b, k=6)
    torch.testing.assert_close(w, torch.sigmoid(torch.gather(x, 1, ids.long())), rtol=0, atol=0)
    # renorm sums to one
    _, wn = orc.router_ref(x, b, k=6, renorm=True)
    torch.testing.assert_close(wn.sum(-1), torch.ones(4), rtol=1e-6, atol=1e-6)


def test_router_gemm_oracle_matches_the_reference_formula():
    """router_gemm_ref rounds the exact (fp64) product once to bf16; the reference's eager
    `(x @ W_g).float()` (router_logits_ref, a bf16 matmul on the CPU) accumulates in fp32 and
    rounds once too.  They agree within one bf16 ulp everywhere and exactly almost everywhere,
    and the routing of the oracle is router_ref on its own logits."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 1024, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(384, 1024, generator=g)).to(torch.bfloat16)
    b = 0.1 * torch.randn(384, generator=g)
    ids, wt, lg = orc.router_gemm_ref(x, w, b)
    ref = orc.router_logits_ref(x, w.t())
    torch.testing.assert_close(lg, ref, rtol=2 ** -7, atol=1e-4)
    assert (lg == ref).float().mean().item() > 0.99
    rid, rw = orc.router_ref(lg, b)
    assert torch.equal(ids, rid) and torch.equal(wt, rw)
