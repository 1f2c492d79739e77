"""Expert maps, fused router+maps, activation expansion and the prologue API on the GPU:
bit-exact against the CPU oracle (counts, offsets, p2u, u2p; (expert, token, slot) order)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from kb_testutil import np_of
from kolibri_b200 import _lib, ops
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu

MODES = [ops.KB_MAPS_AUTO, ops.KB_MAPS_SINGLE_CTA, ops.KB_MAPS_MULTI_CTA, ops.KB_MAPS_TWO_KERNEL]


def check_maps(ids_cpu, got, E=384):
    c, off, p2u, u2p = got
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(ids_cpu, E)
    if c is not None:
        np.testing.assert_array_equal(np_of(c), rc)
    np.testing.assert_array_equal(np_of(off), roff)
    np.testing.assert_array_equal(np_of(p2u), rp2u)
    if u2p is not None:
        np.testing.assert_array_equal(np_of(u2p), ru2p)


def ids_config1(T):
    logits, bias = wl.router_inputs(T, seed=1)
    return orc.router_ref(logits, bias)[0]


@pytest.mark.parametrize("T", [1, 64, 4096, 65536])
@pytest.mark.parametrize("mode", MODES)
def test_maps_config1(T, mode):
    ids = ids_config1(T)
    if mode == ops.KB_MAPS_SINGLE_CTA and T * 6 > 12288:
        with pytest.raises(Exception):
            ops.expert_maps(ids.cuda(), 384, mode=mode)
        return
    check_maps(ids, ops.expert_maps(ids.cuda(), 384, mode=mode))


@pytest.mark.parametrize("T", [1, 64, 4096])
def test_maps_golden_offsets(T):
    g = np.load(GOLDEN / f"maps_c1_T{T}.npz")
    ids = torch.from_numpy(g["ids"]).cuda()
    _, off, p2u, _ = ops.expert_maps(ids, 384)
    np.testing.assert_array_equal(np_of(off), g["offsets"])
    o = g["offsets"]
    ref = g["p2u_expert_slot_token"]
    got = np_of(p2u)
    for e in range(384):
        assert set(got[o[e]:o[e + 1]].tolist()) == set(ref[o[e]:o[e + 1]].tolist())


@pytest.mark.parametrize("T", [16, 64, 512, 1152, 98304])
def test_maps_reference_invariant_sizes(T):
    torch.manual_seed(42)
    ids = torch.randint(0, 384, (T, 6), dtype=torch.int32)
    for mode in (ops.KB_MAPS_AUTO, ops.KB_MAPS_MULTI_CTA, ops.KB_MAPS_TWO_KERNEL):
        check_maps(ids, ops.expert_maps(ids.cuda(), 384, mode=mode))


def test_maps_edge_cases():
    one = torch.full((5000, 6), 7, dtype=torch.int32)
    for mode in (ops.KB_MAPS_AUTO, ops.KB_MAPS_MULTI_CTA, ops.KB_MAPS_TWO_KERNEL):
        check_maps(one, ops.expert_maps(one.cuda(), 384, mode=mode))
    bad = torch.from_numpy(np.random.default_rng(0).integers(-3, 390, size=(700, 6)).astype(np.int32))
    for mode in MODES:
        check_maps(bad, ops.expert_maps(bad.cuda(), 384, mode=mode))
    empty = torch.zeros((0, 6), dtype=torch.int32)
    c, off, p2u, u2p = ops.expert_maps(empty.cuda(), 384)
    assert np.all(np_of(off) == 0) and np.all(np_of(c) == 0) and p2u.numel() == 0
    # other E and k
    g = torch.Generator().manual_seed(1)
    for E, k in ((256, 6), (512, 8), (100, 3), (384, 1), (384, 32)):
        ids = torch.randint(0, E, (999, k), generator=g, dtype=torch.int32)
        for mode in MODES:
            if mode == ops.KB_MAPS_SINGLE_CTA and ids.numel() > 12288:
                continue  # the single-CTA path holds at most 12288 selections
            check_maps(ids, ops.expert_maps(ids.cuda(), E, mode=mode), E)


def test_maps_repeated_calls_reuse_workspace():
    # The arrival counters must reset themselves: alternate sizes many times.
    for i in range(6):
        T = (70000, 3000, 513)[i % 3]
        ids = torch.randint(0, 384, (T, 6), dtype=torch.int32)
        for mode in (ops.KB_MAPS_MULTI_CTA, ops.KB_MAPS_TWO_KERNEL):
            check_maps(ids, ops.expert_maps(ids.cuda(), 384, mode=mode))


def test_maps_workspace_shared_across_paths_and_experts():
    # One workspace buffer serves every path, T, E and K in turn: what a call leaves in it
    # must never leak into the next one (zero zone restored, scratch rewritten).
    g = torch.Generator().manual_seed(3)
    cases = [(70000, 384, 6, ops.KB_MAPS_MULTI_CTA), (513, 512, 8, ops.KB_MAPS_TWO_KERNEL),
             (3000, 128, 6, ops.KB_MAPS_MULTI_CTA), (70000, 384, 32, ops.KB_MAPS_TWO_KERNEL),
             (1, 384, 6, ops.KB_MAPS_MULTI_CTA), (40000, 512, 6, ops.KB_MAPS_MULTI_CTA),
             (700, 100, 3, ops.KB_MAPS_MULTI_CTA), (70000, 384, 6, ops.KB_MAPS_MULTI_CTA)]
    for T, E, k, mode in cases:
        ids = torch.randint(0, E, (T, k), generator=g, dtype=torch.int32)
        check_maps(ids, ops.expert_maps(ids.cuda(), E, mode=mode), E)
        logits = torch.randn(min(T, 5000), E, generator=g)
        ids_r, _, c, off, p2u, u2p = ops.router_maps(logits.cuda(), None, k=min(k, 8), mode=mode)
        check_maps(ids_r.cpu(), (c, off, p2u, u2p), E)


@pytest.mark.parametrize("T", [1, 32, 33, 256, 4096, 65536])
@pytest.mark.parametrize("mode", MODES)
def test_router_maps_fused(T, mode):
    logits, bias = wl.router_inputs(T, seed=1)
    if mode == ops.KB_MAPS_SINGLE_CTA and T * 6 > 12288:
        return
    for renorm in (False, True):
        ids, w, c, off, p2u, u2p = ops.router_maps(logits.cuda(), bias.cuda(), renorm=renorm,
                                                   mode=mode)
        rid, rw = orc.router_ref(logits, bias, renorm=renorm)
        assert torch.equal(ids.cpu(), rid)
        torch.testing.assert_close(w.cpu(), rw, rtol=1e-6, atol=0)
        check_maps(rid, (c, off, p2u, u2p))


@pytest.mark.parametrize("E,k", [(384, 6), (256, 8), (128, 6), (512, 6)])
@pytest.mark.parametrize("T", [33, 4096, 65536])
@pytest.mark.parametrize("mode", [ops.KB_MAPS_HYBRID_ROUTER, ops.KB_MAPS_WARP_ROUTER])
def test_router_maps_forced_fallback_paths(mode, T, E, k):
    """The routing paths AUTO takes only when the tile kernel does not apply, forced: the
    hybrid-router and the warp-per-token-router persistent kernels, bit-exact against the
    oracle (ids, maps) and within 1e-6 (weights), the path confirmed by kb_maps_describe."""
    import ctypes
    path = ctypes.c_int(-1)
    _lib.check(_lib.load().kb_maps_describe(T, E, k, 1, mode, ctypes.byref(path), None, None),
               "kb_maps_describe")
    assert path.value in (mode, ops.KB_MAPS_WARP_ROUTER, ops.KB_MAPS_TWO_KERNEL)
    if mode == ops.KB_MAPS_HYBRID_ROUTER and E in (128, 256, 384, 512):
        assert path.value == ops.KB_MAPS_HYBRID_ROUTER
    logits, bias = wl.router_inputs(T, seed=3, E=E)
    ids, w, c, off, p2u, u2p = ops.router_maps(logits.cuda(), bias.cuda(), k=k, mode=mode)
    rid, rw = orc.router_ref(logits, bias, k=k)
    assert torch.equal(ids.cpu(), rid)
    torch.testing.assert_close(w.cpu(), rw, rtol=1e-6, atol=0)
    check_maps(rid, (c, off, p2u, u2p), E)


def test_expansion_and_prologue(api):
    T, H = 300, 6144
    g = torch.Generator().manual_seed(11)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits, bias = wl.router_inputs(T, seed=12)
    xc = x.cuda()
    out = api.fused_moe_prologue(xc, logits.cuda(), bias.cuda())
    permuted, w, ids, off, p2u, u2p = out
    rid, rw = orc.router_ref(logits, bias)
    assert torch.equal(ids.cpu(), rid)
    torch.testing.assert_close(w.cpu(), rw, rtol=1e-6, atol=0)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, 384)
    np.testing.assert_array_equal(np_of(off), roff)
    np.testing.assert_array_equal(np_of(p2u), rp2u)
    np.testing.assert_array_equal(np_of(u2p), ru2p)
    assert torch.equal(permuted.cpu(), orc.expansion_ref(x, rp2u))
    # reference prologue invariants A-D (fusions/03_moe_prologue/benchmark_and_verify.py:66-86)
    _, wn, *_ = api.fused_moe_prologue(xc, logits.cuda(), bias.cuda(), norm_topk_prob=True)
    assert (wn.sum(-1) - 1).abs().max().item() < 1e-4
    # stand-alone expansion on other dtypes / row sizes
    for dt, h in ((torch.float16, 2560), (torch.bfloat16, 6144), (torch.float32, 7)):
        xx = torch.randn(50, h, generator=g).to(dt)
        pp = torch.from_numpy(orc.expert_maps_ref(torch.randint(0, 384, (50, 6), generator=g), 384)[2])
        got = ops.expand_rows(xx.cuda(), pp.cuda())
        assert torch.equal(got.cpu(), orc.expansion_ref(xx, pp.numpy()))


def test_reference_map_entry_points(api):
    ids = torch.randint(0, 384, (1152, 6), dtype=torch.int32)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(ids, 384)
    idc = ids.cuda()
    for fn in (lambda: api.kolibri_build_expert_maps(idc, 384),
               lambda: api.trtllm_build_expert_maps_b32(idc, 384),
               lambda: api.kolibri_multi_block_build_expert_maps(idc, 384, max_blocks=128),
               lambda: api.kolibri_multi_block_build_expert_maps(idc, 384, max_blocks=-64),
               lambda: api.kolibri_dispatch_map(idc, 384),
               lambda: api.kolibri_dispatch_map(idc, 384, force_multi_block=True)):
        p2u, u2p, off = fn()
        assert off.dtype == torch.int64 and off.numel() == 385
        np.testing.assert_array_equal(np_of(off), roff)
        np.testing.assert_array_equal(np_of(p2u), rp2u)
        np.testing.assert_array_equal(np_of(u2p), ru2p)
    p2u, u2p, off = api.kolibri_multi_block_build_expert_maps(idc, 384, return_inverse_map=False)
    assert u2p.numel() == 0
    small = ids[:40].contiguous()
    p2u, u2p, off = api.kolibri_dispatch_map(small.cuda(), 384, force_single_block=True)
    np.testing.assert_array_equal(np_of(p2u), orc.expert_maps_ref(small, 384)[2])


@pytest.mark.parametrize("T", [1, 40, 4096])
def test_router_dispatch_entry_point(T, api):
    # kernels/cuda/kolibri_router_dispatch.py:49-64: (permuted rows, permuted scales, p2u, offsets)
    g = torch.Generator().manual_seed(T)
    x = torch.randn(T, 2048, generator=g).to(torch.bfloat16)
    logits, bias = wl.router_inputs(T, seed=5)
    out, scales, p2u, off = api.fused_kolibri_router_dispatch(x.cuda(), logits.cuda(), bias.cuda())
    rid, rw = orc.router_ref(logits, bias)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, 384)
    np.testing.assert_array_equal(np_of(off), roff)
    np.testing.assert_array_equal(np_of(p2u), rp2u)
    assert torch.equal(out.cpu(), orc.expansion_ref(x, rp2u))
    src = torch.from_numpy(rp2u).long()
    ref_scales = rw.reshape(-1)[(src % T) * 6 + src // T]
    torch.testing.assert_close(scales.cpu(), ref_scales, rtol=1e-6, atol=0)
    with pytest.raises(RuntimeError, match="384 experts"):
        api.fused_kolibri_router_dispatch(x.cuda(), logits[:, :256].contiguous().cuda(),
                                          bias[:256].contiguous().cuda())


def _adversarial_logits(E, T=320, seed=0):
    """Rows that stress the candidate pass: NaN / inf / -0 rows, displaced ties, the top
    picks packed into one 16-expert group, and coarse integer logits (ties everywhere)."""
    g = torch.Generator().manual_seed(seed + E)
    x = torch.randn(T, E, generator=g)
    x[0, E // 3] = float("nan")
    x[0, 7] = float("inf")
    x[1, :] = -float("inf")
    x[2, ::3] = float("nan")
    x[3, :] = 0.0
    x[3, ::2] = -0.0
    x[4, E // 2:] = float("inf")
    for r in range(16, 80):                      # equal low-index scores displaced later
        x[r] = 0.0
        x[r, :40] = 3.0
        x[r, 60 + r % (E - 70)] = 5.0 + (r % 3)
        x[r, E - 1 - r % 8] = 4.0
    for r in range(80, 144):                     # up to 12 winners inside one group
        grp = r % (E // 16)
        x[r] = torch.randn(E, generator=g) - 10.0
        n = 1 + r % 12
        x[r, grp * 16: grp * 16 + n] = 10.0 + torch.arange(n).float()
    x[144:] = torch.randint(-3, 4, (T - 144, E), generator=g).float()
    return x


@pytest.mark.parametrize("E", [128, 256, 384])
@pytest.mark.parametrize("k", [6, 8])
def test_router_maps_adversarial_rows(E, k):
    x = _adversarial_logits(E)
    g = torch.Generator().manual_seed(E + k)
    biases = [None, torch.randint(-1, 2, (E,), generator=g).float()]
    biases[1][::5] = -0.0
    for bias in biases:
        rid, rw = orc.router_ref(x, bias, k=k)
        rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, E)
        for mode in (ops.KB_MAPS_AUTO, ops.KB_MAPS_MULTI_CTA):
            ids, w, c, off, p2u, u2p = ops.router_maps(
                x.cuda(), None if bias is None else bias.cuda(), k=k, mode=mode)
            assert torch.equal(ids.cpu(), rid), \
                f"rows {torch.nonzero((ids.cpu() != rid).any(1))[:8].flatten().tolist()}"
            torch.testing.assert_close(w.cpu(), rw, rtol=1e-6, atol=0, equal_nan=True)
            check_maps(rid, (c, off, p2u, u2p), E)


def test_router_maps_tile_path_tails():
    # Token counts around the 32-row tile and CTA boundaries of the multi-CTA path.
    for T in (32, 33, 63, 65, 4736, 4767, 148 * 32 * 3 + 5):
        logits, bias = wl.router_inputs(T, seed=T)
        ids, w, c, off, p2u, u2p = ops.router_maps(logits.cuda(), bias.cuda(),
                                                   mode=ops.KB_MAPS_MULTI_CTA)
        rid, rw = orc.router_ref(logits, bias)
        assert torch.equal(ids.cpu(), rid), T
        torch.testing.assert_close(w.cpu(), rw, rtol=1e-6, atol=0)
        check_maps(rid, (c, off, p2u, u2p))


@pytest.mark.parametrize("T", [800, 4096, 65536])
@pytest.mark.parametrize("E", [128, 256, 384, 512])
def test_maps_ids_paths(T, E):
    """Maps from ids above the single-CTA size: the tile map phases (AUTO, MULTI_CTA; E in
    {128, 256, 384}) and the warp-per-token persistent kernel's map phases (forced with
    KB_MAPS_WARP_ROUTER), on routed ids (distinct experts per token), on ids that repeat an
    expert inside a token and on ids outside [0, E)."""
    g = torch.Generator().manual_seed(T + E)
    scores = torch.rand(T, E, generator=g)
    routed = torch.topk(scores, 6, dim=-1).indices.to(torch.int32)
    dups = routed.clone()
    dups[::7, 1] = dups[::7, 0]                  # one expert twice in every 7th token
    bad = routed.clone()
    bad[::5, 2] = -1
    bad[::9, 4] = E + 3
    for ids in (routed, dups, bad):
        for mode in (ops.KB_MAPS_AUTO, ops.KB_MAPS_MULTI_CTA, ops.KB_MAPS_WARP_ROUTER):
            check_maps(ids, ops.expert_maps(ids.cuda(), E, mode=mode), E)
