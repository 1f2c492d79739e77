"""The decode chain on the GPU: every stage of every layer checked against the CPU oracle on
the inputs that stage actually received (the router GEMM, on the tensor cores by default or on
cuBLAS, is checked to bf16 rounding; everything after it is checked on its GPU output), for
SWA and RNoPE layers, and the CUDA-graph replay checked against the eager run."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from kb_testutil import assert_bf16_close, assert_chain_close, np_of
from kolibri_b200 import decode_chain as dc
from kolibri_b200 import workloads as wl
from oracle import kolibri_oracle as orc

pytestmark = pytest.mark.gpu


def _cpu(t):
    return None if t is None else t.detach().cpu()


def make_checker(seen, layers_to_check=None):
    def check(i, stage, t):
        seen.append((i, stage))
        if layers_to_check is not None and i not in layers_to_check:
            return
        c = {k: _cpu(v) for k, v in t.items()}
        if stage in ("sandwich", "post_moe"):
            rs, rn = (orc.sandwich_ref if stage == "sandwich" else orc.post_moe_pre_attn_ref)(
                c["a"], c["residual"], c["g1"], c["g2"], eps=wl.EPS)
            inter = F.rms_norm(c["a"], (c["a"].shape[-1],), c["g1"], eps=wl.EPS)
            assert_chain_close(c["sum"], rs, inter, f"layer {i} {stage} sum")
            assert_chain_close(c["norm"], rn, inter, f"layer {i} {stage} norm")
        elif stage == "qk":
            rq, rk = orc.qk_norm_rope_ref(c["q"], c["k"], c["gq"], c["gk"], c["pos"], eps=wl.EPS)
            assert_bf16_close(c["q_out"], rq, f"layer {i} q")
            assert_bf16_close(c["k_out"], rk, f"layer {i} k")
        elif stage == "gate":
            ref = orc.router_logits_ref(c["x"].float(), c["w"].float())
            # the GEMM accumulates in another order; both round to bf16 before the cast.
            torch.testing.assert_close(c["logits"], ref, rtol=2.0 ** -7, atol=2e-3)
            assert torch.equal(c["logits"], c["logits"].to(torch.bfloat16).float())
        elif stage == "router_maps":
            rid, rw = orc.router_ref(c["logits"], c["bias"])
            assert torch.equal(c["ids"], rid), f"layer {i} ids"
            torch.testing.assert_close(c["w"], rw, rtol=1e-6, atol=0)
            rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, wl.NUM_EXPERTS)
            np.testing.assert_array_equal(np_of(c["counts"]), rc)
            np.testing.assert_array_equal(np_of(c["offsets"]), roff)
            np.testing.assert_array_equal(np_of(c["p2u"]), rp2u)
            np.testing.assert_array_equal(np_of(c["u2p"]), ru2p)
        elif stage == "expansion":
            assert torch.equal(c["permuted"], orc.expansion_ref(c["x"], np_of(c["p2u"])))
    return check


@pytest.mark.parametrize("T,gate", [(1, "tcgen05"), (3, "tcgen05"), (40, "tcgen05"),
                                    (40, "cublas")])
def test_chain_stages_match_oracle(T, gate):
    dev = torch.device("cuda")
    layers = dc.make_layers(5, dev)   # layer 4 is the RNoPE (full-attention) layer
    assert [L.rnope for L in layers] == [False, False, False, False, True]
    chain = dc.DecodeChain(T, layers, dev, gate=gate)
    seen = []
    chain.run_layers(torch.cuda.current_stream(), record=make_checker(seen))
    torch.cuda.synchronize()
    assert len(seen) == 5 * 6


@pytest.mark.parametrize("T", [256, 8192])
def test_chain_stages_benchmark_sizes(T):
    """The stage path at the benchmark's larger batches: every stage of the first and of the
    last layer (the RNoPE layer) checked against the oracle on the inputs it received."""
    dev = torch.device("cuda")
    layers = dc.make_layers(5, dev)
    chain = dc.DecodeChain(T, layers, dev)
    seen = []
    chain.run_layers(torch.cuda.current_stream(), record=make_checker(seen, {0, 4}))
    torch.cuda.synchronize()
    assert len(seen) == 5 * 6


def test_chain_graph_replay_matches_eager():
    dev = torch.device("cuda")
    layers = dc.make_layers(10, dev)
    chain = dc.DecodeChain(2, layers, dev)
    s = torch.cuda.Stream()
    chain.run_layers(s)
    torch.cuda.synchronize()
    eager = [chain.r.clone(), chain.nxt.clone(), chain.ids.clone(), chain.p2u.clone(),
             chain.permuted.clone()]
    g = chain.capture(s)
    chain.r.zero_()
    chain.ids.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, [chain.r, chain.nxt, chain.ids, chain.p2u, chain.permuted]):
        assert torch.equal(a, b)


def test_chain_without_gate_gemm():
    dev = torch.device("cuda")
    chain = dc.DecodeChain(4, dc.make_layers(5, dev), dev, gate_gemm=False, expansion=False)
    seen = []
    chain.run_layers(torch.cuda.current_stream(), record=make_checker(seen))
    torch.cuda.synchronize()
    assert len(seen) == 5 * 4
    assert chain.launches_per_layer() == 4


@pytest.mark.parametrize("T,n_layers", [(1, 5), (2, 5), (4, 5), (1, 50), (4, 50)])
def test_decode_chain_kernel_matches_stages(T, n_layers):
    """kb_decode_chain (one launch for all layers) against the stage-by-stage path, up to the
    benchmark's 50 layers: the routing-independent state is bit-identical, every layer's
    logits agree with cuBLAS to bf16 rounding and with the CPU oracle, and the last layer's
    router, maps and expansion match the oracle on the kernel's own logits."""
    dev = torch.device("cuda")
    layers = dc.make_layers(n_layers, dev)
    chain = dc.DecodeChain(T, layers, dev)
    s = torch.cuda.Stream()
    ref_logits = []

    def keep(i, stage, t):
        if stage == "gate":
            ref_logits.append((t["x"].detach().cpu(), t["logits"].detach().cpu()))
    chain.run_layers(s, record=keep)
    torch.cuda.synchronize()
    ref = {n: getattr(chain, n).clone() for n in ("r", "nxt", "h", "moe_in", "q_out", "k_out")}
    for n in ("r", "nxt", "h", "moe_in", "q_out", "k_out", "ids", "logits", "p2u"):
        getattr(chain, n).zero_()
    trace = torch.full((n_layers, T, wl.NUM_EXPERTS), float("nan"), device=dev)
    chain.run_mega(s, trace=trace)
    chain.run_mega(s)            # a second call on the same workspace
    torch.cuda.synchronize()
    for n, v in ref.items():
        assert torch.equal(getattr(chain, n), v), n
    tr = trace.cpu()
    for i, (x, lg) in enumerate(ref_logits):
        assert torch.equal(tr[i], tr[i].to(torch.bfloat16).float())
        torch.testing.assert_close(tr[i], lg, rtol=2.0 ** -7, atol=2e-3)
        ref_cpu = orc.router_logits_ref(x.float(), layers[i].w_gate_t.t().float().cpu())
        torch.testing.assert_close(tr[i], ref_cpu, rtol=2.0 ** -7, atol=2e-3)
    last = tr[-1]
    assert torch.equal(chain.logits.cpu(), last)
    rid, rw = orc.router_ref(last, layers[-1].gate_bias.cpu())
    assert torch.equal(chain.ids.cpu(), rid)
    torch.testing.assert_close(chain.w.cpu(), rw, rtol=1e-6, atol=0)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, wl.NUM_EXPERTS)
    np.testing.assert_array_equal(np_of(chain.counts), rc)
    np.testing.assert_array_equal(np_of(chain.offsets), roff)
    np.testing.assert_array_equal(np_of(chain.p2u), rp2u)
    np.testing.assert_array_equal(np_of(chain.u2p), ru2p)
    assert torch.equal(chain.permuted.cpu(), orc.expansion_ref(chain.moe_in.cpu(), rp2u))


def test_decode_chain_kernel_rejects_large_batches():
    dev = torch.device("cuda")
    chain = dc.DecodeChain(5, dc.make_layers(1, dev), dev)
    with pytest.raises(ValueError):
        chain.run_mega(torch.cuda.current_stream())


def _tied_layers(case, dev):
    """One layer whose router rows make the kernel's candidate filter meet ties, NaN and
    small expert counts: (E, K, layers)."""
    E, K = {"all_equal": (384, 6), "tie40": (384, 6), "tie20": (384, 8),
            "nan_inf": (384, 6), "e40": (40, 6), "e24": (24, 8), "e8": (8, 8)}[case]
    layers = dc.make_layers(1, dev, E=E)
    L = layers[0]
    g = torch.Generator(device="cpu").manual_seed(11)
    if case == "all_equal":        # every score equal: more than 32 candidates
        L.w_gate_t[:] = L.w_gate_t[0].clone()
        L.gate_bias.zero_()
    elif case in ("tie40", "tie20"):
        n = 40 if case == "tie40" else 20
        S = torch.randperm(E, generator=g)[:n].to(dev)
        L.w_gate_t[S] = L.w_gate_t[0].clone()
        L.gate_bias[S] = 10.0     # the tied set on top; tie40 overflows the 32 candidates
    elif case == "nan_inf":
        S = torch.randperm(E, generator=g)[:5].to(dev)
        L.gate_bias[S[:3]] = float("nan")
        L.gate_bias[S[3:]] = float("-inf")
    return E, K, layers


@pytest.mark.parametrize("case", ["all_equal", "tie40", "tie20", "nan_inf", "e40", "e24", "e8"])
@pytest.mark.parametrize("T", [1, 3])
def test_decode_chain_kernel_routing_ties_and_small_E(case, T):
    """kb_decode_chain's router on rows with tied scores (more and fewer than 32 keys at the
    threshold), NaN and -inf biases, and expert counts below 32 * K: ids, weights, maps and
    expansion against the oracle on the kernel's own logits."""
    dev = torch.device("cuda")
    E, K, layers = _tied_layers(case, dev)
    chain = dc.DecodeChain(T, layers, dev, E=E, K=K)
    s = torch.cuda.Stream()
    trace = torch.full((1, T, E), float("nan"), device=dev)
    chain.run_mega(s, trace=trace)
    torch.cuda.synchronize()
    last = trace[0].cpu()
    bias = layers[0].gate_bias.cpu()
    rid, rw = orc.router_ref(last, bias, k=K)
    assert torch.equal(chain.ids.cpu(), rid)
    torch.testing.assert_close(chain.w.cpu(), rw, rtol=1e-6, atol=0)
    rc, roff, rp2u, ru2p = orc.expert_maps_ref(rid, E)
    np.testing.assert_array_equal(np_of(chain.counts), rc)
    np.testing.assert_array_equal(np_of(chain.offsets), roff)
    np.testing.assert_array_equal(np_of(chain.p2u), rp2u)
    np.testing.assert_array_equal(np_of(chain.u2p), ru2p)
    assert torch.equal(chain.permuted.cpu(), orc.expansion_ref(chain.moe_in.cpu(), rp2u))
    if case == "all_equal":
        assert rid.tolist() == [list(range(K))] * T


@pytest.mark.parametrize("T", [1, 32, 256])
def test_chain_with_expert_parallel_exchange(T):
    """The token-sharded layer on one rank: the exchange stage's MoE output equals the one-GPU
    finalize(expand(moe_in)) of the layer's own routing bit for bit, every other stage matches
    the oracle, and the CUDA-graph replay equals the eager run."""
    from kolibri_b200 import ops
    from kolibri_b200.ep import PeerExpertParallel
    dev = torch.device("cuda")
    layers = dc.make_layers(5, dev)
    ep = PeerExpertParallel(wl.NUM_EXPERTS, wl.TOP_K, wl.HIDDEN, max_tokens=T, device=dev)
    try:
        chain = dc.DecodeChain(T, layers, dev, ep=ep)
        seen = []
        check = make_checker(seen)

        def rec(i, stage, t):
            if stage == "ep":
                seen.append((i, stage))
                ref = ops.moe_finalize(ops.expand_rows(t["x"], t["p2u"]), t["u2p"], t["w"])
                assert torch.equal(t["out"], ref), f"layer {i} exchange"
            else:
                check(i, stage, t)
        s = torch.cuda.Stream()
        chain.run_layers(s, record=rec)
        torch.cuda.synchronize()
        assert len(seen) == 5 * 6
        eager = [chain.r.clone(), chain.nxt.clone(), chain.moe_out_ep.clone()]
        g = chain.capture(s)
        chain.r.zero_()
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(eager, [chain.r, chain.nxt, chain.moe_out_ep]):
            assert torch.equal(a, b)
        assert ep.pg.status() == 0
        del g
    finally:
        ep.close()
