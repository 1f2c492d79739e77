"""Expert-parallel dispatch/combine (kolibri_b200.ep) on two CPU ranks over gloo: the exchange
logic (splits from the all-gathered counts, the row and metadata all-to-alls, the grouping
by local expert and the way back) with the four local operations done by the CPU oracle.
The identity experts make combine(dispatch(x)) = sum_k w[t, k] * x[t] exactly in fp32."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import kolibri_oracle as orc


class OracleOps:
    """CPU restatements of the four local operations (test infrastructure)."""

    def __init__(self, E):
        self.E = E

    def router_maps(self, logits, bias, k):
        ids, w = orc.router_ref(logits, bias, k=k)
        c, off, p2u, u2p = orc.expert_maps_ref(ids, self.E)
        return (ids, w, torch.from_numpy(c).int(), torch.from_numpy(off).long(),
                torch.from_numpy(p2u).int(), torch.from_numpy(u2p).int())

    def expert_maps(self, ids, n):
        c, off, p2u, u2p = orc.expert_maps_ref(ids, n)
        return (torch.from_numpy(c).int(), torch.from_numpy(off).long(),
                torch.from_numpy(p2u).int(), torch.from_numpy(u2p).int())

    def expand_rows(self, x, p2u):
        return orc.expansion_ref(x, np.asarray(p2u))

    def finalize(self, rows, u2p, w):
        return orc.finalize_ref(rows, u2p, w)


def _worker(rank, world, port, T, E, K, H, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kolibri_b200.ep import ExpertParallel
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(T, H, generator=g)
        logits = torch.randn(T, E, generator=g)
        bias = 0.1 * torch.randn(E, generator=g)
        ep = ExpertParallel(E, K, local_ops=OracleOps(E))
        d = ep.dispatch(x, logits, bias)
        Er = E // world
        # every received row belongs to this rank's experts, grouped by expert
        exp = d.meta[:, 0]
        assert bool(((exp >= rank * Er) & (exp < (rank + 1) * Er)).all())
        grouped_exp = exp[d.group_p2u.long()] - rank * Er
        assert bool((grouped_exp[1:] >= grouped_exp[:-1]).all())
        assert torch.equal(torch.bincount(grouped_exp.long(), minlength=Er).cumsum(0),
                           d.expert_offsets[1:])
        # the closed-form placement of the peer-memory kernels reproduces the grouping
        ids_l, _, counts, _, p2u, _ = OracleOps(E).router_maps(logits, bias, K)
        permuted = orc.expansion_ref(x, np.asarray(p2u))
        all_counts = [torch.empty_like(counts) for _ in range(world)]
        dist.all_gather(all_counts, counts)
        all_perm = [torch.empty_like(permuted) for _ in range(world)]
        dist.all_gather(all_perm, permuted)
        grouped, dest = orc.ep_placement_ref(torch.stack(all_counts).numpy(), world)
        assert len(grouped[rank]) == d.rows.shape[0]
        for gpos, (sender, i) in enumerate(grouped[rank]):
            assert torch.equal(d.rows[gpos], all_perm[sender][i])
            assert dest[sender][i] == (rank, gpos)
        out = ep.combine(d, d.rows)           # identity experts
        ids, w = orc.router_ref(logits, bias, k=K)
        ref = x * w.sum(-1, keepdim=True)
        assert torch.equal(d.ids, ids)
        torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
        q.put((rank, "ok", sum(d.recv_splits)))
    except Exception as e:  # report to the parent, then leave the group cleanly
        q.put((rank, repr(e), 0))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_expert_parallel_dispatch_combine_gloo_2_ranks():
    world, T, E, K, H = 2, 64, 16, 4, 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, E, K, H, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] == "ok" for r in res), res
    assert sum(r[2] for r in res) == world * T * K  # every routed row reached its owner
