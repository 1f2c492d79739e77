"""Expert-parallel dispatch/combine over NCCL on two GPUs (skipped with fewer): with identity
experts, combine(dispatch(x)) equals, bit for bit, the one-GPU path finalize(expand(x)) of the
same routing; every received row belongs to the receiving rank's experts."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from kolibri_b200 import ops
        from kolibri_b200.ep import ExpertParallel
        from kolibri_b200 import workloads as wl
        T, E, K, H = 512, 384, 6, 6144
        g = torch.Generator().manual_seed(7 + rank)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
        logits, bias = wl.router_inputs(T, seed=20 + rank)
        logits, bias = logits.to(dev), bias.to(dev)
        ep = ExpertParallel(E, K)
        d = ep.dispatch(x, logits, bias)
        out = ep.combine(d, d.rows)
        ids, w, c, off, p2u, u2p = ops.router_maps(logits, bias)
        ref = ops.moe_finalize(ops.expand_rows(x, p2u), u2p, w)
        Er = E // world
        exp = d.meta[:, 0]
        owned = bool(((exp >= rank * Er) & (exp < (rank + 1) * Er)).all())
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(out, ref)) and owned and torch.equal(d.ids, ids),
               sum(d.recv_splits)))
    except Exception as e:
        q.put((rank, repr(e), 0))
    finally:
        dist.destroy_process_group()


def test_expert_parallel_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] is True for r in res), res
    assert sum(r[2] for r in res) == 2 * 512 * 6
