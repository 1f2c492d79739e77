"""The expert-parallel exchange on peer memory (kb_ep_counts_allgather, kb_ep_dispatch,
kb_ep_combine) against the one-GPU path and against the collective exchange
(ExpertParallel over NCCL):

  * one rank (no process group): the received rows are the expansion of x by the maps,
    segments = the expert offsets, and combine(dispatch(x)) with identity experts equals
    finalize(expand(x)) bit for bit, over several calls (epochs) and inside a CUDA graph;
  * two GPUs (skipped with fewer): rows, segments and combine output bit-identical to
    ExpertParallel's, and combine(dispatch(x)) = finalize(expand(x)) of each rank's routing,
    with a different token count on each rank and an empty rank; the fused router + maps +
    count all-gather against NCCL's all-gather of the same counts.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H = 384, 6, 6144


def _inputs(T, seed, dev):
    from kolibri_b200 import workloads as wl
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    logits, bias = wl.router_inputs(T, seed=seed + 1)
    return x, logits.to(dev), bias.to(dev)


def _one_gpu_reference(x, logits, bias):
    from kolibri_b200 import ops
    ids, w, counts, offsets, p2u, u2p = ops.router_maps(logits, bias, k=K)
    permuted = ops.expand_rows(x, p2u)
    return counts, offsets, permuted, ops.moe_finalize(permuted, u2p, w)


@pytest.mark.parametrize("T", [1, 4, 100, 2048])
def test_single_rank_exchange_matches_local_path(T):
    from kolibri_b200.ep import PeerExpertParallel
    dev = torch.device("cuda")
    ep = PeerExpertParallel(E, K, H, max_tokens=2048, device=dev)
    try:
        for call in range(3):                      # successive epochs on one buffer
            x, logits, bias = _inputs(T, 10 * call + T, dev)
            d = ep.dispatch(x, logits, bias)
            out = ep.combine(d, d.rows)
            counts, offsets, permuted, ref = _one_gpu_reference(x, logits, bias)
            torch.cuda.synchronize()
            assert torch.equal(d.gathered[0], counts)
            assert torch.equal(d.expert_offsets, offsets)
            R = d.num_rows()
            assert R == T * K
            assert torch.equal(d.rows[:R], permuted)
            assert torch.equal(out, ref)
        assert ep.pg.status() == 0
    finally:
        ep.close()


@pytest.mark.parametrize("E_,K_,H_,dtype", [(256, 8, 4096, torch.bfloat16),
                                             (128, 4, 2048, torch.float32),
                                             (384, 6, 6144, torch.float16)])
def test_single_rank_exchange_other_shapes(E_, K_, H_, dtype):
    """Other expert counts, top-K, widths and dtypes: rows = the expansion, combine output =
    the one-GPU finalize, bit for bit."""
    from kolibri_b200 import ops
    from kolibri_b200.ep import PeerExpertParallel
    dev = torch.device("cuda")
    T = 300
    ep = PeerExpertParallel(E_, K_, H_, dtype=dtype, max_tokens=T, device=dev)
    try:
        g = torch.Generator().manual_seed(17)
        x = torch.randn(T, H_, generator=g).to(dtype).to(dev)
        logits = torch.randn(T, E_, generator=g).to(dev)
        bias = (0.1 * torch.randn(E_, generator=g)).to(dev)
        d = ep.dispatch(x, logits, bias)
        out = ep.combine(d, d.rows)
        ids, w, counts, offsets, p2u, u2p = ops.router_maps(logits, bias, k=K_)
        permuted = ops.expand_rows(x, p2u)
        ref = ops.moe_finalize(permuted, u2p, w)
        torch.cuda.synchronize()
        R = d.num_rows()
        assert R == T * K_
        assert torch.equal(d.expert_offsets, offsets)
        assert torch.equal(d.rows[:R], permuted)
        assert torch.equal(out, ref)
        assert ep.pg.status() == 0
    finally:
        ep.close()


def test_single_rank_exchange_in_cuda_graph():
    from kolibri_b200.ep import PeerExpertParallel
    from kolibri_b200 import ops
    dev = torch.device("cuda")
    T = 256
    ep = PeerExpertParallel(E, K, H, max_tokens=T, device=dev)
    try:
        x, logits, bias = _inputs(T, 3, dev)
        ops.reserve_workspace(T)
        s = torch.cuda.Stream()
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        with torch.cuda.stream(s):
            d = ep.dispatch(x, logits, bias)
            ep.combine(d, d.rows, out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            d = ep.dispatch(x, logits, bias)
            ep.combine(d, d.rows, out)
        out.zero_()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        _, _, _, ref = _one_gpu_reference(x, logits, bias)
        assert torch.equal(out, ref)
        assert ep.pg.status() == 0
        del g
    finally:
        ep.close()


@pytest.mark.parametrize("T", [1, 64, 4096, 65536])
def test_router_maps_allgather_single_rank(T):
    """kb_router_maps_allgather (fused into the tile kernel's tail at large T): the maps equal
    kb_router_maps', and gathered[0] = counts, over successive calls."""
    from kolibri_b200 import ops
    from kolibri_b200.ep import PeerGroup
    from kolibri_b200 import workloads as wl
    dev = torch.device("cuda")
    pg = PeerGroup(E, K, 0, 16, device=dev)
    try:
        gathered = torch.full((1, E), -7, dtype=torch.int32, device=dev)
        for call in range(3):
            logits, bias = wl.router_inputs(T, seed=50 + call)
            logits, bias = logits.to(dev), bias.to(dev)
            got = ops.router_maps_allgather(pg.addr, logits, bias, gathered, k=K)
            ref = ops.router_maps(logits, bias, k=K)
            torch.cuda.synchronize()
            for a, b in zip(got, ref):
                assert torch.equal(a, b)
            assert torch.equal(gathered[0], ref[2])
        assert pg.status() == 0
        for _ in range(3):                       # the device barrier of a one-rank group
            pg.barrier()
        torch.cuda.synchronize()
        assert pg.status() == 0
    finally:
        pg.close()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    ep = None
    try:
        from kolibri_b200.ep import ExpertParallel, PeerExpertParallel
        ep = PeerExpertParallel(E, K, H, max_tokens=1024, device=dev)
        ref_ep = ExpertParallel(E, K)
        ok = True
        # token counts per call and rank: equal, different, one rank empty
        for call, Ts in enumerate(([512, 512], [1024, 300], [0, 700], [1, 1])):
            T = Ts[rank]
            x, logits, bias = _inputs(T, 100 * call + rank, dev)
            d = ep.dispatch(x, logits, bias)
            out = ep.combine(d, d.rows)
            if T > 0:
                _, _, _, ref = _one_gpu_reference(x, logits, bias)
            else:
                ref = torch.empty(0, H, dtype=torch.bfloat16, device=dev)
            # the collective path on the same routing (both ranks take part, or neither)
            r = ref_ep.dispatch(x, logits, bias) if min(Ts) > 0 else None
            torch.cuda.synchronize()
            R = d.num_rows()
            ok &= torch.equal(out, ref)
            if r is not None:
                ok &= R == r.rows.shape[0]
                ok &= torch.equal(d.rows[:R], r.rows)
                ok &= torch.equal(d.expert_offsets, r.expert_offsets)
                ok &= torch.equal(ref_ep.combine(r, r.rows), ref)
        ok &= ep.pg.status() == 0
        # the fused router + maps + count all-gather against NCCL's all-gather
        from kolibri_b200 import ops
        from kolibri_b200 import workloads as wl
        for T in (64, 4096, 65536):
            logits, bias = wl.router_inputs(T, seed=70 + rank)
            logits, bias = logits.to(dev), bias.to(dev)
            gathered = torch.empty(world, E, dtype=torch.int32, device=dev)
            _, _, counts, *_ = ops.router_maps_allgather(ep.pg.addr, logits, bias, gathered, k=K)
            ref = torch.empty(world, E, dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(ref, counts)
            torch.cuda.synchronize()
            ok &= torch.equal(gathered, ref)
        for _ in range(5):                       # device barriers across the two GPUs
            ep.pg.barrier()
        torch.cuda.synchronize()
        ok &= ep.pg.status() == 0
        q.put((rank, bool(ok)))
    except Exception as e:  # report, then leave the group cleanly
        q.put((rank, repr(e)))
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def _run_two(target):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    return res


def test_peer_exchange_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run_two(_worker)
    assert all(r[1] is True for r in res), res


def test_exchange_error_word_reported_and_sticky():
    """A pre-set error word (as a wait that gave up leaves it): the count all-gather writes
    gathered = -1, later calls do nothing, and the status reads KB_WS_TIMEOUT."""
    from kolibri_b200 import _lib
    from kolibri_b200.ep import PeerExpertParallel
    dev = torch.device("cuda")
    ep = PeerExpertParallel(E, K, H, max_tokens=64, device=dev)
    try:
        x, logits, bias = _inputs(64, 5, dev)
        d = ep.dispatch(x, logits, bias)
        ep.combine(d, d.rows)
        torch.cuda.synchronize()
        assert ep.pg.status() == _lib.KB_WS_CLEAN
        err = torch.as_tensor(_ErrWord(ep.pg._own), device=dev)
        err.fill_(_lib.KB_WS_TIMEOUT)
        ep.gathered.fill_(5)
        ep.dispatch(x, logits, bias)
        torch.cuda.synchronize()
        assert bool((ep.gathered == -1).all())
        assert ep.pg.status() == _lib.KB_WS_TIMEOUT
    finally:
        ep.close()


def test_exchange_rejects_invalid_counts():
    """Counts that cannot be right (negative) stop the dispatch with KB_WS_CAPACITY."""
    from kolibri_b200 import _lib
    from kolibri_b200.ep import PeerExpertParallel
    dev = torch.device("cuda")
    ep = PeerExpertParallel(E, K, H, max_tokens=64, device=dev)
    try:
        x, logits, bias = _inputs(64, 6, dev)
        from kolibri_b200 import ops
        ids, w, counts, offsets, p2u, u2p = ops.router_maps(logits, bias, k=K)
        bad = torch.full((1, E), -3, dtype=torch.int32, device=dev)
        _lib.check(ep.pg._lib.kb_ep_dispatch(ep.pg.addr, x.data_ptr(), 64, p2u.data_ptr(),
                                             bad.data_ptr(), ep.recv_offsets.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream),
                   "kb_ep_dispatch")
        torch.cuda.synchronize()
        assert ep.pg.status() == _lib.KB_WS_CAPACITY
    finally:
        ep.close()


class _ErrWord:
    """The 4-byte error word at the start of an exchange buffer, as a torch view."""

    def __init__(self, ptr):
        self.__cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (ptr, False),
                                         "version": 3, "strides": None}
