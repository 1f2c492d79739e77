"""Expert-parallel dispatch and combine of the MoE prologue across ranks (one process per GPU).

Rank r of N owns experts [r*E/N, (r+1)*E/N) (48 per GPU for E = 384 on 8 GPUs) and routes
its own tokens.  The only collectives are the two the path needs (NCCL on GPUs):

  dispatch  1. local router + expert maps over all E experts and the expansion: the permuted
               rows come out sorted by expert, hence already grouped by owner rank
            2. all-gather of the per-expert counts [E] -> [N, E]; every rank derives the send
               and receive row counts of the all-to-all from it, with no further round trip
            3. all-to-all of the permuted rows and of their metadata (expert id, routing
               weight, origin row = slot*T + token on the sender)
            4. the owner groups the received rows of each of its experts across senders
               (expert maps over the received expert ids, then an expansion): contiguous
               per-expert segments and their offsets, ready for the expert GEMMs
  combine   5. the owner ungroups the expert outputs and sends them back (the reverse
               all-to-all), and every sender finalizes its tokens: out[t] =
               sum_k w[t, k] * row(u2p[k*T + t])

The reference repository runs on one GPU and has no such path; the layout follows the
(expert, token, slot) order of its maps (kernels/cuda/customKolibriBuildExpertMapsKernel.cu:
96-156) and its finalize (benchmarks/11_profile_2block_e2e.py:259-262).

The local steps go through a `LocalOps` object.  The default one calls the libkolibri_b200
kernels (CUDA tensors only, no fallback); the CPU tests of the exchange logic substitute
CPU implementations of the same four operations.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


class LocalOps:
    """The four local operations of the path, on the libkolibri_b200 kernels."""

    def router_maps(self, logits, bias, k):
        from . import ops
        ids, w, counts, offsets, p2u, u2p = ops.router_maps(logits, bias, k=k)
        return ids, w, counts, offsets, p2u, u2p

    def expert_maps(self, ids, num_experts):
        from . import ops
        return ops.expert_maps(ids, num_experts)

    def expand_rows(self, x, p2u):
        from . import ops
        return ops.expand_rows(x, p2u)

    def finalize(self, rows, u2p, w):
        from . import ops
        return ops.moe_finalize(rows, u2p, w)


@dataclass
class Dispatched:
    """What dispatch() returns: the sender-side state for combine() and the owner's rows."""
    # sender side
    T: int
    ids: torch.Tensor          # int32 [T, K] routed experts (global ids)
    weights: torch.Tensor      # fp32 [T, K]
    u2p: torch.Tensor          # int32 [K*T] local unpermuted -> permuted row
    send_splits: list          # rows sent to each rank
    recv_splits: list          # rows received from each rank
    # owner side
    rows: torch.Tensor         # [R, H] received rows grouped by local expert
    expert_offsets: torch.Tensor  # int64 [E/N + 1] segments of `rows` per local expert
    meta: torch.Tensor         # int32 [R, 3] received (expert, weight bits, origin), sender order
    group_p2u: torch.Tensor    # int32 [R] grouped position -> received row
    group_u2p: torch.Tensor    # int32 [R] received row -> grouped position


class ExpertParallel:
    """Dispatch/combine for one MoE layer with E experts and top-K routing over `group`."""

    def __init__(self, num_experts: int = 384, top_k: int = 6,
                 group: Optional[dist.ProcessGroup] = None, local_ops: Optional[LocalOps] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError("num_experts must be a multiple of the world size")
        self.E, self.K = num_experts, top_k
        self.Er = num_experts // self.world
        self.ops = local_ops or LocalOps()

    # ------------------------------------------------------------------------------------
    def dispatch(self, x: torch.Tensor, logits: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> Dispatched:
        T, H = x.shape
        N, Er, K = self.world, self.Er, self.K
        ids, w, counts, offsets, p2u, u2p = self.ops.router_maps(logits, bias, K)
        permuted = self.ops.expand_rows(x, p2u)                   # [T*K, H], expert order
        # metadata of every permuted row: expert, weight bits, origin (slot*T + token)
        p2u_l = p2u.long()
        tok, slot = p2u_l % T, p2u_l // T
        flat = tok * K + slot
        meta = torch.stack([ids.reshape(-1)[flat].int(),
                            w.reshape(-1)[flat].contiguous().view(torch.int32),
                            p2u.int()], dim=1).contiguous()
        # counts of every rank, then the splits of both directions
        counts_all = torch.empty(N * self.E, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(counts_all, counts.contiguous(), group=self.group)
        per_owner = counts_all.view(N, N, Er).sum(-1).cpu()       # [sender, owner]
        send_splits = per_owner[self.rank].tolist()
        recv_splits = per_owner[:, self.rank].tolist()
        R = int(sum(recv_splits))
        recv_rows = torch.empty(R, H, dtype=x.dtype, device=x.device)
        recv_meta = torch.empty(R, 3, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_rows, permuted, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_splits, send_splits, group=self.group)
        # group the received rows by local expert (stable: sender, then sender's order)
        local_ids = (recv_meta[:, 0] - self.rank * Er).contiguous().view(R, 1)
        if R:
            _, loff, gp2u, gu2p = self.ops.expert_maps(local_ids, Er)
            rows = self.ops.expand_rows(recv_rows, gp2u)
        else:
            loff = torch.zeros(Er + 1, dtype=torch.int64, device=x.device)
            gp2u = torch.empty(0, dtype=torch.int32, device=x.device)
            gu2p = torch.empty(0, dtype=torch.int32, device=x.device)
            rows = recv_rows
        return Dispatched(T=T, ids=ids, weights=w, u2p=u2p, send_splits=send_splits,
                          recv_splits=recv_splits, rows=rows, expert_offsets=loff,
                          meta=recv_meta, group_p2u=gp2u, group_u2p=gu2p)

    def combine(self, d: Dispatched, expert_out: torch.Tensor) -> torch.Tensor:
        """expert_out: [R, H] outputs of the local experts in the grouped order of d.rows."""
        R, H = expert_out.shape
        back_rows = (self.ops.expand_rows(expert_out, d.group_u2p) if R
                     else expert_out)                             # received (sender) order
        mine = torch.empty(d.T * self.K, H, dtype=expert_out.dtype, device=expert_out.device)
        dist.all_to_all_single(mine, back_rows.contiguous(), d.send_splits, d.recv_splits,
                               group=self.group)
        return self.ops.finalize(mine, d.u2p, d.weights)
