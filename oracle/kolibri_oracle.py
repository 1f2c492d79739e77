"""CPU oracle for the Kolibri non-GEMM MoE decode path.

TEST INFRASTRUCTURE ONLY.  This module is the checker, never the thing measured or shipped:
only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
it.  The product path (profiling-moe_b200/) never imports it and has no CPU fallback.

Each function restates the reference's PyTorch-eager definition of one hot-path stage (cited
file:line, relative to the reference repository root) and runs it on the CPU:

  router_ref               benchmarks/01_benchmark_router.py:33-37 with the lower-index tie-break
                           of kernels/cuda/moeTopKFuncs.cuh:54-61 (stable descending sort; torch.topk
                           does not order ties) and the optional renorm of
                           kernels/triton/fused_kolibri_router.py:84-92
  router_eager_reference   benchmarks/01_benchmark_router.py:33-37 verbatim (torch.topk); the timed
                           CPU baseline, identical to router_ref whenever no scores tie
  expert_maps_ref          counts/offsets of benchmarks/09_benchmark_build_expert_maps.py:18-28, the
                           slot-major unpermuted row of benchmarks/08_benchmark_router_dispatch.py:29-41,
                           ordered (expert, token, slot) like the CUB rank kernel
                           kernels/cuda/customKolibriBuildExpertMapsKernel.cu:96-156; ids outside
                           [0, E) skipped as in kernels/cuda/customKolibriBuildExpertMapsKernels.cuh:42-48
  expansion_ref            fusions/03_moe_prologue/fused/custom_moe_prologue.cu:453-478 (x[p2u % T])
  qk_norm_rope_ref         scratch/diag_rope_fusion.py:31-38 (per-head RMSNorm then NeoX RoPE);
                           positions=None is the RNoPE identity, i.e. the per-head F.rms_norm of
                           benchmarks/11_profile_2block_e2e.py:195-196
  sandwich_ref             fusions/01_sandwich_norm/baseline/trtllm_baseline.py:78-95
  add_post_moe_norm_ref    fusions/02_post_moe_norm/baseline/trtllm_baseline.py:77-90
  post_moe_pre_attn_ref    benchmarks/11_profile_2block_e2e.py:269-270 then :229-231
                           (out = h + RMSNorm(moe_out); next = RMSNorm(out))
  router_logits_ref        benchmarks/11_profile_2block_e2e.py:242-243 ((x @ W_g).float())
  finalize_ref             benchmarks/11_profile_2block_e2e.py:259-262 (weighted combine by u2p)
  ep_placement_ref         where the expert-parallel exchange puts every routed row (no reference
                           counterpart: the reference runs on one GPU); the order an all-to-all of
                           the expert-sorted rows (expert_maps_ref order) followed by a stable
                           grouping by local expert produces, written as the closed formula the
                           peer-memory kernels use, so the CPU tests can check the formula against
                           the collective exchange

Pinning: tests/golden/ holds outputs of the reference's own eager functions (extracted from
the reference sources by tests/golden/make_golden.py) at the benchmark seeds; the oracle is
checked against them in tests/test_oracle_golden.py.
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------------------
# Router
# --------------------------------------------------------------------------------------
def router_ref(logits: torch.Tensor, bias: Optional[torch.Tensor], k: int = 6,
               renorm: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """-> (ids int32 [T,k], weights fp32 [T,k]).  Ties: lower expert index first; NaN first."""
    x = logits.float()
    scores = x + bias.float() if bias is not None else x
    order = torch.sort(scores, dim=-1, descending=True, stable=True).indices[:, :k]
    w = torch.sigmoid(torch.gather(x, -1, order))
    if renorm:
        w = w * (1.0 / (w.sum(dim=-1, keepdim=True) + 1e-20))
    return order.to(torch.int32), w


def router_eager_reference(x: torch.Tensor, bias: torch.Tensor, k: int = 6):
    """The reference's eager router as written (torch.topk, int64 ids)."""
    scores = x + bias
    topk_ids = torch.topk(scores, k=k, dim=-1).indices
    topk_weights = torch.sigmoid(torch.gather(x, -1, topk_ids))
    return topk_ids, topk_weights


# --------------------------------------------------------------------------------------
# Expert maps
# --------------------------------------------------------------------------------------
def expert_maps_ref(ids, num_experts: int = 384):
    """ids [T,k] (any integer array) -> (counts int32 [E], offsets int64 [E+1],
    p2u int32 [T*k], u2p int32 [T*k]) as numpy arrays.

    p2u[r] = slot*T + token of the r-th row in (expert, token, slot) order, -1 past the
    last valid row; u2p[slot*T + token] = r, -1 for an id outside [0, E)."""
    ids = np.asarray(ids.cpu() if isinstance(ids, torch.Tensor) else ids).astype(np.int64)
    T, k = ids.shape
    E = int(num_experts)
    flat = ids.reshape(-1)                      # selection s = token*k + slot
    valid = (flat >= 0) & (flat < E)
    counts = np.bincount(flat[valid], minlength=E).astype(np.int32)
    offsets = np.zeros(E + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    sel = np.nonzero(valid)[0]
    order = sel[np.argsort(flat[sel], kind="stable")]   # (expert, token, slot)
    tok, slot = order // k, order % k
    unperm = slot * T + tok
    p2u = np.full(T * k, -1, dtype=np.int32)
    p2u[: order.size] = unperm
    u2p = np.full(T * k, -1, dtype=np.int32)
    u2p[unperm] = np.arange(order.size, dtype=np.int32)
    return counts, offsets, p2u, u2p


def maps_eager_reference(ids: torch.Tensor, num_experts: int = 384):
    """The map part of benchmarks/08_benchmark_router_dispatch.py:24-49 on the CPU (slot-major
    flatten, stable argsort, bincount, cumsum) plus the inverse map: the eager counterpart of
    kb_expert_maps that the timed CPU baseline runs.  -> (counts, offsets, p2u, u2p)."""
    T, k = ids.shape
    flat_experts = ids.t().contiguous().view(-1).long()
    order = torch.argsort(flat_experts, stable=True)
    p2u = order.to(torch.int32)
    counts = torch.bincount(flat_experts, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, dim=0)
    u2p = torch.empty(T * k, dtype=torch.int32)
    u2p[order] = torch.arange(T * k, dtype=torch.int32)
    return counts, offsets, p2u, u2p


def router_maps_eager_reference(logits: torch.Tensor, bias: torch.Tensor, k: int = 6,
                                num_experts: int = 384):
    """The reference's eager router + dispatch-map path on the CPU, the baseline that the
    timed CPU arm runs: benchmarks/01_benchmark_router.py:33-37 (torch.topk router) followed
    by the map part of benchmarks/08_benchmark_router_dispatch.py:24-49 (slot-major flatten,
    stable argsort, bincount, cumsum), plus the inverse map the kernels also produce.
    Multi-threaded through torch's intra-op pool.  -> (ids, w, counts, offsets, p2u, u2p)."""
    T = logits.shape[0]
    ids, w = router_eager_reference(logits, bias, k)
    flat_experts = ids.t().contiguous().view(-1)
    order = torch.argsort(flat_experts, stable=True)
    p2u = order.to(torch.int32)            # slot-major position = slot*T + token
    counts = torch.bincount(flat_experts, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(counts, dim=0)
    u2p = torch.empty(T * k, dtype=torch.int32)
    u2p[order] = torch.arange(T * k, dtype=torch.int32)
    return ids, w, counts, offsets, p2u, u2p


def expansion_ref(x: torch.Tensor, p2u) -> torch.Tensor:
    """out[r] = x[p2u[r] % T]; rows with p2u outside [0, rows) are zero."""
    p = torch.as_tensor(np.asarray(p2u), dtype=torch.int64)
    T = x.shape[0]
    out = torch.zeros((p.numel(),) + tuple(x.shape[1:]), dtype=x.dtype)
    ok = (p >= 0) & (p < p.numel())
    out[ok] = x[p[ok] % T]
    return out


# --------------------------------------------------------------------------------------
# Q/K RMSNorm + NeoX RoPE
# --------------------------------------------------------------------------------------
def rope_inv_freq_ref(theta: float, head_dim: int) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))


def _head_norm_rope(x: torch.Tensor, w: torch.Tensor, pos: Optional[torch.Tensor], eps: float,
                    theta: float) -> torch.Tensor:
    T, H, D = x.shape
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    if pos is None:
        return y.to(torch.bfloat16)
    inv = rope_inv_freq_ref(theta, D)
    ang = pos.float()[:, None] * inv[None]            # [T, D/2]
    cos, sin = ang.cos()[:, None], ang.sin()[:, None]  # [T, 1, D/2]
    y1, y2 = y[..., : D // 2], y[..., D // 2:]
    return torch.cat([y1 * cos - y2 * sin, y2 * cos + y1 * sin], -1).to(torch.bfloat16)


def qk_norm_rope_ref(q, k, gamma_q, gamma_k, positions: Optional[torch.Tensor],
                     eps: float = 1e-6, theta: float = 10000.0):
    """q [T,Hq,D], k [T,Hkv,D] bf16 -> (q', k') bf16; positions None = RNoPE (identity)."""
    return (_head_norm_rope(q, gamma_q, positions, eps, theta),
            _head_norm_rope(k, gamma_k, positions, eps, theta))


# --------------------------------------------------------------------------------------
# Residual norms
# --------------------------------------------------------------------------------------
def sandwich_ref(attn_out, residual_in, gamma1, gamma2, eps: float = 1e-6):
    """-> (updated_residual, moe_in)."""
    d = attn_out.shape[-1]
    post_attn = F.rms_norm(attn_out, (d,), gamma1, eps=eps)
    updated_residual = residual_in + post_attn
    moe_in = F.rms_norm(updated_residual, (d,), gamma2, eps=eps)
    return updated_residual, moe_in


def add_post_moe_norm_ref(routed_out, shared_out, gamma, eps: float = 1e-6):
    d = routed_out.shape[-1]
    return F.rms_norm(routed_out + shared_out, (d,), gamma, eps=eps)


def post_moe_pre_attn_ref(moe_out, h, gamma_post_moe, gamma_pre_attn, eps: float = 1e-6):
    """-> (out, next): out = h + RMSNorm(moe_out)*g_pm ; next = RMSNorm(out)*g_pa."""
    d = moe_out.shape[-1]
    out = h + F.rms_norm(moe_out, (d,), gamma_post_moe, eps=eps)
    nxt = F.rms_norm(out, (d,), gamma_pre_attn, eps=eps)
    return out, nxt


def router_logits_ref(x: torch.Tensor, w_gate: torch.Tensor) -> torch.Tensor:
    return (x @ w_gate).float()


def router_gemm_ref(x: torch.Tensor, w_gate_t: torch.Tensor, bias: Optional[torch.Tensor],
                    k: int = 6, renorm: bool = False):
    """The gate GEMM + router of benchmarks/11_profile_2block_e2e.py:241-246: logits =
    (moe_in @ W_g).float() with W_g = w_gate_t.T, i.e. an exact product rounded once to bf16
    (the fp64 product stands in for the exact one), then router_ref on those logits.
    -> (ids, w, logits fp32 [T, E])."""
    logits = (x.double() @ w_gate_t.double().t()).to(torch.bfloat16).float()
    ids, w = router_ref(logits, bias, k=k, renorm=renorm)
    return ids, w, logits


def finalize_ref(expert_out: torch.Tensor, u2p, weights: torch.Tensor) -> torch.Tensor:
    """(expert_out[u2p.view(K, T)].float() * weights.float().t().unsqueeze(-1)).sum(0).to(dtype);
    slots whose u2p is negative contribute zero."""
    T, K = weights.shape
    perm = torch.as_tensor(u2p).view(K, T).long()
    valid = (perm >= 0).unsqueeze(-1)
    rows = expert_out[perm.clamp(min=0)].float() * valid
    return (rows * weights.float().t().unsqueeze(-1)).sum(0).to(expert_out.dtype)


# --------------------------------------------------------------------------------------
# Expert-parallel exchange: placement of the routed rows
# --------------------------------------------------------------------------------------
def ep_placement_ref(counts_all, world: int):
    """counts_all int [N, E] (every rank's per-expert counts) -> for every owner rank o, the
    list of (sender q, sender's permuted row i) in the owner's grouped order, and for every
    sender q, dest[q][i] = (owner, grouped row) of its permuted row i.

    Grouped row of sender q's permuted row i of expert e on owner o = e // (E/N):
        (S[e] - S[o*Er]) + sum_{q' < q} c[q'][e] + (i - loff_q[e])
    with tot[e] = sum_q c[q][e], S its exclusive scan, loff_q the exclusive scan of c[q]."""
    c = np.asarray(counts_all, dtype=np.int64)
    N, E = c.shape
    assert N == world and E % N == 0
    Er = E // N
    tot = c.sum(0)
    S = np.concatenate([[0], np.cumsum(tot)])
    loff = np.concatenate([np.zeros((N, 1), np.int64), np.cumsum(c, 1)], 1)
    before = np.concatenate([np.zeros((1, E), np.int64), np.cumsum(c, 0)[:-1]], 0)
    grouped = [[None] * int(S[(o + 1) * Er] - S[o * Er]) for o in range(N)]
    dest = []
    for q in range(N):
        dq = []
        for e in range(E):
            o = e // Er
            for j in range(int(c[q, e])):
                gpos = int(S[e] - S[o * Er] + before[q, e] + j)
                grouped[o][gpos] = (q, int(loff[q, e] + j))
                dq.append((o, gpos))
        dest.append(dq)
    return grouped, dest
