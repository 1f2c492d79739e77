"""Torch-facing wrappers over the libkolibri_b200 C ABI.

Each function validates its tensors, allocates outputs with the PyTorch caching allocator,
and launches on the current CUDA stream of the input's device.  Nothing here computes on
the host: every result comes from the sm_100a kernels.
"""
from __future__ import annotations

import threading
from typing import Optional, Tuple

import torch

from ._lib import (KB_BF16, KB_F16, KB_F32, KB_MAPS_AUTO, KB_MAPS_HYBRID_ROUTER,
                   KB_MAPS_MULTI_CTA, KB_MAPS_SINGLE_CTA, KB_MAPS_TWO_KERNEL, KB_MAPS_WARP_ROUTER,
                   KB_NOALLOC_REZERO, check, load)

__all__ = [
    "router", "expert_maps", "router_maps", "expand_rows", "qk_norm_rope", "rope_inv_freq",
    "residual_norm_pair", "add_rms_norm", "reserve_workspace", "set_pdl", "expert_maps_noalloc",
    "set_wait_limit", "workspace_status",
    "moe_finalize", "expand_rows_scaled", "router_maps_allgather", "router_gemm",
    "KB_MAPS_AUTO", "KB_MAPS_SINGLE_CTA", "KB_MAPS_MULTI_CTA", "KB_MAPS_TWO_KERNEL",
    "KB_MAPS_HYBRID_ROUTER", "KB_MAPS_WARP_ROUTER",
]

_DTYPE_CODE = {torch.bfloat16: KB_BF16, torch.float16: KB_F16, torch.float32: KB_F32}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def _contig(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def set_pdl(enable: bool) -> bool:
    """Turn programmatic dependent launch on or off for later launches; returns the old value."""
    return bool(load().kb_set_pdl(int(bool(enable))))


def set_wait_limit(polls: int) -> int:
    """Poll limit of the kernels' bounded waits for later launches (0 = the defaults);
    returns the previous setting."""
    return int(load().kb_set_wait_limit(int(polls)))


def workspace_status(workspace: Optional[torch.Tensor], kind: int = 0,
                     device: Optional[torch.device] = None) -> int:
    """The error word of a workspace (kind 0: maps / router+maps, 1: decode chain, 2: the
    static scratch of expert_maps_noalloc on `device`): 0 clean, 1 a bounded wait gave up,
    2 misaligned decode-chain weights.  Waits for the current stream."""
    import ctypes
    dev = workspace.device if workspace is not None else (device or torch.device("cuda"))
    out = ctypes.c_int(-1)
    with torch.cuda.device(dev):
        check(load().kb_workspace_status(_p(workspace), int(kind), ctypes.byref(out),
                                         _stream(dev)), "kb_workspace_status")
    return out.value


# ----------------------------------------------------------------------------------------
# Workspace: one zero-filled byte buffer per (device, stream), grown on demand.  The map
# kernels leave it zero-filled after every call.  Grow it before CUDA-graph capture with
# reserve_workspace(); growing during capture is refused.
# ----------------------------------------------------------------------------------------
_WS_LOCK = threading.Lock()
_WS: dict = {}


def _workspace(nbytes: int, device: torch.device, tag: str = "maps") -> torch.Tensor:
    stream = _stream(device)
    key = (device.index, stream, tag)
    with _WS_LOCK:
        buf = _WS.get(key)
        if buf is None or buf.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "kolibri_b200 workspace must grow during CUDA graph capture; call "
                    "reserve_workspace() with the largest T before capturing")
            buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            _WS[key] = buf
        return buf


def reserve_workspace(T: int, num_experts: int = 384, k: int = 6,
                      device: Optional[torch.device] = None) -> None:
    """Pre-allocate the expert-map workspace for up to T tokens on the current stream."""
    device = torch.device(device or torch.device("cuda", torch.cuda.current_device()))
    lib = load()
    need = max(lib.kb_expert_maps_workspace_bytes(T, num_experts, k),
               lib.kb_router_maps_workspace_bytes(T, num_experts, k))
    _workspace(need, device)


# ----------------------------------------------------------------------------------------
# Router and expert maps
# ----------------------------------------------------------------------------------------
def _check_logits(logits: torch.Tensor, bias: Optional[torch.Tensor]) -> Tuple[int, int]:
    _cuda(logits, "logits")
    if logits.dim() != 2:
        raise ValueError("logits must be 2D [num_tokens, num_experts]")
    if logits.dtype != torch.float32:
        raise ValueError("logits must be float32")
    _contig(logits, "logits")
    T, E = logits.shape
    if bias is not None:
        _cuda(bias, "bias")
        if bias.dtype != torch.float32 or bias.numel() != E or bias.device != logits.device:
            raise ValueError(f"bias must be float32 [{E}] on {logits.device}")
        _contig(bias, "bias")
    return T, E


def router(logits: torch.Tensor, bias: Optional[torch.Tensor] = None, k: int = 6,
           renorm: bool = False, w_dtype: torch.dtype = torch.float32):
    """Top-k of (logits + bias) per row; weights = sigmoid(logits[ids]).  -> (ids int32, w)."""
    T, E = _check_logits(logits, bias)
    dev = logits.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=w_dtype, device=dev)
    if w_dtype not in _DTYPE_CODE:
        raise ValueError("w_dtype must be float32, bfloat16 or float16")
    check(load().kb_router(_p(logits), _p(bias), _p(ids), _p(w), _DTYPE_CODE[w_dtype], T, E, k,
                           int(bool(renorm)), _stream(dev)), "kb_router")
    return ids, w


def router_gemm(x: torch.Tensor, w_gate: torch.Tensor, bias: Optional[torch.Tensor] = None,
                k: int = 6, renorm: bool = False, route: bool = True, logits: bool = True):
    """Router projection on the tensor cores with the routing fused into its epilogue:
    logits = (x @ w_gate.T) rounded to bf16 and widened to fp32, then the top-k router on
    them.  x bf16 [T, H], w_gate bf16 [E, H] (nn.Linear layout).
    -> (ids int32 [T, k] or None, w fp32 [T, k] or None, logits fp32 [T, E] or None)."""
    _cuda(x, "x")
    _cuda(w_gate, "w_gate")
    if x.dim() != 2 or w_gate.dim() != 2 or x.shape[1] != w_gate.shape[1]:
        raise ValueError("x must be [num_tokens, hidden] and w_gate [num_experts, hidden]")
    if x.dtype != torch.bfloat16 or w_gate.dtype != torch.bfloat16:
        raise ValueError("x and w_gate must be bfloat16")
    if w_gate.device != x.device:
        raise ValueError("x and w_gate must be on the same device")
    _contig(x, "x")
    _contig(w_gate, "w_gate")
    T, H = x.shape
    E = w_gate.shape[0]
    if bias is not None:
        _cuda(bias, "bias")
        if bias.dtype != torch.float32 or bias.numel() != E or bias.device != x.device:
            raise ValueError(f"bias must be float32 [{E}] on {x.device}")
        _contig(bias, "bias")
    if not route and not logits:
        raise ValueError("router_gemm needs route=True or logits=True")
    dev = x.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev) if route else None
    w = torch.empty((T, k), dtype=torch.float32, device=dev) if route else None
    lg = torch.empty((T, E), dtype=torch.float32, device=dev) if logits else None
    lib = load()
    with torch.cuda.device(dev):
        need = lib.kb_router_gemm_workspace_bytes(T, H, E, k if route else 1)
        ws = _workspace(need, dev, "rgemm")
        check(lib.kb_router_gemm(_p(x), _p(w_gate), _p(bias), _p(lg), _p(ids), _p(w), _p(ws),
                                 ws.numel(), T, H, E, k, int(bool(renorm)), _stream(dev)),
              "kb_router_gemm")
    return ids, w, lg


def _maps_outputs(T: int, E: int, k: int, dev, counts: bool, inverse: bool):
    c = torch.empty((E,), dtype=torch.int32, device=dev) if counts else None
    off = torch.empty((E + 1,), dtype=torch.int64, device=dev)
    p2u = torch.empty((T * k,), dtype=torch.int32, device=dev)
    u2p = torch.empty((T * k,), dtype=torch.int32, device=dev) if inverse else None
    return c, off, p2u, u2p


def expert_maps(ids: torch.Tensor, num_experts: int = 384, mode: int = KB_MAPS_AUTO,
                counts: bool = True, inverse: bool = True):
    """Stable expert maps of top-k ids [T, k].  -> (counts, offsets, p2u, u2p).

    p2u[r] = k*T + t of the r-th row in (expert, token, slot) order; u2p is its inverse,
    indexed by k*T + t; offsets int64 [E+1]; counts int32 [E] (None if counts=False).
    """
    _cuda(ids, "token_selected_experts")
    if ids.dtype != torch.int32:
        raise ValueError("token_selected_experts must be int32")
    _contig(ids, "token_selected_experts")
    if ids.dim() != 2:
        raise ValueError("token_selected_experts must be 2D [num_tokens, top_k]")
    T, k = ids.shape
    E = int(num_experts)
    dev = ids.device
    c, off, p2u, u2p = _maps_outputs(T, E, k, dev, counts, inverse)
    lib = load()
    need = lib.kb_expert_maps_workspace_bytes(T, E, k)
    ws = _workspace(need, dev) if need else None
    check(lib.kb_expert_maps(_p(ids), _p(c), _p(off), _p(p2u), _p(u2p), _p(ws),
                             0 if ws is None else ws.numel(), T, E, k, int(mode), _stream(dev)),
          "kb_expert_maps")
    return c, off, p2u, u2p


def expert_maps_noalloc(ids: torch.Tensor, c: torch.Tensor, off: torch.Tensor,
                        p2u: torch.Tensor, u2p: Optional[torch.Tensor] = None,
                        num_experts: int = 384, rezero: bool = False) -> None:
    """expert_maps into caller-provided outputs through kb_expert_maps_noalloc: the
    library's static device scratch replaces the workspace, so the call allocates no
    device memory.  c int32 [E] (or None), off int64 [E+1], p2u/u2p int32 [T*k]."""
    _cuda(ids, "token_selected_experts")
    if ids.dtype != torch.int32 or ids.dim() != 2:
        raise ValueError("token_selected_experts must be 2D int32 [num_tokens, top_k]")
    _contig(ids, "token_selected_experts")
    T, k = ids.shape
    E = int(num_experts)
    for t, n, dt, name in ((c, E, torch.int32, "counts"), (off, E + 1, torch.int64, "offsets"),
                           (p2u, T * k, torch.int32, "p2u"), (u2p, T * k, torch.int32, "u2p")):
        if t is None:
            if name in ("offsets", "p2u"):
                raise ValueError(f"{name} is required")
            continue
        _cuda(t, name)
        _contig(t, name)
        if t.dtype != dt or t.numel() != n:
            raise ValueError(f"{name} must be {dt} with {n} elements")
        if t.device != ids.device:
            raise ValueError(f"{name} must be on {ids.device}")
    with torch.cuda.device(ids.device):  # the library resolves the scratch of the current device
        check(load().kb_expert_maps_noalloc(_p(ids), _p(c), _p(off), _p(p2u), _p(u2p), T, E, k,
                                            KB_NOALLOC_REZERO if rezero else 0,
                                            _stream(ids.device)),
              "kb_expert_maps_noalloc")


def router_maps(logits: torch.Tensor, bias: Optional[torch.Tensor] = None, k: int = 6,
                renorm: bool = False, mode: int = KB_MAPS_AUTO, inverse: bool = True):
    """Router and expert maps in one pass.  -> (ids, w, counts, offsets, p2u, u2p)."""
    T, E = _check_logits(logits, bias)
    dev = logits.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    c, off, p2u, u2p = _maps_outputs(T, E, k, dev, True, inverse)
    lib = load()
    need = lib.kb_router_maps_workspace_bytes(T, E, k)
    ws = _workspace(need, dev) if need else None
    check(lib.kb_router_maps(_p(logits), _p(bias), _p(ids), _p(w), _p(c), _p(off), _p(p2u),
                             _p(u2p), _p(ws), 0 if ws is None else ws.numel(), T, E, k,
                             int(bool(renorm)), int(mode), _stream(dev)), "kb_router_maps")
    return ids, w, c, off, p2u, u2p


def router_maps_allgather(group_addr: int, logits: torch.Tensor, bias: Optional[torch.Tensor],
                          gathered: torch.Tensor, k: int = 6, renorm: bool = False,
                          mode: int = KB_MAPS_AUTO):
    """router_maps on this rank's tokens plus the all-gather of every rank's counts into
    gathered int32 [N, E] (group_addr: address of a kb_ep_group_t, see ep.PeerGroup), fused
    into one kernel on the tile path.  -> (ids, w, counts, offsets, p2u, u2p)."""
    T, E = _check_logits(logits, bias)
    dev = logits.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    c, off, p2u, u2p = _maps_outputs(T, E, k, dev, True, True)
    lib = load()
    need = lib.kb_router_maps_workspace_bytes(T, E, k)
    ws = _workspace(need, dev) if need else None
    check(lib.kb_router_maps_allgather(group_addr, _p(logits), _p(bias), _p(ids), _p(w), _p(c),
                                       _p(off), _p(p2u), _p(u2p), _p(ws),
                                       0 if ws is None else ws.numel(), T, int(bool(renorm)),
                                       int(mode), _p(gathered), _stream(dev)),
          "kb_router_maps_allgather")
    return ids, w, c, off, p2u, u2p


def expand_rows(x: torch.Tensor, p2u: torch.Tensor) -> torch.Tensor:
    """out[r] = x[p2u[r] % T] for every permuted row r (T = x.shape[0])."""
    _cuda(x, "unpermuted_input")
    _cuda(p2u, "permuted_row_to_unpermuted_row")
    _contig(x, "unpermuted_input")
    _contig(p2u, "permuted_row_to_unpermuted_row")
    if p2u.dtype != torch.int32:
        raise ValueError("permuted_row_to_unpermuted_row must be int32")
    T = x.shape[0]
    rows = p2u.numel()
    row_bytes = (x.numel() // max(T, 1)) * x.element_size()
    out = torch.empty((rows,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    check(load().kb_expand_rows(_p(x), _p(out), _p(p2u), T, rows, row_bytes,
                                _stream(x.device)), "kb_expand_rows")
    return out


def expand_rows_scaled(x: torch.Tensor, p2u: torch.Tensor, weights: torch.Tensor):
    """(out, scales): out[r] = x[p2u[r] % T] and scales[r] = weights[p2u[r] % T, p2u[r] // T],
    in one pass (weights fp32 [T, K], p2u int32 [T*K])."""
    _cuda(x, "unpermuted_input")
    _cuda(p2u, "permuted_row_to_unpermuted_row")
    _cuda(weights, "weights")
    for t, n in ((x, "unpermuted_input"), (p2u, "permuted_row_to_unpermuted_row"),
                 (weights, "weights")):
        _contig(t, n)
    if p2u.dtype != torch.int32 or weights.dtype != torch.float32 or weights.dim() != 2:
        raise ValueError("p2u must be int32 and weights float32 [T, K]")
    T, K = weights.shape
    if x.shape[0] != T or p2u.numel() != T * K:
        raise ValueError("x must hold T rows and p2u T*K entries")
    row_bytes = (x.numel() // max(T, 1)) * x.element_size()
    out = torch.empty((T * K,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    scales = torch.empty(T * K, dtype=torch.float32, device=x.device)
    check(load().kb_expand_rows_scaled(_p(x), _p(out), _p(p2u), _p(weights), _p(scales), T, K,
                                       row_bytes, _stream(x.device)), "kb_expand_rows_scaled")
    return out, scales


def moe_finalize(expert_out: torch.Tensor, u2p: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """Weighted combine of the K expert-output rows of every token.

    expert_out [T*K, H] (permuted order), u2p int32 [K*T] (slot*T + token -> permuted row),
    weights fp32 [T, K]  ->  out [T, H] = sum_k expert_out[u2p[k*T+t]] * w[t, k] (fp32, in
    slot order, one rounding)."""
    _cuda(expert_out, "expert_out")
    _cuda(u2p, "u2p")
    _cuda(weights, "weights")
    for t, n in ((expert_out, "expert_out"), (u2p, "u2p"), (weights, "weights")):
        _contig(t, n)
    if u2p.dtype != torch.int32 or weights.dtype != torch.float32 or weights.dim() != 2:
        raise ValueError("u2p must be int32 and weights float32 [T, K]")
    if expert_out.dtype not in _DTYPE_CODE:
        raise ValueError("expert_out must be bfloat16, float16 or float32")
    T, K = weights.shape
    H = expert_out.shape[-1]
    if expert_out.numel() != T * K * H or u2p.numel() != T * K:
        raise ValueError("expert_out must hold T*K rows and u2p T*K entries")
    out = torch.empty((T, H), dtype=expert_out.dtype, device=expert_out.device)
    check(load().kb_moe_finalize(_p(expert_out), _p(u2p), _p(weights), _p(out), T, K, H,
                                 _DTYPE_CODE[expert_out.dtype], _stream(expert_out.device)),
          "kb_moe_finalize")
    return out


# ----------------------------------------------------------------------------------------
# Q/K norm + RoPE
# ----------------------------------------------------------------------------------------
_INV_FREQ: dict = {}


def rope_inv_freq(theta: float, head_dim: int, device: torch.device) -> torch.Tensor:
    """inv_freq = 1 / theta^(arange(0, D, 2) / D), evaluated by torch in fp32 on the host
    (the expression of the RoPE reference), cached on the device."""
    key = (float(theta), int(head_dim), device.type, device.index)
    t = _INV_FREQ.get(key)
    if t is None:
        inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
        t = inv.to(device=device, dtype=torch.float32).contiguous()
        _INV_FREQ[key] = t
    return t


def _heads_view(x: torch.Tensor, name: str):
    if x.dim() != 3:
        raise ValueError(f"{name} must be [num_tokens, num_heads, head_dim]")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16")
    T, H, D = x.shape
    if x.stride(2) != 1 or (H > 1 and x.stride(1) != D):
        raise ValueError(f"{name} must have contiguous heads (strides [*, head_dim, 1])")
    return T, H, D, x.stride(0)


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, gamma_q: torch.Tensor,
                 gamma_k: torch.Tensor, position_ids: Optional[torch.Tensor],
                 eps: float = 1e-6, theta: float = 10000.0, inplace: bool = False):
    """Per-head RMSNorm of q [T,Hq,D] and k [T,Hkv,D] then NeoX RoPE at position_ids
    (None = RNoPE identity).  -> (q_out, k_out)."""
    _cuda(q, "q")
    _cuda(k, "k")
    Tq, Hq, D, qs = _heads_view(q, "q")
    Tk, Hkv, Dk, ks = _heads_view(k, "k")
    if Tq != Tk or D != Dk:
        raise ValueError("q and k must agree on num_tokens and head_dim")
    for g, n in ((gamma_q, "gamma_q"), (gamma_k, "gamma_k")):
        _cuda(g, n)
        if g.dtype != torch.bfloat16 or g.numel() != D:
            raise ValueError(f"{n} must be bfloat16 [{D}]")
        _contig(g, n)
    dev = q.device
    pos = None
    inv = None
    if position_ids is not None:
        _cuda(position_ids, "position_ids")
        pos = position_ids.reshape(-1)
        if pos.dtype != torch.int32:
            pos = pos.to(torch.int32)
        pos = pos.contiguous()
        if pos.numel() != Tq:
            raise ValueError("position_ids must hold one position per token")
        inv = rope_inv_freq(theta, D, dev)
    if inplace:
        qo, ko, qos, kos = q, k, qs, ks
    else:
        qo = torch.empty((Tq, Hq, D), dtype=q.dtype, device=dev)
        ko = torch.empty((Tq, Hkv, D), dtype=k.dtype, device=dev)
        qos, kos = Hq * D, Hkv * D
        if qs != qos or ks != kos:
            # Out of place with a strided input: normalise a contiguous copy in place.
            qo.copy_(q)
            ko.copy_(k)
            q, k, qs, ks = qo, ko, qos, kos
    check(load().kb_qk_norm_rope(_p(q), _p(qo), _p(k), _p(ko), _p(gamma_q), _p(gamma_k),
                                 _p(pos), _p(inv), Tq, Hq, Hkv, D, qs, ks, float(eps),
                                 _stream(dev)), "kb_qk_norm_rope")
    return qo, ko


# ----------------------------------------------------------------------------------------
# Residual norms
# ----------------------------------------------------------------------------------------
def _rows(a: torch.Tensor, name: str):
    _cuda(a, name)
    _contig(a, name)
    if a.dtype not in _DTYPE_CODE:
        raise ValueError(f"Unsupported dtype: only bfloat16, float16, and float32 are supported")
    H = a.shape[-1]
    return a.numel() // max(H, 1), H


def _same(a: torch.Tensor, b: torch.Tensor, name: str) -> None:
    _cuda(b, name)
    _contig(b, name)
    if b.shape != a.shape or b.dtype != a.dtype or b.device != a.device:
        raise ValueError(f"{name} must match the first input's shape, dtype and device")


def _gamma(g: torch.Tensor, a: torch.Tensor, H: int, name: str) -> None:
    _cuda(g, name)
    _contig(g, name)
    if g.dtype != a.dtype or g.numel() != H:
        raise ValueError(f"{name} must have size equal to hidden_dim and the input dtype")


def residual_norm_pair(a: torch.Tensor, residual: torch.Tensor, g1: torch.Tensor,
                       g2: torch.Tensor, eps: float = 1e-6):
    """sum = residual + RMSNorm(a)*g1 ; norm = RMSNorm(sum)*g2.  -> (sum, norm)."""
    T, H = _rows(a, "attn_out")
    _same(a, residual, "residual_in")
    _gamma(g1, a, H, "gamma1")
    _gamma(g2, a, H, "gamma2")
    s = torch.empty_like(residual)
    n = torch.empty_like(a)
    check(load().kb_residual_norm_pair(_p(a), _p(residual), _p(g1), _p(g2), _p(s), _p(n), T, H,
                                       float(eps), _DTYPE_CODE[a.dtype], _stream(a.device)),
          "kb_residual_norm_pair")
    return s, n


def add_rms_norm(a: torch.Tensor, b: torch.Tensor, g: torch.Tensor, eps: float = 1e-6,
                 return_sum: bool = False):
    """out = RMSNorm(a + b)*g (the sum rounded to the dtype first).  -> out or (out, sum)."""
    T, H = _rows(a, "routed_out")
    _same(a, b, "shared_out")
    _gamma(g, a, H, "gamma")
    out = torch.empty_like(a)
    s = torch.empty_like(a) if return_sum else None
    check(load().kb_add_rms_norm(_p(a), _p(b), _p(g), _p(out), _p(s), T, H, float(eps),
                                 _DTYPE_CODE[a.dtype], _stream(a.device)), "kb_add_rms_norm")
    return (out, s) if return_sum else out
