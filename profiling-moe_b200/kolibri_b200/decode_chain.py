"""The 50-layer non-GEMM decode chain of a Kolibri-style MoE decoder on one GPU.

It follows the layer loop of the reference's end-to-end harness
(benchmarks/11_profile_2block_e2e.py:215-280, decoder_layer and forward) restricted to the
stages between the GEMMs, with the layer schedule of config.json:29-80 (every fifth layer is
full attention without RoPE).  Per layer i, on one stream:

  1. sandwich norm      h = r + RMSNorm(attn_out)*g_post_attn ; moe_in = RMSNorm(h)*g_pre_moe
                        (R1_sandwich_norm, :232-234)
  2. Q/K norm + RoPE    q', k' = per-head RMSNorm then NeoX RoPE at the token positions, or
                        the RNoPE identity on full-attention layers (attention(), :190-199)
  3. router GEMM        logits = (moe_in @ W_g[i]).float()        (gate_gemm, :241-242)
  4. router + maps      top-6 of logits + bias, sigmoid weights, counts/offsets/p2u/u2p
                        (R2_moe_prologue, :244-246)
     gate="tcgen05" (default): kb_router_gemm computes 3 and the router of 4 in one launch
     (tensor-core GEMM, routing in its epilogue), then kb_expert_maps builds the maps from the
     ids; gate="cublas": torch.matmul, the cast to fp32 and kb_router_maps, as the reference
     runs it.
  5. expansion          permuted[r] = moe_in[p2u[r] % T]            (R2, optional)
     or, token-sharded over ranks (ep=PeerExpertParallel), the expert-parallel exchange:
                        count all-gather, dispatch of the routed rows to their owners,
                        identity experts, combine back and finalize, whose output is the
                        layer's moe_out (finalize :259-262)
  6. post-MoE + next    r = h + RMSNorm(moe_out)*g_post_ffn ; nxt = RMSNorm(r)*g_input_ln
                        (R3_post_moe_norm :264-266 fused with the next layer's
                        input_layernorm :222-227)

The attention and expert GEMMs are outside this path: attn_out, moe_out and the projected
q/k are fixed synthetic stand-ins (one buffer each, shared by all layers), while the residual
stream r and the router inputs flow from layer to layer, so every layer depends on the one
before.  Every stage is a libkolibri_b200 kernel launched through the C ABI (with gate="cublas"
the router GEMM is torch.matmul instead).  `capture()` records the whole chain in
one CUDA graph; launches keep programmatic-dependent-launch edges inside it.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from . import _lib
from . import ops
from . import workloads as wl


@dataclass
class LayerWeights:
    g_post_attn: torch.Tensor   # bf16 [H]
    g_pre_moe: torch.Tensor     # bf16 [H]
    g_post_ffn: torch.Tensor    # bf16 [H]
    g_input_ln: torch.Tensor    # bf16 [H]  (the next layer's input_layernorm)
    g_q: torch.Tensor           # bf16 [D]
    g_k: torch.Tensor           # bf16 [D]
    w_gate_t: torch.Tensor      # bf16 [E, H] (nn.Linear layout: logits = x @ w_gate_t.T)
    gate_bias: torch.Tensor     # fp32 [E]
    rnope: bool


def make_layers(n_layers: int, device: torch.device, seed: int = 4, H: int = wl.HIDDEN,
                E: int = wl.NUM_EXPERTS, D: int = wl.HEAD_DIM) -> List[LayerWeights]:
    """Random-init layer weights with the benchmark distributions (gammas 1+N(0,0.02),
    W_g N(0,0.02) stored [E, H], gate bias N(0,0.1)), drawn from one generator on `device`."""
    g = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16

    def gamma(n):
        return (1.0 + 0.02 * torch.randn(n, generator=g, device=device)).to(bf)

    layers = []
    for i in range(n_layers):
        layers.append(LayerWeights(
            g_post_attn=gamma(H), g_pre_moe=gamma(H), g_post_ffn=gamma(H), g_input_ln=gamma(H),
            g_q=gamma(D), g_k=gamma(D),
            w_gate_t=(0.02 * torch.randn(E, H, generator=g, device=device)).to(bf).contiguous(),
            gate_bias=(0.1 * torch.randn(E, generator=g, device=device)).contiguous(),
            rnope=wl.is_rnope_layer(i)))
    return layers


class DecodeChain:
    """Buffers and launch sequence of the chain for a fixed batch of T tokens."""

    def __init__(self, T: int, layers: List[LayerWeights], device: torch.device,
                 seed: int = 5, expansion: bool = True, gate_gemm: bool = True,
                 H: int = wl.HIDDEN, Hq: int = wl.HQ, Hkv: int = wl.HKV, D: int = wl.HEAD_DIM,
                 E: int = wl.NUM_EXPERTS, K: int = wl.TOP_K, eps: float = wl.EPS,
                 theta: float = wl.ROPE_THETA, ep=None, gate: str = "tcgen05"):
        self.T, self.H, self.Hq, self.Hkv, self.D, self.E, self.K = T, H, Hq, Hkv, D, E, K
        self.eps, self.layers, self.device = float(eps), layers, device
        self.expansion, self.gate_gemm = expansion and ep is None, gate_gemm
        if gate not in ("tcgen05", "cublas"):
            raise ValueError("gate must be 'tcgen05' or 'cublas'")
        self.gate = gate if gate_gemm else None
        self.ep = ep
        if ep is not None and (ep.H != H or ep.E != E or ep.K != K or
                               T > ep.pg.max_tokens or ep.dtype != torch.bfloat16):
            raise ValueError("the expert-parallel group does not match the chain's shapes")
        self.lib = _lib.load()
        g = torch.Generator(device=device).manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape, scale=1.0):
            return (scale * torch.randn(*shape, generator=g, device=device)).to(bf).contiguous()

        # Synthetic stand-ins for the GEMM outputs, and the residual stream.
        self.attn_out = rnd(T, H)
        self.moe_out = rnd(T, H, scale=0.5)
        self.q = rnd(T, Hq, D)
        self.k = rnd(T, Hkv, D)
        self.pos = torch.randint(0, wl.MAX_POSITION, (T,), generator=g, device=device,
                                 dtype=torch.int32)
        self.r0 = rnd(T, H)
        self.r = torch.empty_like(self.r0)
        self.h = torch.empty_like(self.r0)
        self.moe_in = torch.empty_like(self.r0)
        self.nxt = torch.empty_like(self.r0)
        self.q_out = torch.empty_like(self.q)
        self.k_out = torch.empty_like(self.k)
        self.logits_bf = torch.empty(T, E, dtype=bf, device=device)
        # Without the gate GEMM the router reads fixed logits (non-GEMM-only timing).
        self.logits = (torch.randn(T, E, generator=g, device=device) if not gate_gemm
                       else torch.empty(T, E, dtype=torch.float32, device=device))
        self.ids = torch.empty(T, K, dtype=torch.int32, device=device)
        self.w = torch.empty(T, K, dtype=torch.float32, device=device)
        self.counts = torch.empty(E, dtype=torch.int32, device=device)
        self.offsets = torch.empty(E + 1, dtype=torch.int64, device=device)
        self.p2u = torch.empty(T * K, dtype=torch.int32, device=device)
        self.u2p = torch.empty(T * K, dtype=torch.int32, device=device)
        self.permuted = torch.empty(T * K, H, dtype=bf, device=device) if self.expansion else None
        self.moe_out_ep = torch.empty(T, H, dtype=bf, device=device) if ep is not None else None
        self.ws_bytes = int(max(self.lib.kb_router_maps_workspace_bytes(T, E, K),
                                self.lib.kb_expert_maps_workspace_bytes(T, E, K)))
        self.ws = torch.zeros(max(self.ws_bytes, 256), dtype=torch.uint8, device=device)
        self.gws_bytes = (int(self.lib.kb_router_gemm_workspace_bytes(T, H, E, K))
                          if self.gate == "tcgen05" else 0)
        self.gws = (torch.zeros(self.gws_bytes, dtype=torch.uint8, device=device)
                    if self.gws_bytes else None)
        self.inv_freq = ops.rope_inv_freq(theta, D, device)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    # ------------------------------------------------------------------------------------
    def launches_per_layer(self) -> int:
        """Kernels of this library launched per layer (the cuBLAS GEMM and cast excluded)."""
        _, launches, _ = self._describe(route=self.gate != "tcgen05" or self.ep is not None)
        # the exchange: dispatch, combine send + finalize (the count all-gather rides on the
        # router + maps launch on its single-CTA and tile paths, one more launch elsewhere)
        extra = 0
        if self.ep is not None:
            p, _, grid = self._describe()      # the tile path reports KB_MAPS_MULTI_CTA
            fused = p == _lib.KB_MAPS_SINGLE_CTA or (p == _lib.KB_MAPS_MULTI_CTA and
                                                      grid >= self.ep.world)
            extra = 3 + (0 if fused else 1)
        gate = 1 if self.gate == "tcgen05" else 0     # kb_router_gemm
        return 3 + gate + launches + (1 if self.expansion else 0) + extra

    def _describe(self, route: bool = True):
        import ctypes
        p, n, gsz = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.check(self.lib.kb_maps_describe(self.T, self.E, self.K, int(route), _lib.KB_MAPS_AUTO,
                                             ctypes.byref(p), ctypes.byref(n), ctypes.byref(gsz)),
                   "kb_maps_describe")
        return p.value, n.value, gsz.value

    def run_layers(self, stream: torch.cuda.Stream,
                   record: Optional[Callable[[int, str, dict], None]] = None) -> None:
        """Enqueue the whole chain on `stream`.  record(i, stage, tensors) is called after
        each stage with the stage's inputs and outputs (eager runs only)."""
        lib, T, H, E, K = self.lib, self.T, self.H, self.E, self.K
        st = stream.cuda_stream
        bf16 = _lib.KB_BF16
        with torch.cuda.stream(stream):
            self.r.copy_(self.r0)
            for i, L in enumerate(self.layers):
                if record:
                    r_in = self.r.clone()
                _lib.check(lib.kb_residual_norm_pair(
                    self.attn_out.data_ptr(), self.r.data_ptr(), L.g_post_attn.data_ptr(),
                    L.g_pre_moe.data_ptr(), self.h.data_ptr(), self.moe_in.data_ptr(), T, H,
                    self.eps, bf16, st), "kb_residual_norm_pair")
                if record:
                    record(i, "sandwich", dict(a=self.attn_out, residual=r_in, g1=L.g_post_attn,
                                               g2=L.g_pre_moe, sum=self.h, norm=self.moe_in))
                pos = None if L.rnope else self.pos
                inv = None if L.rnope else self.inv_freq
                _lib.check(lib.kb_qk_norm_rope(
                    self.q.data_ptr(), self.q_out.data_ptr(), self.k.data_ptr(),
                    self.k_out.data_ptr(), L.g_q.data_ptr(), L.g_k.data_ptr(),
                    None if pos is None else pos.data_ptr(),
                    None if inv is None else inv.data_ptr(), T, self.Hq, self.Hkv, self.D,
                    self.Hq * self.D, self.Hkv * self.D, self.eps, st), "kb_qk_norm_rope")
                if record:
                    record(i, "qk", dict(q=self.q, k=self.k, gq=L.g_q, gk=L.g_k, pos=pos,
                                         q_out=self.q_out, k_out=self.k_out))
                routed = False   # ids and weights already written by kb_router_gemm
                if self.gate == "cublas":
                    torch.matmul(self.moe_in, L.w_gate_t.t(), out=self.logits_bf)
                    self.logits.copy_(self.logits_bf)
                elif self.gate == "tcgen05":
                    routed = self.ep is None
                    _lib.check(lib.kb_router_gemm(
                        self.moe_in.data_ptr(), L.w_gate_t.data_ptr(), L.gate_bias.data_ptr(),
                        self.logits.data_ptr(), self.ids.data_ptr() if routed else None,
                        self.w.data_ptr() if routed else None, self.gws.data_ptr(),
                        self.gws_bytes, T, H, E, K, 0, st), "kb_router_gemm")
                if self.gate_gemm and record:
                    record(i, "gate", dict(x=self.moe_in, w=L.w_gate_t.t(), logits=self.logits))
                if routed:
                    _lib.check(lib.kb_expert_maps(
                        self.ids.data_ptr(), self.counts.data_ptr(), self.offsets.data_ptr(),
                        self.p2u.data_ptr(), self.u2p.data_ptr(), self.ws.data_ptr(),
                        self.ws_bytes, T, E, K, _lib.KB_MAPS_AUTO, st), "kb_expert_maps")
                elif self.ep is None:
                    _lib.check(lib.kb_router_maps(
                        self.logits.data_ptr(), L.gate_bias.data_ptr(), self.ids.data_ptr(),
                        self.w.data_ptr(), self.counts.data_ptr(), self.offsets.data_ptr(),
                        self.p2u.data_ptr(), self.u2p.data_ptr(), self.ws.data_ptr(),
                        self.ws_bytes, T, E, K, 0, _lib.KB_MAPS_AUTO, st), "kb_router_maps")
                else:   # the count all-gather of the exchange rides on the same launch
                    _lib.check(lib.kb_router_maps_allgather(
                        self.ep.pg.addr, self.logits.data_ptr(), L.gate_bias.data_ptr(),
                        self.ids.data_ptr(), self.w.data_ptr(), self.counts.data_ptr(),
                        self.offsets.data_ptr(), self.p2u.data_ptr(), self.u2p.data_ptr(),
                        self.ws.data_ptr(), self.ws_bytes, T, 0, _lib.KB_MAPS_AUTO,
                        self.ep.gathered.data_ptr(), st), "kb_router_maps_allgather")
                if record:
                    record(i, "router_maps", dict(logits=self.logits, bias=L.gate_bias,
                                                  ids=self.ids, w=self.w, counts=self.counts,
                                                  offsets=self.offsets, p2u=self.p2u,
                                                  u2p=self.u2p))
                if self.expansion:
                    _lib.check(lib.kb_expand_rows(self.moe_in.data_ptr(),
                                                  self.permuted.data_ptr(), self.p2u.data_ptr(),
                                                  T, T * K, H * 2, st), "kb_expand_rows")
                    if record:
                        record(i, "expansion", dict(x=self.moe_in, p2u=self.p2u,
                                                    permuted=self.permuted))
                moe_out = self.moe_out
                if self.ep is not None:
                    ep = self.ep
                    _lib.check(lib.kb_ep_dispatch(ep.pg.addr, self.moe_in.data_ptr(), T,
                                                  self.p2u.data_ptr(), ep.gathered.data_ptr(),
                                                  ep.recv_offsets.data_ptr(), st),
                               "kb_ep_dispatch")
                    # identity experts: the owner returns the rows it received
                    _lib.check(lib.kb_ep_combine(ep.pg.addr, ep.rows.data_ptr(),
                                                 ep.gathered.data_ptr(), T, self.u2p.data_ptr(),
                                                 self.w.data_ptr(), self.moe_out_ep.data_ptr(),
                                                 bf16, st), "kb_ep_combine")
                    moe_out = self.moe_out_ep
                    if record:
                        record(i, "ep", dict(x=self.moe_in, u2p=self.u2p, w=self.w,
                                             p2u=self.p2u, out=self.moe_out_ep))
                if record:
                    h_in = self.h.clone()
                _lib.check(lib.kb_residual_norm_pair(
                    moe_out.data_ptr(), self.h.data_ptr(), L.g_post_ffn.data_ptr(),
                    L.g_input_ln.data_ptr(), self.r.data_ptr(), self.nxt.data_ptr(), T, H,
                    self.eps, bf16, st), "kb_residual_norm_pair")
                if record:
                    record(i, "post_moe", dict(a=moe_out, residual=h_in, g1=L.g_post_ffn,
                                               g2=L.g_input_ln, sum=self.r, norm=self.nxt))

    # ------------------------------------------------------------------------------------
    # The whole chain in one launch (kb_decode_chain), for T <= 4.
    # ------------------------------------------------------------------------------------
    MEGA_MAX_T = 4

    def _mega_setup(self):
        if getattr(self, "_mega", None) is not None:
            return self._mega
        import ctypes
        descs = (_lib.ChainLayer * len(self.layers))()
        for i, L in enumerate(self.layers):
            descs[i] = _lib.ChainLayer(
                L.g_post_attn.data_ptr(), L.g_pre_moe.data_ptr(), L.g_post_ffn.data_ptr(),
                L.g_input_ln.data_ptr(), L.g_q.data_ptr(), L.g_k.data_ptr(),
                L.w_gate_t.data_ptr(), L.gate_bias.data_ptr(), int(L.rnope), 0)
        raw = torch.frombuffer(bytearray(ctypes.string_at(descs, ctypes.sizeof(descs))),
                               dtype=torch.uint8)
        dev_descs = raw.to(self.device)
        ws = torch.zeros(int(self.lib.kb_decode_chain_workspace_bytes()), dtype=torch.uint8,
                         device=self.device)
        self._mega = (dev_descs, ws)
        return self._mega

    def run_mega(self, stream: torch.cuda.Stream, trace: Optional[torch.Tensor] = None) -> None:
        """Enqueue the whole chain as one kb_decode_chain launch on `stream` (T <= 4).
        trace: optional fp32 [layers, T, E] receiving every layer's logits."""
        if self.T > self.MEGA_MAX_T:
            raise ValueError(f"kb_decode_chain takes at most {self.MEGA_MAX_T} tokens")
        descs, ws = self._mega_setup()
        P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        with torch.cuda.stream(stream):
            _lib.check(self.lib.kb_decode_chain(
                descs.data_ptr(), len(self.layers), P(self.attn_out), P(self.moe_out), P(self.q),
                P(self.k), P(self.pos), P(self.inv_freq), P(self.r0), P(self.r), P(self.h),
                P(self.moe_in), P(self.nxt), P(self.q_out), P(self.k_out), P(self.logits),
                P(self.ids), P(self.w), P(self.counts), P(self.offsets), P(self.p2u), P(self.u2p),
                P(self.permuted), P(trace), ws.data_ptr(), ws.numel(), self.T, self.H, self.Hq,
                self.Hkv, self.D, self.E, self.K, self.eps, stream.cuda_stream),
                "kb_decode_chain")

    def capture(self, stream: torch.cuda.Stream) -> torch.cuda.CUDAGraph:
        """Run the chain once eagerly (library set-up, cuBLAS handles), then record it in one
        CUDA graph on `stream`."""
        self.run_layers(stream)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self.run_layers(stream)
        self.graph = g
        return g
