"""Seeded synthetic inputs with the shapes and distributions of the benchmark configurations.

All tensors are drawn on the CPU from torch.Generator().manual_seed(seed) in a fixed order
and then copied where needed, so CPU checkers and GPU kernels see bit-identical inputs.
The reference measures on real Kolibri-1 weights and activations (downloaded from the Hub
by benchmarks/weights_loader.py); there is no network here, so these stand in for them.

  router     logits fp32 [T, 384] ~ N(0,1), bias fp32 [384] ~ N(0, 0.1)
  qk         q bf16 [T, 64, 128], k bf16 [T, 8, 128] ~ N(0,1); gammas bf16 [128] ~ 1+N(0,0.02);
             positions int32 uniform in [0, 8192)
  norms      attn_out, residual bf16 [T, 6144] ~ N(0,1); moe_out ~ N(0, 0.5);
             four gammas bf16 [6144] ~ 1+N(0,0.02)
  chain      per layer a router weight W_g bf16 [6144, 384] ~ N(0, 0.02)
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch

NUM_EXPERTS = 384
TOP_K = 6
HIDDEN = 6144
HQ, HKV, HEAD_DIM = 64, 8, 128
EPS = 1e-6
ROPE_THETA = 10000.0
MAX_POSITION = 8192
NUM_LAYERS = 50


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def router_inputs(T: int, seed: int = 0, E: int = NUM_EXPERTS):
    g = _gen(seed)
    logits = torch.randn(T, E, generator=g, dtype=torch.float32)
    bias = 0.1 * torch.randn(E, generator=g, dtype=torch.float32)
    return logits, bias


def qk_inputs(T: int, seed: int = 2, hq: int = HQ, hkv: int = HKV, d: int = HEAD_DIM):
    g = _gen(seed)
    q = torch.randn(T, hq, d, generator=g).to(torch.bfloat16)
    k = torch.randn(T, hkv, d, generator=g).to(torch.bfloat16)
    gq = (1.0 + 0.02 * torch.randn(d, generator=g)).to(torch.bfloat16)
    gk = (1.0 + 0.02 * torch.randn(d, generator=g)).to(torch.bfloat16)
    pos = torch.randint(0, MAX_POSITION, (T,), generator=g, dtype=torch.int32)
    return q, k, gq, gk, pos


@dataclass
class NormInputs:
    attn_out: torch.Tensor
    residual: torch.Tensor
    moe_out: torch.Tensor
    g_post_attn: torch.Tensor
    g_pre_moe: torch.Tensor
    g_post_moe: torch.Tensor
    g_pre_attn: torch.Tensor


def norm_inputs(T: int, seed: int = 3, H: int = HIDDEN) -> NormInputs:
    g = _gen(seed)
    attn_out = torch.randn(T, H, generator=g).to(torch.bfloat16)
    residual = torch.randn(T, H, generator=g).to(torch.bfloat16)
    moe_out = (0.5 * torch.randn(T, H, generator=g)).to(torch.bfloat16)
    gammas = [(1.0 + 0.02 * torch.randn(H, generator=g)).to(torch.bfloat16) for _ in range(4)]
    return NormInputs(attn_out, residual, moe_out, *gammas)


def router_weight(layer: int, seed: int = 4, H: int = HIDDEN, E: int = NUM_EXPERTS):
    g = _gen(seed * 1000 + layer)
    return (0.02 * torch.randn(H, E, generator=g)).to(torch.bfloat16)


def is_rnope_layer(layer: int) -> bool:
    """Every fifth layer is full attention without RoPE (config.json layer_types)."""
    return (layer + 1) % 5 == 0


def digest(*tensors: torch.Tensor) -> str:
    """SHA-256 over the raw bytes of CPU tensors (input pinning for golden fixtures)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous().cpu()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.view(torch.int16).numpy().tobytes())
    return h.hexdigest()
