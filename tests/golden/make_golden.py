"""Generate the golden fixtures in this directory from the reference's own eager code.

Run with the reference checkout named by the KOLIBRI_REFERENCE environment variable
(required; there is no default path):

    KOLIBRI_REFERENCE=<path to the profiling-moe checkout> python tests/golden/make_golden.py

The reference scripts import CUDA extensions at module level, so each eager function is
pulled out of its source file with `ast` (only that function's definition is executed) and
run on the CPU at the benchmark seeds.  Inputs are regenerated from seeds on the test side;
the fixtures store a SHA-256 of them so that a generator change fails loudly.

Functions used (paths relative to the reference root):
  benchmarks/01_benchmark_router.py            eager_kolibri_router          (router)
  benchmarks/08_benchmark_router_dispatch.py   eager_kolibri_router, eager_router_dispatch
  benchmarks/09_benchmark_build_expert_maps.py eager_build_expert_maps       (offsets)
  fusions/01_sandwich_norm/baseline/trtllm_baseline.py  eager_pytorch_baseline (sandwich)
  fusions/02_post_moe_norm/baseline/trtllm_baseline.py  eager_pytorch_baseline (post-MoE)
  scratch/diag_rope_fusion.py                  ref                            (Q/K norm + RoPE)
  benchmarks/11_profile_2block_e2e.py:195-196  per-head F.rms_norm (RNoPE), :229-231 and
                                               :269-270 (post-MoE + pre-attention pair)
"""
from __future__ import annotations

import ast
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "profiling-moe_b200"))
from kolibri_b200 import workloads as wl  # noqa: E402

def _reference_root() -> Path:
    root = os.environ.get("KOLIBRI_REFERENCE")
    if not root:
        raise SystemExit("set KOLIBRI_REFERENCE to the reference checkout (no default path)")
    return Path(root)


REF = _reference_root()


def extract(rel: str, name: str, extra_globals: dict | None = None):
    """Compile only `def name(...)` from a reference source file and return the function."""
    src = (REF / rel).read_text()
    tree = ast.parse(src)
    node = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == name)
    node.decorator_list = []
    mod = ast.Module(body=[node], type_ignores=[])
    g = {"torch": torch, "F": F, "Tuple": tuple}
    if extra_globals:
        g.update(extra_globals)
    exec(compile(mod, f"{rel}:{name}", "exec"), g)
    return g[name]


class _CpuTorch(types.SimpleNamespace):
    """torch with device='cuda' dropped from arange (the RoPE reference builds its
    frequency table on the GPU; the arithmetic is the same on the CPU)."""

    def __getattr__(self, item):
        return getattr(torch, item)

    @staticmethod
    def arange(*args, device=None, **kw):
        return torch.arange(*args, **kw)


def main() -> None:
    out = {}

    # ---------------- router, config 0 (T=128, seed 0) ----------------
    eager01 = extract("benchmarks/01_benchmark_router.py", "eager_kolibri_router")
    eager08 = extract("benchmarks/08_benchmark_router_dispatch.py", "eager_kolibri_router")
    logits, bias = wl.router_inputs(128, seed=0)
    ids, w = eager01(logits, bias, 6)
    w08, ids08 = eager08(logits, bias, topk=6)
    assert torch.equal(ids, ids08) and torch.equal(w, w08)
    np.savez_compressed(HERE / "router_c0.npz", inputs_sha=wl.digest(logits, bias),
                        ids=ids.to(torch.int32).numpy(), w=w.numpy())
    out["router_c0"] = ids.shape

    # ---------------- expert maps, config 1 (seed 1), T in {1, 64, 4096} ----------------
    disp08 = extract("benchmarks/08_benchmark_router_dispatch.py", "eager_router_dispatch",
                     {"eager_kolibri_router": eager08})
    maps09 = extract("benchmarks/09_benchmark_build_expert_maps.py", "eager_build_expert_maps")
    for T in (1, 64, 4096):
        logits, bias = wl.router_inputs(T, seed=1)
        ids, _ = eager01(logits, bias, 6)
        x = torch.arange(T, dtype=torch.float32)[:, None].repeat(1, 2)  # hidden 2: row id
        perm_x, perm_w, p2u08, off08 = disp08(x, logits, bias, topk=6, num_experts=384)
        off09 = maps09(ids.to(torch.int32).to(torch.int64), num_experts=384, topk=6)
        assert torch.equal(off08, off09)
        np.savez_compressed(HERE / f"maps_c1_T{T}.npz", inputs_sha=wl.digest(logits, bias),
                            ids=ids.to(torch.int32).numpy(), offsets=off09.numpy(),
                            p2u_expert_slot_token=p2u08.numpy(),
                            permuted_weights=perm_w.numpy(),
                            permuted_token=perm_x[:, 0].to(torch.int64).numpy())
        out[f"maps_c1_T{T}"] = off09.shape

    # ---------------- Q/K norm + RoPE, config 2 (seed 2), T=4 ----------------
    T = 4
    q, k, gq, gk, pos = wl.qk_inputs(T, seed=2)
    D = wl.HEAD_DIM
    pc = types.SimpleNamespace(rms_norm_eps=wl.EPS, rope_theta=wl.ROPE_THETA)

    def diag_ref(positions):
        return extract("scratch/diag_rope_fusion.py", "ref",
                       {"torch": _CpuTorch(), "b": T, "D": D, "pc": pc, "pos": positions})

    ref_swa = diag_ref(pos)
    q_swa = ref_swa(q.reshape(T, -1), wl.HQ, gq).view(T, wl.HQ, D)
    k_swa = ref_swa(k.reshape(T, -1), wl.HKV, gk).view(T, wl.HKV, D)
    ref_zero = diag_ref(torch.zeros(T, dtype=torch.int32))
    q_zero = ref_zero(q.reshape(T, -1), wl.HQ, gq).view(T, wl.HQ, D)
    k_zero = ref_zero(k.reshape(T, -1), wl.HKV, gk).view(T, wl.HKV, D)
    # RNoPE as the harness computes it: per-head F.rms_norm (no rotation).
    q_rn = F.rms_norm(q.view(T, wl.HQ, D), (D,), gq, wl.EPS)
    k_rn = F.rms_norm(k.view(T, wl.HKV, D), (D,), gk, wl.EPS)
    assert torch.equal(q_zero, q_rn) and torch.equal(k_zero, k_rn)
    np.savez_compressed(HERE / "qk_c2_T4.npz", inputs_sha=wl.digest(q, k, gq, gk, pos),
                        q_swa=q_swa.view(torch.int16).numpy(), k_swa=k_swa.view(torch.int16).numpy(),
                        q_rnope=q_rn.view(torch.int16).numpy(), k_rnope=k_rn.view(torch.int16).numpy())
    out["qk_c2_T4"] = q_swa.shape

    # ---------------- sandwich + post-MoE norms, config 3 (seed 3), T=2 ----------------
    T = 2
    ni = wl.norm_inputs(T, seed=3)
    sand = extract("fusions/01_sandwich_norm/baseline/trtllm_baseline.py", "eager_pytorch_baseline")
    post = extract("fusions/02_post_moe_norm/baseline/trtllm_baseline.py", "eager_pytorch_baseline")
    h, x = sand(ni.attn_out, ni.residual, ni.g_post_attn, ni.g_pre_moe, eps=wl.EPS)
    moe = post(ni.attn_out, ni.moe_out, ni.g_post_moe, eps=wl.EPS)
    # post-MoE + next layer's input_layernorm (harness :269-270 then :229-231)
    d = wl.HIDDEN
    o = h + F.rms_norm(ni.moe_out, (d,), ni.g_post_moe, wl.EPS)
    nxt = F.rms_norm(o, (d,), ni.g_pre_attn, wl.EPS)
    sha = wl.digest(ni.attn_out, ni.residual, ni.moe_out, ni.g_post_attn, ni.g_pre_moe,
                    ni.g_post_moe, ni.g_pre_attn)
    np.savez_compressed(HERE / "norms_c3_T2.npz", inputs_sha=sha,
                        sandwich_h=h.view(torch.int16).numpy(), sandwich_x=x.view(torch.int16).numpy(),
                        add_post_moe=moe.view(torch.int16).numpy(),
                        pair_out=o.view(torch.int16).numpy(), pair_next=nxt.view(torch.int16).numpy())
    out["norms_c3_T2"] = h.shape

    for k_, v in out.items():
        print(f"{k_}: {tuple(v)}")


if __name__ == "__main__":
    main()
