"""Load every reference-named entry point of this package by file path, the way the
reference's harness loads its fusions (benchmarks/11_profile_2block_e2e.py:72-88): the
fusion directories start with digits and are not importable as packages.

    from kolibri_b200.api import load_api
    api = load_api()
    api.fused_sandwich_norm(...), api.fused_moe_prologue(...), api.fused_kolibri_router(...)
"""
from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

_MODULES = {
    "fused_sandwich_norm": "fusions/01_sandwich_norm/fused/fused_sandwich_norm.py",
    "fused_post_moe_norm": "fusions/02_post_moe_norm/fused/fused_post_moe_norm.py",
    "fused_moe_prologue": "fusions/03_moe_prologue/fused/fused_moe_prologue.py",
    "fused_qk_norm_rope": "fusions/04_qk_norm_rope/fused/fused_qk_norm_rope.py",
    "kolibri_multi_block_build_expert_maps":
        "kernels/cuda/multi_block_expert_maps/kolibri_multi_block_build_expert_maps.py",
}


def load_module_from_path(name: str, rel: str):
    spec = importlib.util.spec_from_file_location(f"kolibri_b200_api_{name}", ROOT / rel)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load_api() -> types.SimpleNamespace:
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    import kernels
    from kernels.cuda import kolibri_build_expert_maps as kbem
    from kernels.cuda import kolibri_router_dispatch as krd
    from kernels.kolibri_cuda_router import kolibri_cuda_ops

    mods = {k: load_module_from_path(k, v) for k, v in _MODULES.items()}
    ns = types.SimpleNamespace(
        fused_kolibri_router=kernels.fused_kolibri_router,
        kolibri_cuda_ops=kolibri_cuda_ops,
        kolibri_build_expert_maps=kbem.kolibri_build_expert_maps,
        trtllm_build_expert_maps_b32=kbem.trtllm_build_expert_maps_b32,
        kolibri_activation_expansion_cuda=kbem.kolibri_activation_expansion,
        kolibri_multi_block_build_expert_maps=mods["kolibri_multi_block_build_expert_maps"]
        .kolibri_multi_block_build_expert_maps,
        fused_sandwich_norm=mods["fused_sandwich_norm"].fused_sandwich_norm,
        fused_add_post_moe_norm=mods["fused_post_moe_norm"].fused_add_post_moe_norm,
        fused_post_moe_pre_attn_norm=mods["fused_post_moe_norm"].fused_post_moe_pre_attn_norm,
        kolibri_router=mods["fused_moe_prologue"].kolibri_router,
        kolibri_dispatch_map=mods["fused_moe_prologue"].kolibri_dispatch_map,
        kolibri_activation_expansion=mods["fused_moe_prologue"].kolibri_activation_expansion,
        fused_moe_prologue=mods["fused_moe_prologue"].fused_moe_prologue,
        fused_qk_norm_rope=mods["fused_qk_norm_rope"].fused_qk_norm_rope,
        fused_kolibri_router_dispatch=krd.fused_kolibri_router_dispatch,
        apply_qk_norm_rope_qkv=mods["fused_qk_norm_rope"].apply_qk_norm_rope_qkv,
    )
    return ns
