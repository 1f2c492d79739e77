"""C-ABI library checks that need no GPU: it loads, exports exactly what include/kolibri_b200.h
declares, and rejects bad arguments on the host before any CUDA call.  Also checks that the
reference-named Python entry points keep the reference's signatures."""
from __future__ import annotations

import inspect
import re
import subprocess

import pytest

from conftest import REPO
from kolibri_b200 import _lib

HEADER = REPO / "include" / "kolibri_b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^KB_API[^(]*?\b(kb_\w+)\s*\(", text, flags=re.M))


def test_library_built_and_loads():
    assert _lib.LIB_PATH.exists(), "run __graft_entry__.build() first"
    lib = _lib.load()
    assert lib.kb_version() == 10000


def test_exports_match_header():
    declared = header_symbols()
    assert declared == set(_lib.SIGNATURES), "ctypes signatures and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert declared <= exported, f"missing exports: {declared - exported}"
    assert {s for s in exported if s.startswith("kb_")} == declared


def test_status_strings():
    lib = _lib.load()
    for code in (_lib.KB_OK, _lib.KB_ERR_INVALID_ARG, _lib.KB_ERR_UNSUPPORTED,
                 _lib.KB_ERR_ALIGNMENT, _lib.KB_ERR_WORKSPACE, _lib.KB_ERR_TOO_LARGE):
        assert lib.kb_status_str(code)
    with pytest.raises(_lib.KolibriError):
        _lib.check(_lib.KB_ERR_UNSUPPORTED, "x")


def test_host_validation_without_gpu():
    lib = _lib.load()
    # Each call is rejected by argument checks before touching CUDA.
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, -1, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, 4, 384, 40, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, 4, 600, 6, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, 4, 4, 6, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, 4, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert lib.kb_router(None, None, None, None, _lib.KB_F32, 1 << 29, 384, 6, 0, None) == _lib.KB_ERR_TOO_LARGE
    assert lib.kb_expert_maps(None, None, None, None, None, None, 0, 4, 384, 6, 9, None) == _lib.KB_ERR_INVALID_ARG
    assert lib.kb_expand_rows(None, None, None, 4, -1, 16, None) == _lib.KB_ERR_INVALID_ARG
    assert lib.kb_qk_norm_rope(None, None, None, None, None, None, None, None, 1, 64, 8, 96, 0, 0,
                               1e-6, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_residual_norm_pair(None, None, None, None, None, None, 1, 64, 1e-6, 7, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_add_rms_norm(None, None, None, None, None, 1, 0, 1e-6, 0, None) == _lib.KB_ERR_INVALID_ARG
    # kb_router_gemm: (x, w_gate, bias, logits, ids, weights, ws, ws_bytes, T, H, E, K, renorm, st)
    fake = 1 << 20   # never dereferenced: every call below is refused before any launch
    rg = lib.kb_router_gemm
    assert rg(None, fake, None, fake, None, None, fake, 1 << 24, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert rg(fake, fake, None, None, None, None, fake, 1 << 24, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert rg(fake, fake, None, None, fake, None, fake, 1 << 24, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_INVALID_ARG
    assert rg(fake, fake, None, None, fake, fake, fake, 1 << 24, 4, 6144, 384, 9, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert rg(fake, fake, None, None, fake, fake, fake, 1 << 24, 4, 6112, 384, 6, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert rg(fake, fake, None, None, fake, fake, fake, 1 << 24, 4, 6144, 320 + 8, 6, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert rg(fake, fake, None, None, fake, fake, fake, 1 << 24, 4, 6144, 576, 6, 0, None) == _lib.KB_ERR_UNSUPPORTED
    assert rg(fake, fake, None, None, fake, fake, fake, 1 << 24, 1 << 20, 6144, 384, 6, 0, None) == _lib.KB_ERR_TOO_LARGE
    assert rg(fake + 8, fake, None, None, fake, fake, fake, 1 << 24, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_ALIGNMENT
    assert rg(fake, fake, None, None, fake, fake, fake + 16, 1 << 24, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_ALIGNMENT
    need = lib.kb_router_gemm_workspace_bytes(4, 6144, 384, 6)
    assert rg(fake, fake, None, None, fake, fake, fake, need - 256, 4, 6144, 384, 6, 0, None) == _lib.KB_ERR_WORKSPACE


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.kb_expert_maps_workspace_bytes(0, 384, 6) == 0
    prev = 0
    for T in (1, 64, 4096, 65536, 262144):
        ws = lib.kb_router_maps_workspace_bytes(T, 384, 6)
        assert ws >= prev
        prev = ws
    assert lib.kb_expert_maps_workspace_bytes(65536, 384, 6) > 0
    # router GEMM: a fixed 256 KB zero zone, then the split partials and rounded logits (small
    # T) or the tile candidates (more tiles than SMs)
    for T in (1, 32, 256, 4096, 8192, 65536):
        assert lib.kb_router_gemm_workspace_bytes(T, 6144, 384, 6) >= 256 * 1024


def test_reference_signatures(api):
    def params(f):
        return [(n, p.default) for n, p in inspect.signature(f).parameters.items()]

    # kernels/triton/fused_kolibri_router.py:98-104
    assert params(api.fused_kolibri_router) == [
        ("x", inspect.Parameter.empty), ("bias", None), ("k", 6), ("norm_topk_prob", False),
        ("output_dtype", None)]
    assert list(inspect.signature(api.fused_sandwich_norm).parameters) == [
        "attn_out", "residual_in", "gamma1", "gamma2", "eps"]
    assert inspect.signature(api.fused_sandwich_norm).parameters["eps"].default == 1e-5
    assert list(inspect.signature(api.fused_add_post_moe_norm).parameters) == [
        "routed_out", "shared_out", "gamma", "eps"]
    assert list(inspect.signature(api.kolibri_dispatch_map).parameters) == [
        "token_selected_experts", "num_experts", "force_single_block", "force_multi_block"]
    assert list(inspect.signature(api.fused_moe_prologue).parameters)[:3] == [
        "unpermuted_input", "router_logits", "router_bias"]
    assert list(inspect.signature(api.kolibri_router).parameters)[:2] == ["scores", "bias"]
    assert list(inspect.signature(api.kolibri_multi_block_build_expert_maps).parameters) == [
        "token_selected_experts", "num_experts", "max_blocks", "return_inverse_map"]
    for name in ("forward", "forward_vA", "forward_vB", "forward_vFloat4"):
        assert list(inspect.signature(getattr(api.kolibri_cuda_ops, name)).parameters) == [
            "logits", "bias", "topk"]


def test_product_never_imports_oracle():
    pkg = REPO / "profiling-moe_b200"
    for p in pkg.rglob("*.py"):
        src = p.read_text()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", src, re.M), p


def _ep_group(world=2, rank=0, E=384, K=6, max_tokens=64, row_bytes=12288, bufs=None):
    import ctypes
    if bufs is None:
        bufs = [0x100000 * (q + 1) for q in range(min(world, _lib.KB_MAX_RANKS))]  # fakes
    arr = (ctypes.c_void_p * _lib.KB_MAX_RANKS)(*(bufs + [None] * (_lib.KB_MAX_RANKS - len(bufs))))
    g = _lib.EpGroup(world, rank, E, K, max_tokens, row_bytes, arr)
    return g, ctypes.addressof(g)


def test_ep_host_validation_without_gpu():
    """kb_ep_* reject a bad group or bad arguments before any CUDA call."""
    lib = _lib.load()
    g, a = _ep_group(world=9)
    assert lib.kb_ep_counts_allgather(a, 16, 16, None) == _lib.KB_ERR_INVALID_ARG
    g, a = _ep_group(world=2, rank=2)
    assert lib.kb_ep_counts_allgather(a, 16, 16, None) == _lib.KB_ERR_INVALID_ARG
    g, a = _ep_group(world=3, E=384 + 1)                     # E not a multiple of N
    assert lib.kb_ep_counts_allgather(a, 16, 16, None) == _lib.KB_ERR_UNSUPPORTED
    g, a = _ep_group(row_bytes=12290)
    assert lib.kb_ep_dispatch(a, 16, 4, 16, 16, 16, None) == _lib.KB_ERR_ALIGNMENT
    g, a = _ep_group(bufs=[0x100000, 0x100008])              # peer buffer not 256-aligned
    assert lib.kb_ep_dispatch(a, 16, 4, 16, 16, 16, None) == _lib.KB_ERR_ALIGNMENT
    g, a = _ep_group(bufs=[0x100000, 0])
    assert lib.kb_ep_combine(a, 16, 16, 4, 16, 16, 16, _lib.KB_BF16, None) == _lib.KB_ERR_INVALID_ARG
    g, a = _ep_group(max_tokens=64)
    assert lib.kb_ep_dispatch(a, 16, 65, 16, 16, 16, None) == _lib.KB_ERR_INVALID_ARG   # T > max
    assert lib.kb_ep_dispatch(a, 24, 4, 16, 16, 16, None) == _lib.KB_ERR_ALIGNMENT      # x
    assert lib.kb_ep_combine(a, 16, 16, 4, 16, 16, 16, 9, None) == _lib.KB_ERR_UNSUPPORTED
    assert lib.kb_ep_counts_allgather(None, 16, 16, None) == _lib.KB_ERR_INVALID_ARG
    g, a = _ep_group(world=8, max_tokens=1 << 26)             # N*T*K overflows int32
    assert lib.kb_ep_counts_allgather(a, 16, 16, None) == _lib.KB_ERR_TOO_LARGE
    assert lib.kb_ep_alloc(0, None) == _lib.KB_ERR_INVALID_ARG
    assert lib.kb_ipc_export(None, None) == _lib.KB_ERR_INVALID_ARG


def test_ep_buffer_bytes():
    """One rank's buffer: control + tagged counts, N*T*K received rows, T*K returned rows."""
    lib = _lib.load()
    assert lib.kb_ep_buffer_bytes(0, 384, 6, 64, 16) == 0
    assert lib.kb_ep_buffer_bytes(9, 384, 6, 64, 16) == 0
    for N, T in ((1, 1), (2, 512), (8, 4096)):
        b = lib.kb_ep_buffer_bytes(N, 384, 6, T, 12288)
        rows = N * T * 6 + T * 6
        assert rows * 12288 <= b <= rows * 12288 + 2 * 8 * 384 * 8 + 4096
        assert b % 256 == 0


def test_router_gemm_plan():
    """The router GEMM's tile shape on a 148-SM B200 (the library's fallback count without a
    GPU): 192-expert tiles, and enough hidden splits for about one CTA per SM while the grid
    fits the SMs (a cooperative launch); more tiles than SMs take one split."""
    import ctypes
    lib = _lib.load()
    expect = {1: (192, 48, 96), 32: (192, 48, 96), 256: (192, 32, 128), 1024: (192, 8, 128),
              4096: (192, 2, 128), 8192: (192, 1, 128), 20000: (192, 1, 314)}
    for T, want in expect.items():
        bn, ks, grid = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        assert lib.kb_router_gemm_describe(T, 6144, 384, 6, ctypes.byref(bn), ctypes.byref(ks),
                                           ctypes.byref(grid)) == 0
        assert (bn.value, ks.value, grid.value) == want, T
