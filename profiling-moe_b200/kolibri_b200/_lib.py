"""ctypes binding of libkolibri_b200.so (the C ABI declared in include/kolibri_b200.h).

Loading never falls back to anything: a missing or unloadable library raises, so a GPU
path cannot silently run without the CUDA kernels.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libkolibri_b200.so"

KB_OK = 0
KB_ERR_INVALID_ARG = -1
KB_ERR_UNSUPPORTED = -2
KB_ERR_ALIGNMENT = -3
KB_ERR_WORKSPACE = -4
KB_ERR_TOO_LARGE = -5
KB_ERR_SCRATCH_LIMIT = -6
KB_NOALLOC_REZERO = 1
KB_WS_MAPS, KB_WS_CHAIN, KB_WS_NOALLOC, KB_WS_EP, KB_WS_RGEMM = 0, 1, 2, 3, 4
KB_WS_CLEAN, KB_WS_TIMEOUT, KB_WS_MISALIGNED, KB_WS_CAPACITY = 0, 1, 2, 3
KB_MAX_RANKS = 8
KB_IPC_HANDLE_BYTES = 64

KB_BF16, KB_F16, KB_F32 = 0, 1, 2
KB_MAPS_AUTO, KB_MAPS_SINGLE_CTA, KB_MAPS_MULTI_CTA, KB_MAPS_TWO_KERNEL = 0, 1, 2, 3
KB_MAPS_HYBRID_ROUTER, KB_MAPS_WARP_ROUTER = 4, 5

# name -> (restype, argtypes); must match include/kolibri_b200.h one for one.
SIGNATURES = {
    "kb_status_str": (c_char_p, [c_int]),
    "kb_version": (c_int, []),
    "kb_set_pdl": (c_int, [c_int]),
    "kb_workspace_status": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "kb_set_wait_limit": (c_int64, [c_int64]),
    "kb_router": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int, c_int,
                          c_int, c_void_p]),
    "kb_expert_maps_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "kb_expert_maps": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_size_t, c_int64, c_int, c_int, c_int, c_void_p]),
    "kb_router_maps_workspace_bytes": (c_size_t, [c_int64, c_int, c_int]),
    "kb_router_maps": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_size_t, c_int64, c_int, c_int,
                               c_int, c_int, c_void_p]),
    "kb_router_gemm_workspace_bytes": (c_size_t, [c_int64, c_int, c_int, c_int]),
    "kb_router_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                               c_void_p, c_size_t, c_int64, c_int, c_int, c_int, c_int,
                               c_void_p]),
    "kb_router_gemm_describe": (c_int, [c_int64, c_int, c_int, c_int, c_void_p, c_void_p,
                                        c_void_p]),
    "kb_maps_describe": (c_int, [c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                 c_void_p]),
    "kb_expert_maps_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int64, c_int, c_int, c_int, c_void_p]),
    "kb_moe_finalize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int64,
                                c_int, c_void_p]),
    "kb_expand_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                               c_void_p]),
    "kb_expand_rows_scaled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int64, c_int, c_int64, c_void_p]),
    "kb_qk_norm_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_int64,
                                c_int64, c_float, c_void_p]),
    "kb_residual_norm_pair": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_int64, c_int64, c_float, c_int, c_void_p]),
    "kb_add_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                c_int64, c_float, c_int, c_void_p]),
    "kb_ep_buffer_bytes": (c_size_t, [c_int, c_int, c_int, c_int64, c_int64]),
    "kb_ep_alloc": (c_int, [c_size_t, c_void_p]),
    "kb_ep_free": (c_int, [c_void_p]),
    "kb_ipc_export": (c_int, [c_void_p, c_void_p]),
    "kb_ipc_import": (c_int, [c_void_p, c_void_p]),
    "kb_ipc_close": (c_int, [c_void_p]),
    "kb_ep_counts_allgather": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "kb_router_maps_allgather": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_size_t, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "kb_ep_dispatch": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                               c_void_p]),
    "kb_ep_recv_rows": (c_int, [c_void_p, c_void_p]),
    "kb_ep_barrier": (c_int, [c_void_p, c_void_p]),
    "kb_ep_combine": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                              c_void_p, c_int, c_void_p]),
    "kb_decode_chain_workspace_bytes": (c_size_t, []),
    "kb_decode_chain": (c_int, [c_void_p, c_int] + [c_void_p] * 22 + [c_void_p, c_size_t, c_int64,
                                c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_void_p]),
}


class ChainLayer(ctypes.Structure):
    """kb_chain_layer_t: one layer's weights for kb_decode_chain (device pointers)."""
    _fields_ = [("g_post_attn", c_void_p), ("g_pre_moe", c_void_p), ("g_post_ffn", c_void_p),
                ("g_input_ln", c_void_p), ("g_q", c_void_p), ("g_k", c_void_p),
                ("w_gate_t", c_void_p), ("gate_bias", c_void_p), ("rnope", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class EpGroup(ctypes.Structure):
    """kb_ep_group_t: the ranks' exchange buffers as mapped in this process."""
    _fields_ = [("world", c_int), ("rank", c_int), ("num_experts", c_int), ("top_k", c_int),
                ("max_tokens", c_int64), ("row_bytes", c_int64),
                ("buf", c_void_p * KB_MAX_RANKS)]


class KolibriError(RuntimeError):
    """A libkolibri_b200 entry point returned a non-zero status."""

    def __init__(self, what: str, status: int, message: str):
        super().__init__(f"{what}: {message} (status {status})")
        self.status = status


_LIB = None


def load() -> ctypes.CDLL:
    """Load the shared library once and declare every signature."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -m kolibri_b200.build` "
                "(or __graft_entry__.build())")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def check(status: int, what: str) -> None:
    if status != KB_OK:
        raise KolibriError(what, status, load().kb_status_str(status).decode())


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)
