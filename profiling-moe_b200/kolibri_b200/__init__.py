"""kolibri_b200 — sm_100a kernels for the non-GEMM MoE decode path of Kolibri-style layers.

The compute lives in libkolibri_b200.so (C ABI, include/kolibri_b200.h); this package binds
it with ctypes (`_lib`) and wraps it for torch tensors (`ops`).  The reference-compatible
entry points (kernels.*, fusions.*) sit next to this package and call `ops`.
"""
from ._lib import KolibriError, LIB_PATH, load  # noqa: F401
from . import ops  # noqa: F401
from .ops import *  # noqa: F401,F403

__version__ = "1.0.0"
