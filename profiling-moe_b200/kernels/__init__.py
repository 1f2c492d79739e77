"""Drop-in for the reference's `kernels` package (kernels/__init__.py): re-exports the router.

The reference's Triton kernel is replaced by the sm_100a CUDA router of libkolibri_b200."""
from . import _root  # noqa: F401
from .fused_kolibri_router import fused_kolibri_router

__all__ = ["fused_kolibri_router"]
