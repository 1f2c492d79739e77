# Re-export, as the reference's kernels/kolibri_cuda_router.py does.
from .cuda.kolibri_cuda_router import kolibri_cuda_ops

__all__ = ["kolibri_cuda_ops"]
