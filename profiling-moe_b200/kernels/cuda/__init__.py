from .kolibri_cuda_router import kolibri_cuda_ops

__all__ = ["kolibri_cuda_ops"]
