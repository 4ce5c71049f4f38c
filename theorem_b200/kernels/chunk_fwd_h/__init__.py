"""chunk_fwd_h on B200: drop-in for kernels/chunk_fwd_h/kernel.py."""
from .kernel import CHUNK_SIZE, SHAPE_CONFIGS, custom_kernel

__all__ = ["custom_kernel", "SHAPE_CONFIGS", "CHUNK_SIZE"]
