"""chunk_fwd_o on B200: drop-in for kernels/chunk_fwd_o/kernel.py."""
from .kernel import DEFAULT_CONFIG, SHAPE_CONFIGS, custom_kernel

__all__ = ["custom_kernel", "SHAPE_CONFIGS", "DEFAULT_CONFIG"]
