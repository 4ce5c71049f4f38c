"""causal_conv1d on B200: drop-in for kernels/causal_conv1d/kernel.py."""
from .kernel import SHAPE_CONFIGS, custom_kernel

__all__ = ["custom_kernel", "SHAPE_CONFIGS"]
