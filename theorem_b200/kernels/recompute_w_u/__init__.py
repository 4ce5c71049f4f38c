"""recompute_w_u on B200: drop-in for kernels/recompute_w_u/kernel.py."""
from .kernel import BT, SHAPE_CONFIGS, SHAPE_LIST, custom_kernel

__all__ = ["custom_kernel", "SHAPE_CONFIGS", "SHAPE_LIST", "BT"]
