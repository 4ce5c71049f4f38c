"""Depthwise causal 1D convolution on B200 (sm_100a CUDA via the C ABI).

Drop-in for the reference's ``kernels/causal_conv1d/kernel.py``: same
``custom_kernel(data)`` contract (kernel.py:170-230) -- ``data = (x, weight,
bias)`` with x [B, D, S], weight [D, W], bias [D], all contiguous float32 on
the GPU; returns a new float32 [B, D, S] tensor; asserts like the reference.

``SHAPE_CONFIGS`` keeps the reference's keys (kernel.py:136-151) so tools that
import or patch it keep working. Launch shapes are chosen in C++ (one thread
per 8 outputs, 256 threads per block); the table records that choice and is
not read at launch.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from theorem_b200 import ops

__all__ = ["custom_kernel", "SHAPE_CONFIGS"]

_CFG = {"OUTPUTS_PER_THREAD": 8, "THREADS": 256}
SHAPE_CONFIGS: Dict[Tuple[int, int, int, int], dict] = {
    (1, 64, 64, 4): dict(_CFG), (2, 128, 128, 4): dict(_CFG), (1, 256, 256, 3): dict(_CFG),
    (1, 128, 64, 8): dict(_CFG), (4, 64, 128, 4): dict(_CFG),
    (1, 1536, 2048, 4): dict(_CFG), (1, 2560, 2048, 4): dict(_CFG), (1, 2560, 4096, 4): dict(_CFG),
}


def custom_kernel(data: tuple) -> torch.Tensor:
    """out[b,d,t] = bias[d] + sum_k weight[d,k] * x[b,d,t-W+1+k] (zero left pad)."""
    x, weight, bias = data
    assert x.is_contiguous(), "x must be contiguous (B, D, S)"
    assert weight.is_contiguous(), "weight must be contiguous (D, W)"
    assert bias.is_contiguous(), "bias must be contiguous (D,)"
    assert x.dtype == torch.float32 == weight.dtype == bias.dtype
    return ops.causal_conv1d(x, weight, bias, activation=None, layout="bds")
