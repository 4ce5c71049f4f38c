"""Gated-DeltaNet chunkwise output on B200 (tcgen05 MMA, TMEM accumulators).

Drop-in for the reference's ``kernels/chunk_fwd_o/kernel.py``:
``custom_kernel(data)`` with data = dict(q, k [B,T,H,K], v [B,T,H,V],
g [B,T,H], h [B,NT,H,K,V], scale, ...) float32 on the GPU returns
o [B,T,H,V] float32 (kernel.py:146-212). ``SHAPE_CONFIGS`` /
``DEFAULT_CONFIG`` keep the reference's names (kernel.py:38-49; the
autotuner reads DEFAULT_CONFIG); launch shapes are fixed in C++.
"""
from __future__ import annotations

from typing import Any, Dict

import torch

from theorem_b200 import ops

__all__ = ["custom_kernel", "SHAPE_CONFIGS", "DEFAULT_CONFIG"]

DEFAULT_CONFIG: Dict[str, int] = {"BT": 64, "BV": 64, "THREADS": 128}
SHAPE_CONFIGS = {k: dict(DEFAULT_CONFIG) for k in [(1, 64, 1, 64, 64), (2, 128, 4, 64, 64),
                                                   (1, 256, 4, 64, 128), (2, 512, 3, 64, 64),
                                                   (2, 1024, 3, 64, 64)]}


def custom_kernel(data: Dict[str, Any]) -> torch.Tensor:
    q, k, v, g, h = data["q"], data["k"], data["v"], data["g"], data["h"]
    scale = float(data["scale"])
    assert q.is_cuda and k.is_cuda and v.is_cuda and g.is_cuda and h.is_cuda, \
        "all inputs must be on a CUDA device"
    assert q.dtype == torch.float32, "fp32 expected"
    B, T, H, K = q.shape
    NT = h.shape[1]
    assert T % 64 == 0, f"T={T} must be divisible by BT=64"
    assert NT == T // 64, f"NT={NT} must equal T/BT={T // 64}"
    return ops.chunk_fwd_o(q, k, v, g, h, scale)
