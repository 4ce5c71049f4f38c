"""Gated-DeltaNet inter-chunk state recurrence on B200 (state resident in TMEM).

Drop-in for the reference's ``kernels/chunk_fwd_h/kernel.py``:
``custom_kernel(data)`` with data = dict(k [B,T,H,K], v [B,T,H,V],
g [B,T,H], B, T, H, K, V) float32 returns h [B, T/64, H, K, V] float32, the
state after each chunk (kernel.py:141-191). ``SHAPE_CONFIGS`` keeps the
reference's keys (kernel.py:40-48); launch shapes are fixed in C++.
"""
from __future__ import annotations

import torch

from theorem_b200 import ops

CHUNK_SIZE = 64
__all__ = ["custom_kernel", "SHAPE_CONFIGS", "CHUNK_SIZE"]

_KEYS = [(1, 64, 1, 64, 64), (2, 128, 4, 64, 64), (1, 256, 4, 64, 128), (2, 512, 3, 64, 64),
         (2, 1024, 3, 64, 64)]
SHAPE_CONFIGS = {k: {"CTA_PER": "(b,h,V-tile)", "THREADS": 128} for k in _KEYS}


def custom_kernel(data) -> torch.Tensor:
    k, v, g = data["k"], data["v"], data["g"]
    T = data["T"]
    assert T % CHUNK_SIZE == 0, f"T={T} must be divisible by {CHUNK_SIZE}"
    k, v, g = k.contiguous(), v.contiguous(), g.contiguous()
    assert k.dtype == torch.float32
    assert v.dtype == torch.float32
    assert g.dtype == torch.float32
    return ops.chunk_fwd_h(k, v, g, mode=0)
