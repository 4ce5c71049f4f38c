"""Gated-DeltaNet WY recompute of (w, u) on B200 (tcgen05 MMA, TMEM accumulators).

Drop-in for the reference's ``kernels/recompute_w_u/kernel.py``:
``custom_kernel(data)`` takes the reference's ``Data`` (any object with
``k, v, beta, A, g`` attributes; k [B,T,H,K], v [B,T,H,V], beta/g [B,T,H],
A [B,T,H,64], float32, contiguous) and returns the tuple ``(w, u)``
(kernel.py:246-248). ``SHAPE_LIST`` / ``SHAPE_CONFIGS`` keep the reference's
entries (kernel.py:42-67); launch shapes are fixed in C++ (one CTA per
(b, h, 64-chunk), 128 threads) and the table is informational.
"""
from __future__ import annotations

import torch

from theorem_b200 import ops

BT = 64
__all__ = ["custom_kernel", "SHAPE_CONFIGS", "SHAPE_LIST", "BT"]

SHAPE_LIST = [
    {"B": 1, "T": 64, "H": 2, "K": 64, "V": 64},
    {"B": 2, "T": 128, "H": 4, "K": 64, "V": 64},
    {"B": 1, "T": 256, "H": 4, "K": 64, "V": 128},
    {"B": 1, "T": 64, "H": 1, "K": 64, "V": 64},
    {"B": 2, "T": 512, "H": 3, "K": 64, "V": 64},
    {"B": 2, "T": 1024, "H": 3, "K": 64, "V": 64},
]
SHAPE_CONFIGS: dict = {tuple(s.values()): {"CTA_PER": "chunk", "THREADS": 128} for s in SHAPE_LIST}


def custom_kernel(data) -> tuple[torch.Tensor, torch.Tensor]:
    """w = A @ (k * beta * exp(g)), u = A @ (v * beta) per 64-token chunk."""
    k, v, beta, A, g = data.k, data.v, data.beta, data.A, data.g
    assert k.is_contiguous() and v.is_contiguous() and A.is_contiguous()
    assert beta.is_contiguous() and g.is_contiguous()
    return ops.recompute_w_u(k, v, beta, A, g, a_mode=0)
