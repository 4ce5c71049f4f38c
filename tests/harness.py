"""Restatement of the reference harness's comparison (utils.py:30-83, verbose_allclose)
and of eval.py's per-shape test loop (eval.py:85-117), for the GPU parity tests.

A result passes when container type/length, shape and dtype match and every
finite element satisfies |r - e| <= atol + rtol * |e| with identical NaN/Inf
patterns -- the same rule the reference's ``eval.py test`` applies.
"""
from __future__ import annotations

import torch


def verbose_allclose(received, expected, rtol: float, atol: float) -> list[str]:
    if isinstance(received, (tuple, list)) or isinstance(expected, (tuple, list)):
        if type(received) is not type(expected) or len(received) != len(expected):
            return [f"container mismatch: {type(received).__name__} vs {type(expected).__name__}"]
        out = []
        for i, (r, e) in enumerate(zip(received, expected)):
            out += [f"[{i}] {m}" for m in verbose_allclose(r, e, rtol, atol)]
        return out
    if not torch.is_tensor(received) or not torch.is_tensor(expected):
        return [f"type mismatch: {type(received)} vs {type(expected)}"]
    if received.shape != expected.shape:
        return [f"shape mismatch: {tuple(received.shape)} vs {tuple(expected.shape)}"]
    reasons = []
    if received.dtype != expected.dtype:
        reasons.append(f"dtype mismatch: {received.dtype} vs {expected.dtype}")
    r = received.detach().float().cpu()
    e = expected.detach().float().cpu()
    if (torch.isnan(r) ^ torch.isnan(e)).any():
        reasons.append("NaN pattern mismatch")
    if (torch.isinf(r) ^ torch.isinf(e)).any():
        reasons.append("Inf pattern mismatch")
    fin = torch.isfinite(r) & torch.isfinite(e)
    diff = torch.where(fin, (r - e).abs(), torch.zeros_like(r))
    bad = fin & (diff > atol + rtol * e.abs())
    if bad.any():
        reasons.append(f"{int(bad.sum())} elements exceed tolerance; max|diff|={float(diff.max()):.3e}")
    return reasons


def assert_close(received, expected, rtol: float, atol: float, what: str = "") -> None:
    reasons = verbose_allclose(received, expected, rtol, atol)
    assert not reasons, f"{what}: " + "; ".join(reasons)
