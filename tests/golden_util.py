"""Helpers to read the golden fixtures under tests/golden/ and regenerate inputs."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from oracle import inputs as oin

GOLDEN = Path(__file__).resolve().parent / "golden"
_MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())
_ARRAYS: dict = {}


def cases(op: str, kind: str | None = None):
    """List of (index, shape dict) for an op, optionally only 'test' or 'benchmark'."""
    out = []
    for i, c in enumerate(_MANIFEST[op]["cases"]):
        if kind is None or c["kind"] == kind:
            out.append((i, dict(c["shape"])))
    return out


def tolerances(op: str):
    t = _MANIFEST[op]["tolerances"]
    return float(t["rtol"]), float(t["atol"])


def arrays(op: str):
    if op not in _ARRAYS:
        _ARRAYS[op] = dict(np.load(GOLDEN / f"{op}.npz"))
    return _ARRAYS[op]


def regenerate(op: str, shape: dict):
    """CPU inputs for a fixture case (same generators the fixture was made with)."""
    kw = {k: v for k, v in shape.items() if k != "seed"}
    seed = shape["seed"]
    if op == "causal_conv1d":
        return oin.conv_inputs(seed=seed, **kw)
    if op == "recompute_w_u":
        return oin.wu_inputs(seed=seed, **kw)
    if op == "chunk_fwd_h":
        return oin.h_inputs(seed=seed, **kw)
    if op == "chunk_fwd_o":
        return oin.o_inputs(seed=seed, **kw)
    raise ValueError(op)


def input_tensors(op: str, data) -> dict:
    if op == "causal_conv1d":
        return dict(zip(("x", "weight", "bias"), data))
    names = {"recompute_w_u": ("k", "v", "beta", "A", "g"),
             "chunk_fwd_h": ("k", "v", "g"),
             "chunk_fwd_o": ("q", "k", "v", "g", "h")}[op]
    return {n: data[n] for n in names}


def check_inputs(op: str, idx: int, data) -> None:
    """Assert regenerated inputs match the checksums stored with the fixture."""
    arr = arrays(op)
    for name, t in input_tensors(op, data).items():
        a = t.detach().double().reshape(-1).numpy()
        got = np.array([a.sum(), np.abs(a).sum(), (a * a).sum()])
        np.testing.assert_allclose(got, arr[f"c{idx}_in_{name}"], rtol=1e-12, atol=1e-9,
                                   err_msg=f"{op} case {idx} input {name} regenerated differently")


def compare(op: str, idx: int, name: str, result, rtol: float, atol: float) -> float:
    """Compare ``result`` (any array/tensor of the output's shape) with the stored
    reference samples: elementwise |r-e| <= atol + rtol|e| at the sampled points
    and the stored sum / sum|x| to a relative 1e-4. Returns max |diff| seen."""
    arr = arrays(op)
    if torch.is_tensor(result):
        result = result.detach().to("cpu").double().numpy()
    flat = np.asarray(result, np.float64).reshape(-1)
    idxs = arr[f"c{idx}_out_{name}_idx"]
    exp = arr[f"c{idx}_out_{name}_val"]
    stats = arr[f"c{idx}_out_{name}_stats"]
    assert flat.size == int(stats[3]), f"{op} case {idx} {name}: size {flat.size} != {int(stats[3])}"
    got = flat[idxs]
    diff = np.abs(got - exp)
    bad = diff > atol + rtol * np.abs(exp)
    assert not bad.any(), (f"{op} case {idx} {name}: {int(bad.sum())} samples out of tolerance; "
                           f"max|diff|={diff.max():.3e}")
    s = np.array([flat.sum(), np.abs(flat).sum()])
    np.testing.assert_allclose(s[1], stats[1], rtol=max(rtol, 1e-4))
    assert abs(s[0] - stats[0]) <= max(rtol, 1e-4) * stats[1] + 1e-6
    return float(diff.max())
