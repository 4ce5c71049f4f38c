"""Generate the golden fixtures from the reference's own PyTorch ``ref_kernel``s.

Run in a checkout that has the reference next to it (the reference is NOT
available where the GPU tests run; only the fixtures travel):

    python tests/golden/make_golden.py --reference <path to yhinai/Theorem>

For every shape in each op's ``task.yml`` (tests + benchmarks) it

1. builds the inputs on the CPU. For recompute_w_u and chunk_fwd_o it calls
   the reference's own generators (``generate_data`` / ``_build_inputs`` with
   ``device="cpu"``) and asserts that ``oracle.inputs`` reproduces them bit for
   bit; causal_conv1d and chunk_fwd_h generators hard-code ``cuda:0``, so the
   ``oracle.inputs`` CPU restatement supplies them;
2. runs the reference ``ref_kernel`` on those CPU tensors;
3. stores, per output: the full tensor when it has <= 4096 elements, else 4096
   evenly spaced samples, plus sum / sum|x| / sum x^2 (float64) -- and input
   checksums so a test can tell that it regenerated the same inputs.

It also runs the reference's NumPy conv restatement
(scripts/cpu_reference.py) against its torch ref at atol=1e-4, as that script
does with --validate-against-pytorch.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch
import yaml

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import inputs as oin  # noqa: E402

NSAMP = 4096
OPS = ("causal_conv1d", "recompute_w_u", "chunk_fwd_h", "chunk_fwd_o")


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def sample(t: torch.Tensor) -> dict:
    a = t.detach().double().reshape(-1).numpy()
    n = a.size
    idx = np.arange(n) if n <= NSAMP else np.linspace(0, n - 1, NSAMP).astype(np.int64)
    return {"idx": idx.astype(np.int64), "val": a[idx].astype(np.float64),
            "stats": np.array([a.sum(), np.abs(a).sum(), (a * a).sum(), n], np.float64)}


def checksum(t: torch.Tensor) -> np.ndarray:
    a = t.detach().double().reshape(-1).numpy()
    return np.array([a.sum(), np.abs(a).sum(), (a * a).sum()], np.float64)


def build(op: str, shape: dict, ref):
    kw = {k: v for k, v in shape.items() if k != "seed"}
    seed = shape["seed"]
    if op == "causal_conv1d":
        data = oin.conv_inputs(seed=seed, **kw)
        ins = dict(zip(("x", "weight", "bias"), data))
        outs = {"out": ref.ref_kernel(data)}
    elif op == "recompute_w_u":
        d_ref = ref.generate_data(device="cpu", seed=seed, **kw)
        d_my = oin.wu_inputs(seed=seed, **kw)
        for name in ("k", "v", "beta", "A", "g"):
            assert torch.equal(getattr(d_ref, name), d_my[name]), f"{op} {shape}: {name} differs"
        ins = {n: getattr(d_ref, n) for n in ("k", "v", "beta", "A", "g")}
        w, u = ref.ref_kernel(d_ref)
        outs = {"w": w, "u": u, "A": d_ref.A}
    elif op == "chunk_fwd_h":
        data = oin.h_inputs(seed=seed, **kw)
        ins = {n: data[n] for n in ("k", "v", "g")}
        outs = {"h": ref.ref_kernel(data)}
    elif op == "chunk_fwd_o":
        d_ref = ref._build_inputs(device="cpu", seed=seed, **kw)
        d_my = oin.o_inputs(seed=seed, **kw)
        for name in ("q", "k", "v", "g", "h"):
            assert torch.equal(d_ref[name], d_my[name]), f"{op} {shape}: {name} differs"
        assert d_ref["scale"] == d_my["scale"]
        ins = {n: d_ref[n] for n in ("q", "k", "v", "g", "h")}
        outs = {"o": ref.ref_kernel(d_ref)}
    else:
        raise ValueError(op)
    return ins, outs


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--reference", required=True, type=Path)
    p.add_argument("--out", default=str(HERE), type=Path)
    args = p.parse_args()
    refroot = args.reference.resolve()
    torch.set_num_threads(8)

    # Reference NumPy restatement vs its torch ref (scripts/cpu_reference.py:66-83).
    cpu_ref = _load(refroot / "scripts" / "cpu_reference.py", "_thm_cpu_reference")
    conv_ref = _load(refroot / "kernels" / "causal_conv1d" / "reference.py", "_thm_ref_conv")
    for shp in cpu_ref.TEST_SHAPES:
        x, w, b = cpu_ref._gen_inputs(**shp)
        out_np = cpu_ref.causal_conv1d_numpy(x, w, b)
        out_t = conv_ref.ref_kernel((torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b)))
        assert np.abs(out_np - out_t.numpy()).max() <= 1e-4

    manifest = {}
    for op in OPS:
        ref = _load(refroot / "kernels" / op / "reference.py", f"_thm_ref_{op}")
        task = yaml.safe_load((refroot / "kernels" / op / "task.yml").read_text())
        shapes = list(task["shapes"]["tests"]) + list(task["shapes"]["benchmarks"])
        arrays = {}
        cases = []
        for i, shape in enumerate(shapes):
            ins, outs = build(op, shape, ref)
            for n, t in ins.items():
                arrays[f"c{i}_in_{n}"] = checksum(t)
            for n, t in outs.items():
                s = sample(t)
                arrays[f"c{i}_out_{n}_idx"] = s["idx"]
                arrays[f"c{i}_out_{n}_val"] = s["val"]
                arrays[f"c{i}_out_{n}_stats"] = s["stats"]
            cases.append({"shape": shape, "inputs": sorted(ins), "outputs": sorted(outs),
                          "kind": "test" if i < len(task["shapes"]["tests"]) else "benchmark"})
            print(f"{op:14s} {shape}  ok")
        np.savez_compressed(args.out / f"{op}.npz", **arrays)
        manifest[op] = {"cases": cases, "tolerances": task.get("tolerances")}
    (args.out / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
