"""GPU parity: chunk_fwd_h through the C ABI (reference recurrence and delta rule)."""
import numpy as np
import pytest
import torch

from oracle import ops as orc
from tests import golden_util as gu
from tests.harness import assert_close
from tests.synth import deltanet_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2


@pytest.mark.parametrize("idx,shape", gu.cases("chunk_fwd_h"))
def test_dropin_matches_reference_fixture(idx, shape):
    from theorem_b200.kernels.chunk_fwd_h import custom_kernel
    d = gu.regenerate("chunk_fwd_h", shape)
    dd = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    h = custom_kernel(dd)
    B, T, H, K, V = (d[n] for n in "BTHKV")
    assert h.dtype == torch.float32 and h.shape == (B, T // 64, H, K, V)
    gu.compare("chunk_fwd_h", idx, "h", h, TOL, TOL)
    ref = orc.chunk_fwd_h(d["k"], d["v"], d["g"])
    assert_close(h.cpu().double(), torch.from_numpy(ref), TOL, TOL, "oracle")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K,V", [(64, 64), (128, 128), (64, 128), (128, 64)])
def test_reference_mode_shapes(dtype, K, V):
    from theorem_b200 import ops
    d = gu.regenerate("chunk_fwd_h", dict(B=2, T=320, H=3, K=K, V=V, seed=K + V))
    k, v = d["k"].to(dtype), d["v"].to(dtype)
    h = ops.chunk_fwd_h(k.to(DEV), v.to(DEV), d["g"].to(DEV), mode=0)
    ref = orc.chunk_fwd_h(k.float(), v.float(), d["g"])
    assert_close(h.cpu().double(), torch.from_numpy(ref), TOL, TOL, f"{dtype} K={K} V={V}")


def _delta_inputs(B, T, H, K, V, seed, dtype):
    """k, w, u, g as the chain produces them (config 2 distributions), rounded to dtype."""
    d = deltanet_inputs(B, T, H, K, V, seed, dtype=dtype)
    k, v, beta, g = d["k"], d["v"], d["beta"], d["g"]
    A = orc.build_A(k.float(), beta, g, 1)
    w, u = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    w = torch.from_numpy(w).to(dtype)
    u = torch.from_numpy(u).to(dtype)
    gen = torch.Generator().manual_seed(seed + 1)
    h0 = torch.randn(B, H, K, V, generator=gen) * (0.1 ** 0.5)
    return k, w, u, g, h0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("K,V", [(64, 64), (128, 128), (64, 128), (128, 64)])
@pytest.mark.parametrize("with_h0", [True, False])
def test_delta_rule(dtype, K, V, with_h0):
    from theorem_b200 import ops
    k, w, u, g, h0 = _delta_inputs(2, 256, 2, K, V, K + 2 * V + with_h0, dtype)
    h, vn, fin = ops.chunk_fwd_h(k.to(DEV), u.to(DEV), g.to(DEV), w=w.to(DEV),
                                 h0=h0.to(DEV) if with_h0 else None, mode=1, want_v_new=True, want_final=True)
    rh, rvn, rfin = orc.chunk_fwd_h_delta(k.float(), w.float(), u.float(), g, h0 if with_h0 else None)
    assert vn.dtype == dtype
    assert_close(h.cpu().double(), torch.from_numpy(rh), TOL, TOL, "h")
    assert_close(vn.float().cpu().double(), torch.from_numpy(rvn), TOL, TOL, "v_new")
    assert_close(fin.cpu().double(), torch.from_numpy(rfin), TOL, TOL, "final")


def test_config3_bf16():
    """B2 T1024 H3 K=V=64 bf16 / fp32 state with h0."""
    from theorem_b200 import ops
    k, w, u, g, h0 = _delta_inputs(2, 1024, 3, 64, 64, 3, torch.bfloat16)
    h, vn, fin = ops.chunk_fwd_h(k.to(DEV), u.to(DEV), g.to(DEV), w=w.to(DEV), h0=h0.to(DEV), mode=1,
                                 want_v_new=True, want_final=True)
    rh, rvn, rfin = orc.chunk_fwd_h_delta(k.float(), w.float(), u.float(), g, h0)
    assert_close(h.cpu().double(), torch.from_numpy(rh), TOL, TOL, "h")
    assert_close(fin.cpu().double(), torch.from_numpy(rfin), TOL, TOL, "final")


def test_delta_reduces_to_reference_recurrence():
    """w = 0, u = v, h0 = 0: h_delta[:, c+1] == h_ref[:, c], final == h_ref[:, -1]."""
    from theorem_b200 import ops
    d = gu.regenerate("chunk_fwd_h", dict(B=1, T=512, H=2, K=64, V=64, seed=77))
    k, v, g = (d[n].to(DEV) for n in ("k", "v", "g"))
    href = ops.chunk_fwd_h(k, v, g, mode=0)
    hd, vn, fin = ops.chunk_fwd_h(k, v, g, w=torch.zeros_like(k), mode=1, want_v_new=True, want_final=True)
    assert torch.all(hd[:, 0] == 0)
    assert_close(hd[:, 1:].cpu(), href[:, :-1].cpu(), 1e-5, 1e-5, "shifted states")
    assert_close(fin.cpu(), href[:, -1].cpu(), 1e-5, 1e-5, "final")
    assert torch.equal(vn, v)


@pytest.mark.parametrize("mode", [0, 1])
def test_bf16_state_output(mode):
    """h stored in bf16 (the chain's layout) equals the fp32 h rounded to bf16."""
    from theorem_b200 import ops
    k, w, u, g, h0 = _delta_inputs(2, 512, 2, 128, 128, 31 + mode, torch.bfloat16)
    args = dict(mode=mode)
    if mode == 1:
        args.update(w=w.to(DEV), h0=h0.to(DEV))
    r32 = ops.chunk_fwd_h(k.to(DEV), u.to(DEV), g.to(DEV), **args)
    r16 = ops.chunk_fwd_h(k.to(DEV), u.to(DEV), g.to(DEV), h_dtype=torch.bfloat16, **args)
    h32 = r32[0] if mode == 1 else r32
    h16 = r16[0] if mode == 1 else r16
    assert h16.dtype == torch.bfloat16
    assert torch.equal(h16, h32.to(torch.bfloat16))
