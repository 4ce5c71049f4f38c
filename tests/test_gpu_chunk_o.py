"""GPU parity: chunk_fwd_o through the C ABI vs the reference fixtures and the oracle."""
import numpy as np
import pytest
import torch

from oracle import ops as orc
from tests import golden_util as gu
from tests.harness import assert_close
from tests.synth import deltanet_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2  # task.yml rtol = atol


@pytest.mark.parametrize("idx,shape", gu.cases("chunk_fwd_o"))
def test_dropin_matches_reference_fixture(idx, shape):
    from theorem_b200.kernels.chunk_fwd_o import custom_kernel
    d = gu.regenerate("chunk_fwd_o", shape)
    dd = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    o = custom_kernel(dd)
    assert o.dtype == torch.float32 and o.shape == d["v"].shape
    gu.compare("chunk_fwd_o", idx, "o", o, TOL, TOL)
    ref = orc.chunk_fwd_o(d["q"], d["k"], d["v"], d["g"], d["h"], d["scale"])
    assert_close(o.cpu().double(), torch.from_numpy(ref), TOL, TOL, "oracle")
    for name in ("q", "k", "v", "g", "h"):
        assert torch.equal(dd[name].cpu(), d[name]), f"input {name} was modified"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K,V", [(64, 64), (64, 128), (128, 128), (128, 64), (64, 256), (128, 192)])
def test_shapes_and_dtypes(dtype, K, V):
    from theorem_b200 import ops
    B, T, H = 2, 192, 3
    d = deltanet_inputs(B, T, H, K, V, seed=K + V, dtype=dtype)
    gen = torch.Generator().manual_seed(1)
    h = torch.randn(B, T // 64, H, K, V, generator=gen) * 0.1
    scale = K ** -0.5
    o = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV), h.to(DEV), scale)
    assert o.dtype == dtype
    ref = orc.chunk_fwd_o(d["q"].float(), d["k"].float(), d["v"].float(), d["g"], h, scale)
    assert_close(o.float().cpu().double(), torch.from_numpy(ref), TOL, TOL, f"{dtype} K={K} V={V}")


def test_config4_full_size_sliced():
    """BASELINE config 4 (B8 T4096 H16 K=V=128 bf16) at full size; checked
    against the oracle on a sample of (b, h) sequences."""
    from theorem_b200 import ops
    B, T, H, K, V = 8, 4096, 16, 128, 128
    d = deltanet_inputs(B, T, H, K, V, seed=4)
    gen = torch.Generator().manual_seed(44)
    h = torch.randn(B, T // 64, H, K, V, generator=gen) * 0.05
    o = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV), h.to(DEV), K ** -0.5)
    oc = o.float().cpu()
    assert torch.isfinite(oc).all()
    for b, hh in [(0, 0), (3, 7), (7, 15)]:
        sl = lambda t: t[b:b + 1, :, hh:hh + 1].float()
        ref = orc.chunk_fwd_o(sl(d["q"]), sl(d["k"]), sl(d["v"]), sl(d["g"]), h[b:b + 1, :, hh:hh + 1],
                              K ** -0.5)
        assert_close(oc[b:b + 1, :, hh:hh + 1].double(), torch.from_numpy(ref), TOL, TOL, f"b={b} h={hh}")


def test_linear_in_v_and_h():
    """o(v1 + v2, h1 + h2) == o(v1, h1) + o(v2, h2) (fp32, tf32 rounding only)."""
    from theorem_b200 import ops
    B, T, H, K, V = 1, 256, 2, 64, 64
    d = gu.regenerate("chunk_fwd_o", dict(B=B, T=T, H=H, K=K, V=V, seed=9))
    dd = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    v2 = torch.randn_like(dd["v"])
    h2 = torch.randn_like(dd["h"]) * 0.1
    f = lambda v, h: ops.chunk_fwd_o(dd["q"], dd["k"], v, dd["g"], h, d["scale"])
    lhs = f(dd["v"] + v2, dd["h"] + h2)
    rhs = f(dd["v"], dd["h"]) + f(v2, h2)
    assert_close(lhs.cpu(), rhs.cpu(), 1e-2, 1e-2, "linearity")


def test_unsupported_head_dim_raises():
    from theorem_b200 import ops
    q = torch.zeros(1, 64, 1, 96, device=DEV)
    with pytest.raises(AssertionError):
        ops.chunk_fwd_o(q, q, torch.zeros(1, 64, 1, 64, device=DEV), torch.zeros(1, 64, 1, device=DEV),
                        torch.zeros(1, 1, 1, 96, 64, device=DEV), 0.1)


@pytest.mark.parametrize("K,V", [(64, 64), (64, 128), (128, 64), (128, 128)])
def test_warp_specialized_bf16_state(K, V):
    """bf16 q/k/v with a bf16 h: the persistent warp-specialized kernel."""
    from theorem_b200 import ops
    B, T, H = 2, 256, 3
    d = deltanet_inputs(B, T, H, K, V, seed=11 * K + V)
    gen = torch.Generator().manual_seed(3)
    h = (torch.randn(B, T // 64, H, K, V, generator=gen) * 0.1).to(torch.bfloat16)
    o = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV), h.to(DEV), K ** -0.5)
    ref = orc.chunk_fwd_o(d["q"].float(), d["k"].float(), d["v"].float(), d["g"], h.float(), K ** -0.5)
    assert o.dtype == torch.bfloat16
    assert_close(o.float().cpu().double(), torch.from_numpy(ref), TOL, TOL, f"K={K} V={V}")


def test_warp_specialized_many_units_per_cta():
    """1024 (b, chunk, h) units over <= 148 persistent CTAs: every ring stage and
    TMEM buffer is reused several times."""
    from theorem_b200 import ops
    B, T, H, K, V = 2, 4096, 8, 128, 128
    d = deltanet_inputs(B, T, H, K, V, seed=21)
    gen = torch.Generator().manual_seed(4)
    h = (torch.randn(B, T // 64, H, K, V, generator=gen) * 0.05).to(torch.bfloat16)
    o = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV), h.to(DEV), K ** -0.5)
    oc = o.float().cpu()
    assert torch.isfinite(oc).all()
    for b, hh in [(0, 0), (1, 5), (1, 7)]:
        sl = lambda t: t[b:b + 1, :, hh:hh + 1].float()
        ref = orc.chunk_fwd_o(sl(d["q"]), sl(d["k"]), sl(d["v"]), sl(d["g"]), h[b:b + 1, :, hh:hh + 1].float(),
                              K ** -0.5)
        assert_close(oc[b:b + 1, :, hh:hh + 1].double(), torch.from_numpy(ref), TOL, TOL, f"b={b} h={hh}")
    # repeated calls give identical results (no state leaks between launches)
    o2 = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), d["g"].to(DEV), h.to(DEV), K ** -0.5)
    assert torch.equal(o, o2)


@pytest.mark.parametrize("K", [64, 128])
def test_fp32_state_keeps_fp32_accuracy(K):
    """bf16 q/k with an fp32 h and v = 0: o = scale e^{g_t} q h. The kernel splits h
    into bf16 hi + lo, so the only error left is the bf16 rounding of o itself."""
    from theorem_b200 import ops
    B, T, H, V = 1, 512, 2, 128
    d = deltanet_inputs(B, T, H, K, V, seed=31 + K)
    gen = torch.Generator().manual_seed(5)
    h = torch.randn(B, T // 64, H, K, V, generator=gen) * 0.3
    v0 = torch.zeros(B, T, H, V, dtype=torch.bfloat16)
    o = ops.chunk_fwd_o(d["q"].to(DEV), d["k"].to(DEV), v0.to(DEV), d["g"].to(DEV), h.to(DEV), K ** -0.5)
    ref = torch.from_numpy(orc.chunk_fwd_o(d["q"].float(), d["k"].float(), v0.float(), d["g"], h, K ** -0.5))
    err = (o.float().cpu().double() - ref).abs()
    bound = 2.0 ** -8 * ref.abs() + 1e-6
    assert bool((err <= bound).all()), f"max excess {float((err - bound).max())}"
