"""GPU parity: recompute_w_u through the C ABI vs the reference fixtures and the oracle."""
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


class _Data:  # stands in for the reference's Data dataclass (attribute access only)
    def __init__(self, d):
        self.__dict__.update(d)


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u"))
def test_dropin_matches_reference_fixture(idx, shape):
    from theorem_b200.kernels.recompute_w_u import custom_kernel
    d = gu.regenerate("recompute_w_u", shape)
    dd = _Data({k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()})
    out = custom_kernel(dd)
    assert isinstance(out, tuple) and len(out) == 2
    w, u = out
    assert w.dtype == torch.float32 and w.shape == d["k"].shape and u.shape == d["v"].shape
    gu.compare("recompute_w_u", idx, "w", w, TOL, TOL)
    gu.compare("recompute_w_u", idx, "u", u, TOL, TOL)
    rw, ru = orc.recompute_w_u(d["k"], d["v"], d["beta"], d["A"], d["g"])
    assert_close(w.cpu().double(), torch.from_numpy(rw), 1e-3, 1e-4, "w vs oracle")
    assert_close(u.cpu().double(), torch.from_numpy(ru), 1e-3, 1e-4, "u vs oracle")


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u", "test"))
def test_fused_A_reference_sign_matches_build_A(idx, shape):
    """a_mode=-1 builds A = (I - M)^-1 in-kernel: A_out == the reference's _build_A."""
    from theorem_b200 import ops
    d = gu.regenerate("recompute_w_u", shape)
    k, v, beta, g = (d[n].to(DEV) for n in ("k", "v", "beta", "g"))
    A_out = torch.empty_like(d["A"], device=DEV)
    w, u = ops.recompute_w_u(k, v, beta, None, g, a_mode=-1, A_out=A_out)
    gu.compare("recompute_w_u", idx, "A", A_out, 1e-4, 1e-5)
    gu.compare("recompute_w_u", idx, "w", w, TOL, TOL)
    gu.compare("recompute_w_u", idx, "u", u, TOL, TOL)


def _baseline_case(B, T, H, K, V, seed, dtype):
    d = deltanet_inputs(B, T, H, K, V, seed, dtype=dtype)
    return d["k"], d["v"], d["beta"], d["g"]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("sign", [1, -1])
@pytest.mark.parametrize("K,V", [(64, 64), (64, 128), (128, 64), (128, 128)])
def test_fused_A_baseline_distributions(dtype, sign, K, V):
    from theorem_b200 import ops
    B, T, H = 2, 256, 3
    k, v, beta, g = _baseline_case(B, T, H, K, V, K * 3 + V + sign, dtype)
    A_out = torch.empty(B, T, H, 64, device=DEV)
    w, u = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), None, g.to(DEV), a_mode=sign, A_out=A_out)
    A = orc.build_A(k.float(), beta, g, sign)
    rw, ru = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    assert w.dtype == dtype and u.dtype == dtype
    assert_close(A_out.cpu().double(), torch.from_numpy(A), 1e-3, 1e-4, "A")
    assert_close(w.float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w")
    assert_close(u.float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u")


def test_config2_bf16():
    """B2 T512 H3 K=V=64 bf16 in, fp32 accumulate, A = (I + M)^-1."""
    from theorem_b200 import ops
    k, v, beta, g = _baseline_case(2, 512, 3, 64, 64, 2, torch.bfloat16)
    w, u = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), None, g.to(DEV), a_mode=1)
    A = orc.build_A(k.float(), beta, g, 1)
    rw, ru = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    assert_close(w.float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w")
    assert_close(u.float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u")


@pytest.mark.parametrize("K,V", [(64, 64), (128, 128)])
def test_given_A_bf16_operands(K, V):
    """a_mode=0 with bf16 k, v and an fp32 A (converted to bf16 in shared memory)."""
    from theorem_b200 import ops
    k, v, beta, g = _baseline_case(1, 128, 2, K, V, 5, torch.bfloat16)
    A = torch.from_numpy(orc.build_A(k.float(), beta, g, 1)).float()
    w, u = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), A.to(DEV), g.to(DEV), a_mode=0)
    rw, ru = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    assert_close(w.float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w")
    assert_close(u.float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u")


@pytest.mark.parametrize("sign", [1, -1])
def test_fused_many_units_per_cta(sign):
    """2048 (b, chunk, h) units over <= 148 persistent CTAs (both math groups,
    every ring stage and TMEM buffer reused many times); A_out checked too."""
    from theorem_b200 import ops
    B, T, H, K, V = 4, 2048, 16, 128, 128
    k, v, beta, g = _baseline_case(B, T, H, K, V, 40 + sign, torch.bfloat16)
    A_out = torch.empty(B, T, H, 64, device=DEV)
    w, u = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), None, g.to(DEV), a_mode=sign, A_out=A_out)
    w2, u2 = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), None, g.to(DEV), a_mode=sign)
    assert torch.equal(w, w2) and torch.equal(u, u2)
    for b, hh in [(0, 0), (2, 9), (3, 15)]:
        sl = lambda t: t[b:b + 1, :, hh:hh + 1].float()
        A = orc.build_A(sl(k), sl(beta), sl(g), sign)
        rw, ru = orc.recompute_w_u(sl(k), sl(v), sl(beta), A, sl(g))
        assert_close(A_out[b:b + 1, :, hh:hh + 1].cpu().double(), torch.from_numpy(A), 1e-3, 1e-4, "A")
        assert_close(w[b:b + 1, :, hh:hh + 1].float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w")
        assert_close(u[b:b + 1, :, hh:hh + 1].float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u")


@pytest.mark.parametrize("sign", [1, -1])
def test_fused_A_steep_gates(sign):
    """Chunks whose gates span more than 120 keep one exponential per M entry
    (the two-factor decay would leave fp32 range); mixed with gentle chunks."""
    from theorem_b200 import ops
    B, T, H, K, V = 1, 256, 2, 128, 128
    d = deltanet_inputs(B, T, H, K, V, seed=60 + sign)
    gen = torch.Generator().manual_seed(61)
    inc = -3.0 * torch.rand(B, T, H, generator=gen)
    inc[:, 64:128] *= 0.01
    g = inc.reshape(B, T // 64, 64, H).cumsum(2).reshape(B, T, H).contiguous()
    k, v, beta = d["k"], d["v"], d["beta"]
    w, u = ops.recompute_w_u(k.to(DEV), v.to(DEV), beta.to(DEV), None, g.to(DEV), a_mode=sign)
    A = orc.build_A(k.float(), beta, g, sign)
    rw, ru = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    assert_close(w.float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w")
    assert_close(u.float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u")
