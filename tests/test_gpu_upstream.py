"""GPU parity of the upstream producers of the path's inputs: build_A (the
reference's `_build_A`, kernels/recompute_w_u/reference.py:48-91) and the
chunk-local cumulative gate (kernels/chunk_fwd_h/reference.py:41-45,
kernels/recompute_w_u/reference.py:103-106)."""
import pytest
import torch

from oracle import ops as orc
from tests import golden_util as gu
from tests.harness import assert_close
from tests.synth import deltanet_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u"))
def test_build_A_matches_reference_fixture(idx, shape):
    """fp32 A against the reference's own _build_A outputs stored in the fixtures."""
    from theorem_b200 import ops
    d = gu.regenerate("recompute_w_u", shape)
    A = ops.build_A(d["k"].to(DEV), d["beta"].to(DEV), d["g"].to(DEV), sign=-1)
    assert A.shape == d["A"].shape and A.dtype == torch.float32
    gu.compare("recompute_w_u", idx, "A", A, 1e-4, 1e-5)
    assert_close(A.cpu(), d["A"], 1e-4, 1e-5, "A vs generator")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K", [64, 128])
@pytest.mark.parametrize("sign", [-1, 1])
def test_build_A_against_oracle(dtype, K, sign):
    from theorem_b200 import ops
    d = deltanet_inputs(2, 256, 3, K, 64, seed=K + sign + (dtype == torch.bfloat16), dtype=dtype)
    A = ops.build_A(d["k"].to(DEV), d["beta"].to(DEV), d["g"].to(DEV), sign=sign)
    ref = orc.build_A(d["k"].float(), d["beta"], d["g"], sign)
    assert_close(A.cpu().double(), torch.from_numpy(ref), 1e-4, 1e-5, f"{dtype} K={K} sign={sign}")


def test_build_A_feeds_recompute_w_u():
    """recompute_w_u with A from build_A (the reference contract, a_mode 0) equals
    recompute_w_u forming A in-kernel (a_mode -1)."""
    from theorem_b200 import ops
    d = gu.regenerate("recompute_w_u", dict(B=2, T=512, H=3, K=64, V=64, seed=4052))
    k, v, beta, g = (d[n].to(DEV) for n in ("k", "v", "beta", "g"))
    A = ops.build_A(k, beta, g, sign=-1)
    w0, u0 = ops.recompute_w_u(k, v, beta, A, g, a_mode=0)
    w1, u1 = ops.recompute_w_u(k, v, beta, None, g, a_mode=-1)
    assert_close(w0.cpu(), w1.cpu(), 1e-4, 1e-5, "w")
    assert_close(u0.cpu(), u1.cpu(), 1e-4, 1e-5, "u")


def _wu_increments(B, T, H, K, V, seed):
    """The per-token gate increments of recompute_w_u/reference.py:94-106, drawn in
    the generator's order (k, v, beta, then raw g)."""
    gen = torch.Generator().manual_seed(int(seed))
    torch.randn(B, T, H, K, generator=gen)
    torch.randn(B, T, H, V, generator=gen)
    torch.randn(B, T, H, generator=gen)
    return -torch.rand(B, T, H, generator=gen, dtype=torch.float32) * 0.05


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u"))
def test_chunk_local_cumsum_reproduces_reference_gates(idx, shape):
    from theorem_b200 import ops
    d = gu.regenerate("recompute_w_u", shape)
    kw = {k: v for k, v in shape.items() if k != "seed"}
    inc = _wu_increments(seed=shape["seed"], **kw)
    g = ops.chunk_local_cumsum(inc.to(DEV))
    assert_close(g.cpu(), d["g"], 1e-6, 1e-6, "g")


@pytest.mark.parametrize("B,T,H", [(1, 64, 1), (2, 192, 3), (3, 512, 16), (1, 128, 64), (2, 64, 33)])
def test_chunk_local_cumsum_shapes_scale_in_place(B, T, H):
    from theorem_b200 import ops
    gen = torch.Generator().manual_seed(B * T + H)
    inc = torch.randn(B, T, H, generator=gen)
    ref = inc.reshape(B, T // 64, 64, H).double().cumsum(2).reshape(B, T, H) * 0.0625
    x = inc.to(DEV)
    out = ops.chunk_local_cumsum(x, scale=0.0625)
    assert_close(out.cpu().double(), ref, 1e-5, 1e-5, "cumsum")
    y = ops.chunk_local_cumsum(x, scale=0.0625, out=x)  # in place
    assert y.data_ptr() == x.data_ptr()
    assert torch.equal(y, out)


def test_gates_into_the_chain_ops():
    """cumsum -> build_A(+1) -> recompute_w_u (a_mode 0) == recompute_w_u (a_mode +1)."""
    from theorem_b200 import ops
    d = deltanet_inputs(1, 256, 2, 128, 128, seed=8)
    gen = torch.Generator().manual_seed(9)
    inc = torch.nn.functional.logsigmoid(torch.randn(1, 256, 2, generator=gen)) / 16
    g = ops.chunk_local_cumsum(inc.to(DEV))
    k, v, beta = d["k"].to(DEV), d["v"].to(DEV), d["beta"].to(DEV)
    A = ops.build_A(k, beta, g, sign=1)
    w0, u0 = ops.recompute_w_u(k, v, beta, A, g, a_mode=0)
    w1, u1 = ops.recompute_w_u(k, v, beta, None, g, a_mode=1)
    assert_close(w0.float().cpu(), w1.float().cpu(), 1e-2, 1e-2, "w")
    assert_close(u0.float().cpu(), u1.float().cpu(), 1e-2, 1e-2, "u")
