"""The fp32 CPU baseline (oracle/eager.py) agrees with the float64 oracle."""
import numpy as np
import torch

from oracle import eager, ops
from tests import golden_util as gu
from tests.synth import deltanet_inputs


def _close(a, b, tol=1e-4):
    np.testing.assert_allclose(np.asarray(a.double() if torch.is_tensor(a) else a), np.asarray(b), rtol=tol, atol=tol)


def test_reference_ops():
    x, w, b = gu.regenerate("causal_conv1d", dict(B=2, D=32, S=100, W=4, seed=1))
    _close(eager.causal_conv1d_bds(x, w, b), ops.causal_conv1d(x, w, b))
    d = gu.regenerate("chunk_fwd_h", dict(B=2, T=256, H=2, K=64, V=64, seed=2))
    _close(eager.chunk_fwd_h(d["k"], d["v"], d["g"]), ops.chunk_fwd_h(d["k"], d["v"], d["g"]))
    d = gu.regenerate("chunk_fwd_o", dict(B=1, T=128, H=2, K=64, V=64, seed=3))
    args = (d["q"], d["k"], d["v"], d["g"], d["h"], d["scale"])
    _close(eager.chunk_fwd_o(*args), ops.chunk_fwd_o(*args), 1e-3)
    _close(eager.chunk_fwd_o_exact_decay(*args), ops.chunk_fwd_o(*args), 1e-3)
    d = gu.regenerate("recompute_w_u", dict(B=1, T=128, H=2, K=64, V=64, seed=4))
    w_e, u_e = eager.recompute_w_u(d["k"], d["v"], d["beta"], d["A"], d["g"])
    w_o, u_o = ops.recompute_w_u(d["k"], d["v"], d["beta"], d["A"], d["g"])
    _close(w_e, w_o)
    _close(u_e, u_o)
    _close(eager.wy_matrix(d["k"], d["beta"], d["g"], -1), ops.build_A(d["k"], d["beta"], d["g"], -1))


def test_chain():
    B, T, H, K = 1, 128, 2, 64
    D = H * K
    gen = torch.Generator().manual_seed(0)
    xs = [torch.randn(B, T, D, generator=gen) for _ in range(3)]
    cw = [torch.randn(D, 4, generator=gen) * 0.5 for _ in range(3)]
    cb = [torch.randn(D, generator=gen) * 0.3 for _ in range(3)]
    d = deltanet_inputs(B, T, H, K, K, 5, dtype=torch.float32)
    args = (*xs, cw[0], cb[0], cw[1], cb[1], cw[2], cb[2], d["beta"], d["g"], H, K, K)
    o_e, f_e = eager.gated_delta_chain(*args)
    o_o, f_o = ops.gated_delta_chain(*args)
    _close(o_e, o_o, 1e-3)
    _close(f_e, f_o, 1e-3)
