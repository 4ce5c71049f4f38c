"""Pin the CPU oracle (oracle/ops.py) to the reference's own ref_kernel outputs.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py
from the reference's ``ref_kernel``s (fp32 torch on CPU). The oracle computes
in float64, so the agreement bar is far tighter than the task tolerance.
"""
import numpy as np
import pytest

from oracle import ops
from tests import golden_util as gu

RTOL, ATOL = 2e-5, 2e-5


@pytest.mark.parametrize("idx,shape", gu.cases("causal_conv1d"))
def test_conv_oracle_matches_reference(idx, shape):
    data = gu.regenerate("causal_conv1d", shape)
    gu.check_inputs("causal_conv1d", idx, data)
    out = ops.causal_conv1d(*data)
    gu.compare("causal_conv1d", idx, "out", out, RTOL, ATOL)


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u"))
def test_wu_oracle_matches_reference(idx, shape):
    d = gu.regenerate("recompute_w_u", shape)
    gu.check_inputs("recompute_w_u", idx, d)
    w, u = ops.recompute_w_u(d["k"], d["v"], d["beta"], d["A"], d["g"])
    gu.compare("recompute_w_u", idx, "w", w, RTOL, ATOL)
    gu.compare("recompute_w_u", idx, "u", u, RTOL, ATOL)


@pytest.mark.parametrize("idx,shape", gu.cases("recompute_w_u"))
def test_build_A_oracle_matches_reference(idx, shape):
    """oracle.build_A(sign=-1) == the reference's upstream _build_A."""
    d = gu.regenerate("recompute_w_u", shape)
    A = ops.build_A(d["k"], d["beta"], d["g"], sign=-1)
    gu.compare("recompute_w_u", idx, "A", A, RTOL, ATOL)


@pytest.mark.parametrize("idx,shape", gu.cases("chunk_fwd_h"))
def test_h_oracle_matches_reference(idx, shape):
    d = gu.regenerate("chunk_fwd_h", shape)
    gu.check_inputs("chunk_fwd_h", idx, d)
    h = ops.chunk_fwd_h(d["k"], d["v"], d["g"])
    gu.compare("chunk_fwd_h", idx, "h", h, RTOL, ATOL)


@pytest.mark.parametrize("idx,shape", gu.cases("chunk_fwd_o"))
def test_o_oracle_matches_reference(idx, shape):
    d = gu.regenerate("chunk_fwd_o", shape)
    gu.check_inputs("chunk_fwd_o", idx, d)
    o = ops.chunk_fwd_o(d["q"], d["k"], d["v"], d["g"], d["h"], d["scale"])
    gu.compare("chunk_fwd_o", idx, "o", o, RTOL, ATOL)


def test_delta_h_reduces_to_reference_recurrence():
    """w = 0, u = v, h0 = 0: delta rule == reference recurrence, shifted by one chunk."""
    d = gu.regenerate("chunk_fwd_h", dict(B=2, T=256, H=3, K=64, V=64, seed=7))
    h_ref = ops.chunk_fwd_h(d["k"], d["v"], d["g"])
    h_pre, vnew, final = ops.chunk_fwd_h_delta(d["k"], 0 * d["k"], d["v"], d["g"])
    np.testing.assert_allclose(h_pre[:, 1:], h_ref[:, :-1], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(final, h_ref[:, -1], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(vnew, d["v"].double().numpy(), rtol=0, atol=0)
    assert np.all(h_pre[:, 0] == 0)


def test_build_A_signs_are_inverses():
    """(I + sign*M) A == I for both conventions, chunk by chunk."""
    d = gu.regenerate("recompute_w_u", dict(B=1, T=128, H=2, K=64, V=64, seed=3))
    k, beta, g = (d[n].double().numpy() for n in ("k", "beta", "g"))
    for sign in (-1, 1):
        A = ops.build_A(k, beta, g, sign)
        Ac = ops._to_chunks(A)
        kc, bc, gc = ops._to_chunks(k), ops._to_chunks(beta), ops._to_chunks(g)
        M = np.tril((kc @ kc.swapaxes(-1, -2)) * bc[..., :, None] * ops._decay(gc), -1)
        L = np.eye(64) + sign * M
        np.testing.assert_allclose(L @ Ac, np.broadcast_to(np.eye(64), L.shape), atol=1e-10)


def test_conv_silu_and_channel_last_layouts_agree():
    x, w, b = gu.regenerate("causal_conv1d", dict(B=2, D=48, S=70, W=4, seed=11))
    a = ops.causal_conv1d(x, w, b, "silu")
    c = ops.causal_conv1d(x.transpose(1, 2).contiguous(), w, b, "silu", layout="bsd")
    np.testing.assert_allclose(a, c.transpose(0, 2, 1), rtol=0, atol=0)
    plain = ops.causal_conv1d(x, w, b)
    np.testing.assert_allclose(a, plain / (1 + np.exp(-plain)), rtol=1e-15)
