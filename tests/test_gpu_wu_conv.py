"""GPU parity: recompute_w_u with the v projection's causal conv folded in
(thm_recompute_w_u_conv_fwd) against the two launches it replaces
(thm_causal_conv1d_fwd on x_v, then thm_recompute_w_u_fwd) and the oracle.

The fused kernel forms v with the conv kernel's bf16 arithmetic, so w, u and A
must equal the two-launch path's bit for bit; the oracle check holds the chain
to the north star's 1e-2."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ops as orc
from tests.harness import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2


def _inputs(B, T, H, K, V, seed, gate_scale=1.0 / 16):
    gen = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, T, H, K, generator=gen), dim=-1).to(torch.bfloat16)
    xv = torch.randn(B, T, H * V, generator=gen).to(torch.bfloat16)
    cw = torch.randn(H * V, 4, generator=gen) * 0.5
    cb = torch.randn(H * V, generator=gen) * 0.3
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    inc = F.logsigmoid(torch.randn(B, T, H, generator=gen)) * gate_scale
    g = inc.reshape(B, T // 64, 64, H).cumsum(2).reshape(B, T, H).contiguous()
    return k, xv, cw, cb, beta, g


def _two_launch(k, xv, cw, cb, beta, g, act, a_mode):
    from theorem_b200 import ops
    B, T, H, K = k.shape
    v = ops.causal_conv1d(xv, cw, cb, act, "bsd", 0).view(B, T, H, -1)
    A = torch.empty(B, T, H, 64, device=k.device)
    w, u = ops.recompute_w_u(k, v.contiguous(), beta, None, g, a_mode=a_mode, A_out=A)
    return w, u, A, v


@pytest.mark.parametrize("K,V", [(128, 128), (64, 128), (128, 64), (64, 64)])
@pytest.mark.parametrize("act", ["silu", None])
def test_equals_conv_then_recompute_w_u(K, V, act):
    from theorem_b200 import ops
    B, T, H = 2, 320, 3  # 5 chunks per sequence; sequence 1 starts mid-batch (zero conv history)
    k, xv, cw, cb, beta, g = (t.to(DEV) for t in _inputs(B, T, H, K, V, seed=K + V + (act is None)))
    w1, u1, A1, _ = _two_launch(k, xv, cw, cb, beta, g, act, 1)
    A2 = torch.empty_like(A1)
    w2, u2 = ops.recompute_w_u_conv(k, xv, cw, cb, beta, g, act, a_mode=1, A_out=A2)
    assert torch.equal(w1, w2), "w differs from the two-launch path"
    assert torch.equal(u1, u2), "u differs from the two-launch path"
    assert torch.equal(A1, A2), "A differs from the two-launch path"


def test_reference_sign_and_many_units():
    """a_mode -1 ((I - M)^-1) and B*T/64*H units well above the SM count, so every CTA
    walks many units through the three-stage ring."""
    from theorem_b200 import ops
    B, T, H, K, V = 2, 4096, 16, 128, 128
    k, xv, cw, cb, beta, g = (t.to(DEV) for t in _inputs(B, T, H, K, V, seed=11))
    w1, u1, _, _ = _two_launch(k, xv, cw, cb, beta, g, "silu", -1)
    w2, u2 = ops.recompute_w_u_conv(k, xv, cw, cb, beta, g, "silu", a_mode=-1)
    assert torch.equal(w1, w2) and torch.equal(u1, u2)
    w3, u3 = ops.recompute_w_u_conv(k, xv, cw, cb, beta, g, "silu", a_mode=-1)
    assert torch.equal(w2, w3) and torch.equal(u2, u3), "repeated calls differ"


def test_matches_oracle():
    """The fused op against the oracle's conv then recompute_w_u (A built in fp64),
    with the conv output rounded to bf16 as the chain stores it."""
    from theorem_b200 import ops
    B, T, H, K, V = 1, 192, 2, 128, 128
    k, xv, cw, cb, beta, g = _inputs(B, T, H, K, V, seed=5)
    w, u = ops.recompute_w_u_conv(*(t.to(DEV) for t in (k, xv, cw, cb, beta, g)), "silu", a_mode=1)
    # oracle conv on the channel-last projection, SiLU, rounded to bf16 as the chain stores v
    vo = orc.causal_conv1d(xv.float().numpy(), cw.numpy(), cb.numpy(), "silu", layout="bsd")
    v = torch.from_numpy(np.asarray(vo)).reshape(B, T, H, V).to(torch.bfloat16).float()
    A = orc.build_A(k.float(), beta, g, 1)
    rw, ru = orc.recompute_w_u(k.float(), v, beta, A, g)
    assert_close(w.float().cpu().double(), torch.from_numpy(rw), TOL, TOL, "w vs oracle")
    assert_close(u.float().cpu().double(), torch.from_numpy(ru), TOL, TOL, "u vs oracle")


def test_rejects_unsupported():
    from theorem_b200 import ops
    k, xv, cw, cb, beta, g = (t.to(DEV) for t in _inputs(1, 64, 2, 128, 128, seed=1))
    with pytest.raises(Exception):
        ops.recompute_w_u_conv(k, xv, cw[:, :3].contiguous(), cb, beta, g, "silu", a_mode=1)  # width 3
    with pytest.raises(Exception):
        ops.recompute_w_u_conv(k, xv, cw, cb, beta, g, "silu", a_mode=0)


def test_single_chunk_sequences():
    """T = 64: every unit is a sequence start, so each reads a zero conv history (the
    4-D TMA fills the rows before t = 0 of every sequence, not the previous one's)."""
    from theorem_b200 import ops
    B, T, H, K, V = 3, 64, 5, 128, 128
    k, xv, cw, cb, beta, g = (t.to(DEV) for t in _inputs(B, T, H, K, V, seed=31))
    w1, u1, _, _ = _two_launch(k, xv, cw, cb, beta, g, "silu", 1)
    w2, u2 = ops.recompute_w_u_conv(k, xv, cw, cb, beta, g, "silu", a_mode=1)
    assert torch.equal(w1, w2) and torch.equal(u1, u2)
