"""GPU parity of the whole gated-DeltaNet layer forward (theorem_b200.chain):
causal_conv1d(+SiLU, +L2 norm) on q, k -> recompute_w_u with the v conv folded in
(in-kernel WY solve) -> the fused chunk_fwd_h + chunk_fwd_o kernel (or the v conv,
recompute_w_u, chunk_fwd_h and chunk_fwd_o as separate kernels),
against the float64 oracle chain (oracle.ops.gated_delta_chain) at the north
star's bf16 tolerance rtol = atol = 1e-2 (kernels/chunk_fwd_o/task.yml, applied
as eval.py:85-117 does through verbose_allclose).

The oracle rounds to bf16 exactly the intermediates the CUDA chain stores in
bf16 (conv outputs, w, u, v_new); everything else it keeps in float64."""
import numpy as np
import pytest
import torch

from oracle import ops as orc
from tests.harness import assert_close
from tests.synth import chain_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2


def _bf(a):
    return torch.from_numpy(np.asarray(a)).to(torch.bfloat16).double().numpy()


def _oracle_seq(xs, cw, cb, beta, g, b, h, K, V, h0=None):
    """Oracle chain of sequence (b, h): the conv is depthwise and the L2 norm is per
    head, so the head's own channels are all the oracle needs."""
    cq, cv = slice(h * K, (h + 1) * K), slice(h * V, (h + 1) * V)
    xq, xk, xv = (x[b:b + 1, :, s].float().cpu() for x, s in zip(xs, (cq, cq, cv)))
    ws = [cw[0][cq].cpu(), cw[1][cq].cpu(), cw[2][cv].cpu()]
    bs = [cb[0][cq].cpu(), cb[1][cq].cpu(), cb[2][cv].cpu()]
    be = beta[b:b + 1, :, h:h + 1].cpu()
    gg = g[b:b + 1, :, h:h + 1].cpu()
    hh0 = None if h0 is None else h0[b:b + 1, h:h + 1].cpu().double().numpy()
    return orc.gated_delta_chain(xq, xk, xv, ws[0], bs[0], ws[1], bs[1], ws[2], bs[2], be, gg, 1, K, V,
                                 h0=hh0, round_bf16=_bf)


@pytest.mark.parametrize("fused", [True, False])
def test_chain_matches_oracle_every_sequence(fused):
    from theorem_b200.chain import GatedDeltaNetForward
    B, T, H, K = 2, 512, 3, 128
    xq, xk, xv, cw, cb, beta, g = chain_inputs(B, T, H, K, K, 4, 21, DEV)
    layer = GatedDeltaNetForward(H, K, K, cw, cb, fused=fused)
    assert layer.uses_fused(torch.bfloat16) == fused
    gen = torch.Generator(device=DEV).manual_seed(5)
    h0 = torch.randn(B, H, K, K, generator=gen, device=DEV) * 0.1 ** 0.5
    o, fin = layer(xq, xk, xv, beta, g, h0=h0)
    for b in range(B):
        for h in range(H):
            ro, rfin = _oracle_seq((xq, xk, xv), cw, cb, beta, g, b, h, K, K, h0=h0)
            assert_close(o[b:b + 1, :, h:h + 1].float().cpu().double(), torch.from_numpy(ro), TOL, TOL,
                         f"o b={b} h={h}")
            assert_close(fin[b:b + 1, h:h + 1].cpu().double(), torch.from_numpy(rfin), TOL, TOL,
                         f"final b={b} h={h}")


def test_chain_config5_sampled_sequences():
    """BASELINE config 5 at full size (B=16, T=8192, H=16, K=V=128, D=2048, W=4,
    h0 = 0): the layer runs on the whole batch, four (b, h) sequences spread over
    the batch and heads (each 128 chunks of carried state) are checked against the
    oracle chain in full."""
    from theorem_b200.chain import GatedDeltaNetForward
    B, T, H, K = 16, 8192, 16, 128
    xq, xk, xv, cw, cb, beta, g = chain_inputs(B, T, H, K, K, 4, 1234, DEV)
    layer = GatedDeltaNetForward(H, K, K, cw, cb)
    assert layer.uses_fused(torch.bfloat16)
    o, fin = layer(xq, xk, xv, beta, g)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(o.float()).all()) and bool(torch.isfinite(fin).all())
    for b, h in [(0, 0), (5, 7), (11, 3), (15, 15)]:
        ro, rfin = _oracle_seq((xq, xk, xv), cw, cb, beta, g, b, h, K, K)
        assert_close(o[b:b + 1, :, h:h + 1].float().cpu().double(), torch.from_numpy(ro), TOL, TOL,
                     f"o b={b} h={h}")
        assert_close(fin[b:b + 1, h:h + 1].cpu().double(), torch.from_numpy(rfin), TOL, TOL,
                     f"final b={b} h={h}")


def test_conv_width_3_keeps_the_v_conv_separate():
    """The conv-folded recompute_w_u is built for conv width 4; another width runs the v
    conv and recompute_w_u as separate launches and keeps the fused state/output kernel,
    still against the oracle."""
    from theorem_b200.chain import GatedDeltaNetForward
    B, T, H, K = 1, 192, 2, 128
    xq, xk, xv, cw, cb, beta, g = chain_inputs(B, T, H, K, K, 3, 8, DEV)
    layer = GatedDeltaNetForward(H, K, K, cw, cb)
    assert layer.uses_fused(torch.bfloat16) and not layer.folds_v_conv(torch.bfloat16)
    o, fin = layer(xq, xk, xv, beta, g)
    for h in range(H):
        ro, rfin = _oracle_seq((xq, xk, xv), cw, cb, beta, g, 0, h, K, K)
        assert_close(o[:, :, h:h + 1].float().cpu().double(), torch.from_numpy(ro), TOL, TOL, f"o h={h}")
        assert_close(fin[:, h:h + 1].cpu().double(), torch.from_numpy(rfin), TOL, TOL, f"final h={h}")
