"""GPU parity: thm_causal_conv1d_pair_fwd (the q and k projections' convs in one
launch) against two thm_causal_conv1d_fwd calls, bit for bit, and the oracle.

The pair kernel runs the single-conv kernel's strip body on one grid of 2B
sequences, so its outputs must equal the two single launches exactly; shapes the
TMA path does not take (W outside {2, 3, 4}, D * elem % 16 != 0) go through two
single launches inside the entry point."""
import pytest
import torch

from oracle import ops as orc
from tests.harness import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, S, D, W, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    xs = [torch.randn(B, S, D, generator=gen).to(dtype).to(DEV) for _ in range(2)]
    ws = [(torch.randn(D, W, generator=gen) * 0.5).to(DEV) for _ in range(2)]
    bs = [(torch.randn(D, generator=gen) * 0.3).to(DEV) for _ in range(2)]
    return xs, ws, bs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("act", ["silu", None])
@pytest.mark.parametrize("B,S,D,W,G", [
    (1, 77, 256, 4, 128),      # one sequence per conv: the grid's z splits 1 + 1
    (3, 700, 640, 4, 128),     # partial channel block, several strips, partial tiles
    (5, 257, 1024, 3, 64),
    (2, 33, 264, 2, 0),
    (2, 130, 256, 6, 128),     # W = 6: two single-conv launches inside the entry point
    (2, 96, 12, 4, 0),         # D = 12: bf16 rows of 24 B take no TMA map (two single launches)
])
def test_pair_equals_two_single_launches(dtype, act, B, S, D, W, G):
    from theorem_b200 import ops
    (x0, x1), (w0, w1), (b0, b1) = _inputs(B, S, D, W, dtype, seed=B * 1000 + S + D + W + G)
    r0 = ops.causal_conv1d(x0, w0, b0, act, "bsd", G)
    r1 = ops.causal_conv1d(x1, w1, b1, act, "bsd", G)
    p0, p1 = ops.causal_conv1d_pair(x0, w0, b0, x1, w1, b1, act, G)
    assert torch.equal(p0, r0), "first output differs from the single-conv launch"
    assert torch.equal(p1, r1), "second output differs from the single-conv launch"


def test_pair_long_strips_chain_shape():
    """2B = 8 sequences of T = 8192, D = 2048 (H = 16 heads of 128): the grid takes
    512-row strips, as config 5's q and k convs do on one GPU, into caller buffers."""
    from theorem_b200 import ops
    B, S, D = 4, 8192, 2048
    (x0, x1), (w0, w1), (b0, b1) = _inputs(B, S, D, 4, torch.bfloat16, seed=8)
    o0, o1 = torch.empty_like(x0), torch.empty_like(x1)
    ops.causal_conv1d_pair(x0, w0, b0, x1, w1, b1, "silu", 128, out0=o0, out1=o1)
    assert torch.equal(o0, ops.causal_conv1d(x0, w0, b0, "silu", "bsd", 128))
    assert torch.equal(o1, ops.causal_conv1d(x1, w1, b1, "silu", "bsd", 128))


def test_pair_matches_oracle():
    from theorem_b200 import ops
    B, S, D, G = 2, 300, 512, 128
    (x0, x1), (w0, w1), (b0, b1) = _inputs(B, S, D, 4, torch.bfloat16, seed=3)
    p0, p1 = ops.causal_conv1d_pair(x0, w0, b0, x1, w1, b1, "silu", G)
    for p, x, w, b in ((p0, x0, w0, b0), (p1, x1, w1, b1)):
        ref = orc.causal_conv1d(x.float().cpu(), w.cpu(), b.cpu(), "silu", layout="bsd")
        ref = orc.l2norm(ref.reshape(B, S, D // G, G)).reshape(B, S, D)
        assert_close(p.float().cpu().double(), torch.from_numpy(ref), 1e-2, 1e-2, "pair vs oracle")


def test_pair_empty_batch_and_rejections():
    from theorem_b200 import ops
    (x0, x1), (w0, w1), (b0, b1) = _inputs(0, 16, 256, 4, torch.bfloat16, seed=1)
    p0, p1 = ops.causal_conv1d_pair(x0, w0, b0, x1, w1, b1, "silu", 128)
    assert p0.shape == (0, 16, 256) and p1.shape == (0, 16, 256)
    (x0, x1), (w0, w1), (b0, b1) = _inputs(1, 16, 256, 4, torch.bfloat16, seed=2)
    with pytest.raises(AssertionError):  # shapes differ
        ops.causal_conv1d_pair(x0, w0, b0, x1[:, :8].contiguous(), w1, b1, "silu", 128)
    with pytest.raises(AssertionError):  # dtypes differ
        ops.causal_conv1d_pair(x0, w0, b0, x1.float(), w1, b1, "silu", 128)
    with pytest.raises(AssertionError):  # L2 group that does not divide D
        ops.causal_conv1d_pair(x0[..., :192].contiguous(), w0[:192].contiguous(), b0[:192].contiguous(),
                               x1[..., :192].contiguous(), w1[:192].contiguous(), b1[:192].contiguous(),
                               "silu", 128)
