"""GPU parity of the sequence-parallel delta rule (theorem_b200.sp) on one GPU:
segment summaries against the oracle, and the segmented layer forward against the
unsegmented kernel and the oracle."""
import numpy as np
import pytest
import torch

from oracle import ops as orc
from tests.harness import assert_close
from tests.synth import deltanet_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-2  # the north star's bf16 tolerance (rtol = atol = 1e-2)


def _inputs(B, T, H, K, V, seed, dtype=torch.bfloat16):
    """Chain-like inputs with a slow gate (about -0.1 per chunk), so that a state
    carried across a segment boundary still matters many chunks later."""
    d = deltanet_inputs(B, T, H, K, V, seed, dtype=dtype)
    q, k, v, beta = d["q"], d["k"], d["v"], d["beta"]
    gen = torch.Generator().manual_seed(seed + 11)
    inc = -0.003 * torch.rand(B, T, H, generator=gen) - 0.0002
    g = inc.reshape(B, T // 64, 64, H).cumsum(2).reshape(B, T, H).contiguous()
    A = orc.build_A(k.float(), beta, g, 1)
    w, u = orc.recompute_w_u(k.float(), v.float(), beta, A, g)
    gen = torch.Generator().manual_seed(seed + 7)
    h0 = torch.randn(B, H, K, V, generator=gen) * 0.3
    return q, k, torch.from_numpy(w).to(dtype), torch.from_numpy(u).to(dtype), g, h0


def test_segment_summary_matches_oracle():
    from theorem_b200 import sp
    q, k, w, u, g, _ = _inputs(2, 512, 2, 128, 128, seed=1)
    M, S = sp.segment_summary(k.to(DEV), w.to(DEV), u.to(DEV), g.to(DEV))
    eye = np.broadcast_to(np.eye(128), (2, 2, 128, 128)).copy()
    _, _, rM = orc.chunk_fwd_h_delta(k.float(), w.float(), np.zeros((2, 512, 2, 128)), g, eye)
    _, _, rS = orc.chunk_fwd_h_delta(k.float(), w.float(), u.float(), g, None)
    assert_close(M.cpu().double(), torch.from_numpy(rM), TOL, TOL, "M")
    assert_close(S.cpu().double(), torch.from_numpy(rS), TOL, TOL, "S")


@pytest.mark.parametrize("R", [1, 2, 4, 8])
def test_segmented_forward_matches_unsegmented(R):
    from theorem_b200 import ops, sp
    q, k, w, u, g, h0 = (t.to(DEV) for t in _inputs(1, 4096, 4, 128, 128, seed=2))
    scale = 128 ** -0.5
    o_ref, f_ref = ops.gated_delta_fwd_ho(q, k, w, u, g, scale, h0=h0, want_final=True)
    o, f = sp.sp_forward_local(q, k, w, u, g, scale, R, h0=h0)
    assert o.shape == o_ref.shape and f.shape == f_ref.shape
    assert_close(o.float().cpu(), o_ref.float().cpu(), TOL, TOL, f"o R={R}")
    assert_close(f.cpu(), f_ref.cpu(), TOL, TOL, f"final R={R}")


def test_segmented_forward_matches_oracle():
    from theorem_b200 import sp
    q, k, w, u, g, h0 = _inputs(2, 1024, 2, 128, 128, seed=3)
    scale = 128 ** -0.5
    o, f = sp.sp_forward_local(*(t.to(DEV) for t in (q, k, w, u, g)), scale, 4, h0=h0.to(DEV))
    bf = lambda a: torch.from_numpy(np.asarray(a)).to(torch.bfloat16).double().numpy()  # noqa: E731
    h, vn, fin = orc.chunk_fwd_h_delta(k.float(), w.float(), u.float(), g, h0)
    ro = orc.chunk_fwd_o(q.float(), k.float(), bf(vn), g, h, scale)
    assert_close(o.float().cpu().double(), torch.from_numpy(ro), TOL, TOL, "o")
    assert_close(f.cpu().double(), torch.from_numpy(fin), TOL, TOL, "final")


def test_segmented_forward_fp32_separate_kernels():
    """fp32, K = V = 64: pass 3 runs chunk_fwd_h -> chunk_fwd_o (no fused kernel)."""
    from theorem_b200 import sp
    q, k, w, u, g, h0 = _inputs(1, 512, 2, 64, 64, seed=4, dtype=torch.float32)
    scale = 64 ** -0.5
    o, f = sp.sp_forward_local(*(t.to(DEV) for t in (q, k, w, u, g)), scale, 4, h0=h0.to(DEV))
    h, vn, fin = orc.chunk_fwd_h_delta(k, w, u, g, h0)
    ro = orc.chunk_fwd_o(q, k, vn, g, h, scale)
    assert_close(o.cpu().double(), torch.from_numpy(ro), TOL, TOL, "o")
    assert_close(f.cpu().double(), torch.from_numpy(fin), TOL, TOL, "final")


def test_delta_h_without_state_output():
    """chunk_fwd_h mode 1 with h = NULL writes only v_new / final."""
    from theorem_b200 import ops
    q, k, w, u, g, h0 = (t.to(DEV) for t in _inputs(2, 256, 2, 128, 128, seed=5))
    h, vn, fin = ops.chunk_fwd_h(k, u, g, w=w, h0=h0, mode=1, want_v_new=True, want_final=True)
    none, vn2, fin2 = ops.chunk_fwd_h(k, u, g, w=w, h0=h0, mode=1, want_v_new=True, want_final=True,
                                      want_h=False)
    assert none is None
    assert torch.equal(vn, vn2) and torch.equal(fin, fin2)


@pytest.mark.parametrize("R,BH,K,V,with_x0,nout", [(7, 16, 128, 128, False, None), (3, 5, 64, 96, True, None),
                                                  (4, 2, 128, 256, True, 3), (1, 3, 32, 32, False, 1)])
def test_prefix_fold_kernel_matches_float64(R, BH, K, V, with_x0, nout):
    """One-launch fold x_{r+1} = M_r x_r + S_r against the same recurrence in float64."""
    from theorem_b200 import ops
    gen = torch.Generator().manual_seed(R * 100 + K)
    Ms = torch.randn(R, BH, K, K, generator=gen) / K ** 0.5
    Ss = torch.randn(R, BH, K, V, generator=gen)
    x0 = torch.randn(BH, K, V, generator=gen) if with_x0 else None
    out = ops.sp_prefix_fold(Ms.cuda(), Ss.cuda(), None if x0 is None else x0.cuda(), nout=nout).cpu().double()
    n = R + 1 if nout is None else nout
    x = torch.zeros(BH, K, V, dtype=torch.float64) if x0 is None else x0.double()
    ref = [x]
    for r in range(n - 1):
        x = torch.matmul(Ms[r].double(), x) + Ss[r].double()
        ref.append(x)
    ref = torch.stack(ref)
    assert out.shape == ref.shape
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-4), float((out - ref).abs().max())


def test_prefix_fold_rejects_unsupported():
    from theorem_b200 import ops
    with pytest.raises(AssertionError):  # K > 128
        ops.sp_prefix_fold(torch.zeros(2, 1, 256, 256).cuda(), torch.zeros(2, 1, 256, 32).cuda())
    with pytest.raises(AssertionError):  # V % 32 != 0
        ops.sp_prefix_fold(torch.zeros(2, 1, 64, 64).cuda(), torch.zeros(2, 1, 64, 48).cuda())


def _maps(R, B, H, K, V, seed):
    gen = torch.Generator().manual_seed(seed)
    Ms = torch.randn(R, B, H, K, K, generator=gen) / K ** 0.5
    Ss = torch.randn(R, B, H, K, V, generator=gen)
    h0 = torch.randn(B, H, K, V, generator=gen)
    return Ms, Ss, h0


@pytest.mark.parametrize("K,V", [(128, 128), (64, 128)])
def test_compose_gpu_fold_matches_float64_branch(K, V):
    """compose() on the GPU (one fold over K + V columns from [I | 0]) against its
    float64 CPU branch (the same products in a Python loop)."""
    from theorem_b200 import sp
    Ms, Ss, _ = _maps(5, 2, 3, K, V, seed=K + V)
    M_gpu, S_gpu = sp.compose(Ms.cuda(), Ss.cuda())
    M_ref, S_ref = sp.compose(Ms.double(), Ss.double())
    assert M_gpu.shape == (2, 3, K, K) and S_gpu.shape == (2, 3, K, V)
    assert torch.allclose(M_gpu.cpu().double(), M_ref, rtol=1e-4, atol=1e-4), float((M_gpu.cpu() - M_ref).abs().max())
    assert torch.allclose(S_gpu.cpu().double(), S_ref, rtol=1e-4, atol=1e-4), float((S_gpu.cpu() - S_ref).abs().max())


@pytest.mark.parametrize("K,V", [(128, 128), (64, 128)])
@pytest.mark.parametrize("with_h0", [True, False])
def test_prefix_state_gpu_matches_float64_branch(K, V, with_h0):
    """prefix_state(upto) on the GPU (the fold over Ms[:upto]) against the float64
    CPU branch, for upto = 0 (the entering state itself), 1 and R (after the last)."""
    from theorem_b200 import sp
    R = 4
    Ms, Ss, h0 = _maps(R, 1, 2, K, V, seed=3 * K + V)
    h0 = h0 if with_h0 else None
    for upto in (0, 1, R):
        got = sp.prefix_state(Ms.cuda(), Ss.cuda(), upto, None if h0 is None else h0.cuda())
        ref = sp.prefix_state(Ms.double(), Ss.double(), upto, None if h0 is None else h0.double())
        assert got.shape == (1, 2, K, V)
        assert torch.allclose(got.cpu().double(), ref, rtol=1e-4, atol=1e-4), (upto, float((got.cpu() - ref).abs().max()))
    starts = sp.prefix_states(Ms.cuda(), Ss.cuda(), None if h0 is None else h0.cuda())
    ref = sp.prefix_states(Ms.double(), Ss.double(), None if h0 is None else h0.double())
    assert torch.allclose(starts.cpu().double(), ref, rtol=1e-4, atol=1e-4)
