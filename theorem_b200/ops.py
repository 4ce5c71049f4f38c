"""Functional host API over the C ABI (torch tensors in, torch tensors out).

Each function validates like the reference launcher it replaces (asserts on
device, dtype, contiguity and shape), allocates its outputs with
``torch.empty`` on the input's device, and launches on torch's current CUDA
stream. Nothing here computes on the CPU.
"""
from __future__ import annotations

import functools

import torch

from . import _lib as L

BT = 64
_ACT = {None: L.THM_ACT_NONE, "none": L.THM_ACT_NONE, "silu": L.THM_ACT_SILU}


def _on_input_device(fn):
    """Run the op with its first tensor argument's device current, so the
    launch (which goes to the current device) and the pointers agree even when
    the caller's current device is another GPU."""
    @functools.wraps(fn)
    def wrapped(*args, **kw):
        t = next((a for a in args if torch.is_tensor(a)), None)
        if t is not None and t.is_cuda and t.device.index != torch.cuda.current_device():
            with torch.cuda.device(t.device):
                return fn(*args, **kw)
        return fn(*args, **kw)
    return wrapped


def _cuda(*ts):
    for t in ts:
        if t is not None:
            assert t.is_cuda, "theorem_b200 ops need CUDA tensors (there is no CPU fallback)"


def _contig(*ts):
    for t in ts:
        if t is not None:
            assert t.is_contiguous(), "inputs must be contiguous"


@_on_input_device
def causal_conv1d(x, weight, bias, activation=None, layout: str = "bds", l2norm_group: int = 0,
                  out=None):
    """Depthwise causal conv (kernels/causal_conv1d/kernel.py:170-230 contract).

    layout "bds": x [B, D, S] fp32 (reference). layout "bsd": x [B, S, D] fp32 or
    bf16 (channel-last chain). weight [D, W], bias [D] fp32. Optional SiLU and
    per-``l2norm_group`` L2 norm (bsd only).
    """
    _cuda(x, weight, bias)
    _contig(x, weight, bias)
    assert weight.dtype == torch.float32 and bias.dtype == torch.float32, "weight/bias must be float32"
    assert x.dim() == 3, "x must be rank 3"
    if layout == "bds":
        B, D, S = x.shape
        lay = L.THM_LAYOUT_BDS
    elif layout == "bsd":
        B, S, D = x.shape
        lay = L.THM_LAYOUT_BSD
    else:
        raise AssertionError(f"unknown layout {layout!r}")
    Dw, W = weight.shape
    assert D == Dw, f"channel mismatch: x has D={D}, weight has D={Dw}"
    assert bias.shape == (D,), f"bias shape {tuple(bias.shape)} != ({D},)"
    if out is None:
        out = torch.empty_like(x)
    st = L.stream_of(x)
    L.check(L.load().thm_causal_conv1d_fwd(L.ptr(x), L.ptr(weight), L.ptr(bias), L.ptr(out), B, D, S, W,
                                           lay, L.dtype_code(x), _ACT[activation], int(l2norm_group), st),
            "thm_causal_conv1d_fwd")
    return out


@_on_input_device
def causal_conv1d_pair(x0, weight0, bias0, x1, weight1, bias1, activation=None, l2norm_group: int = 0,
                       out0=None, out1=None):
    """Two channel-last convs of the same shape in one launch (the layer's q and k
    projections): equal bit for bit to ``causal_conv1d(x0, weight0, bias0, activation,
    "bsd", l2norm_group)`` and the same for x1. x0, x1 [B, S, D] fp32 or bf16 of one
    dtype; weights [D, W] and biases [D] fp32. Returns (out0, out1)."""
    _cuda(x0, weight0, bias0, x1, weight1, bias1, out0, out1)
    _contig(x0, weight0, bias0, x1, weight1, bias1)
    for t in (weight0, bias0, weight1, bias1):
        assert t.dtype == torch.float32, "weight/bias must be float32"
    assert x0.dim() == 3 and x1.shape == x0.shape, "x0, x1 must be [B, S, D] of one shape"
    assert x1.dtype == x0.dtype and x1.device == x0.device, "x0, x1 must share dtype and device"
    B, S, D = x0.shape
    W = weight0.shape[1]
    for wt, bt in ((weight0, bias0), (weight1, bias1)):
        assert wt.shape == (D, W), f"weight shape {tuple(wt.shape)} != ({D}, {W})"
        assert bt.shape == (D,), f"bias shape {tuple(bt.shape)} != ({D},)"
    outs = []
    for o in (out0, out1):
        if o is None:
            o = torch.empty_like(x0)
        assert o.shape == x0.shape and o.dtype == x0.dtype and o.is_contiguous() and o.device == x0.device, \
            "out must match x in shape, dtype and device and be contiguous"
        outs.append(o)
    st = L.stream_of(x0)
    L.check(L.load().thm_causal_conv1d_pair_fwd(L.ptr(x0), L.ptr(weight0), L.ptr(bias0), L.ptr(outs[0]),
                                                L.ptr(x1), L.ptr(weight1), L.ptr(bias1), L.ptr(outs[1]),
                                                B, D, S, W, L.dtype_code(x0), _ACT[activation], int(l2norm_group), st),
            "thm_causal_conv1d_pair_fwd")
    return outs[0], outs[1]


@_on_input_device
def recompute_w_u(k, v, beta, A, g, a_mode: int = 0, w=None, u=None, A_out=None):
    """w = A (k beta e^g), u = A (v beta) per 64-chunk (kernels/recompute_w_u/kernel.py:192-248).

    a_mode 0 reads ``A`` [B,T,H,64] fp32; a_mode -1 / +1 computes
    A = (I -/+ M)^-1 in-kernel (``A`` may be None; ``A_out`` receives it).
    """
    _cuda(k, v, beta, A, g)
    _contig(k, v, beta, A, g)
    B, T, H, K = k.shape
    V = v.shape[-1]
    assert v.shape == (B, T, H, V) and v.dtype == k.dtype
    assert beta.shape == (B, T, H) and g.shape == (B, T, H)
    assert beta.dtype == torch.float32 and g.dtype == torch.float32, "beta / g must be float32"
    assert T % BT == 0, "T must be a multiple of BT (=64)"
    if a_mode == 0:
        assert A is not None and A.shape == (B, T, H, BT) and A.dtype == torch.float32
    w = torch.empty_like(k) if w is None else w
    u = torch.empty_like(v) if u is None else u
    st = L.stream_of(k)
    L.check(L.load().thm_recompute_w_u_fwd(L.ptr(k), L.ptr(v), L.ptr(beta), L.ptr(A) if a_mode == 0 else None,
                                           L.ptr(g), L.ptr(w), L.ptr(u), L.ptr(A_out), B, T, H, K, V,
                                           L.dtype_code(k), int(a_mode), st),
            "thm_recompute_w_u_fwd")
    return w, u


@_on_input_device
def recompute_w_u_conv(k, xv, conv_weight, conv_bias, beta, g, activation=None, a_mode: int = 1, w=None, u=None,
                       A_out=None):
    """recompute_w_u with v = act(causal_conv1d(xv)) formed in the same kernel.

    The layer's v projection ``xv`` [B,T,H*V] bf16 goes through the depthwise causal
    conv (``conv_weight`` [H*V, 4], ``conv_bias`` [H*V] fp32, optional SiLU) and straight
    into u = A (v beta): the chain kernels/causal_conv1d -> kernels/recompute_w_u
    (kernel.py:192-248) without v in HBM. a_mode +1 / -1 computes A in-kernel.
    """
    _cuda(k, xv, conv_weight, conv_bias, beta, g)
    _contig(k, xv, conv_weight, conv_bias, beta, g)
    B, T, H, K = k.shape
    assert k.dtype == torch.bfloat16 and xv.dtype == torch.bfloat16, "bf16 only"
    assert xv.dim() == 3 and xv.shape[:2] == (B, T) and xv.shape[2] % H == 0
    V = xv.shape[2] // H
    Dw, W = conv_weight.shape
    assert Dw == H * V and conv_bias.shape == (H * V,)
    assert conv_weight.dtype == torch.float32 and conv_bias.dtype == torch.float32, "conv weight/bias must be float32"
    assert beta.shape == (B, T, H) and g.shape == (B, T, H)
    assert beta.dtype == torch.float32 and g.dtype == torch.float32, "beta / g must be float32"
    assert T % BT == 0, "T must be a multiple of BT (=64)"
    assert a_mode in (1, -1), "the conv-fused path computes A in-kernel"
    w = torch.empty_like(k) if w is None else w
    u = torch.empty(B, T, H, V, device=k.device, dtype=k.dtype) if u is None else u
    for name, t, shape, dt in (("w", w, (B, T, H, K), k.dtype), ("u", u, (B, T, H, V), k.dtype),
                               ("A_out", A_out, (B, T, H, BT), torch.float32)):
        if t is not None:
            assert t.shape == shape and t.dtype == dt, f"{name} must be {tuple(shape)} {dt}"
            assert t.is_contiguous() and t.device == k.device, f"{name} must be contiguous on {k.device}"
    st = L.stream_of(k)
    L.check(L.load().thm_recompute_w_u_conv_fwd(L.ptr(k), L.ptr(xv), L.ptr(conv_weight), L.ptr(conv_bias),
                                                L.ptr(beta), L.ptr(g), L.ptr(w), L.ptr(u), L.ptr(A_out), B, T, H,
                                                K, V, W, _ACT[activation], int(a_mode), st),
            "thm_recompute_w_u_conv_fwd")
    return w, u


@_on_input_device
def chunk_fwd_h(k, v, g, w=None, h0=None, mode: int = 0, want_v_new: bool = False,
                want_final: bool = False, h=None, v_new=None, h_dtype=torch.float32, want_h: bool = True):
    """Inter-chunk state recurrence (kernels/chunk_fwd_h/kernel.py:141-191).

    mode 0: reference recurrence, returns h [B,NT,H,K,V] of post-update states.
    mode 1: gated delta rule (``v`` is u, ``w`` required), returns
    (h of states entering each chunk, v_new or None, final or None).
    h is stored in ``h_dtype`` (float32, or bfloat16 for the chain); the state
    itself is carried in fp32. ``want_h=False`` (mode 1) writes no per-chunk
    states and returns None for h.
    """
    _cuda(k, v, g, w, h0)
    _contig(k, v, g, w, h0)
    B, T, H, K = k.shape
    V = v.shape[-1]
    assert T % BT == 0, f"T={T} must be divisible by {BT}"
    assert v.shape == (B, T, H, V) and v.dtype == k.dtype and g.shape == (B, T, H)
    assert g.dtype == torch.float32
    NT = T // BT
    assert want_h or mode == 1, "the reference recurrence (mode 0) always returns h"
    if h is None and want_h:
        h = torch.empty(B, NT, H, K, V, device=k.device, dtype=h_dtype)
    if h is not None:
        assert h.shape == (B, NT, H, K, V) and h.dtype in (torch.float32, torch.bfloat16) and h.is_contiguous()
    final = None
    if mode == 1:
        assert w is not None and w.shape == k.shape and w.dtype == k.dtype
        if h0 is not None:
            assert h0.shape == (B, H, K, V) and h0.dtype == torch.float32
        if v_new is not None:
            assert v_new.shape == v.shape and v_new.dtype == v.dtype and v_new.is_contiguous()
        elif want_v_new:
            v_new = torch.empty_like(v)
        if want_final:
            final = torch.empty(B, H, K, V, device=k.device, dtype=torch.float32)
    else:
        assert w is None and h0 is None and v_new is None
    st = L.stream_of(k)
    L.check(L.load().thm_chunk_fwd_h_fwd(L.ptr(k), L.ptr(w), L.ptr(v), L.ptr(g), L.ptr(h0), L.ptr(h),
                                         L.ptr(v_new), L.ptr(final), B, T, H, K, V, L.dtype_code(k),
                                         L.dtype_code(h) if h is not None else L.dtype_code(k), int(mode), st),
            "thm_chunk_fwd_h_fwd")
    if mode == 1:
        return h, v_new, final
    return h


@_on_input_device
def chunk_fwd_o(q, k, v, g, h, scale: float, o=None):
    """Chunkwise output (kernels/chunk_fwd_o/kernel.py:146-212)."""
    _cuda(q, k, v, g, h)
    _contig(q, k, v, g, h)
    B, T, H, K = q.shape
    V = v.shape[-1]
    assert k.shape == q.shape and k.dtype == q.dtype and v.dtype == q.dtype
    assert v.shape == (B, T, H, V) and g.shape == (B, T, H) and g.dtype == torch.float32
    assert T % BT == 0, f"T={T} must be divisible by BT={BT}"
    NT = T // BT
    assert h.shape == (B, NT, H, K, V) and h.dtype in (torch.float32, torch.bfloat16), \
        "h must be [B,NT,H,K,V] float32 (or bfloat16 with bfloat16 q/k/v)"
    if o is None:
        o = torch.empty(B, T, H, V, dtype=q.dtype, device=q.device)
    st = L.stream_of(q)
    L.check(L.load().thm_chunk_fwd_o_fwd(L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(h), L.ptr(o),
                                         float(scale), B, T, H, K, V, L.dtype_code(q), L.dtype_code(h), st),
            "thm_chunk_fwd_o_fwd")
    return o


@_on_input_device
def gated_delta_fwd_ho(q, k, w, u, g, scale: float, h0=None, want_final: bool = False, o=None):
    """chunk_fwd_h (delta rule) and chunk_fwd_o fused in one kernel: returns
    (o, final state or None). Same result as
    ``chunk_fwd_h(k, u, g, w=w, h0=h0, mode=1, want_v_new=True, h_dtype=bf16)``
    followed by ``chunk_fwd_o(q, k, v_new, g, h, scale)``, without writing h or
    v_new (kernels/chunk_fwd_h/kernel.py:141-191 + kernels/chunk_fwd_o/kernel.py:146-212).
    Built for bf16, K = V = 128."""
    _cuda(q, k, w, u, g, h0)
    _contig(q, k, w, u, g, h0)
    B, T, H, K = q.shape
    V = u.shape[-1]
    assert k.shape == q.shape and w.shape == q.shape and u.shape == (B, T, H, V)
    assert k.dtype == q.dtype and w.dtype == q.dtype and u.dtype == q.dtype
    assert g.shape == (B, T, H) and g.dtype == torch.float32
    assert T % BT == 0, f"T={T} must be divisible by BT={BT}"
    if h0 is not None:
        assert h0.shape == (B, H, K, V) and h0.dtype == torch.float32
    if o is None:
        o = torch.empty(B, T, H, V, dtype=q.dtype, device=q.device)
    assert o.shape == (B, T, H, V) and o.dtype == q.dtype and o.is_contiguous()
    final = torch.empty(B, H, K, V, device=q.device, dtype=torch.float32) if want_final else None
    st = L.stream_of(q)
    L.check(L.load().thm_gated_delta_fwd_ho(L.ptr(q), L.ptr(k), L.ptr(w), L.ptr(u), L.ptr(g), L.ptr(h0), L.ptr(o),
                                            L.ptr(final), float(scale), B, T, H, K, V, L.dtype_code(q), st),
            "thm_gated_delta_fwd_ho")
    return o, final


@_on_input_device
def sp_prefix_fold(Ms, Ss, x0=None, nout: int | None = None, out=None):
    """States entering consecutive segments: out[0] = x0 (or 0), out[r+1] =
    Ms[r] out[r] + Ss[r]. Ms [R, BH, K, K], Ss [R, BH, K, V], x0 [BH, K, V] fp32;
    returns out [nout, BH, K, V] (nout <= R + 1, default R + 1). One launch; the
    state of each (bh, 32-column tile) stays in shared memory across the steps."""
    _cuda(Ms, Ss, x0)
    _contig(Ms, Ss, x0)
    R, BH, K, V = Ss.shape
    assert Ms.shape == (R, BH, K, K), f"Ms shape {tuple(Ms.shape)} != {(R, BH, K, K)}"
    assert Ms.dtype == torch.float32 and Ss.dtype == torch.float32, "segment maps must be float32"
    if x0 is not None:
        assert x0.shape == (BH, K, V) and x0.dtype == torch.float32
    nout = R + 1 if nout is None else int(nout)
    assert 1 <= nout <= R + 1
    if out is None:
        out = torch.empty(nout, BH, K, V, device=Ss.device, dtype=torch.float32)
    assert out.shape == (nout, BH, K, V) and out.dtype == torch.float32 and out.is_contiguous()
    st = L.stream_of(Ss)
    L.check(L.load().thm_sp_prefix_fold(L.ptr(Ms), L.ptr(Ss), L.ptr(x0), L.ptr(out), nout, BH, K, V, st),
            "thm_sp_prefix_fold")
    return out


@_on_input_device
def build_A(k, beta, g, sign: int = -1, out=None):
    """Per-chunk WY matrix A = (I + sign*M)^-1, M = strict_tril(beta_i k_i.k_j e^{g_i-g_j})
    (kernels/recompute_w_u/reference.py:48-91 ``_build_A`` is sign = -1). Returns
    A [B,T,H,64] fp32 -- the ``A`` input of ``recompute_w_u`` with a_mode 0."""
    _cuda(k, beta, g)
    _contig(k, beta, g)
    B, T, H, K = k.shape
    assert T % BT == 0, f"T={T} must be divisible by BT={BT}"
    assert beta.shape == (B, T, H) and g.shape == (B, T, H)
    assert beta.dtype == torch.float32 and g.dtype == torch.float32
    assert sign in (-1, 1)
    if out is None:
        out = torch.empty(B, T, H, BT, device=k.device, dtype=torch.float32)
    assert out.shape == (B, T, H, BT) and out.dtype == torch.float32 and out.is_contiguous()
    st = L.stream_of(k)
    L.check(L.load().thm_build_A_fwd(L.ptr(k), L.ptr(beta), L.ptr(g), L.ptr(out), B, T, H, K, L.dtype_code(k),
                                     int(sign), st), "thm_build_A_fwd")
    return out


@_on_input_device
def chunk_local_cumsum(g_inc, scale: float = 1.0, out=None):
    """g[b, c*64+i, h] = scale * sum_{j<=i} g_inc[b, c*64+j, h] per 64-token chunk: the
    chunk-local cumulative gate the reference's generators build
    (kernels/chunk_fwd_h/reference.py:41-45). ``out`` may be ``g_inc`` (in place)."""
    _cuda(g_inc)
    _contig(g_inc)
    assert g_inc.dtype == torch.float32 and g_inc.dim() == 3, "g_inc must be [B,T,H] float32"
    B, T, H = g_inc.shape
    assert T % BT == 0, f"T={T} must be divisible by BT={BT}"
    if out is None:
        out = torch.empty_like(g_inc)
    assert out.shape == g_inc.shape and out.dtype == torch.float32 and out.is_contiguous()
    st = L.stream_of(g_inc)
    L.check(L.load().thm_chunk_local_cumsum_fwd(L.ptr(g_inc), L.ptr(out), B, T, H, float(scale), st),
            "thm_chunk_local_cumsum_fwd")
    return out
