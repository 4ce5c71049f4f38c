"""numpy (float64) restatement of the reference's hot-path ops -- TEST INFRASTRUCTURE.

Every function cites the reference file:line it restates (paths are relative
to the yhinai/Theorem checkout). Inputs may be numpy arrays or torch CPU
tensors of any float dtype; everything is computed in float64 and returned as
float64 numpy arrays. Callers that compare against bf16 kernels pass the
bf16-rounded inputs, so the oracle sees exactly what the kernel saw.

Layouts follow the reference:
    conv   x [B, D, S] (``layout="bds"``) or channel-last x [B, S, D] (``"bsd"``)
    q,k    [B, T, H, K];  v, u, w-like [B, T, H, V|K];  beta, g [B, T, H]
    A      [B, T, H, BT]  (row t of the chunk's 64x64 matrix at position t)
    h      [B, NT, H, K, V]
"""
from __future__ import annotations

import numpy as np

BT = 64  # chunk length (kernels/recompute_w_u/reference.py:31, chunk_fwd_h/reference.py:13)


def _f64(x):
    if x is None:
        return None
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().to("cpu").float().numpy()
    return np.asarray(x, dtype=np.float64)


# --------------------------------------------------------------------------
# causal_conv1d
# --------------------------------------------------------------------------
def silu(x):
    x = _f64(x)
    return x / (1.0 + np.exp(-x))


def causal_conv1d(x, weight, bias, activation: str | None = None, layout: str = "bds"):
    """Depthwise causal conv, zero left-pad of W-1.

    out[b,d,t] = bias[d] + sum_k weight[d,k] * x[b,d,t-W+1+k]
    Restates kernels/causal_conv1d/reference.py:55-81 (F.pad + grouped
    F.conv1d) in the per-tap form of scripts/cpu_reference.py:40-63.
    ``activation="silu"`` applies SiLU to the output (
    the reference has no activation). ``layout="bsd"`` takes/returns the
    channel-last [B, S, D] tensor of the gated-DeltaNet chain.
    """
    x, w, b = _f64(x), _f64(weight), _f64(bias)
    if layout == "bsd":
        x = x.transpose(0, 2, 1)
    B, D, S = x.shape
    Dw, W = w.shape
    assert D == Dw and b.shape == (D,)
    xp = np.pad(x, ((0, 0), (0, 0), (W - 1, 0)))
    out = np.broadcast_to(b[None, :, None], (B, D, S)).copy()
    for k in range(W):
        out += w[None, :, k, None] * xp[:, :, k:k + S]
    if activation == "silu":
        out = silu(out)
    elif activation not in (None, "none"):
        raise ValueError(f"unknown activation {activation!r}")
    if layout == "bsd":
        out = out.transpose(0, 2, 1)
    return np.ascontiguousarray(out)


def l2norm(x, eps: float = 1e-6):
    """x / sqrt(sum(x^2) + eps) over the last axis (the chain's q/k norm)."""
    x = _f64(x)
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + eps)


# --------------------------------------------------------------------------
# helpers: [B, T, H, X] <-> per-chunk [B, NT, H, BT, X]
# --------------------------------------------------------------------------
def _to_chunks(x):
    B, T, H = x.shape[:3]
    rest = x.shape[3:]
    NT = T // BT
    y = x.reshape((B, NT, BT, H) + rest)
    if rest:
        return np.ascontiguousarray(y.transpose(0, 1, 3, 2, 4))
    return np.ascontiguousarray(y.transpose(0, 1, 3, 2))


def _from_chunks(y):
    B, NT, H, bt, X = y.shape
    return np.ascontiguousarray(y.transpose(0, 1, 3, 2, 4).reshape(B, NT * bt, H, X))


def _decay(gc):
    """exp(g_i - g_j) for j <= i, 0 above the diagonal; gc [..., BT]."""
    d = gc[..., :, None] - gc[..., None, :]
    mask = np.tril(np.ones((gc.shape[-1],) * 2, dtype=bool))
    return np.where(mask, np.exp(np.where(mask, d, 0.0)), 0.0)


# --------------------------------------------------------------------------
# WY matrix and recompute_w_u
# --------------------------------------------------------------------------
def build_A(k, beta, g, sign: int = -1):
    """Per-chunk WY matrix, returned in the reference's [B, T, H, BT] storage.

    M = strict_tril(beta_i * (k_i . k_j) * exp(g_i - g_j))
    sign=-1: A = (I - M)^-1  -- kernels/recompute_w_u/reference.py:48-91
             (the reference's upstream producer ``_build_A``);
    sign=+1: A = (I + M)^-1  -- the gated-DeltaNet (FLA) convention written
             in BASELINE.json config 2.
    """
    assert sign in (-1, 1)
    k, beta, g = _f64(k), _f64(beta), _f64(g)
    B, T, H, K = k.shape
    assert T % BT == 0
    kc, bc, gc = _to_chunks(k), _to_chunks(beta), _to_chunks(g)
    kkt = kc @ kc.swapaxes(-1, -2)
    M = np.tril(kkt * bc[..., :, None] * _decay(gc), -1)
    eye = np.eye(BT)
    L = eye + sign * M
    Ainv = np.linalg.solve(L, np.broadcast_to(eye, L.shape))
    Ainv = np.tril(Ainv)  # exact zeros above the diagonal
    return _from_chunks(Ainv)


def recompute_w_u(k, v, beta, A, g):
    """w = A @ (k * beta * exp(g)), u = A @ (v * beta), per 64-chunk.

    Restates kernels/recompute_w_u/reference.py:118-149 (ref_kernel).
    Returns (w [B,T,H,K], u [B,T,H,V]).
    """
    k, v, beta, A, g = map(_f64, (k, v, beta, A, g))
    kc, vc, bc, gc, Ac = map(_to_chunks, (k, v, beta, g, A))
    ks = kc * (bc * np.exp(gc))[..., None]
    vs = vc * bc[..., None]
    return _from_chunks(Ac @ ks), _from_chunks(Ac @ vs)


# --------------------------------------------------------------------------
# chunk_fwd_h
# --------------------------------------------------------------------------
def chunk_fwd_h(k, v, g):
    """Reference inter-chunk recurrence; h[b,c,h] is the POST-update state.

    state = state * exp(g_end) + k_c^T @ (v_c * exp(g_end - g_c))
    Restates kernels/chunk_fwd_h/reference.py:50-97 (vectorised over b, h).
    Returns h [B, NT, H, K, V].
    """
    k, v, g = map(_f64, (k, v, g))
    B, T, H, K = k.shape
    V = v.shape[-1]
    NT = T // BT
    kc, vc, gc = _to_chunks(k), _to_chunks(v), _to_chunks(g)
    h = np.zeros((B, NT, H, K, V))
    state = np.zeros((B, H, K, V))
    for c in range(NT):
        gend = gc[:, c, :, -1]                                   # [B,H]
        vg = vc[:, c] * np.exp(gend[..., None] - gc[:, c])[..., None]
        state = state * np.exp(gend)[..., None, None] + kc[:, c].swapaxes(-1, -2) @ vg
        h[:, c] = state
    return h


def chunk_fwd_h_delta(k, w, u, g, h0=None):
    """Gated delta-rule recurrence (extension, no reference).

    For each chunk c (h_c = state entering the chunk, h_0 = h0):
        v_new_c = u_c - w_c @ h_c
        h_{c+1} = exp(g_last) h_c + (k_c * exp(g_last - g_c))^T @ v_new_c
    Extends the loop of kernels/chunk_fwd_h/reference.py:75-95: with w = 0,
    u = v, h0 = 0 it reduces to it (h_{c+1} here == h[c] there).
    Returns (h_pre [B,NT,H,K,V] with h_pre[:,c] = h_c, v_new [B,T,H,V],
    final [B,H,K,V] = h_NT).
    """
    k, w, u, g = map(_f64, (k, w, u, g))
    B, T, H, K = k.shape
    V = u.shape[-1]
    NT = T // BT
    kc, wc, uc, gc = map(_to_chunks, (k, w, u, g))
    h = np.zeros((B, NT, H, K, V))
    vnew = np.zeros((B, NT, H, BT, V))
    state = np.zeros((B, H, K, V)) if h0 is None else _f64(h0).copy()
    for c in range(NT):
        h[:, c] = state
        vn = uc[:, c] - wc[:, c] @ state
        vnew[:, c] = vn
        gl = gc[:, c, :, -1]
        vs = vn * np.exp(gl[..., None] - gc[:, c])[..., None]
        state = state * np.exp(gl)[..., None, None] + kc[:, c].swapaxes(-1, -2) @ vs
    return h, _from_chunks(vnew), state


# --------------------------------------------------------------------------
# chunk_fwd_o
# --------------------------------------------------------------------------
def chunk_fwd_o(q, k, v, g, h, scale):
    """o = scale * (tril((q k^T) * exp(g_t - g_s)) v + (q * exp(g)) h[c]).

    Restates kernels/chunk_fwd_o/reference.py:80-142: the reference forms
    q*exp(g) and v*exp(-g) and a causal (s <= t) mask; the decay is applied
    here as exp(g_t - g_s) on the masked tile, which is the same quantity.
    h[:, c] is used for chunk c exactly as given (reference.py:113).
    Returns o [B, T, H, V].
    """
    q, k, v, g, h = map(_f64, (q, k, v, g, h))
    qc, kc, vc, gc = map(_to_chunks, (q, k, v, g))
    P = (qc @ kc.swapaxes(-1, -2)) * _decay(gc)
    local = P @ vc
    glob = (qc * np.exp(gc)[..., None]) @ h                 # h [B,NT,H,K,V]
    return _from_chunks(scale * (local + glob))


# --------------------------------------------------------------------------
# chained gated-DeltaNet layer forward (extension)
# --------------------------------------------------------------------------
def gated_delta_chain(xq, xk, xv, wq, bq, wk, bk, wv, bv, beta, g, H, K, V,
                      h0=None, scale=None, sign: int = 1, act: str = "silu",
                      round_bf16=None):
    """causal_conv1d(+SiLU) on q/k/v projections [B,T,D] -> l2norm(q,k) ->
    WY (A, w, u) -> delta-rule h (h0) -> chunk_fwd_o with v_new and h entering
    each chunk. ``round_bf16`` (callable or None) is applied to every
    intermediate the CUDA chain stores in bf16 (conv outputs, w, u, v_new), so
    the oracle sees the same rounded operands. Returns (o [B,T,H,V], final).
    """
    rnd = round_bf16 if round_bf16 is not None else (lambda a: a)
    B, T, D = _f64(xq).shape
    q = causal_conv1d(xq, wq, bq, act, "bsd").reshape(B, T, H, K)
    k = causal_conv1d(xk, wk, bk, act, "bsd").reshape(B, T, H, K)
    v = rnd(causal_conv1d(xv, wv, bv, act, "bsd").reshape(B, T, H, V))
    q = rnd(l2norm(q))
    k = rnd(l2norm(k))
    A = build_A(k, beta, g, sign)
    w, u = recompute_w_u(k, v, beta, A, g)
    w, u = rnd(w), rnd(u)
    h, vnew, final = chunk_fwd_h_delta(k, w, u, g, h0)
    vnew = rnd(vnew)
    if scale is None:
        scale = K ** -0.5
    o = chunk_fwd_o(q, k, vnew, g, h, scale)
    return o, final
