"""Vectorised fp32 torch-CPU form of the reference's eager baselines -- TEST / BASELINE ONLY.

Restates benchmarks/pytorch_baseline.py:121-229 (``_causal_conv1d_eager``,
``_chunk_fwd_h_eager``, ``_chunk_fwd_o_eager``, ``_recompute_w_u_eager``) --
the functions the reference itself times against its kernels -- plus the
pieces the gated-DeltaNet chain needs beyond them (SiLU / L2 norm, the
upstream WY producer of recompute_w_u/reference.py:48-91 with the chain's
sign, and the delta-rule state recurrence). This is what ``bench.py`` times
on the host cores as the CPU baseline ("port" of the reference's own CPU
path); ``oracle.ops`` remains the float64 checker.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

BT = 64


def causal_conv1d_bds(x, weight, bias):
    """pytorch_baseline.py:121-127: F.pad + grouped F.conv1d on [B, D, S]."""
    W = weight.shape[1]
    return F.conv1d(F.pad(x, (W - 1, 0)), weight.unsqueeze(1), bias=bias, groups=x.shape[1])


def causal_conv1d_bsd(x, weight, bias, silu=True):
    """Channel-last [B, S, D] form of the same conv (+ SiLU) for the chain."""
    out = causal_conv1d_bds(x.transpose(1, 2), weight, bias).transpose(1, 2)
    return F.silu(out) if silu else out


def chunk_fwd_h(k, v, g):
    """pytorch_baseline.py:130-168: per-chunk loop, vectorised over (b, h)."""
    B, T, H, K = k.shape
    V = v.shape[-1]
    NT = T // BT
    kc, vc, gc = k.reshape(B, NT, BT, H, K), v.reshape(B, NT, BT, H, V), g.reshape(B, NT, BT, H)
    h = torch.zeros(B, NT, H, K, V)
    state = torch.zeros(B, H, K, V)
    for c in range(NT):
        gend = gc[:, c, -1, :]
        vg = vc[:, c] * torch.exp(gend.unsqueeze(1) - gc[:, c]).unsqueeze(-1)
        upd = torch.matmul(kc[:, c].permute(0, 2, 3, 1), vg.permute(0, 2, 1, 3))
        state = state * torch.exp(gend)[..., None, None] + upd
        h[:, c] = state
    return h


def chunk_fwd_o(q, k, v, g, h, scale):
    """pytorch_baseline.py:171-204: batched masked qk, local + global terms."""
    B, T, H, K = q.shape
    V = v.shape[-1]
    NT = T // BT
    qc = q.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    kc = k.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    vc = v.reshape(B, NT, BT, H, V).permute(0, 1, 3, 2, 4)
    gc = g.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    qg = qc * torch.exp(gc).unsqueeze(-1)
    vg = vc * torch.exp(-gc).unsqueeze(-1)
    causal = torch.tril(torch.ones(BT, BT, dtype=torch.bool))
    qk = torch.matmul(qg, kc.transpose(-1, -2)) * causal
    out = scale * (torch.matmul(qk, vg) + torch.matmul(qg, h))
    return out.permute(0, 1, 3, 2, 4).reshape(B, T, H, V)


def recompute_w_u(k, v, beta, A, g):
    """pytorch_baseline.py:207-229."""
    B, T, H, K = k.shape
    V = v.shape[-1]
    NT = T // BT
    kc = k.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    vc = v.reshape(B, NT, BT, H, V).permute(0, 1, 3, 2, 4)
    bc = beta.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    gc = g.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    Ac = A.reshape(B, NT, BT, H, BT).permute(0, 1, 3, 2, 4)
    u = torch.matmul(Ac, vc * bc.unsqueeze(-1))
    w = torch.matmul(Ac, kc * (bc * torch.exp(gc)).unsqueeze(-1))
    return (w.permute(0, 1, 3, 2, 4).reshape(B, T, H, K), u.permute(0, 1, 3, 2, 4).reshape(B, T, H, V))


def wy_matrix(k, beta, g, sign: int = 1):
    """A = (I + sign * strict_tril(beta_i k_i.k_j e^{g_i - g_j}))^-1 per chunk, [B,T,H,BT].

    Same steps as recompute_w_u/reference.py:48-91 (which uses sign = -1)."""
    B, T, H, K = k.shape
    NT = T // BT
    kc = k.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    bc = beta.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    gc = g.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    lower = torch.tril(torch.ones(BT, BT, dtype=torch.bool), -1)
    d = torch.where(lower, gc.unsqueeze(-1) - gc.unsqueeze(-2), torch.zeros(()))
    m = torch.matmul(kc, kc.transpose(-1, -2)) * bc.unsqueeze(-1) * torch.exp(d) * lower
    eye = torch.eye(BT).expand_as(m)
    a = torch.linalg.solve_triangular(eye + sign * m, eye, upper=False, unitriangular=True)
    return a.permute(0, 1, 3, 2, 4).reshape(B, T, H, BT)


def chunk_fwd_h_delta(k, w, u, g, h0=None):
    """Delta-rule recurrence vectorised over (b, h): (h entering each chunk, v_new, final)."""
    B, T, H, K = k.shape
    V = u.shape[-1]
    NT = T // BT
    kc, wc, uc = (x.reshape(B, NT, BT, H, -1) for x in (k, w, u))
    gc = g.reshape(B, NT, BT, H)
    h = torch.empty(B, NT, H, K, V)
    vnew = torch.empty(B, NT, BT, H, V)
    state = torch.zeros(B, H, K, V) if h0 is None else h0.clone()
    for c in range(NT):
        h[:, c] = state
        vn = uc[:, c] - torch.matmul(wc[:, c].permute(0, 2, 1, 3), state).permute(0, 2, 1, 3)
        vnew[:, c] = vn
        gl = gc[:, c, -1, :]
        vs = vn * torch.exp(gl.unsqueeze(1) - gc[:, c]).unsqueeze(-1)
        state = state * torch.exp(gl)[..., None, None] + torch.matmul(kc[:, c].permute(0, 2, 3, 1),
                                                                      vs.permute(0, 2, 1, 3))
    return h, vnew.reshape(B, T, H, V), state


def chunk_fwd_o_exact_decay(q, k, v, g, h, scale):
    """chunk_fwd_o with the decay exp(g_t - g_s) formed on the masked tile (as the
    B200 kernel does); the reference's q e^g / v e^-g factorisation overflows for
    the chain's long cumulative gates only in extreme cases, but this keeps the
    CPU chain robust."""
    B, T, H, K = q.shape
    V = v.shape[-1]
    NT = T // BT
    qc = q.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    kc = k.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4)
    vc = v.reshape(B, NT, BT, H, V).permute(0, 1, 3, 2, 4)
    gc = g.reshape(B, NT, BT, H).permute(0, 1, 3, 2)
    causal = torch.tril(torch.ones(BT, BT, dtype=torch.bool))
    dec = torch.exp(torch.where(causal, gc.unsqueeze(-1) - gc.unsqueeze(-2), torch.zeros(()))) * causal
    qk = torch.matmul(qc, kc.transpose(-1, -2)) * dec
    out = scale * (torch.matmul(qk, vc) + torch.matmul(qc * torch.exp(gc).unsqueeze(-1), h))
    return out.permute(0, 1, 3, 2, 4).reshape(B, T, H, V)


def gated_delta_chain(xq, xk, xv, wq, bq, wk, bk, wv, bv, beta, g, H, K, V, h0=None, scale=None):
    """conv+SiLU -> l2norm(q, k) -> WY (sign +1) -> w, u -> delta h -> o. fp32 CPU."""
    B, T, _ = xq.shape
    q = causal_conv1d_bsd(xq, wq, bq).reshape(B, T, H, K)
    k = causal_conv1d_bsd(xk, wk, bk).reshape(B, T, H, K)
    v = causal_conv1d_bsd(xv, wv, bv).reshape(B, T, H, V)
    q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6)
    k = k / torch.sqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    A = wy_matrix(k, beta, g, 1)
    w, u = recompute_w_u(k, v, beta, A, g)
    h, vnew, final = chunk_fwd_h_delta(k, w, u, g, h0)
    o = chunk_fwd_o_exact_decay(q, k, vnew, g, h, K ** -0.5 if scale is None else scale)
    return o, final
