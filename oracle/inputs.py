"""Seeded input generators of the reference, restated on the CPU -- TEST INFRASTRUCTURE.

The reference's generators for causal_conv1d and chunk_fwd_h hard-code a
``cuda:0`` torch.Generator (kernels/causal_conv1d/reference.py:24,48;
kernels/chunk_fwd_h/reference.py:31-32), so on a CPU they cannot run; the
functions below draw the same distributions in the same order from a CPU
generator. The recompute_w_u and chunk_fwd_o generators already use a CPU
generator (recompute_w_u/reference.py:97, chunk_fwd_o/reference.py:48); the
restatements below reproduce them bit for bit, which
``tests/golden/make_golden.py`` asserted against the reference itself.

All tensors are float32 CPU tensors; move them to the GPU with ``.to(dev)``.
"""
from __future__ import annotations

import math

import torch

BT = 64


def conv_inputs(B, D, S, W, seed):
    """(x [B,D,S], weight [D,W], bias [D]) ~ N(0,1): causal_conv1d/reference.py:27-52."""
    gen = torch.Generator().manual_seed(int(seed))
    x = torch.randn((B, D, S), generator=gen, dtype=torch.float32)
    w = torch.randn((D, W), generator=gen, dtype=torch.float32)
    b = torch.randn((D,), generator=gen, dtype=torch.float32)
    return x, w, b


def wy_matrix_torch(k, beta, g):
    """fp32 torch form of the upstream WY producer (recompute_w_u/reference.py:48-91).

    A_c = (I - strict_tril(beta_i k_i.k_j exp(g_i - g_j)))^-1, stored [B,T,H,BT].
    Kept in torch fp32 with the reference's operation order so the drop-in
    test feeds the kernel the same A the reference harness would.
    """
    B, T, H, K = k.shape
    NT = T // BT
    kc = k.reshape(B, NT, BT, H, K).permute(0, 1, 3, 2, 4).contiguous()
    bc = beta.reshape(B, NT, BT, H).permute(0, 1, 3, 2).contiguous()
    gc = g.reshape(B, NT, BT, H).permute(0, 1, 3, 2).contiguous()
    kkt = torch.matmul(kc, kc.transpose(-1, -2))
    decay = torch.exp(gc.unsqueeze(-1) - gc.unsqueeze(-2))
    m = kkt * bc.unsqueeze(-1) * decay
    lower = torch.tril(torch.ones(BT, BT, dtype=torch.bool), diagonal=-1)
    m = m * lower
    eye = torch.eye(BT, dtype=k.dtype).expand_as(m)
    a = torch.linalg.solve_triangular(eye - m, eye, upper=False, unitriangular=True)
    return a.permute(0, 1, 3, 2, 4).contiguous().reshape(B, T, H, BT)


def wu_inputs(B, T, H, K, V, seed):
    """dict(k, v, beta, A, g) as recompute_w_u/reference.py:94-115 (generate_data)."""
    gen = torch.Generator().manual_seed(int(seed))
    k = torch.randn(B, T, H, K, generator=gen, dtype=torch.float32) * 0.1
    v = torch.randn(B, T, H, V, generator=gen, dtype=torch.float32) * 0.1
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen, dtype=torch.float32))
    g = -torch.rand(B, T, H, generator=gen, dtype=torch.float32) * 0.05
    g = g.reshape(B, T // BT, BT, H).cumsum(dim=2).reshape(B, T, H)
    A = wy_matrix_torch(k, beta, g)
    return dict(k=k, v=v, beta=beta, A=A, g=g, B=B, T=T, H=H, K=K, V=V)


def h_inputs(B, T, H, K, V, seed):
    """dict(k, v, g, B..V) as chunk_fwd_h/reference.py:15-47 (CPU generator)."""
    gen = torch.Generator().manual_seed(int(seed))
    k = torch.randn(B, T, H, K, generator=gen, dtype=torch.float32) * 0.5
    v = torch.randn(B, T, H, V, generator=gen, dtype=torch.float32) * 0.5
    inc = -0.05 * torch.rand(B, T, H, generator=gen, dtype=torch.float32) - 0.005
    g = torch.cumsum(inc.view(B, T // BT, BT, H), dim=2).reshape(B, T, H).contiguous()
    return dict(k=k, v=v, g=g, B=B, T=T, H=H, K=K, V=V)


def o_inputs(B, T, H, K, V, seed):
    """dict(q, k, v, g, h, scale, ...) as chunk_fwd_o/reference.py:36-77."""
    gen = torch.Generator().manual_seed(int(seed))
    NT = T // BT
    q = torch.randn(B, T, H, K, generator=gen, dtype=torch.float32)
    k = torch.randn(B, T, H, K, generator=gen, dtype=torch.float32)
    v = torch.randn(B, T, H, V, generator=gen, dtype=torch.float32)
    g = torch.randn(B, T, H, generator=gen, dtype=torch.float32) * 0.05
    h = torch.randn(B, NT, H, K, V, generator=gen, dtype=torch.float32) * 0.1
    return dict(q=q, k=k, v=v, g=g, h=h, scale=1.0 / math.sqrt(K), B=B, T=T, H=H,
                K=K, V=V, BT=BT, NT=NT, seed=seed)


def to_device(data, device):
    """Copy every tensor of a dict/tuple input bundle to ``device``."""
    if isinstance(data, dict):
        return {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in data.items()}
    return tuple(t.to(device) for t in data)
