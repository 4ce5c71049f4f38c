"""Seeded CPU inputs with BASELINE.json's distributions (configs 2-5), for tests.

Notation N(m, s2) is mean / variance. g is the within-chunk cumulative sum of
logsigmoid(N(0,1))/16; beta = sigmoid(N(0,1)); q, k are L2-normalised over K.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

BT = 64


def gate(B, T, H, gen):
    inc = F.logsigmoid(torch.randn(B, T, H, generator=gen)) / 16
    return inc.reshape(B, T // BT, BT, H).cumsum(2).reshape(B, T, H).contiguous()


def l2n(x):
    return x / x.norm(dim=-1, keepdim=True)


def deltanet_inputs(B, T, H, K, V, seed, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    q = l2n(torch.randn(B, T, H, K, generator=gen)).to(dtype)
    k = l2n(torch.randn(B, T, H, K, generator=gen)).to(dtype)
    v = torch.randn(B, T, H, V, generator=gen).to(dtype)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    g = gate(B, T, H, gen)
    return dict(q=q, k=k, v=v, beta=beta, g=g)


def chain_inputs(B, T, H, K, V, W, seed, device, dtype=torch.bfloat16):
    """Inputs of the layer forward (BASELINE config 5 distributions), generated on
    ``device`` from a seeded generator: q/k/v projections [B, T, H*K|H*V] ~ N(0,1),
    depthwise conv weights ~ N(0, 1/4), biases ~ N(0, 0.1), beta = sigmoid(N(0,1)),
    g = within-chunk cumsum of logsigmoid(N(0,1))/16."""
    gen = torch.Generator(device=device).manual_seed(seed)
    D, DV = H * K, H * V
    xq = torch.randn(B, T, D, generator=gen, device=device).to(dtype)
    xk = torch.randn(B, T, D, generator=gen, device=device).to(dtype)
    xv = torch.randn(B, T, DV, generator=gen, device=device).to(dtype)
    cw = [torch.randn(n, W, generator=gen, device=device) * 0.5 for n in (D, D, DV)]
    cb = [torch.randn(n, generator=gen, device=device) * 0.1 ** 0.5 for n in (D, D, DV)]
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen, device=device))
    inc = F.logsigmoid(torch.randn(B, T, H, generator=gen, device=device)) / 16
    g = inc.reshape(B, T // BT, BT, H).cumsum(2).reshape(B, T, H).contiguous()
    return xq, xk, xv, cw, cb, beta, g
