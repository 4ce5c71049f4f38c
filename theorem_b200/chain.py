"""Gated-DeltaNet layer forward built from the four C-ABI ops.

The reference runs its three DeltaNet ops only separately, each on its own
random inputs (kernels/*/reference.py); its docs compose them as
recompute_w_u -> chunk_fwd_h -> chunk_fwd_o (docs/ARCHITECTURE.md:200-235)
behind a Mamba-2 causal conv. This module chains them the gated-DeltaNet way:

    q = l2norm(silu(conv(xq)))   k = l2norm(silu(conv(xk)))   v = silu(conv(xv))
    A = (I + strict_tril(beta_i k_i.k_j e^{g_i-g_j}))^-1        (in-kernel)
    w = A (k beta e^g),  u = A (v beta)
    h_c = state entering chunk c (h_0 = h0); v_new = u - w h_c;
    h_{c+1} = e^{g_last} h_c + (k e^{g_last - g})^T v_new
    o = scale (tril(q k^T * e^{g_t - g_s}) v_new + (q e^g) h_c)

Inputs xq, xk, xv are channel-last [B, T, H*K] (bf16 or fp32); beta and g
[B, T, H] fp32 (g already the within-chunk cumulative gate). Intermediates
(q, k, v, w, u, v_new in the input dtype; h [B, T/64, H, K, V] in bf16 for
bf16 inputs -- the state is carried in fp32 inside chunk_fwd_h and only its
stored per-chunk copy is rounded -- else fp32) are kept in buffers reused
across calls with the same shape.

With bf16 inputs and K = V = 128 the last two steps run as one kernel
(ops.gated_delta_fwd_ho): the state recurrence and the output share a pass
over the chunks and h, v_new never reach HBM; with a conv width of 4 the v
conv also runs inside recompute_w_u (ops.recompute_w_u_conv: v is read only
there, so it never reaches HBM). ``fused=False`` keeps the separate v conv,
recompute_w_u, chunk_fwd_h and chunk_fwd_o launches.
"""
from __future__ import annotations

import torch

from . import ops


class GatedDeltaNetForward:
    """Callable layer forward; holds the depthwise conv weights [H*K, W] / [H*V, W]."""

    def __init__(self, H: int, K: int, V: int, conv_weights, conv_biases, activation: str = "silu",
                 scale: float | None = None, fused: bool = True):
        assert len(conv_weights) == 3 and len(conv_biases) == 3, "q, k, v conv weights and biases"
        self.H, self.K, self.V = H, K, V
        self.wq, self.wk, self.wv = (w.contiguous().float() for w in conv_weights)
        self.bq, self.bk, self.bv = (b.contiguous().float() for b in conv_biases)
        self.activation = activation
        self.scale = K ** -0.5 if scale is None else float(scale)
        self.fused = fused
        self._buf: dict = {}

    def uses_fused(self, dtype) -> bool:
        """chunk_fwd_h + chunk_fwd_o as the one fused kernel."""
        return self.fused and dtype == torch.bfloat16 and self.K == 128 and self.V == 128

    def folds_v_conv(self, dtype) -> bool:
        """The v conv inside recompute_w_u (built for conv width 4)."""
        return self.uses_fused(dtype) and self.wv.shape[1] == 4

    def _buffers(self, xq, xv, B, T):
        key = (B, T, xq.dtype, xq.device)
        if self._buf.get("key") != key:
            H, K, V = self.H, self.K, self.V
            dev, dt = xq.device, xq.dtype
            self._buf = dict(
                key=key,
                q=torch.empty(B, T, H, K, device=dev, dtype=dt),
                k=torch.empty(B, T, H, K, device=dev, dtype=dt),
                v=None if self.folds_v_conv(dt) else torch.empty(B, T, H, V, device=dev, dtype=dt),
                w=torch.empty(B, T, H, K, device=dev, dtype=dt),
                u=torch.empty(B, T, H, V, device=dev, dtype=dt),
                h=None if self.uses_fused(dt) else torch.empty(
                    B, T // 64, H, K, V, device=dev, dtype=torch.bfloat16 if dt == torch.bfloat16 else torch.float32),
            )
        return self._buf

    def __call__(self, xq, xk, xv, beta, g, h0=None, out=None, final_state: bool = True):
        B, T, Dq = xq.shape
        H, K, V = self.H, self.K, self.V
        assert Dq == H * K and xk.shape == xq.shape and xv.shape == (B, T, H * V)
        assert T % 64 == 0, "T must be a multiple of the chunk length 64"
        bf = self._buffers(xq, xv, B, T)
        q, k, v = bf["q"], bf["k"], bf["v"]
        ops.causal_conv1d_pair(xq, self.wq, self.bq, xk, self.wk, self.bk, self.activation, K,
                               out0=q.view(B, T, H * K), out1=k.view(B, T, H * K))
        if self.folds_v_conv(xq.dtype):
            w, u = ops.recompute_w_u_conv(k, xv, self.wv, self.bv, beta, g, self.activation, a_mode=1,
                                          w=bf["w"], u=bf["u"])
        else:
            ops.causal_conv1d(xv, self.wv, self.bv, self.activation, "bsd", 0, out=v.view(B, T, H * V))
            w, u = ops.recompute_w_u(k, v, beta, None, g, a_mode=1, w=bf["w"], u=bf["u"])
        if self.uses_fused(xq.dtype):
            return ops.gated_delta_fwd_ho(q, k, w, u, g, self.scale, h0=h0, want_final=final_state, o=out)
        h, v_new, fin = ops.chunk_fwd_h(k, u, g, w=w, h0=h0, mode=1, want_v_new=True, want_final=final_state,
                                        h=bf["h"], v_new=v)
        o = ops.chunk_fwd_o(q, k, v_new, g, h, self.scale, o=out)
        return o, fin

    def forward_from_host(self, xq, xk, xv, beta, g, out, slices: int = 4, h0=None):
        """The layer forward for inputs and output in pinned host memory.

        The batch is cut into ``slices`` groups of sequences and pipelined over three
        streams: the host-to-device copy of group i+1 and the device-to-host copy of
        group i-1 run while group i computes (PCIe is full duplex). Device staging is
        double-buffered; all compute stays on the caller's current stream, which on
        return is ordered after the last copy. Returns ``out`` (and the final states
        [B,H,K,V] fp32 when ``h0`` is given)."""
        B, T, D = xq.shape
        assert B % slices == 0, "B must split into equal groups"
        assert all(t.is_pinned() for t in (xq, xk, xv, beta, g, out)), "host tensors must be pinned"
        bs = B // slices
        dev = torch.device("cuda", torch.cuda.current_device())
        comp = torch.cuda.current_stream(dev)
        if getattr(self, "_host_streams", None) is None:
            self._host_streams = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
        s_in, s_out = self._host_streams
        hosts = (xq, xk, xv, beta, g)
        stage = [[torch.empty((bs,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev) for t in hosts] for _ in range(2)]
        ostage = [torch.empty((bs,) + tuple(out.shape[1:]), dtype=out.dtype, device=dev) for _ in range(2)]
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        finals = []
        for i in range(slices):
            j = i & 1
            lo, hi = i * bs, (i + 1) * bs
            if i >= 2:
                s_in.wait_event(ev_comp[j])  # group i-2 no longer reads this staging set
            with torch.cuda.stream(s_in):
                for d_, h_ in zip(stage[j], hosts):
                    d_.copy_(h_[lo:hi], non_blocking=True)
            ev_in[j].record(s_in)
            comp.wait_event(ev_in[j])
            if i >= 2:
                comp.wait_event(ev_out[j])  # group i-2's output has left this buffer
            _, fin = self(*stage[j], h0=None if h0 is None else h0[lo:hi], out=ostage[j],
                          final_state=h0 is not None)
            if fin is not None:
                finals.append(fin)
            ev_comp[j].record(comp)
            s_out.wait_event(ev_comp[j])
            with torch.cuda.stream(s_out):
                out[lo:hi].copy_(ostage[j], non_blocking=True)
            ev_out[j].record(s_out)
        comp.wait_stream(s_out)
        comp.wait_stream(s_in)
        for t in stage[0] + stage[1] + ostage:
            t.record_stream(comp)
        if h0 is not None:
            return out, torch.cat(finals, 0)
        return out
