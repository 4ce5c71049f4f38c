"""Sequence-parallel gated delta rule: long sequences split along T into segments.

The delta-rule recurrence (kernels/chunk_fwd_h/kernel.py:61-138 extended with the
delta rule, as ``chunk_fwd_h`` mode 1 computes it) is affine in the state:

    h_{c+1} = (e^{g_last} I - K~_c^T w_c) h_c + K~_c^T u_c,   K~_c = k_c e^{g_last - g_c}

so a segment of chunks maps its entering state h to M h + S, with M (K x K) the
product of the per-chunk linear parts and S (K x V) the state it reaches from 0:

    M_r: the recurrence with u = 0 started from h = I   (its final state)
    S_r: the recurrence with the real u started from 0  (its final state)
    h_start(r) = M_{r-1} (... (M_0 h0 + S_0) ...) + S_{r-1}

Three passes, each a batched launch of this library's kernels in which every
segment is one more "sequence" of the batch ([B, T, H, X] viewed as
[B*R, T/R, H, X], a free view since the segments are contiguous in T):

  1. (M_r, S_r) of every segment: two chunk_fwd_h launches, no per-chunk states
     written;
  2. the prefix fold over segments: R-1 small K x K by K x V products per head in
     fp32, one launch of ``ops.sp_prefix_fold`` on the GPU;
  3. state recurrence + output of every segment from its entering state
     (the fused gated_delta_fwd_ho kernel for bf16, K = V = 128).

On one GPU this turns B*H sequences into B*H*R independent CTAs (B = 1, H = 16
fills 16 of 148 SMs; R = 8 fills 128). Across ranks (``sp_forward``) each rank
holds a contiguous part of T, composes its local segments into one (M, S) pair,
and the pairs are all-gathered (NCCL over NVLink on GPUs: 2 MiB per rank at
B = 1, H = 16, K = V = 128) -- the only exchange on the data path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


_CONST: dict = {}


def _constants(k):
    """The zero u and identity h0 of the M summary for k's shape, kept across calls
    (read-only inputs of the kernel, so one copy per shape and device serves all).

    The zero u is as large as k (512 MiB at B = 1, T = 131072, H = 16, K = 128
    in bf16), so at most two shapes are kept; ``release_constants()`` frees them.
    Before an entry is dropped the device is synchronized, so no kernel still in
    flight on any stream reads memory the caching allocator hands out again."""
    B, T, H, K = k.shape
    key = (tuple(k.shape), k.dtype, k.device)
    if key not in _CONST:
        if len(_CONST) >= 2:
            release_constants()
        _CONST[key] = (torch.zeros_like(k),
                       torch.eye(K, device=k.device, dtype=torch.float32).expand(B, H, K, K).contiguous())
    return _CONST[key]


def release_constants():
    """Free the cached M-summary constants (after the kernels using them are done)."""
    for (shape, dtype, dev) in list(_CONST):
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
    _CONST.clear()


def segment_summary(k, w, u, g):
    """(M, S) of each sequence of the batch: M [B,H,K,K], S [B,H,K,V] fp32."""
    zero_u, eye = _constants(k)
    _, _, M = ops.chunk_fwd_h(k, zero_u, g, w=w, h0=eye, mode=1, want_final=True, want_h=False)
    _, _, S = ops.chunk_fwd_h(k, u, g, w=w, h0=None, mode=1, want_final=True, want_h=False)
    return M, S


def _acc_dtype(t):
    return torch.float64 if t.dtype == torch.float64 else torch.float32


def _fold_on_gpu(Ss):
    return Ss.is_cuda and Ss.dtype != torch.float64


def prefix_states(Ms, Ss, h0=None):
    """States entering each of R consecutive segments, [R,B,H,K,V], from the
    segment summaries Ms [R,B,H,K,K], Ss [R,B,H,K,V] and the state h0 entering
    the first (None = 0). On the GPU one ``ops.sp_prefix_fold`` launch; CPU
    tensors (the gloo tests of the multi-rank logic) use torch products."""
    R, B, H, K, V = Ss.shape
    if _fold_on_gpu(Ss):
        x0 = None if h0 is None else h0.float().reshape(B * H, K, V).contiguous()
        out = ops.sp_prefix_fold(Ms.float().reshape(R, B * H, K, K).contiguous(),
                                 Ss.float().reshape(R, B * H, K, V).contiguous(), x0, nout=R)
        return out.reshape(R, B, H, K, V)
    dt = _acc_dtype(Ss)
    out = torch.empty(R, B * H, K, V, dtype=dt, device=Ss.device)
    if h0 is None:
        out[0].zero_()
    else:
        out[0].copy_(h0.reshape(B * H, K, V))
    Mf = Ms.to(dt).reshape(R, B * H, K, K)
    Sf = Ss.to(dt).reshape(R, B * H, K, V)
    for r in range(1, R):
        torch.baddbmm(Sf[r - 1], Mf[r - 1], out[r - 1], out=out[r])  # h_r = M h_{r-1} + S
    return out.reshape(R, B, H, K, V)


def prefix_state(Ms, Ss, upto: int, h0=None):
    """State entering segment ``upto`` (``upto`` = R: the state after the last one)."""
    R, B, H, K, V = Ss.shape
    if _fold_on_gpu(Ss):
        x0 = None if h0 is None else h0.float().reshape(B * H, K, V).contiguous()
        if upto == 0:
            return torch.zeros(B, H, K, V, device=Ss.device) if x0 is None else x0.reshape(B, H, K, V).clone()
        out = ops.sp_prefix_fold(Ms[:upto].float().reshape(upto, B * H, K, K).contiguous(),
                                 Ss[:upto].float().reshape(upto, B * H, K, V).contiguous(), x0)
        return out[upto].reshape(B, H, K, V)
    dt = _acc_dtype(Ss)
    h = torch.zeros(B, H, K, V, dtype=dt, device=Ss.device) if h0 is None else h0.to(dt).clone()
    for r in range(upto):
        h = torch.matmul(Ms[r].to(dt), h) + Ss[r].to(dt)
    return h


def compose(Ms, Ss):
    """(M, S) of R consecutive segments taken as one. On the GPU one fold over
    K + V columns: x_0 = [I | 0], x_{r+1} = M_r x_r + [0 | S_r] ends at
    [prod M | composed S]."""
    if _fold_on_gpu(Ss) and Ss.shape[0] > 1:
        R, B, H, K, V = Ss.shape
        BH = B * H
        eye = torch.eye(K, device=Ss.device, dtype=torch.float32).expand(BH, K, K)
        x0 = torch.cat([eye, torch.zeros(BH, K, V, device=Ss.device)], dim=-1).contiguous()
        Sx = torch.cat([torch.zeros(R, BH, K, K, device=Ss.device), Ss.float().reshape(R, BH, K, V)], dim=-1)
        out = ops.sp_prefix_fold(Ms.float().reshape(R, BH, K, K).contiguous(), Sx.contiguous(), x0)[R]
        return out[..., :K].reshape(B, H, K, K), out[..., K:].reshape(B, H, K, V)
    dt = _acc_dtype(Ss)
    M, S = Ms[0].to(dt), Ss[0].to(dt)
    for r in range(1, Ss.shape[0]):
        M = torch.matmul(Ms[r].to(dt), M)
        S = torch.matmul(Ms[r].to(dt), S) + Ss[r].to(dt)
    return M, S


def exchange(M, S, group=None):
    """All-gather every rank's (M, S) -> (Ms [R,...], Ss [R,...]). Works with any
    torch.distributed backend (nccl on GPUs, gloo on CPUs)."""
    world = dist.get_world_size(group)
    B, H, K, _ = M.shape
    V = S.shape[-1]
    flat = torch.cat([M.reshape(B, H, K * K), S.reshape(B, H, K * V)], dim=-1).contiguous()
    bufs = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(bufs, flat, group=group)
    allp = torch.stack(bufs)
    return allp[..., : K * K].reshape(world, B, H, K, K), allp[..., K * K:].reshape(world, B, H, K, V)


def _split(t, R):
    """[B, T, ...] -> [B*R, T/R, ...] (a view: segments are contiguous in T)."""
    B, T = t.shape[:2]
    return t.reshape(B * R, T // R, *t.shape[2:])


def _output(q, k, w, u, g, scale, h_start):
    """Pass 3 on a batch of segments from their entering states: (o, states after)."""
    K, V = q.shape[-1], u.shape[-1]
    if q.dtype == torch.bfloat16 and K == 128 and V == 128:
        return ops.gated_delta_fwd_ho(q, k, w, u, g, scale, h0=h_start, want_final=True)
    h, vn, fin = ops.chunk_fwd_h(k, u, g, w=w, h0=h_start, mode=1, want_v_new=True, want_final=True,
                                 h_dtype=torch.bfloat16 if q.dtype == torch.bfloat16 else torch.float32)
    return ops.chunk_fwd_o(q, k, vn, g, h, scale), fin


def sp_forward_local(q, k, w, u, g, scale: float, segments: int, h0=None, summaries=None):
    """The layer's state recurrence + output with every sequence cut into
    ``segments`` pieces run side by side on this device. Returns (o [B,T,H,V],
    final state [B,H,K,V]). ``summaries`` (M, S) skips pass 1 when given."""
    B, T, H, K = q.shape
    V = u.shape[-1]
    R = segments
    assert T % (64 * R) == 0, "each segment must hold whole 64-token chunks"
    qs, ks, ws, us, gs = (_split(t, R) for t in (q, k, w, u, g))
    M, S = summaries if summaries is not None else segment_summary(ks, ws, us, gs)
    Ms = M.reshape(B, R, H, K, K).transpose(0, 1)
    Ss = S.reshape(B, R, H, K, V).transpose(0, 1)
    starts = prefix_states(Ms, Ss, h0)                                      # [R, B, H, K, V]
    h_start = starts.transpose(0, 1).reshape(B * R, H, K, V).float().contiguous()
    o, fin = _output(qs, ks, ws, us, gs, scale, h_start)
    return o.reshape(B, T, H, V), fin.reshape(B, R, H, K, V)[:, -1]


def sp_forward(q, k, w, u, g, scale: float, h0=None, local_segments: int = 1, group=None):
    """This rank's part (along T, in rank order) of sequences split across the
    ranks of ``group``: returns (o of this rank's part, state after it; on the
    last rank that is the sequences' final state). Every rank calls it."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    B, T, H, K = q.shape
    V = u.shape[-1]
    R = local_segments
    ks, ws, us, gs = (_split(t, R) for t in (k, w, u, g))
    M, S = segment_summary(ks, ws, us, gs)
    Mr, Sr = compose(M.reshape(B, R, H, K, K).transpose(0, 1), S.reshape(B, R, H, K, V).transpose(0, 1))
    Ms, Ss = exchange(Mr.float().contiguous(), Sr.float().contiguous(), group)
    h_rank = prefix_state(Ms, Ss, rank, h0)
    return sp_forward_local(q, k, w, u, g, scale, R, h0=h_rank, summaries=(M, S))
