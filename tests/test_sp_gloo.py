"""world_size-2 gloo test of the sequence-parallel delta rule (CPU only).

Each rank holds one half (along T) of one sequence, summarises its segment as
(M, S) -- computed here by the oracle, which stands in for the chunk_fwd_h kernel
on CPU -- and calls the library's exchange (all_gather) and prefix fold. The state
entering each rank's segment, and the last rank's final state, must equal the
full-sequence oracle recurrence.
"""
import numpy as np
import pytest
import torch

from tests.test_dist_gloo import _init, _run


def _oracle_summary(k, w, u, g):
    from oracle import ops as orc
    B, T, H, K = k.shape
    eye = np.broadcast_to(np.eye(K), (B, H, K, K)).copy()
    _, _, M = orc.chunk_fwd_h_delta(k, w, np.zeros_like(k), g, eye)
    _, _, S = orc.chunk_fwd_h_delta(k, w, u, g, None)
    return torch.from_numpy(M), torch.from_numpy(S)


def _inputs():
    from tests.synth import deltanet_inputs
    from oracle import ops as orc
    d = deltanet_inputs(2, 512, 2, 64, 48, seed=12, dtype=torch.float32)
    # slow gate (about -0.1 per chunk): the state entering a segment still matters
    inc = -0.003 * torch.rand(2, 512, 2, generator=torch.Generator().manual_seed(5)) - 0.0002
    g = inc.reshape(2, 8, 64, 2).cumsum(2).reshape(2, 512, 2)
    A = orc.build_A(d["k"], d["beta"], g, 1)
    w, u = orc.recompute_w_u(d["k"], d["v"], d["beta"], A, g)
    h0 = np.random.default_rng(3).standard_normal((2, 2, 64, 48)) * 0.3
    return d["k"].double().numpy(), w, u, g.double().numpy(), h0


def _worker_sp(rank, ws, port, q):
    _init(rank, ws, port)
    from theorem_b200 import sp
    from oracle import ops as orc
    k, w, u, g, h0 = _inputs()
    T = k.shape[1]
    L = T // ws
    sl = lambda a: a[:, rank * L:(rank + 1) * L]  # noqa: E731
    M, S = _oracle_summary(sl(k), sl(w), sl(u), sl(g))
    Ms, Ss = sp.exchange(M, S)
    h_start = sp.prefix_state(Ms, Ss, rank, torch.from_numpy(h0))
    h_pre, _, fin = orc.chunk_fwd_h_delta(k, w, u, g, h0)
    expect = h_pre[:, rank * L // 64]
    ok = bool(np.allclose(h_start.numpy(), expect, rtol=1e-9, atol=1e-9))
    if rank > 0:  # the carried state is visible: starting from 0 instead would be wrong
        ok = ok and not np.allclose(sp.prefix_state(Ms, Ss, rank, None).numpy() * 0, expect, atol=1e-3)
    fin_ok = True
    if rank == ws - 1:
        h_end = torch.matmul(M, h_start) + S
        fin_ok = bool(np.allclose(h_end.numpy(), fin, rtol=1e-9, atol=1e-9))
    res = torch.tensor([int(ok and fin_ok)])
    torch.distributed.all_reduce(res, op=torch.distributed.ReduceOp.MIN)
    if rank == 0:
        q.put(("ok", int(res.item()), tuple(Ms.shape), tuple(Ss.shape)))
    torch.distributed.destroy_process_group()


def test_sp_prefix_over_two_ranks_matches_full_sequence():
    status, good, ms_shape, ss_shape = _run(_worker_sp)
    assert status == "ok" and good == 1
    assert ms_shape == (2, 2, 2, 64, 64) and ss_shape == (2, 2, 2, 64, 48)


def test_prefix_state_single_process():
    """Three segments folded in one process (no collective) equal the recurrence."""
    from theorem_b200 import sp
    from oracle import ops as orc
    k, w, u, g, h0 = _inputs()
    T = k.shape[1]
    L = T // 4
    pairs = [_oracle_summary(a[:, r * L:(r + 1) * L], b[:, r * L:(r + 1) * L], c[:, r * L:(r + 1) * L],
                             e[:, r * L:(r + 1) * L]) for r, (a, b, c, e) in enumerate([(k, w, u, g)] * 4)]
    Ms = torch.stack([p[0] for p in pairs])
    Ss = torch.stack([p[1] for p in pairs])
    h_pre, _, fin = orc.chunk_fwd_h_delta(k, w, u, g, h0)
    for r in range(4):
        h = sp.prefix_state(Ms, Ss, r, torch.from_numpy(h0))
        assert np.allclose(h.numpy(), h_pre[:, r * L // 64], rtol=1e-9, atol=1e-9), r
    assert np.allclose(sp.prefix_state(Ms, Ss, 4, torch.from_numpy(h0)).numpy(), fin, rtol=1e-9, atol=1e-9)
