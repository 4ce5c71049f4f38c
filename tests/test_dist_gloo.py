"""world_size-2 gloo tests of the multi-rank host logic (CPU only, no GPU).

The data path has no collective: ranks split the batch (shard_range), each runs
its shard, and only timing (max over ranks) and result checks (gather to rank 0)
communicate. A rank that dies must turn the survivors' next collective into an
error within the process-group timeout, not a hang.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = str(Path(__file__).resolve().parent.parent)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, ws, port, timeout_s=30.0):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws))
    from theorem_b200 import dist as D
    D.init("gloo", timeout_s=timeout_s)
    return D


def _worker_sharded_oracle(rank, ws, port, q):
    """Each rank computes its batch shard of chunk_fwd_h (oracle stands in for the
    kernel on CPU); rank 0 gathers and compares with the unsharded result."""
    import numpy as np
    D = _init(rank, ws, port)
    from oracle import inputs as oin, ops as orc
    d = oin.h_inputs(5, 128, 2, 64, 64, 1)  # B = 5: uneven shards (3 + 2)
    lo, hi = D.shard_range(d["B"], ws, rank)
    h = torch.from_numpy(orc.chunk_fwd_h(d["k"][lo:hi], d["v"][lo:hi], d["g"][lo:hi]))
    full = D.gather_batches(h)
    t = D.max_over_ranks(float(rank + 1))
    if rank == 0:
        ref = orc.chunk_fwd_h(d["k"], d["v"], d["g"])
        q.put(("ok", bool(np.allclose(full.numpy(), ref)), t, tuple(full.shape)))
    torch.distributed.destroy_process_group()


def _worker_dead_rank(rank, ws, port, q):
    """Rank 1 leaves between steps without joining the next collective; rank 0's
    collective must fail with an error inside the timeout."""
    import time
    D = _init(rank, ws, port, timeout_s=5.0)
    D.max_over_ranks(1.0)  # one healthy step together
    if rank == 1:
        os._exit(0)  # dies between steps, nothing in flight
    t0 = time.time()
    try:
        D.max_over_ranks(2.0)
        q.put(("no-error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put(("error", time.time() - t0, type(e).__name__))


def _run(fn, ws=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=fn, args=(r, ws, port, q)) for r in range(ws)]
    for p in ps:
        p.start()
    out = q.get(timeout=timeout)
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_shard_range_covers_exactly():
    from theorem_b200.dist import shard_range
    for n in (0, 1, 5, 16, 17):
        for ws in (1, 2, 3, 8):
            parts = [shard_range(n, ws, r) for r in range(ws)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1


def test_two_rank_sharded_run_gathers_to_reference():
    status, equal, tmax, shape = _run(_worker_sharded_oracle)
    assert status == "ok" and equal
    assert tmax == 2.0
    assert shape == (5, 2, 2, 64, 64)


def test_dead_rank_fails_fast_instead_of_hanging():
    res = _run(_worker_dead_rank)
    assert res[0] == "error", res
    assert res[1] < 60.0
