"""Multi-rank host logic on CPU (gloo, world size 2): sequence sharding, the
end-of-run reduction (max of times, sum of counters), and failure detection on
the host (a rank that never joins the collective makes its peer fail within the
process-group timeout instead of hanging)."""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
    import __graft_entry__
    __graft_entry__.load_package()
    from wavefront_decoding_b200 import parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "reduce":
            a, b = parallel.shard_range(64, world, rank)
            t, c = parallel.reduce_over_ranks([1.5 + rank, 10.0 * rank], [b - a, 7])
            q.put((rank, (a, b), t, c))
        elif mode == "missing_peer":
            if rank == 1:
                q.put((rank, "left"))
                return            # leaves between steps, never joins the collective
            try:
                parallel.reduce_over_ranks([1.0], [1.0])
                q.put((rank, "no error"))
            except Exception as e:  # the collective times out on the host
                q.put((rank, f"error: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda x: x[0])


def test_shard_range():
    from wavefront_decoding_b200.parallel import shard_range
    assert [shard_range(64, 8, r) for r in range(8)] == [(8 * r, 8 * r + 8) for r in range(8)]
    parts = [shard_range(10, 4, r) for r in range(4)]
    assert parts == [(0, 3), (3, 6), (6, 8), (8, 10)]
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def test_reduce_two_ranks_gloo():
    out = _run("reduce")
    assert [o[1] for o in out] == [(0, 32), (32, 64)]
    for _, _, t, c in out:
        assert t == [2.5, 10.0]            # max over ranks
        assert c == [64.0, 14.0]           # sum over ranks


def test_missing_peer_fails_on_host():
    out = _run("missing_peer")
    assert out[1][1] == "left"
    assert out[0][1].startswith("error")
