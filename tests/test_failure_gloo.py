"""Host-side failure detection across ranks (lnsb200.shard.init_group,
StepGuard) on CPU with gloo: the failures are made on the host -- a rank that
never joins, a rank that leaves between steps, a rank that stops arriving --
and the ranks still present must raise ShardError within the deadline
instead of waiting, before launching the step's work.  A collective that a
vanished peer never joins ends with the process group's timeout."""
import os
import socket
import time

import pytest

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _path():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "xlns-ggml-backend_b200"))


def _run(target, world, *args, wait=60):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    t0 = time.monotonic()
    try:
        while len(out) < world and time.monotonic() - t0 < wait:
            try:
                r, v = q.get(timeout=1)
                out[r] = v
            except Exception:
                if not any(p.is_alive() for p in procs) and q.empty():
                    break
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return out


def _never_joins(rank, world, port, q):
    _path()
    from lnsb200 import shard
    if rank == world - 1:
        q.put((rank, "absent"))
        return                                   # this rank never joins
    t0 = time.monotonic()
    try:
        shard.init_group("gloo", rank, world, port, timeout_s=3.0)
        q.put((rank, "joined"))
    except shard.ShardError:
        q.put((rank, ("raised", time.monotonic() - t0)))


def test_rank_never_joins():
    out = _run(_never_joins, 2)
    assert out.get(1) == "absent"
    kind, dt = out[0]
    assert kind == "raised" and dt < 30


def _leaves(rank, world, port, q):
    _path()
    import torch.distributed as dist
    from lnsb200 import shard
    store = shard.init_group("gloo", rank, world, port, timeout_s=20.0)
    guard = shard.StepGuard(store, rank, world, timeout_s=20.0)
    x = torch.ones(4) * (rank + 1)
    guard.enter(0)
    dist.all_reduce(x)                            # step 0: everyone present
    if rank == 1:
        guard.leave()                             # leaves between steps, nothing in flight
        q.put((rank, "left"))
        time.sleep(2)
        return
    t0 = time.monotonic()
    try:
        guard.enter(1)
        q.put((rank, "entered"))
    except shard.ShardError as e:
        q.put((rank, ("raised", list(e.ranks), time.monotonic() - t0, float(x[0]))))
    dist.destroy_process_group()


def test_rank_leaves_between_steps():
    out = _run(_leaves, 2)
    assert out.get(1) == "left"
    kind, ranks, dt, v = out[0]
    assert kind == "raised" and ranks == [1] and dt < 5 and v == 3.0


def _stops_arriving(rank, world, port, q):
    _path()
    from lnsb200 import shard
    store = shard.init_group("gloo", rank, world, port, timeout_s=20.0)
    guard = shard.StepGuard(store, rank, world, timeout_s=1.5)
    guard.enter(0)
    if rank == 2:
        q.put((rank, "stalled"))
        time.sleep(4)                             # alive, but never reaches step 1
        return
    t0 = time.monotonic()
    try:
        guard.enter(1)
        q.put((rank, "entered"))
    except shard.ShardError as e:
        q.put((rank, ("raised", list(e.ranks), time.monotonic() - t0)))


def test_rank_stops_arriving():
    out = _run(_stops_arriving, 3)
    assert out.get(2) == "stalled"
    for r in (0, 1):
        kind, ranks, dt = out[r]
        assert kind == "raised" and ranks == [2] and 1.0 <= dt < 10


def _collective_timeout(rank, world, port, q):
    _path()
    import torch.distributed as dist
    from lnsb200 import shard
    shard.init_group("gloo", rank, world, port, timeout_s=3.0)
    if rank == 1:
        q.put((rank, "skipped"))
        time.sleep(8)                             # never joins the collective
        return
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((rank, "completed"))
    except Exception as e:
        q.put((rank, ("raised", type(e).__name__, time.monotonic() - t0)))


def test_collective_times_out():
    out = _run(_collective_timeout, 2)
    assert out.get(1) == "skipped"
    kind, name, dt = out[0]
    assert kind == "raised" and dt < 30
