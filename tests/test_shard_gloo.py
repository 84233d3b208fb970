"""Output-row sharding across ranks (lnsb200.shard) on CPU with gloo,
world_size 2: each rank computes its row block (with the CPU oracle standing
in for the device kernel), the blocks are all-gathered and permuted back to
ggml order, and the result equals the unsharded op bit for bit -- in base and
in Monte mode (shard-adjusted LFSR seed)."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "xlns-ggml-backend_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import datetime
    import torch.distributed as dist
    import oracle
    from lnsb200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(3)
        K, M, N = 130, 64, 9
        w = oracle.from_f32_16(rng.normal(0, 0.02, (M, K)).astype(np.float32))
        x = oracle.from_f32_16(rng.normal(0, 1, (N, K)).astype(np.float32))
        m0, m1 = shard.row_range(M, world, rank)
        w_km = np.ascontiguousarray(w.T)                          # k-major [K][M], as on the device
        mine = np.ascontiguousarray(shard.shard_weights_kmajor(w_km, M, world, rank).T)   # rows m0..m1
        seed = shard.monte_seed_for_shard(7, oracle.lfsr_jump, M, N, K, rank, world)
        part = oracle.mul_mat16(mode, mine, x, seed=seed)         # [N][m1-m0]
        full = shard.all_gather_rows(torch.from_numpy(part.view(np.int16)), world)
        if rank == 0:
            want = oracle.mul_mat16(mode, w, x, seed=7)
            q.put(bool(np.array_equal(full.numpy().view(np.uint16), want)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["base", "monte"])
def test_row_shard_gather_gloo(mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True


def test_row_range_partitions():
    from lnsb200 import shard
    for M in (1, 7, 64, 1536, 8193):
        for world in (1, 2, 3, 8):
            ranges = [shard.row_range(M, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1


def test_monte_seed_for_shard_refuses_slices():
    """a sharded Monte mul_mat with several slices has no single start state"""
    import oracle
    from lnsb200 import shard
    assert shard.monte_seed_for_shard(7, oracle.lfsr_jump, 64, 4, 16, 1, 2) == oracle.lfsr_jump(7, 32 * 4 * 15)
    with pytest.raises(ValueError):
        shard.monte_seed_for_shard(7, oracle.lfsr_jump, 64, 4, 16, 1, 2, slices=3)
