"""The output-row all-gather fused into the mul_mat store over NVLink peer
memory (lnsb_mul_mat_lns_peers + lnsb_group_barrier) against NCCL's
all-gather, two GPUs (skipped with fewer)."""
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,shape", [("base", "tiled"), ("base", "latency"), ("monte", "tiled"), ("sum32", "tiled"),
                                        ("sum32", "latency")])
def test_peer_gather_two_gpus(mode, shape):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(here, "peer_gather_check.py"), mode, shape]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_group_barrier_times_out_without_a_peer():
    """the peer-flag barrier's wait is bounded: with a peer that never signals
    (two flag arrays on this GPU, rank 1 never runs) the call returns and sets
    the error word instead of hanging"""
    import ctypes
    import time
    import lnsb200
    ks = lnsb200.KernelSet(16, "base")
    f0 = torch.zeros(2, dtype=torch.int32, device="cuda")
    f1 = torch.zeros(2, dtype=torch.int32, device="cuda")
    ptrs = torch.tensor([f0.data_ptr(), f1.data_ptr()], dtype=torch.int64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    st = ks.lib.lnsb_group_barrier(ctypes.c_void_p(ptrs.data_ptr()), 2, 0, 1, ctypes.c_void_p(err.data_ptr()), None)
    torch.cuda.synchronize()
    assert st == 0 and err.item() == 1
    assert f1.cpu().tolist() == [1, 0]                    # rank 0's signal reached "peer" 1's slot
    assert time.time() - t0 < 30
    # with both signals present the barrier passes
    f0.fill_(2)
    err.zero_()
    st = ks.lib.lnsb_group_barrier(ctypes.c_void_p(ptrs.data_ptr()), 2, 0, 2, ctypes.c_void_p(err.data_ptr()), None)
    torch.cuda.synchronize()
    assert st == 0 and err.item() == 0


@pytest.mark.parametrize("fmt,mode", [(16, "base"), (16, "monte"), (16, "sum32"), (16, "lpvip"), (16, "monte_bylpvip"),
                                      (32, "base")])
@pytest.mark.parametrize("K,M,N", [(576, 1536, 512), (70, 1000, 600), (1536, 576, 8), (576, 576, 1)])
def test_peer_store_on_one_gpu(orc, fmt, mode, K, M, N):
    """the fused gather's stores without NVLink: two buffers on this GPU stand
    for two ranks' gather buffers, this call is rank 1 of 2 (columns
    [M, 2M) of rows of 2M codes); both must hold exactly lnsb_mul_mat_lns's
    result there and keep their other columns.  The shapes reach the tiled
    kernel, the key-resident latency kernel (configs[0], a decode mat-vec) and
    the 32-bit accumulator kernel"""
    import numpy as np
    import lnsb200
    ks = lnsb200.KernelSet(fmt, mode)
    ks.upload_tables()
    rng = np.random.default_rng(K + M + N)
    conv = orc.from_f32_16 if fmt == 16 else orc.from_f32_32
    w = conv(rng.normal(0, 0.02, (M, K)).astype(np.float32))
    x = conv(rng.normal(0, 1, (N, K)).astype(np.float32))
    it = np.int16 if fmt == 16 else np.int32
    dt = torch.int16 if fmt == 16 else torch.int32
    wd = torch.from_numpy(np.ascontiguousarray(w.T).view(it)).cuda()
    xd = torch.from_numpy(x.view(it)).cuda()
    want = torch.empty(N * M, dtype=dt, device="cuda")
    ks.mul_mat_lns(wd, xd, want, K, M, N, monte_seed=11)
    bufs = [torch.full((N, 2 * M), 0x1234, dtype=dt, device="cuda") for _ in range(2)]
    ptrs = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    ks.mul_mat_lns_peers(wd, xd, ptrs.data_ptr(), 2, 2 * M, M, K, M, N, monte_seed=11)
    torch.cuda.synchronize()
    for b in bufs:
        assert torch.equal(b[:, M:].contiguous().view(-1), want)
        assert bool((b[:, :M] == 0x1234).all())
