"""Helper run by tests/test_gpu_peer_gather.py under torchrun (one process per
GPU): lnsb_mul_mat_lns_peers + lnsb_group_barrier against NCCL's all-gather
of the same output-row shards, bit for bit, over four steps; exit status 0 =
equal.

Each step multiplies different activations, so a buffer holding an older
step's result cannot pass.  The steps alternate between two gather buffers
by parity and read each step's result on this rank's stream before its next
call -- the write-after-read rule of lnsb_mul_mat_lns_peers (passing barrier
e+1 means every peer has finished reading step e-1's buffer).

    peer_gather_check.py <mode> <tiled|latency>"""
import ctypes
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "xlns-ggml-backend_b200"))


def main():
    import datetime
    import lnsb200
    from lnsb200 import shard
    import torch.distributed._symmetric_memory as symm_mem
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    mode = sys.argv[1] if len(sys.argv) > 1 else "base"
    shape = sys.argv[2] if len(sys.argv) > 2 else "tiled"
    ks = lnsb200.KernelSet(16, mode)
    ks.upload_tables()
    # per rank: the tiled kernel's shape (640 rows x 96 tokens), or the latency
    # kernels' (576 rows x 8 tokens at K = 1536, configs[0] per rank)
    K, M, N = (256, 640, 96) if shape == "tiled" else (1536, 576, 8)
    rng = np.random.default_rng(7 + rank)
    wf = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()
    w = torch.empty(K * M, dtype=torch.int16, device="cuda")
    ks.to_lns_transposed(wf, w, M, K, M)
    out = torch.empty(N * M, dtype=torch.int16, device="cuda")
    gbufs = [symm_mem.empty(N * M * world, dtype=torch.int16, device="cuda") for _ in range(2)]
    for g in gbufs:
        g.fill_(-1)
    hdls = [symm_mem.rendezvous(g, dist.group.WORLD) for g in gbufs]
    fbuf = symm_mem.empty(world, dtype=torch.int32, device="cuda")
    fbuf.zero_()
    fhdl = symm_mem.rendezvous(fbuf, dist.group.WORLD)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    dist.barrier()
    ok = True
    for epoch in (1, 2, 3, 4):
        xf = torch.from_numpy(np.random.default_rng(100 + epoch).normal(0, 1, (N, K)).astype(np.float32)).cuda()
        x = torch.empty(N * K, dtype=torch.int16, device="cuda")
        ks.to_lns(xf, x)
        # this step's expected gather: the plain kernel and NCCL
        ks.mul_mat_lns(w, x, out, K, M, N, monte_seed=5)
        want = shard.all_gather_rows(out.view(N, M), world).contiguous().view(-1)
        b = epoch % 2
        ks.mul_mat_lns_peers(w, x, hdls[b].buffer_ptrs_dev, world, M * world, rank * M, K, M, N, monte_seed=5)
        st = ks.lib.lnsb_group_barrier(ctypes.c_void_p(fhdl.buffer_ptrs_dev), world, rank, epoch,
                                       ctypes.c_void_p(err.data_ptr()), None)
        good = st == 0 and torch.equal(gbufs[b], want)     # the read, on this rank's stream
        torch.cuda.synchronize()
        good = good and err.item() == 0
        if not good:
            print("rank %d epoch %d: status %d, barrier error %d, equal %s" % (rank, epoch, st, err.item(),
                                                                              torch.equal(gbufs[b], want)), flush=True)
        ok = ok and good
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
