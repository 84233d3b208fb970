"""The output-row all-gather fused into the mul_mat store over NVLink peer
memory (lnsb_mul_mat_lns_peers + lnsb_group_barrier) against NCCL's
all-gather, two GPUs (skipped with fewer)."""
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["base", "monte"])
def test_peer_gather_two_gpus(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(here, "peer_gather_check.py"), mode]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
