"""Expert parallelism on real GPUs: NCCL all-to-all dispatch/combine and the peer-memory exchange vs the
single-GPU layer, and a skipped step that makes the peers' bounded exchange waits run out (status 1)
(tests/ep_worker.py under torchrun, one rank per visible GPU, 2 to 8). Skipped with one GPU."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_ep_nccl_matches_single_gpu():
    n = min(torch.cuda.device_count(), 8)
    while 384 % n:
        n -= 1
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           os.path.join(ROOT, "tests", "ep_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(" ok: ") == n
    assert r.stdout.count("exchange wait expired after") == n - 1
