"""One model partitioned over two GPUs (bench.py under torchrun, two layers of
cfg4): rank 0's merged whole-model arrays (kept indices, beta, requantised
K/V rows) must equal one GPU's bit for bit, for the copy-engine merge into
rank 0's buffer and for the NCCL send/recv merge. Needs two GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("gather", ["peer", "nccl"])
def test_partitioned_model_equals_one_gpu(gather):
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           "bench.py", "--gpus", "2", "--layers", "2", "--steps", "2", "--warmup", "3", "--no-e2e", "--no-cpu",
           "--gather", gather]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=700)
    assert p.returncode == 0, p.stderr[-3000:]
    lines = [json.loads(l) for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout[-2000:]
    line = lines[0]
    assert line["n_gpus"] == 2
    assert line["gather_check"] == "rank 0's whole-model arrays identical to one GPU's", line["gather_check"]
