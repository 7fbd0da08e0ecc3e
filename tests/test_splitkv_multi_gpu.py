"""Split-KV decode on 2 GPUs: the peer-memory exchange and the NCCL
collective baseline (skipped with fewer GPUs)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_kv_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(HERE, "splitkv_ranks.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    print(r.stdout[-2000:], r.stderr[-2000:])
    assert r.returncode == 0
    assert r.stdout.count("vs one-GPU") == 2 * 3   # 2 ranks x (p2p, collective, p2p-graph)
