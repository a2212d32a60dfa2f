"""Batch split and sequence split on every GPU of the box (2 to 8), one process per
GPU: the sequence split with both exchanges (NVLink peer memory, NCCL all-gather).

Skipped with fewer than two GPUs.  The ranks run tests/mgpu_worker.py under
torch.distributed.run on 127.0.0.1; NVLS stays off (NCCL_NVLS_ENABLE=0).
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_multi_gpu_batch_and_sequence_split():
    """One rank per GPU of the box (2 to 8)."""
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "mgpu_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    # per rank: the batch split, then the sequence-split calls of mgpu_worker's cases
    # (6 over peer memory at b2 h128, 3 over the all-gather, 3 over peer memory at b3 h64)
    assert r.stdout.count("'ok': True") == world * (1 + 6 + 3 + 3), r.stdout
