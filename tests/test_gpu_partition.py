"""Multi-GPU attention partition (config 5's layout) on 2 GPUs: KV-head
partition and KV-head x sequence-part partition, each rank's engine against
an unpartitioned engine (runs tests/partition_worker.py under torchrun)."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    import torch
    return torch.cuda.device_count()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("seq_parts", [1, 2])
def test_partition_two_gpus(seq_parts):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "partition_worker.py"),
           f"--seq-parts={seq_parts}"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert "PARTITION_OK" in r.stdout
