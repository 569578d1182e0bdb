"""Multi-GPU attention partition (config 5's layout) on 2, 4 and 8 GPUs:
KV-head partition and KV-head x sequence-part partition, each rank's engine
against an unpartitioned engine (runs tests/partition_worker.py under
torchrun); layouts needing more GPUs than the box has are skipped."""
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


# (ranks, sequence parts): KV heads over 2 / 4 ranks, KV heads x sequence
# halves over 2 / 4 / 8 ranks (config 5's 8-GPU layout)
LAYOUTS = [(2, 1), (2, 2), (4, 1), (4, 2), (8, 2)]


@pytest.mark.parametrize("world,seq_parts", LAYOUTS, ids=[f"{w}gpu-parts{p}" for w, p in LAYOUTS])
def test_partition(world, seq_parts):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "partition_worker.py"),
           f"--seq-parts={seq_parts}"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert "PARTITION_OK" in r.stdout
