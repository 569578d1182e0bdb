"""Multi-GPU attention partition (config 5's layout) on 2, 4 and 8 GPUs:
KV-head partition and KV-head x sequence-part partition, each rank's engine
against an unpartitioned engine (runs tests/partition_worker.py under
torchrun), with the decode-step exchanges over peer memory (the default) and
over NCCL (VVQ2_PEER=0); layouts needing more GPUs than the box has are
skipped.  A last case makes the failure on the host: one rank skips a
decode step, and the other must come back with the bounded wait's error
instead of hanging."""
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


def _run(world, seq_parts, peer, *extra):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", VVQ2_PEER="1" if peer else "0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "partition_worker.py"),
           f"--seq-parts={seq_parts}", *extra]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    return r


@pytest.mark.parametrize("peer", [True, False], ids=["peer", "nccl"])
@pytest.mark.parametrize("world,seq_parts", LAYOUTS, ids=[f"{w}gpu-parts{p}" for w, p in LAYOUTS])
def test_partition(world, seq_parts, peer):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    r = _run(world, seq_parts, peer)
    assert r.returncode == 0
    assert "PARTITION_OK" in r.stdout


def test_partition_peer_wait_gives_up():
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    r = _run(2, 1, True, "--skip-step-rank=1")
    assert r.returncode == 0
    assert "PEER_TIMEOUT_OK" in r.stdout
