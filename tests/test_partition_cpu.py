"""Host side of the multi-GPU attention partition (config 5), on CPU with a
world-size-2 gloo group: the ownership plan covers every head and key once,
and per-rank partial attention over its (heads, sequence part) merged with
the (O, LSE) rule after an all-gather equals full causal attention; the
engine's own interleave helpers (compiled for the host) agree with that
plan.  The partitioned GPU path itself is tested in test_gpu_partition.py."""
import os
import shutil
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "vibevoice.cpp_b200"))
import partition as PT  # noqa: E402


def test_plan_covers_each_head_and_key_once():
    for world, seq_parts, nq, nkv in [(2, 1, 28, 4), (4, 1, 28, 4), (8, 2, 28, 4), (2, 2, 14, 2)]:
        seen_q, seen_kv = {}, {}
        for r in range(world):
            p = PT.plan(r, world, seq_parts, nq, nkv)
            for h in p["q_heads"]:
                seen_q[(h, p["part"])] = seen_q.get((h, p["part"]), 0) + 1
            for h in p["kv_heads"]:
                seen_kv[(h, p["part"])] = seen_kv.get((h, p["part"]), 0) + 1
        assert sorted(seen_q) == [(h, s) for h in range(nq) for s in range(seq_parts)]
        assert set(seen_q.values()) == {1} and set(seen_kv.values()) == {1}
    n = 27000
    k0, k1 = PT.keys_of_part(0, 2, n), PT.keys_of_part(1, 2, n)
    assert len(k0) + len(k1) == n and not set(k0.tolist()) & set(k1.tolist())
    for part, keys in ((0, k0), (1, k1)):
        assert len(keys) == PT.part_count(part, n)
        # cache index of each held position = the part's positions below it
        for i in (0, 1, 63, 64, 200, len(keys) - 1):
            assert PT.part_count(part, int(keys[i])) == i
    # causal prefill work (queries at or after each key) is balanced across
    # the parts, where a split at the middle gives 3:1
    work = [int(np.sum(n - k)) for k in (k0, k1)]
    assert abs(work[0] - work[1]) / sum(work) < 0.01, work
    with pytest.raises(ValueError):
        PT.plan(0, 3, 1, 28, 4)
    for world in (2, 4, 8):
        feats = [f for r in range(world) for f in PT.ffn_range(r, world, 18944)]
        assert feats == list(range(18944))
    with pytest.raises(ValueError):
        PT.ffn_range(0, 8, 4864 + 64)


def test_engine_interleave_matches_plan(tmp_path):
    """The engine's own interleave helpers (common.cuh, compiled for the host:
    the functions its local_row() and the kernels call) against the plan
    above: which part stores a position, its cache index in that part, and a
    row's (pos, cidx, kvlen) as each part sees it."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc not available")
    root = Path(__file__).resolve().parent.parent
    exe, dump = tmp_path / "zz_host", tmp_path / "zz.bin"
    r = subprocess.run([nvcc, "-std=c++17", "-O1", "-I", str(root / "vibevoice.cpp_b200" / "csrc"),
                        str(root / "tests" / "zz_rows_host.cu"), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    n = 1300                                   # five 256-position periods and a ragged tail
    assert subprocess.run([str(exe), str(n), str(dump)]).returncode == 0
    got = np.fromfile(dump, np.int32).reshape(n, 9)
    keys = [PT.keys_of_part(s, 2, n + 1) for s in (0, 1)]
    for p in range(n):
        part, c0, c1 = got[p, :3]
        assert part == PT.part_of(p) and c0 == PT.part_count(0, p) and c1 == PT.part_count(1, p), p
        for s in (0, 1):
            lpos, lcidx, lkv = got[p, 3 + 3 * s:6 + 3 * s]
            held = keys[s][keys[s] <= p]
            # the part's last key at or before p; the row's own index if it stores p; keys below p + 1
            assert lpos == len(held) - 1, (p, s)
            assert lcidx == (len(held) - 1 if PT.part_of(p) == s else -1), (p, s)
            assert lkv == len(held), (p, s)


def _worker(rank, world, port, seq_parts, q_all, k_all, v_all, q_pos, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nq, T, hd = q_all.shape
        nkv, n, _ = k_all.shape
        p = PT.plan(rank, world, seq_parts, nq, nkv)
        keys = PT.keys_of_part(p["part"], seq_parts, n)
        G = nq // nkv
        o = np.zeros((len(p["q_heads"]), T, hd))
        l = np.zeros((len(p["q_heads"]), T))
        for i, h in enumerate(p["q_heads"]):
            kvh = h // G
            o[i], l[i] = PT.partial_attention(q_all[h], k_all[kvh][keys], v_all[kvh][keys], q_pos, keys,
                                              1.0 / np.sqrt(hd))
        # every rank contributes its partial; rank 0 merges the parts of each head
        parts = [None] * world
        dist.all_gather_object(parts, (rank, o, l))
        if rank == 0:
            full = np.zeros((nq, T, hd))
            for h in range(nq):
                os_, ls_ = [], []
                for r, po, pl in parts:
                    pr = PT.plan(r, world, seq_parts, nq, nkv)
                    if h in pr["q_heads"]:
                        j = list(pr["q_heads"]).index(h)
                        os_.append(po[j])
                        ls_.append(pl[j])
                full[h] = PT.lse_merge(np.stack(os_), np.stack(ls_))
            out.put(full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("seq_parts", [1, 2])
def test_partitioned_attention_merge_gloo(seq_parts):
    rng = np.random.default_rng(7 + seq_parts)
    nq, nkv, hd, n, T = 4, 2, 16, 300, 40
    q_all = rng.standard_normal((nq, T, hd))
    k_all = rng.standard_normal((nkv, n, hd))
    v_all = rng.standard_normal((nkv, n, hd))
    q_pos = np.sort(rng.choice(n, T, replace=False)).astype(np.int64)   # causal: keys <= pos
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29500 + (os.getpid() % 1000) + seq_parts
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq_parts, q_all, k_all, v_all, q_pos, out))
             for r in range(world)]
    for p in procs:
        p.start()
    full = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    G = nq // nkv
    for h in range(nq):
        ref, _ = PT.partial_attention(q_all[h], k_all[h // G], v_all[h // G], q_pos, np.arange(n), 1.0 / np.sqrt(hd))
        assert np.max(np.abs(full[h] - ref)) < 1e-9
