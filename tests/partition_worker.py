"""One rank of the partitioned-attention GPU test (launched by torchrun from
test_gpu_partition.py): a small 2-layer model partitioned over the ranks
(KV heads x sequence parts, 2 to 8 ranks) against an unpartitioned engine on
the same GPU, through a prefill of 2 x 300 prompt tokens and 6 greedy decode
steps.  With --skip-step-rank=r, rank r sits out one decode step (it stays
alive, between steps, with nothing in flight) and every other rank must get
the bounded peer wait's error back from that step."""
import argparse
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "vibevoice.cpp_b200"))
import synth  # noqa: E402
import vvq2  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq-parts", type=int, default=1)
    ap.add_argument("--skip-step-rank", type=int, default=-1)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    # one KV head per head group (at least 2), 4 q heads per KV head; the FFN
    # splits over every rank
    groups = world // args.seq_parts
    nkv = max(2, groups)
    hp = dict(hidden=512, n_heads=4 * nkv, n_kv_heads=nkv, head_dim=64, ffn=128 * world if world > 8 else 1024,
              n_layers=2, vocab=2048, rope_theta=1.0e6, rms_eps=1.0e-6)
    model = synth.model_q8_0(20261201, hp)
    ids = [vvq2.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    part = vvq2.Engine(hp, device=int(os.environ["LOCAL_RANK"]))
    part.partition(rank, world, args.seq_parts, ids[0])
    ref = vvq2.Engine(hp, device=int(os.environ["LOCAL_RANK"]))
    for eng in (part, ref):
        for li, t in enumerate(model["layers"]):
            eng.set_layer(li, t)
        eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    n, steps = 300, 6
    kvp, kvr = part.kv(2, n + steps + 8), ref.kv(2, n + steps + 8)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, n, hp["hidden"])).astype(np.float32)
    hp_ = part.forward(kvp, [0, 1], x, [0, 0])
    hr = ref.forward(kvr, [0, 1], x, [0, 0])
    err = float(np.max(np.abs(hp_ - hr)) / np.max(np.abs(hr)))
    tok = rng.integers(0, hp["vocab"], size=2).astype(np.int32)
    if args.skip_step_rank >= 0:
        got = None
        if rank != args.skip_step_rank:
            try:
                part.decode_step(kvp, [0, 1], tok)
                got = "returned"
            except Exception as e:  # the engine's error for a wait that ran out
                got = str(e)
        errs = [None] * world
        dist.all_gather_object(errs, got)
        if rank == 0:
            print("errors:", errs, flush=True)
            ok = all(e is not None and "timed out" in e for r, e in enumerate(errs) if r != args.skip_step_rank)
            print("PEER_TIMEOUT_OK" if ok else "PEER_TIMEOUT_FAIL", flush=True)
        dist.barrier()   # no rank frees its exchange buffer while another may still store into it
        dist.destroy_process_group()
        return
    same = 0
    for _ in range(steps):
        tp = part.decode_step(kvp, [0, 1], tok)
        tr = ref.decode_step(kvr, [0, 1], tok)
        same += int(np.sum(tp == tr))
        tok = tr
    print(f"rank {rank}: prefill rel err {err:.2e}, decode tokens identical {same}/{2 * steps}", flush=True)
    ok = err < 3e-3 and same >= 2 * steps - 1
    flags = [None] * world
    dist.all_gather_object(flags, ok)
    if rank == 0:
        print("PARTITION_OK" if all(flags) else "PARTITION_FAIL", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
