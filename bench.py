#!/usr/bin/env python3
"""Benchmark: Qwen2 decode tokens/s on the B200 path.

Workload: the 24-layer Qwen2.5-0.5B-shaped LM (hidden 896, 14/2 heads, hd 64,
ffn 4864 SwiGLU, vocab 151936, tied Q8_0 lm_head), random N(0, 0.02) Q8_0
weights (synthetic, seeded), batch 2 (CFG cond + uncond rows), greedy decode
from an f16 KV cache of --kv positions (default 1024, filled from N(0,1)).
One step = embed -> 24 layers -> output_norm -> lm_head -> argmax for both
rows; tokens/s counts both rows.  The 550 MB of weights per step exceed the
126 MB L2, so every step streams them from HBM (no flush needed).

  value : device-resident loop (token ids stay in HBM), CUDA events on the
          launching stream, max over ranks
  e2e   : the same steps through the C ABI with HOST token buffers
          (vvq2_decode_step: H2D ids, D2H argmax ids every step)
  roofline : the dominant kernel (the persistent decode-step kernel),
          algorithmic bytes per launch / mean launch time from CUDA events,
          vs measured HBM peak; traffic from an ncu capture
  cpu_baseline : the CPU oracle (port of the reference's ggml CPU numerics)
          on this host's cores, bounded sample of decode steps
  prefill, c3 : the 16k-token 7B-shaped prefill layer and config 3's
          batched step (see prefill_measure, c3_measure)

--impl reference times that CPU implementation alone for --warmup + --steps
greedy steps (the reference cannot be built here: its ggml submodule is
absent).  --workload c4 / c5 print the config-4 / config-5 lines; --case
runs small profiling workloads.  Multi-GPU: C2 does not shard, so N GPUs run
N independent replicas (weak scaling, no collectives)."""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import tempfile
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vibevoice.cpp_b200"))

C2 = dict(hidden=896, n_heads=14, n_kv_heads=2, head_dim=64, ffn=4864, n_layers=24, vocab=151936,
          rope_theta=1.0e6, rms_eps=1.0e-6)
SEED = 20261201


C5_LAYER = dict(hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, n_layers=1, vocab=152064,
                rope_theta=1.0e6, rms_eps=1.0e-6)


def measured_tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 1590.0, 1400.0, "fallback"


def prefill_measure(vvq2, synth, torch, local, sh, n_tok, reps=3):
    """One 7B-shaped Q8_0 layer (config 5 dims) over an n_tok causal prompt,
    one tensor-core chunk: CUDA events around the whole layer forward, and
    per-launch events (engine profiling) around the flash-attention and GEMM
    kernels.  Flops: 2*T*N*K per linear, 4*nq*hd*(pos+1) per query row for
    attention (the causal half)."""
    hp = C5_LAYER
    rng = np.random.default_rng(SEED + 5)
    layer = synth.layer_q8_0(rng, hp)
    os.environ["VVQ2_PREFILL_ROWS"] = str(n_tok)   # the whole prompt in one chunk
    eng = vvq2.Engine(hp, device=local)
    del os.environ["VVQ2_PREFILL_ROWS"]
    eng.set_layer(0, layer)
    kv = eng.kv(1, n_tok + 64)
    g = torch.Generator(device="cuda").manual_seed(SEED + 5)
    x = torch.randn((1, n_tok, hp["hidden"]), generator=g, device="cuda", dtype=torch.float32)
    y = torch.empty_like(x)

    def run():
        kv.set_past_len(0, 0)
        eng.forward(kv, [0], x, [0], flags=0, y=y, stream=sh)

    run()
    torch.cuda.synchronize()
    eng.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    e0.record(stream)
    for _ in range(reps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    a_ms, a_fl, a_n = eng.profile_read(2)
    g_ms, g_fl, g_n = eng.profile_read(3)
    eng.profile(False)
    burst, sustained, kind = measured_tensor_peak()
    attn_tf = a_fl / (a_ms / 1000.0) / 1e12 if a_n else None
    gemm_tf = g_fl / (g_ms / 1000.0) / 1e12 if g_n else None
    layer_tf = (a_fl + g_fl) / reps / (ms / 1000.0) / 1e12
    return {
        "workload": f"config-5-shaped layer (7B dims: hidden 3584, 28/4 heads, hd 128, ffn 18944, Q8_0), "
                    f"{n_tok}-token causal prompt, batch 1, one tensor-core chunk",
        "tokens_per_s": round(n_tok / (ms / 1000.0), 1), "ms_per_layer": round(ms, 3),
        "layer_tflops": round(layer_tf, 1),
        "attn": {"kernel": "k_fa_prefill<128> (tcgen05 causal flash attention)",
                 "tflops": round(attn_tf, 1) if attn_tf else None,
                 "frac": round(attn_tf / burst, 4) if attn_tf else None,
                 "ms": round(a_ms / max(a_n, 1), 3), "flops_per_launch": a_fl / max(a_n, 1)},
        "gemm": {"kernel": "k_gemm_ws (persistent tcgen05 GEMM: Q8_0 blocks dequantized in shared memory, "
                           "activations by TMA, 256 x nt tiles, fused RoPE/KV/residual/SwiGLU epilogues)",
                 "tflops": round(gemm_tf, 1) if gemm_tf else None,
                 "frac": round(gemm_tf / burst, 4) if gemm_tf else None},
        "peak_tflops": burst, "peak_kind": f"{kind} bf16 dense burst (sustained {sustained})",
    }


def c1_measure(vvq2, synth, torch, local, sh, n_copies=64, kv_len=512, steps=200, warmup=5):
    """Config 1 -- one Qwen2.5-0.5B-shaped attention layer at batch 2 (CFG
    pair), decode 1 token against an f16 KV cache of 512 positions -- timed
    as the attention-layer step of the persistent decode kernel over
    n_copies DISTINCT copies of the layer (own Q8_0 weights, own KV cache;
    ~175 MB in all, above the 126 MB L2), so each copy's bytes come from HBM.
    The copies carry a 64-wide FFN (the kernel always runs one; its bytes are
    counted) and the stack a 1024-row lm_head (counted).  CUDA events over
    `steps` steps.  The attention phase alone (q hand-over, split-K items,
    merges) is timed from the kernel's own %globaltimer stamps and set
    against the KV bytes it reads."""
    hp = dict(C2, n_layers=n_copies, ffn=64, vocab=1024)
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    rng = np.random.default_rng(SEED + 1)
    eng = vvq2.Engine(hp, device=local)
    wbytes = 0
    for li in range(n_copies):
        L = synth.layer_q8_0_fast(rng, hp)
        wbytes += sum(int(t[0].nbytes) for k, t in L.items() if t is not None and "norm" not in k and "bias" not in k)
        eng.set_layer(li, L)
    head = synth.q8_0_random_tensor(rng, hp["vocab"], H)
    norm = synth.f32_tensor(1.0 + rng.standard_normal(H, dtype=np.float32) * 0.02)
    eng.set_output(norm, head, head)
    kv = eng.kv(2, kv_len + warmup + steps + 8)
    g = torch.Generator(device="cuda").manual_seed(SEED + 1)
    for li in range(n_copies):
        for s in range(2):
            kv.load_prefix(s, li, torch.randn((kv_len, nkv * hd), generator=g, device="cuda"),
                           torch.randn((kv_len, nkv * hd), generator=g, device="cuda"))
    for s in range(2):
        kv.set_past_len(s, kv_len)
    tok = torch.randint(0, hp["vocab"], (2,), dtype=torch.int32, device="cuda", generator=g)
    stream = torch.cuda.current_stream()

    def step():
        # every step decodes position kv_len: the cache stays at 512 past keys (+ the new one)
        for s in range(2):
            kv.set_past_len(s, kv_len)
        eng.decode_step(kv, [0, 1], tok, tok, stream=sh)

    # the step's timeline buffer is set up with its CUDA graph (first step)
    os.environ["VVQ2_MEGA_TRACE"] = "1"
    try:
        for _ in range(warmup):
            step()
    finally:
        del os.environ["VVQ2_MEGA_TRACE"]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    step_us = 1000.0 * e0.elapsed_time(e1) / steps
    tr = eng.mega_trace().astype(np.float64) / 1000.0   # last step, us: [slot][cta]
    kv_bytes = 2 * 2 * nkv * hd * 2 * (kv_len + 1)      # rows x (K, V) x heads x hd x f16 per layer
    layer_bytes = wbytes / n_copies + kv_bytes + int(head[0].nbytes) / n_copies
    hbm, hbm_kind = measured_peaks()
    # attention phase per layer: from the last CTA's QKV tiles (mark 2) to the last CTA's merges (mark 4)
    att_us = float(np.mean([tr[1 + 10 * l + 4].max() - tr[1 + 10 * l + 2].max() for l in range(n_copies)]))
    att_kv = kv_bytes
    del kv, eng
    return {
        "workload": f"config 1: 0.5B-shaped attention layer (hidden 896, 14/2 heads, hd 64, Q8_0 + bias), batch 2, "
                    f"decode 1 token vs an f16 KV cache of {kv_len} positions; {n_copies} distinct layer copies "
                    f"(weights + KV {n_copies * layer_bytes / 1e6:.0f} MB > L2) in one persistent step",
        "layer_us": round(step_us / n_copies, 3), "layer_bytes": int(layer_bytes),
        "achieved_gbs": round(layer_bytes / (step_us / n_copies / 1e6) / 1e9, 1),
        "frac": round(layer_bytes / (step_us / n_copies / 1e6) / 1e9 / hbm, 4), "peak_gbs": hbm, "peak_kind": hbm_kind,
        "attn_phase": {"us_per_layer": round(att_us, 3), "kv_bytes": int(att_kv),
                       "achieved_gbs": round(att_kv / (att_us / 1e6) / 1e9, 1),
                       "frac": round(att_kv / (att_us / 1e6) / 1e9 / hbm, 4),
                       "timed_by": "kernel %globaltimer stamps (last step)"},
    }


def c3_measure(eng, hp, torch, dist, rank, world, sh, steps, warmup=2):
    """Config 3: 64 independent TTS streams (128 rows with their CFG pairs),
    ragged KV lengths uniform in [64, 2048] (a pair shares its length), one
    greedy decode step per stream per iteration.  The streams are split over
    the ranks (data parallel, no collective on the data path); each rank
    decodes its rows as one batched step (tensor-core path, split-K attention
    over each row's own length).  The cache is paged: the rows share a pool
    of exactly the 64-position pages their lengths need (an identity-mapped
    cache would reserve the longest row's pages for every row).  Value: all
    ranks' rows per second, timed as the max over ranks."""
    streams = 64
    mine = [s for s in range(streams) if s % world == rank]
    rows = 2 * len(mine)
    rng = np.random.default_rng(SEED + 3)
    lens_all = rng.integers(64, 2049, size=streams)
    lens = np.repeat(lens_all[mine], 2)
    max_seq = int(lens.max()) + warmup + steps + 8
    pool = int(sum((int(L) + warmup + steps + 63) // 64 for L in lens))
    kv = eng.kv(rows, max_seq, pool_pages=pool)
    w = hp["n_kv_heads"] * hp["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(SEED + 3 + rank)
    for r in range(rows):
        L = int(lens[r])
        for li in range(hp["n_layers"]):
            k = torch.randn((L, w), generator=g, device="cuda", dtype=torch.float32)
            v = torch.randn((L, w), generator=g, device="cuda", dtype=torch.float32)
            kv.load_prefix(r, li, k, v)
        kv.set_past_len(r, L)
    seqs = list(range(rows))
    tok = torch.randint(0, hp["vocab"], (rows,), dtype=torch.int32, device="cuda", generator=g)
    for _ in range(warmup):
        eng.decode_step(kv, seqs, tok, tok, stream=sh)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        eng.decode_step(kv, seqs, tok, tok, stream=sh)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kv.close()
    return {"workload": "config 3: 64 streams x CFG pair (128 rows) of the 0.5B-shaped Q8_0 stack, ragged KV "
                        "64..2048, one greedy step per stream per iteration",
            "value": round(2 * streams * steps / (ms / 1000.0), 1), "unit": "tokens/s",
            "ms_per_step": round(ms / steps, 3), "rows_per_gpu": rows, "n_gpus": world, "steps": steps,
            "kv_pages": {"pool": pool, "identity_would_reserve": rows * ((max_seq + 63) // 64)},
            "scaling": "strong", "parallelism": f"data parallel over {world} GPU(s), no collectives"}


C5 = dict(hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, n_layers=28, vocab=152064,
          rope_theta=1.0e6, rms_eps=1.0e-6)


def c5_measure(vvq2, synth, torch, dist, rank, local, world, sh, T, steps):
    """Config 5: the 7B-shaped Q8_0 ASR stack, causal prefill of T prompt
    embeddings (N(0,1)), then `steps` greedy decode steps of the stream.  At
    N > 1 the attention is partitioned (vvq2_partition): KV heads over 2/4
    GPUs, KV heads x interleaved sequence parts over 8; prefill exchanges
    run on NCCL, the decode step's on peer memory (VVQ2_PEER=0: NCCL);
    each rank decodes the same single stream.  Times are CUDA events on the
    launching stream, max over ranks.  Decode bytes per step: the GGUF
    weights plus the f16 K/V of every key (57,344 B per position)."""
    hp = C5
    eng = vvq2.Engine(hp, device=local)
    seq_parts = 2 if world == 8 else 1
    if world > 1:
        ids = [vvq2.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        eng.partition(rank, world, seq_parts, ids[0])
    rng = np.random.default_rng(SEED + 55)
    wbytes = 0
    for li in range(hp["n_layers"]):
        L = synth.layer_q8_0_fast(rng, hp)
        wbytes += sum(int(t[0].nbytes) for k, t in L.items() if t is not None and "norm" not in k and "bias" not in k)
        eng.set_layer(li, L)
        del L
    head = synth.q8_0_random_tensor(rng, hp["vocab"], hp["hidden"])
    norm = synth.f32_tensor(1.0 + rng.standard_normal(hp["hidden"], dtype=np.float32) * 0.02)
    eng.set_output(norm, head, head)
    wbytes += int(head[0].nbytes)
    # warm-up on a separate cache (NCCL connections, lazily created scratch)
    kvw = eng.kv(1, 512)
    eng.forward(kvw, [0], np.zeros((1, 256, hp["hidden"]), np.float32), [0])
    kvw.close()
    kv = eng.kv(1, T + steps + 16)
    g = torch.Generator(device="cuda").manual_seed(SEED + 5)
    x = torch.randn((1, T, hp["hidden"]), generator=g, device="cuda", dtype=torch.float32)
    y = torch.empty((1, hp["hidden"]), device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream()

    def timed(fn):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    pre_ms = timed(lambda: eng.forward(kv, [0], x, [0], flags=vvq2.ADVANCE | vvq2.LAST_ONLY, y=y, stream=sh))
    del x
    tok = torch.randint(0, hp["vocab"], (1,), dtype=torch.int32, device="cuda", generator=g)
    for _ in range(2):
        eng.decode_step(kv, [0], tok, tok, stream=sh)
    dec_ms = timed(lambda: [eng.decode_step(kv, [0], tok, tok, stream=sh) for _ in range(steps)])
    kv.close()
    lin = 2.0 * T * hp["n_layers"] * hp["hidden"] * (
        hp["n_heads"] * hp["head_dim"] + 2 * hp["n_kv_heads"] * hp["head_dim"] + hp["n_heads"] * hp["head_dim"]
        + 3 * hp["ffn"])
    att = 4.0 * hp["n_heads"] * hp["head_dim"] * T * (T + 1) / 2 * hp["n_layers"]
    burst, _, kind = measured_tensor_peak()
    hbm, hbm_kind = measured_peaks()
    kv_mean = T + 2 + steps / 2
    step_bytes = wbytes + 2.0 * 2 * hp["n_layers"] * hp["n_kv_heads"] * hp["head_dim"] * kv_mean
    dec_s = dec_ms / 1000.0 / steps
    return {
        "workload": f"config 5: 7B-shaped Q8_0 stack (28 layers, hidden 3584, 28/4 heads, hd 128, ffn 18944, "
                    f"vocab 152064), causal prefill of {T} prompt embeddings, then {steps} greedy decode steps, "
                    f"batch 1", "n_gpus": world,
        "partition": "none" if world == 1 else (f"KV heads over {world} GPUs" if seq_parts == 1 else
                                                 f"KV heads x interleaved sequence parts over {world} GPUs"),
        "decode_exchange": None if world == 1 else
        ("nccl" if os.environ.get("VVQ2_PEER", "1").startswith("0") else "peer memory (CUDA IPC), one kernel each"),
        "prefill": {"tokens_per_s": round(T / (pre_ms / 1000.0), 1), "ms": round(pre_ms, 1),
                    "tflops_per_gpu": round((lin + att) / (pre_ms / 1000.0) / 1e12 / world, 1),
                    "frac_of_peak": round((lin + att) / (pre_ms / 1000.0) / 1e12 / world / burst, 4),
                    "peak_tflops": burst, "peak_kind": kind},
        "decode": {"tokens_per_s": round(steps / (dec_ms / 1000.0), 2), "ms_per_step": round(dec_ms / steps, 3),
                   "step_bytes": int(step_bytes),
                   "step_hbm_gbs_per_gpu": round(step_bytes / world / dec_s / 1e9, 1),
                   "frac_of_hbm": round(step_bytes / world / dec_s / 1e9 / hbm, 4), "peak_gbs": hbm,
                   "peak_kind": hbm_kind},
        "data": "synthetic (random Q8_0 blocks, N(0,1) embeddings)"}


def run_c5(args, rank, local, world):
    """--workload c5: config 5's own JSON line (partitioned over the ranks)."""
    import torch
    import torch.distributed as dist

    import synth
    import vvq2

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    r = c5_measure(vvq2, synth, torch, dist, rank, local, world, stream.cuda_stream, args.c5_tokens, args.c5_steps)
    line = {"impl": "ours", "metric": "qwen2_c5_prefill_decode", **r}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


C4 = dict(hidden=1536, n_heads=12, n_kv_heads=2, head_dim=128, ffn=8960, n_layers=28, vocab=151936,
          rope_theta=1.0e6, rms_eps=1.0e-6)


def c4_measure(vvq2, synth, torch, dist, world, local, sh, T, steps):
    """Config 4: the 1.5B-shaped stack (Q5_K attention, Q6_K FFN, Q8_0
    lm_head), batch 2 (the CFG pair): causal prefill of T prompt embeddings
    per row, then `steps` greedy decode steps of both rows.  The prompt
    embeddings stand for text-token embeddings plus projected acoustic
    latents (the connector is not part of this path): N(0, 1) f32.  Each rank
    runs its own replica (the config does not shard); times are CUDA events,
    max over ranks."""
    hp = C4
    eng = vvq2.Engine(hp, device=local)
    rng = np.random.default_rng(SEED + 44)
    wbytes = 0
    for li in range(hp["n_layers"]):
        L = synth.layer_c4_fast(rng, hp)
        wbytes += sum(int(t[0].nbytes) for k, t in L.items() if t is not None and "norm" not in k and "bias" not in k)
        eng.set_layer(li, L)
    head = synth.q8_0_random_tensor(rng, hp["vocab"], hp["hidden"])
    norm = synth.f32_tensor(1.0 + rng.standard_normal(hp["hidden"], dtype=np.float32) * 0.02)
    eng.set_output(norm, head, head)
    wbytes += int(head[0].nbytes)
    stream = torch.cuda.current_stream()
    kvw = eng.kv(2, 512)
    eng.forward(kvw, [0, 1], np.zeros((2, 64, hp["hidden"]), np.float32), [0, 0], stream=sh)
    kvw.close()
    kv = eng.kv(2, T + steps + 16)
    g = torch.Generator(device="cuda").manual_seed(SEED + 4)
    x = torch.randn((2, T, hp["hidden"]), generator=g, device="cuda", dtype=torch.float32)
    y = torch.empty((2, hp["hidden"]), device="cuda", dtype=torch.float32)

    def timed(fn):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    pre_ms = timed(lambda: eng.forward(kv, [0, 1], x, [0, 0], flags=vvq2.ADVANCE | vvq2.LAST_ONLY, y=y, stream=sh))
    tok = torch.randint(0, hp["vocab"], (2,), dtype=torch.int32, device="cuda", generator=g)
    for _ in range(3):
        eng.decode_step(kv, [0, 1], tok, tok, stream=sh)
    dec_ms = timed(lambda: [eng.decode_step(kv, [0, 1], tok, tok, stream=sh) for _ in range(steps)])
    lin = 2.0 * 2 * T * hp["n_layers"] * hp["hidden"] * (
        hp["n_heads"] * hp["head_dim"] + 2 * hp["n_kv_heads"] * hp["head_dim"] + hp["n_heads"] * hp["head_dim"]
        + 3 * hp["ffn"])
    att = 2 * 4.0 * hp["n_heads"] * hp["head_dim"] * T * (T + 1) / 2 * hp["n_layers"]
    burst, _, kind = measured_tensor_peak()
    hbm, hbm_kind = measured_peaks()
    kv_len = T + 3 + steps / 2
    step_bytes = wbytes + 2 * 4.0 * hp["n_layers"] * hp["n_kv_heads"] * hp["head_dim"] * kv_len
    dec_s = dec_ms / 1000.0 / steps
    kv.close()
    return {"workload":
            f"config 4: 1.5B-shaped stack (28 layers, Q5_K attention, Q6_K FFN, Q8_0 lm_head), batch 2 (CFG pair), "
            f"causal prefill of {T} prompt embeddings per row, then {steps} greedy decode steps", "n_gpus": world,
            "parallelism": "replicas only (batch 2 does not shard)",
            "prefill": {"tokens_per_s": round(2 * T / (pre_ms / 1000.0), 1), "ms": round(pre_ms, 2),
                        "tflops": round((lin + att) / (pre_ms / 1000.0) / 1e12, 1),
                        "frac_of_peak": round((lin + att) / (pre_ms / 1000.0) / 1e12 / burst, 4),
                        "peak_tflops": burst, "peak_kind": kind},
            "decode": {"tokens_per_s": round(2 * steps / (dec_ms / 1000.0), 1), "ms_per_step": round(dec_ms / steps, 3),
                       "step_bytes": int(step_bytes), "step_hbm_gbs": round(step_bytes / dec_s / 1e9, 1),
                       "frac_of_hbm": round(step_bytes / dec_s / 1e9 / hbm, 4), "peak_gbs": hbm, "peak_kind": hbm_kind},
            "data": "synthetic (random Q5_K / Q6_K / Q8_0 blocks, N(0,1) prompt embeddings)"}


def run_c4(args, rank, local, world):
    """--workload c4: config 4's own JSON line (replicas over the ranks)."""
    import torch
    import torch.distributed as dist

    import synth
    import vvq2

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600))
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    r = c4_measure(vvq2, synth, torch, dist, world, local, stream.cuda_stream, args.c4_tokens, args.c4_steps)
    line = {"impl": "ours", "metric": "qwen2_c4_prefill_decode", **r}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_case(args):
    """Small single-GPU workloads for kernel profiles (a few GB on the device):
    * decode7b: config-5 dims with args.case_layers layers and a small vocab,
      args.kv keys of N(0,1) K/V per layer, then warm-up + timed greedy
      decode steps of one row through vvq2_decode_step (GEMV graph path:
      k_gemv_stream, k_attn_mma, k_attn_merge);
    * c3: config 3's batched step (128 rows, ragged KV) -- tensor-core GEMMs
      and the tensor-core decode attention.
    Prints one JSON line with the mean step time (CUDA events)."""
    import torch

    import synth
    import vvq2

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    if args.case == "c3":
        hp = C2
        model = synth.model_q8_0(SEED, hp)
        eng = vvq2.Engine(hp, device=0)
        for li, t in enumerate(model["layers"]):
            eng.set_layer(li, t)
        eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
        r = c3_measure(eng, hp, torch, None, 0, 1, stream.cuda_stream, args.steps, warmup=args.warmup)
        print(json.dumps({"case": "c3", "ms_per_step": r["ms_per_step"], "tokens_per_s": r["value"]}), flush=True)
        return 0
    hp = dict(C5)
    hp["n_layers"] = args.case_layers
    hp["vocab"] = 8192
    eng = vvq2.Engine(hp, device=0)
    rng = np.random.default_rng(SEED + 55)
    for li in range(hp["n_layers"]):
        eng.set_layer(li, synth.layer_q8_0_fast(rng, hp))
    head = synth.q8_0_random_tensor(rng, hp["vocab"], hp["hidden"])
    norm = synth.f32_tensor(1.0 + rng.standard_normal(hp["hidden"], dtype=np.float32) * 0.02)
    eng.set_output(norm, head, head)
    T = args.kv
    kv = eng.kv(1, T + args.warmup + args.steps + 8)
    w = hp["n_kv_heads"] * hp["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(SEED + 7)
    for li in range(hp["n_layers"]):
        kv.load_prefix(0, li, torch.randn((T, w), generator=g, device="cuda"),
                       torch.randn((T, w), generator=g, device="cuda"))
    kv.set_past_len(0, T)
    tok = torch.randint(0, hp["vocab"], (1,), dtype=torch.int32, device="cuda", generator=g)
    sh = stream.cuda_stream
    for _ in range(args.warmup):
        eng.decode_step(kv, [0], tok, tok, stream=sh)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        eng.decode_step(kv, [0], tok, tok, stream=sh)
    e1.record(stream)
    torch.cuda.synchronize()
    print(json.dumps({"case": "decode7b", "layers": hp["n_layers"], "kv": T,
                      "ms_per_step": round(e0.elapsed_time(e1) / args.steps, 4)}), flush=True)
    kv.close()
    return 0


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def cpu_decode_rate(model, hp, kv_len, budget_s=15.0, flags=None, steps=64, warmup=0):
    """CPU oracle (test infrastructure) decode tokens/s on this host: `warmup`
    untimed greedy steps of both rows, then up to `steps` timed ones (fewer if
    the time budget runs out first).  Returns (tokens/s, timed steps, threads)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vvq2_oracle as O
    flags = (O.GGML_CPU | O.SIMD) if flags is None else flags
    rng = np.random.default_rng(SEED + 1)
    max_steps = steps
    ora = O.Model(hp, 2, kv_len + warmup + max_steps + 2, flags)
    for li, t in enumerate(model["layers"]):
        ora.set_layer(li, t)
    ora.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    w = hp["n_kv_heads"] * hp["head_dim"]
    for li in range(hp["n_layers"]):
        for s in range(2):
            ora.kv_load(s, li, rng.standard_normal((kv_len, w), dtype=np.float32),
                        rng.standard_normal((kv_len, w), dtype=np.float32))
    for s in range(2):
        ora.set_past_len(s, kv_len)
    tok = rng.integers(0, hp["vocab"], size=2).astype(np.int32)
    for _ in range(warmup):
        pos = [ora.past_len(0), ora.past_len(1)]
        h = ora.forward([0, 1], ora.embed(tok)[:, None, :], pos, output_norm=True)
        tok = ora.lm_head(h[:, 0]).astype(np.int32)
    t0 = time.perf_counter()
    n = 0
    while n < max_steps:
        pos = [ora.past_len(0), ora.past_len(1)]
        h = ora.forward([0, 1], ora.embed(tok)[:, None, :], pos, output_norm=True)
        tok = ora.lm_head(h[:, 0]).astype(np.int32)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return 2 * n / dt, n, cores, (O.simd_isa() if flags & O.SIMD else "generic")


class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        # a private temporary file: the samples are summarised into the JSON line
        self.out = Path(tempfile.gettempdir()) / f"vvq2_clocks_rank{index}_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.out, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.f.close()
            self.text = self.out.read_text() if self.out.exists() else ""
            self.out.unlink(missing_ok=True)

    def summary(self):
        if not self.proc or not getattr(self, "text", ""):
            return None
        rows = [r.split(", ") for r in self.text.strip().splitlines() if r.strip()]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and r[5 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def run_reference(args, rank):
    if rank != 0:
        return 0
    import synth
    model = synth.model_q8_0(SEED, C2)
    # the arm's own --steps/--warmup, each step one greedy decode step of both
    # rows; a 150 s budget bounds the timed part on slow hosts
    rate, n, cores, isa = cpu_decode_rate(model, C2, args.kv, budget_s=150.0, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": "qwen2_decode_tokens_per_s", "value": round(rate, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "warmup": args.warmup, "ms_per_step": round(2000.0 / rate, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->f32 (ggml q8_0 dot)",
        "data": "synthetic", "config": workload_config(args),
        "cpu_baseline": {"value": round(rate, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{n} greedy decode steps x 2 rows of the full C2 stack (ggml CPU numerics, "
                                   f"SIMD kernels: {isa} Q8_0 dot, AVX2/F16C f16 flash attention)"},
        "e2e": {"value": round(rate, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's ggml CPU backend cannot be built here (ggml submodule absent); "
                "this is the CPU restatement of its numerics (oracle/) with SIMD integer dots and f16 "
                "attention as ggml's x86 backend runs them, all host threads",
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args):
    return {"workload": "C2: Qwen2.5-0.5B-shaped 24-layer LM, Q8_0 (tied lm_head), batch 2 CFG greedy decode",
            "model": "qwen2.5-0.5b-shaped (random init)", "global_batch": 2 * args.gpus, "kv_len": args.kv,
            "seq_len": args.kv, "parallelism": f"replicas x{args.gpus}" if args.gpus > 1 else "single",
            "l2": "weights 550 MB/step > 126 MB L2: streamed from HBM each step, no flush"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--kv", type=int, default=1024)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--prefill-tokens", type=int, default=16384)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-c3", action="store_true")
    ap.add_argument("--no-c1", action="store_true")
    ap.add_argument("--no-c4", action="store_true")
    ap.add_argument("--no-c5", action="store_true")
    ap.add_argument("--workload", default="c2", choices=["c2", "c4", "c5"])
    ap.add_argument("--case", default=None, choices=["decode7b", "c3"],
                    help="small single-GPU workload for kernel profiles (see run_case)")
    ap.add_argument("--case-layers", type=int, default=2)
    ap.add_argument("--c4-tokens", type=int, default=1024)
    ap.add_argument("--c4-steps", type=int, default=512)
    ap.add_argument("--c5-tokens", type=int, default=27000)
    ap.add_argument("--c5-steps", type=int, default=2048)
    ap.add_argument("--c3-steps", type=int, default=10)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, local, world = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.case:
        return run_case(args)
    if args.workload == "c5":
        return run_c5(args, rank, local, world)
    if args.workload == "c4":
        return run_c4(args, rank, local, world)

    import torch
    import torch.distributed as dist

    import synth
    import vvq2

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    hp = C2
    model = synth.model_q8_0(SEED, hp)
    eng = vvq2.Engine(hp, device=local)
    for li, t in enumerate(model["layers"]):
        eng.set_layer(li, t)
    eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    prof_steps = 20
    total = args.warmup + args.steps * 2 + prof_steps + 8
    kv = eng.kv(2, args.kv + total)
    w = hp["n_kv_heads"] * hp["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(SEED + rank)
    for li in range(hp["n_layers"]):
        for s in range(2):
            k = torch.randn((args.kv, w), generator=g, device="cuda", dtype=torch.float32)
            v = torch.randn((args.kv, w), generator=g, device="cuda", dtype=torch.float32)
            kv.load_prefix(s, li, k, v)
    for s in range(2):
        kv.set_past_len(s, args.kv)
    # a real stream object: handle 0 would mean "the library's own stream" and the
    # events below would not see the work
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    assert sh != 0
    tok = torch.randint(0, hp["vocab"], (2,), dtype=torch.int32, device="cuda")

    def steps(n):
        for _ in range(n):
            eng.decode_step(kv, [0, 1], tok, tok, stream=sh)

    # clocks are sampled over the whole GPU part of the run (warm-up, timed
    # steps, e2e, profiling pass, c3 and prefill fields)
    clk = ClockSampler(local).__enter__()
    steps(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = vvq2.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    launches = vvq2.launches() - l0
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = 2 * world * args.steps / (ms / 1000.0)

    # e2e: host token buffers through the C ABI (H2D ids + D2H argmax ids per step)
    host_tok = tok.cpu().numpy().astype(np.int32)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        host_tok = eng.decode_step(kv, [0, 1], host_tok, stream=sh)
    e3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)
    if world > 1:
        t = torch.tensor([ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = 2 * world * args.steps / (ms_e2e / 1000.0)

    # roofline of the dominant kernel: CUDA events around every launch on the
    # launching stream (kind 0: the persistent decode-step kernel, or the GEMVs
    # of the per-phase graph; kind 1: per-phase attention launches)
    eng.profile(True)
    tok.copy_(torch.from_numpy(host_tok).cuda())
    for _ in range(prof_steps):
        eng.decode_step(kv, [0, 1], tok, tok, stream=sh)
    g_ms, g_bytes, g_n = eng.profile_read(0)
    a_ms, a_bytes, a_n = eng.profile_read(1)
    eng.profile(False)
    peak, peak_kind = measured_peaks()
    achieved = (g_bytes / g_n) / (g_ms / g_n / 1000.0) / 1e9 if g_n else None
    persistent = g_n > 0 and launches == args.steps   # one launch per step
    traffic = None
    tf = ROOT / "profiles" / ("decode_mega_c2_traffic.json" if persistent else "gemv_q8_0_c2_traffic.json")
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")
    kname = ("k_decode_mega (persistent decode step: streamed Q8_0 GEMV tiles, split-K flash-decode, "
             "fused RMSNorm/RoPE/SwiGLU/residual/argmax)" if persistent else
             "k_gemv (fused RMSNorm + Q8_0 GEMV + epilogue)")

    line = {
        "metric": "qwen2_decode_tokens_per_s", "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (exactly dequantized Q8_0 int8 weights x f32 activations), f16 K/V",
        "data": "synthetic (seeded random-init weights of the architecture)",
        "config": workload_config(argparse.Namespace(**{**vars(args), "gpus": world})),
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1) if achieved else None, "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4) if achieved else None,
                     "traffic": traffic, "kernel": kname,
                     "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": round(g_bytes / g_n) if g_n else None,
                     "mean_launch_us": round(1000.0 * g_ms / g_n, 3) if g_n else None,
                     "attn_decode": {"achieved_gbs": round(a_bytes / (a_ms / 1000.0) / 1e9, 1) if a_n else None,
                                     "mean_launch_us": round(1000.0 * a_ms / a_n, 3) if a_n else None},
                     "step_hbm_gbs": round(synth.weight_bytes(model) * 1.0 / (ms / args.steps / 1000.0) / 1e9, 1)},
    }
    if not args.no_c3:
        line["c3"] = c3_measure(eng, hp, torch, dist, rank, world, sh, args.c3_steps)
    if not args.no_c1:
        c1 = c1_measure(vvq2, synth, torch, local, sh)
        line["c1"] = c1
        line["roofline"]["attn_decode"] = {"achieved_gbs": c1["attn_phase"]["achieved_gbs"],
                                           "frac": c1["attn_phase"]["frac"],
                                           "us_per_layer": c1["attn_phase"]["us_per_layer"],
                                           "source": "c1: attention phase of the persistent step, 64 layer copies"}
    if not args.no_prefill:
        line["prefill"] = prefill_measure(vvq2, synth, torch, local, sh, args.prefill_tokens)
    clk.__exit__(None, None, None)
    line["clocks"] = clk.summary()
    if world == 1 and not args.no_c4:
        line["c4"] = c4_measure(vvq2, synth, torch, dist, world, local, sh, args.c4_tokens, args.c4_steps)
    if world == 1 and not args.no_c5:
        line["c5"] = c5_measure(vvq2, synth, torch, dist, rank, local, world, sh, args.c5_tokens, args.c5_steps)
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, n, cores, isa = cpu_decode_rate(model, hp, args.kv)
        line["cpu_baseline"] = {"value": round(rate, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": f"{n} greedy decode steps x 2 rows of the full C2 stack, ggml CPU "
                                          f"numerics with SIMD kernels ({isa} Q8_0 dot, AVX2/F16C f16 flash "
                                          f"attention; oracle/, OpenMP over {cores} threads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
