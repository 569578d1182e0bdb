#!/usr/bin/env python3
"""Regenerate the golden fixtures under tests/golden/ (run in the build
container, where the vibevoice.cpp reference tree and gguf-py are present).

  python tests/golden/make_golden.py --reference /path/to/vibevoice.cpp

Fixtures (all small .npz files, committed):
  dequant.npz   random Q8_0 / Q5_K / Q6_K blocks and gguf-py's numpy
                dequantization of them (gguf.quants.dequantize), plus f32 rows
                and gguf-py's Q8_0.quantize_blocks bytes (documented there as
                bit-exact with ggml-quants.c).
  rope.npz      NEOX RoPE goldens from the reference's own generator
                tests/dump_rope_reference.py (function rope_neox, fp64), at its
                default shape (dim 64, 4 heads, seq 128, theta 1e6, seed 2025)
                and at head_dim 128 with positions up to 32767.
  qwen2_layer0.npz  the reference's tests/dump_qwen2_reference.py fixture (HF
                Qwen2DecoderLayer, hidden 128, 4/2 heads, hd 32, ffn 384, seq 64,
                seed 1234), read back from the GGUF it writes.
"""
from __future__ import annotations

import argparse
import importlib.util
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_dequant(rng: np.random.Generator) -> None:
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    out = {}
    specs = {"q8_0": (T.Q8_0, 34, [0]), "q5_K": (T.Q5_K, 176, [0, 2]), "q6_K": (T.Q6_K, 210, [208])}
    for name, (qt, bsize, f16_offsets) in specs.items():
        nb = 96
        raw = rng.integers(0, 256, size=(nb, bsize), dtype=np.uint8)
        for off in f16_offsets:        # finite, modest scales
            d = (rng.standard_normal(nb) * 0.01).astype(np.float16)
            if name != "q6_K" and off == 0 and name == "q5_K":
                d = np.abs(d)
            raw[:, off:off + 2] = d.view(np.uint8).reshape(nb, 2)
        deq = quants.dequantize(raw.reshape(-1), qt).astype(np.float32)
        out[f"{name}_blocks"] = raw.reshape(-1)
        out[f"{name}_deq"] = deq.reshape(-1)
    x = (rng.standard_normal((64, 32)) * rng.uniform(0.01, 3.0, size=(64, 1))).astype(np.float32)
    x[3] = 0.0                                             # all-zero block
    out["q8_0_quant_src"] = x.reshape(-1)
    out["q8_0_quant_bytes"] = quants.Q8_0.quantize_blocks(x).reshape(-1).astype(np.uint8)
    np.savez_compressed(HERE / "dequant.npz", **out)


def make_rope(ref: Path) -> None:
    mod = _load_module(ref / "tests" / "dump_rope_reference.py", "dump_rope_reference")
    out = {}
    # the reference generator's own default case
    rng = np.random.default_rng(2025)
    x = rng.standard_normal((128, 4, 64)).astype(np.float32)
    pos = np.arange(128).astype(np.int32)
    out["d64_x"], out["d64_pos"], out["d64_y"] = x, pos, mod.rope_neox(x, pos, 1.0e6)
    # head_dim 128 at long-context positions (7B / 1.5B shapes)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((64, 2, 128)).astype(np.float32)
    pos = np.sort(rng.integers(0, 32768, size=64)).astype(np.int32)
    out["d128_x"], out["d128_pos"], out["d128_y"] = x, pos, mod.rope_neox(x, pos, 1.0e6)
    np.savez_compressed(HERE / "rope.npz", **out)


def make_qwen2_layer(ref: Path) -> None:
    import gguf

    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "qwen2_layer0.gguf"
        subprocess.run([sys.executable, str(ref / "tests" / "dump_qwen2_reference.py"),
                        "--out", str(path)], check=True)
        rd = gguf.GGUFReader(str(path))
        out = {}
        for t in rd.tensors:
            out[t.name] = np.array(t.data)
        meta = {}
        for k, f in rd.fields.items():
            if k.startswith("qwen2."):
                meta[k] = f.contents()
    np.savez_compressed(HERE / "qwen2_layer0.npz",
                        hparams=np.array([meta["qwen2.hidden_size"], meta["qwen2.n_heads"],
                                          meta["qwen2.n_kv_heads"], meta["qwen2.head_dim"],
                                          meta["qwen2.intermediate_size"], meta["qwen2.test.seq_len"],
                                          meta["qwen2.test.batch"]], dtype=np.int64),
                        rope_theta=np.float32(meta["qwen2.rope_theta"]),
                        rms_eps=np.float32(meta["qwen2.rms_norm_eps"]),
                        **out)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="vibevoice.cpp source tree")
    args = ap.parse_args()
    ref = Path(args.reference)
    make_dequant(np.random.default_rng(20261201))
    make_rope(ref)
    make_qwen2_layer(ref)
    for p in sorted(HERE.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size} bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
