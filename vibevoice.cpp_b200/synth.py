"""Seeded synthetic Qwen2 weights in GGUF block formats (numpy only).

The benchmark configurations use random-initialised weights of the real
architecture (there are no checkpoints offline): weights N(0, 0.02) f32,
q/k/v biases N(0, 0.02), RMSNorm weights 1 + N(0, 0.02), quantized to Q8_0
with the ggml reference rounding (d = amax/127 stored f16, q = roundf(x/d)),
which is bit-exact with gguf-py's Q8_0.quantize_blocks."""
from __future__ import annotations

import numpy as np

F32, F16, Q8_0, Q5_K, Q6_K = 0, 1, 8, 13, 14


def _roundf(v: np.ndarray) -> np.ndarray:
    """C roundf (half away from zero), exact for |v| < 2^23."""
    a = np.abs(v)
    f = np.floor(a)
    return np.sign(v) * (f + np.floor(2.0 * (a - f)))


def q8_0(w: np.ndarray) -> np.ndarray:
    """f32 [rows, cols] -> raw Q8_0 bytes [rows, cols/32*34] (quantize_row_q8_0_ref)."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    b = w.reshape(-1, 32)
    d = (np.abs(b).max(axis=1, keepdims=True) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _roundf((b * idv).astype(np.float32)).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def f32_tensor(a: np.ndarray):
    a = np.ascontiguousarray(a, np.float32)
    return (a.view(np.uint8).reshape(-1), F32, a.shape[-1], 1 if a.ndim == 1 else a.shape[0])


def q8_0_tensor(rng, rows: int, cols: int, std: float = 0.02, chunk: int = 8192):
    out = np.empty((rows, cols // 32 * 34), np.uint8)
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        out[r0:r1] = q8_0((rng.standard_normal((r1 - r0, cols), dtype=np.float32) * std))
    return (out.reshape(-1), Q8_0, cols, rows)


def layer_q8_0(rng, hp: dict, bias: bool = True) -> dict:
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    g = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.02)
    return {
        "attn_norm": f32_tensor(1.0 + g(H)),
        "attn_q": q8_0_tensor(rng, nq * hd, H),
        "attn_k": q8_0_tensor(rng, nkv * hd, H),
        "attn_v": q8_0_tensor(rng, nkv * hd, H),
        "attn_o": q8_0_tensor(rng, H, nq * hd),
        "attn_q_bias": f32_tensor(g(nq * hd)) if bias else None,
        "attn_k_bias": f32_tensor(g(nkv * hd)) if bias else None,
        "attn_v_bias": f32_tensor(g(nkv * hd)) if bias else None,
        "ffn_norm": f32_tensor(1.0 + g(H)),
        "ffn_gate": q8_0_tensor(rng, F, H),
        "ffn_up": q8_0_tensor(rng, F, H),
        "ffn_down": q8_0_tensor(rng, H, F),
    }


def q8_0_random_tensor(rng, rows: int, cols: int, std: float = 0.02):
    """Random Q8_0 blocks without a float pass (for large timing models):
    uniform int8 quants and f16 scales ~ std*2.5/127, the scale a block of
    N(0, std) values gets.  Statistically close to q8_0_tensor, much faster."""
    nb = rows * (cols // 32)
    raw = np.frombuffer(rng.bytes(nb * 34), np.uint8).reshape(nb, 34).copy()
    d = (rng.uniform(0.8, 1.2, size=nb) * std * 2.5 / 127).astype(np.float16)
    raw[:, :2] = d.view(np.uint8).reshape(-1, 2)
    raw[:, 2:] = np.where(raw[:, 2:] == 128, 127, raw[:, 2:])   # int8 -128 excluded, as in ggml's quantizer
    return (raw.reshape(-1), Q8_0, cols, rows)


def layer_q8_0_fast(rng, hp: dict) -> dict:
    """layer_q8_0 with random Q8_0 bytes (q8_0_random_tensor)."""
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    g = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.02)
    return {
        "attn_norm": f32_tensor(1.0 + g(H)),
        "attn_q": q8_0_random_tensor(rng, nq * hd, H),
        "attn_k": q8_0_random_tensor(rng, nkv * hd, H),
        "attn_v": q8_0_random_tensor(rng, nkv * hd, H),
        "attn_o": q8_0_random_tensor(rng, H, nq * hd),
        "attn_q_bias": f32_tensor(g(nq * hd)),
        "attn_k_bias": f32_tensor(g(nkv * hd)),
        "attn_v_bias": f32_tensor(g(nkv * hd)),
        "ffn_norm": f32_tensor(1.0 + g(H)),
        "ffn_gate": q8_0_random_tensor(rng, F, H),
        "ffn_up": q8_0_random_tensor(rng, F, H),
        "ffn_down": q8_0_random_tensor(rng, H, F),
    }


def kquant_random_tensor(rng, qtype: int, rows: int, cols: int):
    """Random Q5_K / Q6_K super-blocks for timing models: random quant and
    scale bytes, f16 super-block scales chosen so that |w| stays below ~0.04
    (the range of N(0, 0.02) weights).  Every byte pattern is a valid block."""
    nb = rows * (cols // 256)
    if qtype == Q5_K:
        # block_q5_K: d, dmin (f16), scales[12] (6-bit sc/m), qh[32], qs[128]
        raw = np.frombuffer(rng.bytes(nb * 176), np.uint8).reshape(nb, 176).copy()
        d = (rng.uniform(0.8, 1.2, size=nb) * 2.0e-5).astype(np.float16)
        dmin = (rng.uniform(0.8, 1.2, size=nb) * 1.0e-5).astype(np.float16)
        raw[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        raw[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    elif qtype == Q6_K:
        # block_q6_K: ql[128], qh[64], scales[16] (int8), d (f16)
        raw = np.frombuffer(rng.bytes(nb * 210), np.uint8).reshape(nb, 210).copy()
        d = (rng.uniform(0.8, 1.2, size=nb) * 1.0e-5).astype(np.float16)
        raw[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    else:
        raise ValueError("qtype must be Q5_K or Q6_K")
    return (raw.reshape(-1), qtype, cols, rows)


def layer_c4_fast(rng, hp: dict) -> dict:
    """Config-4 layer with random blocks: Q5_K attention, Q6_K FFN."""
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    g = lambda *s: (rng.standard_normal(s, dtype=np.float32) * 0.02)
    return {
        "attn_norm": f32_tensor(1.0 + g(H)),
        "attn_q": kquant_random_tensor(rng, Q5_K, nq * hd, H),
        "attn_k": kquant_random_tensor(rng, Q5_K, nkv * hd, H),
        "attn_v": kquant_random_tensor(rng, Q5_K, nkv * hd, H),
        "attn_o": kquant_random_tensor(rng, Q5_K, H, nq * hd),
        "attn_q_bias": f32_tensor(g(nq * hd)),
        "attn_k_bias": f32_tensor(g(nkv * hd)),
        "attn_v_bias": f32_tensor(g(nkv * hd)),
        "ffn_norm": f32_tensor(1.0 + g(H)),
        "ffn_gate": kquant_random_tensor(rng, Q6_K, F, H),
        "ffn_up": kquant_random_tensor(rng, Q6_K, F, H),
        "ffn_down": kquant_random_tensor(rng, Q6_K, H, F),
    }


def model_q8_0(seed: int, hp: dict, n_layers: int | None = None) -> dict:
    """Full LM: layers, output_norm, tied Q8_0 lm_head / token embedding."""
    rng = np.random.default_rng(seed)
    n = hp["n_layers"] if n_layers is None else n_layers
    layers = [layer_q8_0(rng, hp) for _ in range(n)]
    head = q8_0_tensor(rng, hp["vocab"], hp["hidden"])
    norm = f32_tensor(1.0 + rng.standard_normal(hp["hidden"], dtype=np.float32) * 0.02)
    return {"layers": layers, "output_norm": norm, "lm_head": head, "tok_embd": head}


def tensor_bytes(spec) -> int:
    return 0 if spec is None else int(spec[0].nbytes)


def weight_bytes(model: dict) -> int:
    n = sum(tensor_bytes(t) for L in model["layers"] for t in L.values())
    return n + tensor_bytes(model["output_norm"]) + tensor_bytes(model["lm_head"])
