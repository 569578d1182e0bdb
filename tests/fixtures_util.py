"""Shared helpers for the parity tests: golden-layer loading and seeded
synthetic Qwen2 weights in GGUF block formats (quantized by the oracle's
quantizers or gguf-py's bit-exact Q8_0 quantizer)."""
from __future__ import annotations

import numpy as np

import vvq2_oracle as O

LAYER_NAMES = ["attn_norm", "attn_q", "attn_q_bias", "attn_k", "attn_k_bias", "attn_v",
               "attn_v_bias", "attn_o", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]


def golden_layer(z):
    """(hparams dict, tensors dict name -> (raw, type, ne0, ne1), x, y, pos) from
    the reference's dump_qwen2_reference.py fixture (f32 weights)."""
    hidden, nh, nkv, hd, ffn, seq, batch = [int(v) for v in z["hparams"]]
    hp = dict(hidden=hidden, n_heads=nh, n_kv_heads=nkv, head_dim=hd, ffn=ffn, n_layers=1,
              vocab=0, rope_theta=float(z["rope_theta"]), rms_eps=float(z["rms_eps"]))
    t = {}
    for n in LAYER_NAMES:
        a = np.ascontiguousarray(z["weight." + n], np.float32)
        ne1, ne0 = (a.shape if a.ndim == 2 else (1, a.shape[0]))
        t[n] = (a.view(np.uint8).reshape(-1), O.F32, ne0, ne1)
    return hp, t, z["test.input"], z["test.expected_output"], z["test.position_ids"]


def q8_0_bytes(w: np.ndarray) -> np.ndarray:
    """gguf-py's Q8_0 quantizer if present (bit-exact with ggml), else the oracle's."""
    try:
        from gguf import quants
        rows, cols = w.shape
        return quants.Q8_0.quantize_blocks(w.reshape(-1, 32)).reshape(rows, -1).astype(np.uint8)
    except Exception:
        return O.quantize(O.Q8_0, w)


def quant_tensor(w: np.ndarray, qtype: int):
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    raw = q8_0_bytes(w) if qtype == O.Q8_0 else O.quantize(qtype, w)
    return (np.ascontiguousarray(raw).reshape(-1), qtype, cols, rows)


def f32_tensor(a: np.ndarray):
    a = np.ascontiguousarray(a, np.float32)
    return (a.view(np.uint8).reshape(-1), O.F32, a.shape[-1], 1 if a.ndim == 1 else a.shape[0])


def random_layer(rng, hp, wtype=O.Q8_0, attn_type=None, ffn_type=None, bias=True, std=0.02,
                 with_ffn=True):
    """Seeded Qwen2 layer: weights N(0, std), q/k/v bias N(0, std), norm weights 1 + N(0, 0.02)."""
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    at = attn_type if attn_type is not None else wtype
    ft = ffn_type if ffn_type is not None else wtype
    g = lambda *s: (rng.standard_normal(s) * std).astype(np.float32)
    t = {
        "attn_norm": f32_tensor(1.0 + g(H)),
        "attn_q": quant_tensor(g(nq * hd, H), at),
        "attn_k": quant_tensor(g(nkv * hd, H), at),
        "attn_v": quant_tensor(g(nkv * hd, H), at),
        "attn_o": quant_tensor(g(H, nq * hd), at),
        "attn_q_bias": f32_tensor(g(nq * hd)) if bias else None,
        "attn_k_bias": f32_tensor(g(nkv * hd)) if bias else None,
        "attn_v_bias": f32_tensor(g(nkv * hd)) if bias else None,
        "ffn_norm": f32_tensor(1.0 + g(H)),
    }
    if with_ffn:
        t["ffn_gate"] = quant_tensor(g(F, H), ft)
        t["ffn_up"] = quant_tensor(g(F, H), ft)
        t["ffn_down"] = quant_tensor(g(H, F), ft)
    return t


def rel_err(a: np.ndarray, b: np.ndarray) -> float:
    """max |a - b| / max |b|  (normwise max relative error)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def cos_sim(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))


C1 = dict(hidden=896, n_heads=14, n_kv_heads=2, head_dim=64, ffn=4864, n_layers=1, vocab=151936,
          rope_theta=1.0e6, rms_eps=1.0e-6)
C2 = dict(C1, n_layers=24)
C4 = dict(hidden=1536, n_heads=12, n_kv_heads=2, head_dim=128, ffn=8960, n_layers=28,
          vocab=151936, rope_theta=1.0e6, rms_eps=1.0e-6)
C5 = dict(hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, n_layers=28,
          vocab=152064, rope_theta=1.0e6, rms_eps=1.0e-6)
