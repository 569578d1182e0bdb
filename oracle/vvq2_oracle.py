"""ctypes binding of the CPU oracle (oracle/vvq2_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs as the checker.  The product path never imports
this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "libvvq2_oracle.so"

F32, F16, Q8_0, Q5_K, Q6_K = 0, 1, 8, 13, 14
ACT_GGML, KV_F16, Q_F16, FA_F16ACC, ROPE_GGML, NO_FFN, SIMD = 1, 2, 4, 8, 16, 32, 64
# what the reference's CPU backend computes (ggml semantics on every op)
GGML_CPU = ACT_GGML | KV_F16 | Q_F16 | FA_F16ACC | ROPE_GGML
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q5_K: (256, 176), Q6_K: (256, 210)}


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int), ("ne0", C.c_int64), ("ne1", C.c_int64)]


class Layer(C.Structure):
    _fields_ = [(n, Tensor) for n in (
        "attn_norm", "attn_q", "attn_q_bias", "attn_k", "attn_k_bias", "attn_v", "attn_v_bias",
        "attn_o", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")]


class HParams(C.Structure):
    _fields_ = [("hidden", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("n_layers", C.c_int), ("vocab", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "vvo_dequantize": (I, [I, P, I64, P]),
            "vvo_quantize_q8_0": (I, [P, I64, P]),
            "vvo_quantize_q8_K": (I, [P, I64, P]),
            "vvo_quantize_q5_K": (I, [P, I64, P]),
            "vvo_quantize_q6_K": (I, [P, I64, P]),
            "vvo_matvec": (I, [P, P, P, I]),
            "vvo_rms_norm": (None, [P, P, I, F, P]),
            "vvo_rope_neox": (None, [P, I, I, I, F, I, P]),
            "vvo_simd_isa": (C.c_char_p, []),
            "vvo_fp32_to_fp16": (C.c_uint16, [F]),
            "vvo_fp16_to_fp32": (F, [C.c_uint16]),
            "vvo_model_new": (P, [P, I, I, I]),
            "vvo_model_free": (None, [P]),
            "vvo_model_set_layer": (I, [P, I, P]),
            "vvo_model_set_output": (I, [P, P, P, P]),
            "vvo_kv_load": (I, [P, I, I, P, P, I]),
            "vvo_kv_read": (I, [P, I, I, P, P, I]),
            "vvo_set_past_len": (I, [P, I, I]),
            "vvo_past_len": (I, [P, I]),
            "vvo_forward": (I, [P, I, P, I, P, P, I, I, I, I, P]),
            "vvo_lm_head": (I, [P, I, P, P, P]),
            "vvo_embed": (I, [P, I, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def row_bytes(qtype: int, n: int) -> int:
    be, bb = BLOCK[qtype]
    assert n % be == 0
    return n // be * bb


def dequantize(qtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw)
    out = np.empty(n, np.float32)
    rc = lib().vvo_dequantize(qtype, _p(raw), n, _p(out))
    assert rc == 0, rc
    return out


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    """f32 [rows, cols] -> raw GGUF bytes [rows, row_bytes]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    if qtype == F32:
        return x.view(np.uint8).reshape(rows, -1).copy()
    if qtype == F16:
        return x.astype(np.float16).view(np.uint8).reshape(rows, -1).copy()
    out = np.empty((rows, row_bytes(qtype, cols)), np.uint8)
    fn = {Q8_0: lib().vvo_quantize_q8_0, Q5_K: lib().vvo_quantize_q5_K, Q6_K: lib().vvo_quantize_q6_K}[qtype]
    rc = fn(_p(x), x.size, _p(out))
    assert rc == 0, rc
    return out


def quantize_q8_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size // 256 * 292, np.uint8)
    assert lib().vvo_quantize_q8_K(_p(x), x.size, _p(out)) == 0
    return out


def tensor(raw: np.ndarray, qtype: int, ne0: int, ne1: int) -> Tensor:
    return Tensor(raw.ctypes.data if raw is not None else None, qtype, ne0, ne1)


def matvec(raw: np.ndarray, qtype: int, ne0: int, ne1: int, x: np.ndarray, flags: int) -> np.ndarray:
    t = tensor(raw, qtype, ne0, ne1)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(ne1, np.float32)
    assert lib().vvo_matvec(C.byref(t), _p(x), _p(y), flags) == 0
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().vvo_rms_norm(_p(x), _p(w), x.size, eps, _p(y))
    return y


def _vec(spec):
    """f32 vector of an optional (raw, type, ne0, ne1) bias / norm spec."""
    if spec is None or spec[0] is None:
        return None
    raw, qt, ne0, ne1 = spec
    return dequantize(qt, raw, ne0 * max(ne1, 1))


def connector(x: np.ndarray, fc1, fc1_b, norm, fc2, fc2_b, flags: int = 0) -> np.ndarray:
    """SpeechConnector (src/vibevoice_tts.cpp:464-501, run_speech_connector):
    y = fc2(rms_norm(fc1(x) + b1, eps 1e-6) * norm) + b2, per row of x [batch][latent];
    fc* are (raw GGUF bytes, type, ne0, ne1) specs."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    b1, g, b2 = _vec(fc1_b), _vec(norm), _vec(fc2_b)
    out = []
    for row in x:
        h = matvec(fc1[0], fc1[1], fc1[2], fc1[3], row, flags)
        if b1 is not None:
            h = (h + b1).astype(np.float32)
        h = rms_norm(h, g if g is not None else np.ones_like(h), 1e-6)
        y = matvec(fc2[0], fc2[1], fc2[2], fc2[3], h, flags)
        if b2 is not None:
            y = (y + b2).astype(np.float32)
        out.append(y)
    return np.stack(out)


def eos(x: np.ndarray, fc1, fc1_b, fc2, fc2_b, flags: int = 0) -> np.ndarray:
    """EOS classifier (src/vibevoice_tts.cpp:503-537, run_eos_classifier):
    p = sigmoid(fc2(relu(fc1(x) + b1)) + b2) per row of x [batch][hidden]."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    b1, b2 = _vec(fc1_b), _vec(fc2_b)
    out = []
    for row in x:
        h = matvec(fc1[0], fc1[1], fc1[2], fc1[3], row, flags)
        if b1 is not None:
            h = (h + b1).astype(np.float32)
        h = np.maximum(h, np.float32(0))
        z = matvec(fc2[0], fc2[1], fc2[2], fc2[3], h, flags)
        if b2 is not None:
            z = (z + b2).astype(np.float32)
        out.append(np.float32(1) / (np.float32(1) + np.exp(-z.astype(np.float32))))
    return np.concatenate(out).astype(np.float32)


def rope_neox(x: np.ndarray, pos: int, theta: float, flags: int) -> np.ndarray:
    """x [n_heads, hd] at one position."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().vvo_rope_neox(_p(x), x.shape[0], x.shape[1], int(pos), theta, flags, _p(y))
    return y


def simd_isa() -> str:
    """Instruction set of the SIMD Q8_0 dot on this CPU (flag SIMD)."""
    return lib().vvo_simd_isa().decode()


def fp16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


class Model:
    """Stateful oracle: weights (borrowed raw GGUF bytes) + per-row resident KV."""

    LAYER_FIELDS = [f[0] for f in Layer._fields_]

    def __init__(self, hp: dict, n_rows: int, max_seq: int, flags: int):
        self.hp = dict(hp)
        self._h = HParams(hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"],
                          hp.get("ffn", 0), hp["n_layers"], hp.get("vocab", 0),
                          hp.get("rope_theta", 1.0e6), hp.get("rms_eps", 1.0e-6))
        self.m = lib().vvo_model_new(C.byref(self._h), n_rows, max_seq, flags)
        assert self.m, "vvo_model_new failed"
        self._keep = []
        self.flags = flags

    def __del__(self):
        if getattr(self, "m", None):
            lib().vvo_model_free(self.m)
            self.m = None

    def set_layer(self, li: int, tensors: dict) -> None:
        """tensors: name -> (raw uint8 array or None, qtype, ne0, ne1)."""
        lay = Layer()
        for name in self.LAYER_FIELDS:
            spec = tensors.get(name)
            if spec is None or spec[0] is None:
                setattr(lay, name, Tensor(None, 0, 0, 0))
                continue
            raw, qt, ne0, ne1 = spec
            raw = np.ascontiguousarray(raw)
            self._keep.append(raw)
            setattr(lay, name, Tensor(raw.ctypes.data, qt, ne0, ne1))
        assert lib().vvo_model_set_layer(self.m, li, C.byref(lay)) == 0

    def set_output(self, output_norm=None, lm_head=None, tok_embd=None) -> None:
        ts = []
        for spec in (output_norm, lm_head, tok_embd):
            if spec is None:
                ts.append(None)
                continue
            raw, qt, ne0, ne1 = spec
            raw = np.ascontiguousarray(raw)
            self._keep.append(raw)
            ts.append(Tensor(raw.ctypes.data, qt, ne0, ne1))
        args = [C.byref(t) if t is not None else None for t in ts]
        assert lib().vvo_model_set_output(self.m, *args) == 0

    def kv_load(self, row: int, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert lib().vvo_kv_load(self.m, row, layer, _p(k), _p(v), k.shape[0]) == 0

    def kv_read(self, row: int, layer: int, n_pos: int):
        w = self.hp["n_kv_heads"] * self.hp["head_dim"]
        k = np.empty((n_pos, w), np.float32)
        v = np.empty((n_pos, w), np.float32)
        assert lib().vvo_kv_read(self.m, row, layer, _p(k), _p(v), n_pos) == 0
        return k, v

    def set_past_len(self, row: int, n: int) -> None:
        assert lib().vvo_set_past_len(self.m, row, n) == 0

    def past_len(self, row: int) -> int:
        return lib().vvo_past_len(self.m, row)

    def forward(self, rows, x: np.ndarray, pos_start, first_layer=0, n_layers=None,
                output_norm=False, advance=True) -> np.ndarray:
        rows = np.ascontiguousarray(rows, np.int32)
        x = np.ascontiguousarray(x, np.float32)          # [n_sel, n_tok, hidden]
        assert x.ndim == 3 and x.shape[0] == rows.size
        pos = np.ascontiguousarray(pos_start, np.int32)
        if n_layers is None:
            n_layers = self.hp["n_layers"] - first_layer
        y = np.empty_like(x)
        rc = lib().vvo_forward(self.m, rows.size, _p(rows), x.shape[1], _p(x), _p(pos),
                               first_layer, n_layers, int(output_norm), int(advance), _p(y))
        if rc != 0:
            raise ValueError(f"vvo_forward rc={rc}")
        return y

    def lm_head(self, h: np.ndarray, want_logits=False):
        h = np.ascontiguousarray(h, np.float32).reshape(-1, self.hp["hidden"])
        n = h.shape[0]
        am = np.empty(n, np.int32)
        lg = np.empty((n, self.hp["vocab"]), np.float32) if want_logits else None
        assert lib().vvo_lm_head(self.m, n, _p(h), _p(lg) if want_logits else None, _p(am)) == 0
        return (am, lg) if want_logits else am

    def embed(self, tok) -> np.ndarray:
        tok = np.ascontiguousarray(tok, np.int32)
        out = np.empty((tok.size, self.hp["hidden"]), np.float32)
        assert lib().vvo_embed(self.m, tok.size, _p(tok), _p(out)) == 0
        return out
