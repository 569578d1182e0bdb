"""ctypes binding of libvvq2.so (include/vvq2_capi.h) for tests, bench and
Python callers.  There is no fallback: if the shared library is missing or
no sm_100 device is present, calls raise."""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libvvq2.so"

F32, F16, Q8_0, Q5_K, Q6_K = 0, 1, 8, 13, 14
ADVANCE, OUTPUT_NORM, LAST_ONLY = 1, 2, 4

LAYER_FIELDS = ["attn_norm", "attn_q", "attn_q_bias", "attn_k", "attn_k_bias", "attn_v",
                "attn_v_bias", "attn_o", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"]


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int), ("ne0", C.c_int64), ("ne1", C.c_int64)]


class LayerWeights(C.Structure):
    _fields_ = [(n, Tensor) for n in LAYER_FIELDS]


class HParams(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("intermediate_size", C.c_int), ("n_layers", C.c_int),
                ("vocab_size", C.c_int), ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float)]


class VVQ2Error(RuntimeError):
    def __init__(self, rc: int, msg: str):
        super().__init__(f"vvq2 error {rc}: {msg}")
        self.rc = rc


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} not built (run make -C vibevoice.cpp_b200)")
        L = C.CDLL(str(LIB_PATH))
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "vvq2_init": (I, [P, I, P]),
            "vvq2_free": (None, [P]),
            "vvq2_set_layer": (I, [P, I, P]),
            "vvq2_set_output": (I, [P, P, P, P]),
            "vvq2_kv_init": (I, [P, I, I, P]),
            "vvq2_kv_init_paged": (I, [P, I, I, I, P]),
            "vvq2_kv_free_pages": (I, [P]),
            "vvq2_kv_free": (None, [P]),
            "vvq2_kv_load_prefix": (I, [P, I, I, P, P, I]),
            "vvq2_kv_read": (I, [P, I, I, P, P, I]),
            "vvq2_kv_set_past_len": (I, [P, I, I]),
            "vvq2_kv_past_len": (I, [P, I]),
            "vvq2_forward": (I, [P, P, P, I, I, P, P, I, I, I, P, P]),
            "vvq2_lm_head": (I, [P, I, P, P, P, P]),
            "vvq2_embed": (I, [P, I, P, P, P]),
            "vvq2_decode_step": (I, [P, P, P, I, P, P, P]),
            "vvq2_dequantize": (I, [I, P, I64, P]),
            "vvq2_rope_neox": (I, [P, I, I, I, P, F, P]),
            "vvq2_rms_norm": (I, [P, P, I, I, F, P]),
            "vvq2_backend_selected": (I, []),
            "vvq2_device_count": (I, []),
            "vvq2_version": (C.c_char_p, []),
            "vvq2_last_error": (C.c_char_p, []),
            "vvq2_kernel_launches": (I64, []),
            "vvq2_profile": (I, [P, I]),
            "vvq2_debug_gemm": (I, [I, P, I, I, P, I, P]),
            "vvq2_debug_gemv_mma": (I, [P, I, I, P, I, P]),
            "vvq2_attention_decode_noalloc": (I, [P, P, P, P, I, P, I, I, I, I, I, P, P, P]),
            "vvq2_profile_read": (I, [P, I, P, P, P]),
            "vvq2_mega_trace": (I, [P, P, C.c_int64, P, P]),
            "vvq2_nccl_unique_id": (I, [P]),
            "vvq2_partition": (I, [P, I, I, I, P]),
            "vvq2_set_connector": (I, [P, P, P, P, P, P]),
            "vvq2_connector": (I, [P, P, I, P, P]),
            "vvq2_set_eos": (I, [P, P, P, P, P]),
            "vvq2_eos": (I, [P, P, I, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _chk(rc: int) -> int:
    if rc < 0:
        raise VVQ2Error(rc, lib().vvq2_last_error().decode())
    return rc


def _p(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):          # torch tensor (device or host)
        return a.data_ptr()
    return a.ctypes.data


def launches() -> int:
    return lib().vvq2_kernel_launches()


class Engine:
    """One vvq2_ctx: hparams + device-resident weights."""

    def __init__(self, hp: dict, device: int = 0):
        self.hp = dict(hp)
        h = HParams(hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp.get("ffn", 0),
                    hp["n_layers"], hp.get("vocab", 0), hp.get("rope_theta", 1.0e6),
                    hp.get("rms_eps", 1.0e-6))
        ptr = C.c_void_p()
        _chk(lib().vvq2_init(C.byref(h), device, C.byref(ptr)))
        self.ctx = ptr.value

    def close(self):
        if getattr(self, "ctx", None):
            lib().vvq2_free(self.ctx)
            self.ctx = None

    def __del__(self):
        self.close()

    @staticmethod
    def _tensor(spec) -> Tensor:
        if spec is None or spec[0] is None:
            return Tensor(None, 0, 0, 0)
        raw, qt, ne0, ne1 = spec
        raw = np.ascontiguousarray(raw)
        return Tensor(raw.ctypes.data, qt, ne0, ne1), raw

    def set_layer(self, li: int, tensors: dict) -> None:
        lw = LayerWeights()
        keep = []
        for n in LAYER_FIELDS:
            t = self._tensor(tensors.get(n))
            if isinstance(t, tuple):
                keep.append(t[1])
                t = t[0]
            setattr(lw, n, t)
        _chk(lib().vvq2_set_layer(self.ctx, li, C.byref(lw)))

    def set_output(self, output_norm=None, lm_head=None, tok_embd=None) -> None:
        ts, keep = [], []
        for spec in (output_norm, lm_head, tok_embd):
            t = self._tensor(spec)
            if isinstance(t, tuple):
                keep.append(t[1])
                t = t[0]
            ts.append(t)
        # a tied table: same array object for lm_head and tok_embd -> same pointer
        _chk(lib().vvq2_set_output(self.ctx, *[C.byref(t) if t.data else None for t in ts]))

    def _tensors(self, specs):
        ts, keep = [], []
        for spec in specs:
            t = self._tensor(spec)
            if isinstance(t, tuple):
                keep.append(t[1])
                t = t[0]
            ts.append(t)
        return [C.byref(t) if t.data else None for t in ts], keep

    def set_connector(self, fc1_w, fc1_b, norm_w, fc2_w, fc2_b) -> None:
        """SpeechConnector weights (src/vibevoice_tts.cpp:464-501)."""
        args, keep = self._tensors((fc1_w, fc1_b, norm_w, fc2_w, fc2_b))
        _chk(lib().vvq2_set_connector(self.ctx, *args))

    def connector(self, x, y=None, stream=None):
        """x [batch][latent] -> y [batch][hidden] = fc2(rms_norm(fc1 x + b1) * norm) + b2."""
        if not hasattr(x, "data_ptr"):
            x = np.ascontiguousarray(x, np.float32)
        batch = x.shape[0]
        if y is None:
            y = np.empty((batch, self.hp["hidden"]), np.float32)
        _chk(lib().vvq2_connector(self.ctx, _p(x), batch, _p(y), stream))
        return y

    def set_eos(self, fc1_w, fc1_b, fc2_w, fc2_b) -> None:
        """EOS classifier weights (src/vibevoice_tts.cpp:503-537)."""
        args, keep = self._tensors((fc1_w, fc1_b, fc2_w, fc2_b))
        _chk(lib().vvq2_set_eos(self.ctx, *args))

    def eos(self, x, p=None, stream=None):
        """x [batch][hidden] -> p [batch] = sigmoid(fc2(relu(fc1 x + b1)) + b2)."""
        if not hasattr(x, "data_ptr"):
            x = np.ascontiguousarray(x, np.float32)
        batch = x.shape[0]
        if p is None:
            p = np.empty(batch, np.float32)
        _chk(lib().vvq2_eos(self.ctx, _p(x), batch, _p(p), stream))
        return p

    def profile(self, enable: bool) -> None:
        _chk(lib().vvq2_profile(self.ctx, int(enable)))

    def profile_read(self, kind: int):
        ms, by, n = C.c_double(), C.c_double(), C.c_int64()
        _chk(lib().vvq2_profile_read(self.ctx, kind, C.byref(ms), C.byref(by), C.byref(n)))
        return ms.value, by.value, n.value

    def partition(self, rank: int, world: int, seq_parts: int, nccl_id: bytes) -> None:
        """Attention partition over `world` GPUs (one Engine per process and GPU):
        rank r holds KV-head group r // seq_parts and sequence part r % seq_parts.
        Call on every rank before set_layer / kv()."""
        buf = C.create_string_buffer(bytes(nccl_id), NCCL_ID_BYTES)
        _chk(lib().vvq2_partition(self.ctx, rank, world, seq_parts, C.cast(buf, C.c_void_p)))

    def mega_trace(self) -> np.ndarray:
        """[slots][grid] %globaltimer stamps of the last persistent decode step."""
        g, sl = C.c_int(), C.c_int()
        _chk(lib().vvq2_mega_trace(self.ctx, None, 0, C.byref(g), C.byref(sl)))
        out = np.zeros((sl.value, g.value), np.uint64)
        _chk(lib().vvq2_mega_trace(self.ctx, _p(out), out.size, None, None))
        return out

    def kv(self, n_seqs: int, max_seq: int, pool_pages: int = 0) -> "KV":
        """pool_pages > 0: a paged cache whose sequences share that many pages."""
        return KV(self, n_seqs, max_seq, pool_pages)

    def forward(self, kv: "KV", seqs, x, pos_start, first_layer=0, n_layers=None, flags=ADVANCE,
                y=None, stream=None):
        seqs = np.ascontiguousarray(seqs, np.int32)
        pos = np.ascontiguousarray(pos_start, np.int32)
        if n_layers is None:
            n_layers = self.hp["n_layers"] - first_layer
        if hasattr(x, "data_ptr"):
            n_tok = x.shape[1]
            xp = x
        else:
            x = np.ascontiguousarray(x, np.float32)
            n_tok = x.shape[1]
            xp = x
        if y is None:
            shape = (seqs.size, self.hp["hidden"]) if flags & LAST_ONLY else (seqs.size, n_tok, self.hp["hidden"])
            y = np.empty(shape, np.float32)
        _chk(lib().vvq2_forward(self.ctx, kv.kv, _p(seqs), seqs.size, n_tok, _p(xp), _p(pos),
                                first_layer, n_layers, flags, _p(y), stream))
        return y

    def lm_head(self, h, want_logits=False):
        h = np.ascontiguousarray(h, np.float32).reshape(-1, self.hp["hidden"])
        n = h.shape[0]
        am = np.empty(n, np.int32)
        lg = np.empty((n, self.hp["vocab"]), np.float32) if want_logits else None
        _chk(lib().vvq2_lm_head(self.ctx, n, _p(h), _p(lg), _p(am), None))
        return (am, lg) if want_logits else am

    def embed(self, tok) -> np.ndarray:
        tok = np.ascontiguousarray(tok, np.int32)
        out = np.empty((tok.size, self.hp["hidden"]), np.float32)
        _chk(lib().vvq2_embed(self.ctx, tok.size, _p(tok), _p(out), None))
        return out

    def decode_step(self, kv: "KV", seqs, tokens_in, tokens_out=None, stream=None):
        seqs = np.ascontiguousarray(seqs, np.int32)
        if not hasattr(tokens_in, "data_ptr"):
            tokens_in = np.ascontiguousarray(tokens_in, np.int32)
        if tokens_out is None:
            tokens_out = np.empty(seqs.size, np.int32)
        _chk(lib().vvq2_decode_step(self.ctx, kv.kv, _p(seqs), seqs.size, _p(tokens_in), _p(tokens_out),
                                    stream))
        return tokens_out


class KV:
    """vvq2_kv: f16 paged resident KV cache for n_seqs sequences (pool_pages >
    0: the sequences take pages from a shared pool as they grow)."""

    def __init__(self, eng: Engine, n_seqs: int, max_seq: int, pool_pages: int = 0):
        self.eng = eng
        ptr = C.c_void_p()
        if pool_pages > 0:
            _chk(lib().vvq2_kv_init_paged(eng.ctx, n_seqs, max_seq, pool_pages, C.byref(ptr)))
        else:
            _chk(lib().vvq2_kv_init(eng.ctx, n_seqs, max_seq, C.byref(ptr)))
        self.kv = ptr.value

    def free_pages(self) -> int:
        return lib().vvq2_kv_free_pages(self.kv)

    def close(self):
        if getattr(self, "kv", None):
            lib().vvq2_kv_free(self.kv)
            self.kv = None

    def __del__(self):
        self.close()

    def load_prefix(self, seq: int, layer: int, k, v) -> None:
        """k, v: f32 [n_pos][n_kv*hd], numpy (host) or torch (host or device)."""
        if not hasattr(k, "data_ptr"):
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
        _chk(lib().vvq2_kv_load_prefix(self.kv, seq, layer, _p(k), _p(v), k.shape[0]))

    def read(self, seq: int, layer: int, n_pos: int):
        w = self.eng.hp["n_kv_heads"] * self.eng.hp["head_dim"]
        k = np.empty((n_pos, w), np.float32)
        v = np.empty((n_pos, w), np.float32)
        _chk(lib().vvq2_kv_read(self.kv, seq, layer, _p(k), _p(v), n_pos))
        return k, v

    def set_past_len(self, seq: int, n: int) -> None:
        _chk(lib().vvq2_kv_set_past_len(self.kv, seq, n))

    def past_len(self, seq: int) -> int:
        return _chk(lib().vvq2_kv_past_len(self.kv, seq))


NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (make it on one rank, share it with the others)."""
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    _chk(lib().vvq2_nccl_unique_id(C.cast(buf, C.c_void_p)))
    return buf.raw


def dequantize(qtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw)
    out = np.empty(n, np.float32)
    _chk(lib().vvq2_dequantize(qtype, _p(raw), n, _p(out)))
    return out


def rope_neox(x: np.ndarray, pos: np.ndarray, theta: float) -> np.ndarray:
    """x f32 [n_tok][n_heads][hd], pos int32 [n_tok]."""
    x = np.ascontiguousarray(x, np.float32)
    pos = np.ascontiguousarray(pos, np.int32)
    y = np.empty_like(x)
    _chk(lib().vvq2_rope_neox(_p(x), x.shape[0], x.shape[1], x.shape[2], _p(pos), theta, _p(y)))
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    rows = x.size // x.shape[-1]
    _chk(lib().vvq2_rms_norm(_p(x), _p(w), rows, x.shape[-1], eps, _p(y)))
    return y


def debug_gemm(qtype: int, raw: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """y = x . W^T through the tcgen05 prefill GEMM (test hook)."""
    raw = np.ascontiguousarray(raw)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty((x.shape[0], n), np.float32)
    _chk(lib().vvq2_debug_gemm(qtype, _p(raw), n, k, _p(x), x.shape[0], _p(y)))
    return y


def debug_gemv_mma(raw: np.ndarray, n: int, k: int, x: np.ndarray) -> np.ndarray:
    """y = x . W^T (1-2 rows, Q8_0) through the tensor-core decode GEMV math (test hook)."""
    raw = np.ascontiguousarray(raw)
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty((x.shape[0], n), np.float32)
    _chk(lib().vvq2_debug_gemv_mma(_p(raw), n, k, _p(x), x.shape[0], _p(y)))
    return y
