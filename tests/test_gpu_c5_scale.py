"""Config-5 scale: one 7B-shaped layer (hidden 3584, 28 q / 4 KV heads,
head_dim 128) over a 16,384-token causal prompt in ONE tensor-core chunk --
the prompt the bench's prefill figure times (src/vibevoice_asr.cpp:554-652
runs the ASR prompt through the same layer).

The layer's O-projection is the identity and its FFN is zero, so the layer
output minus its input is exactly the causal attention output.  On a sample
of query rows (the first and last of the prompt, page and chunk boundaries,
random rows) it is checked, for every head, against softmax(q k^T / sqrt(hd))
v evaluated in f64 over the keys the GPU stored in its cache, with q
recomputed exactly from the input (RMSNorm, Q8_0 projection + bias, NEOX RoPE
with ggml's theta recurrence, rounded to f16 as ggml's flash attention does).
The stored K/V rows at the sampled positions are checked against the same
exact projections.  Tolerance: the tensor-core prefill path's bound, 5e-3 of
the max |value| (f16 activations and f16-rounded dequantized weights, f32
accumulation)."""
import os

import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import rel_err

pytestmark = pytest.mark.gpu

HP = dict(hidden=3584, n_heads=28, n_kv_heads=4, head_dim=128, ffn=18944, n_layers=1, vocab=0,
          rope_theta=1.0e6, rms_eps=1.0e-6)
T = 16384
TOL = 5e-3


def _q8_zero(rows, cols):
    return (np.zeros(rows * (cols // 32) * 34, np.uint8), O.Q8_0, cols, rows)


def _f16_eye(n):
    a = np.eye(n, dtype=np.float16)
    return (a.view(np.uint8).reshape(-1), 1, n, n)   # ggml type 1 = F16


def test_c5_16k_prefill_attention_sampled(vv):
    import synth
    H, nq, nkv, hd, F = HP["hidden"], HP["n_heads"], HP["n_kv_heads"], HP["head_dim"], HP["ffn"]
    G = nq // nkv
    rng = np.random.default_rng(16384)
    lay = synth.layer_q8_0(rng, dict(HP, ffn=32))   # attention weights; FFN replaced below
    lay["attn_o"] = _f16_eye(H)
    lay["ffn_gate"] = _q8_zero(F, H)
    lay["ffn_up"] = _q8_zero(F, H)
    lay["ffn_down"] = _q8_zero(H, F)
    os.environ["VVQ2_PREFILL_ROWS"] = str(T)   # the whole prompt in one chunk
    try:
        eng = vv.Engine(HP)
    finally:
        del os.environ["VVQ2_PREFILL_ROWS"]
    eng.set_layer(0, lay)
    kv = eng.kv(1, T + 64)
    x = rng.standard_normal((1, T, H), dtype=np.float32)
    y = eng.forward(kv, [0], x, [0])
    att = (y - x)[0]                     # [T][nq * hd]
    k_gpu, v_gpu = kv.read(0, 0, T)      # [T][nkv * hd], f16 values
    k_gpu = k_gpu.reshape(T, nkv, hd).astype(np.float64)
    v_gpu = v_gpu.reshape(T, nkv, hd).astype(np.float64)

    norm = np.frombuffer(lay["attn_norm"][0].tobytes(), np.float32)
    bias = {n: np.frombuffer(lay[f"attn_{n}_bias"][0].tobytes(), np.float32) for n in "qkv"}

    def proj(name, r):
        xn = O.rms_norm(x[0, r], norm, HP["rms_eps"])
        return O.matvec(*lay[f"attn_{name}"], xn, 0) + bias[name]

    rows = sorted(set([0, 1, 63, 64, 65, 4095, 4096, 8191, 12287, T - 2, T - 1] +
                      rng.integers(0, T, size=9).tolist()))
    worst_att = worst_kv = 0.0
    for r in rows:
        q = O.rope_neox(proj("q", r).reshape(nq, hd), r, HP["rope_theta"], O.ROPE_GGML)
        q = q.astype(np.float16).astype(np.float64)
        k_ex = O.rope_neox(proj("k", r).reshape(nkv, hd), r, HP["rope_theta"], O.ROPE_GGML)
        v_ex = proj("v", r).reshape(nkv, hd)
        worst_kv = max(worst_kv, rel_err(k_gpu[r], k_ex), rel_err(v_gpu[r], v_ex))
        ref = np.empty((nq, hd))
        for h in range(nq):
            kh, vh = k_gpu[: r + 1, h // G], v_gpu[: r + 1, h // G]
            s = kh @ q[h] / np.sqrt(hd)
            p = np.exp(s - s.max())
            ref[h] = (p / p.sum()) @ vh
        e = rel_err(att[r].reshape(nq, hd), ref)
        worst_att = max(worst_att, e)
        assert e < TOL, (r, e)
    print(f"16k prefill: {len(rows)} sampled rows x {nq} heads, attention max rel err {worst_att:.2e}, "
          f"stored K/V vs exact projection {worst_kv:.2e}")
    assert worst_kv < TOL
