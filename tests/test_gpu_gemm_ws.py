"""The persistent many-row GEMM (gemm_ws.cu: 256 weight rows x up to 256
token rows per tile, weight blocks dequantized in shared memory, two TMEM
accumulators) -- the prefill path's linears for chunks of more than 256 rows
(src/qwen2.cpp:19-26,274-276,349; the FFN at :33-40).

The plain product is checked against numpy on the same f16-rounded operands
for every weight type, with partial token and weight tiles and with more
tiles than SMs (each CTA then walks several tiles and its producers run
ahead across tile boundaries).  The fused epilogues (QKV + bias + NEOX RoPE +
K/V append, residual, SwiGLU) are checked through whole layers against the
CPU oracle with the kernel forced on at any tile count."""
import os

import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C1, C4, quant_tensor, random_layer, rel_err

pytestmark = pytest.mark.gpu

GPU_MODE = O.KV_F16 | O.Q_F16 | O.ROPE_GGML


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q5_K, O.Q6_K, O.F16, O.F32])
@pytest.mark.parametrize("t,n,k", [(300, 256, 768), (700, 600, 1024), (2048, 2560, 256)])
def test_gemm_ws_vs_numpy(vv, qt, t, n, k):
    rng = np.random.default_rng(t * 13 + n + qt)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw, _, _, _ = quant_tensor(w, qt)
    x = rng.standard_normal((t, k)).astype(np.float32)
    got = vv.debug_gemm(qt, raw, n, k, x)
    wd = O.dequantize(qt, raw, n * k).reshape(n, k)
    ref = f16(x) @ f16(wd).T
    assert rel_err(got, ref) < 1e-5, rel_err(got, ref)


def _engine(vv, hp):
    os.environ["VVQ2_WS_MIN_TILES"] = "1"   # the persistent kernel at any tile count
    try:
        return vv.Engine(hp)
    finally:
        del os.environ["VVQ2_WS_MIN_TILES"]


SHAPES = {
    "c1-hd64-q8_0": (dict(C1, n_layers=1), O.Q8_0, None),
    "c4-hd128-q5k-q6k": (dict(C4, n_layers=1, ffn=2048), O.Q6_K, O.Q5_K),
    "hd32-q8_0": (dict(hidden=512, n_heads=16, n_kv_heads=4, head_dim=32, ffn=1024, n_layers=1, vocab=0,
                       rope_theta=1.0e6, rms_eps=1.0e-6), O.Q8_0, None),
}


@pytest.mark.parametrize("name", list(SHAPES))
def test_gemm_ws_layer_epilogues_vs_oracle(vv, name):
    """2 sequences x 300 prompt tokens after a 40-position prefix through one
    layer whose four GEMMs all run on the persistent kernel, then a decode
    step that reads the K/V rows its QKV epilogue appended."""
    hp, wt, at = SHAPES[name]
    rng = np.random.default_rng(sum(map(ord, name)))
    t = random_layer(rng, hp, wt, attn_type=at)
    eng = _engine(vv, hp)
    eng.set_layer(0, t)
    past, n = 40, 300
    kv = eng.kv(2, past + n + 8)
    ora = O.Model(hp, 2, past + n + 8, GPU_MODE)
    ora.set_layer(0, t)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(2):
        k = rng.standard_normal((past, w)).astype(np.float32)
        v = rng.standard_normal((past, w)).astype(np.float32)
        kv.load_prefix(s, 0, k, v)
        ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, past)
        ora.set_past_len(s, past)
    x = rng.standard_normal((2, n, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [0, 1], x, [past, past])
    ref = ora.forward([0, 1], x, [past, past])
    err = rel_err(got, ref)
    print(f"{name}: prefill rel err {err:.2e}")
    assert err < 5e-3
    x1 = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
    g1 = eng.forward(kv, [0, 1], x1, [past + n, past + n])
    r1 = ora.forward([0, 1], x1, [past + n, past + n])
    assert rel_err(g1, r1) < 5e-3
