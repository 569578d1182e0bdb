"""Tensor-core (tcgen05) prefill path: the dequant GEMM against numpy on the
same f16-rounded operands, and whole layers with many token rows against the
CPU oracle (chunked prefill, the shape of the ASR / voice-clone prompts)."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C1, golden_layer, quant_tensor, random_layer, rel_err

pytestmark = pytest.mark.gpu

GPU_MODE = O.KV_F16 | O.Q_F16 | O.ROPE_GGML


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q5_K, O.Q6_K, O.F16, O.F32])
@pytest.mark.parametrize("t,n,k", [(1, 128, 256), (37, 200, 512), (300, 256, 768)])
def test_gemm_tc_vs_numpy(vv, qt, t, n, k):
    rng = np.random.default_rng(t * 7 + n)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw, _, _, _ = quant_tensor(w, qt)
    x = rng.standard_normal((t, k)).astype(np.float32)
    got = vv.debug_gemm(qt, raw, n, k, x)
    wd = O.dequantize(qt, raw, n * k).reshape(n, k)
    ref = f16(x) @ f16(wd).T
    assert rel_err(got, ref) < 1e-5, rel_err(got, ref)


def test_prefill_layer_vs_oracle_c1_shape(vv):
    """200 prompt tokens x 2 sequences through one 0.5B-shaped Q8_0 layer."""
    rng = np.random.default_rng(11)
    hp = dict(C1)
    t = random_layer(rng, hp, O.Q8_0)
    eng = vv.Engine(hp)
    eng.set_layer(0, t)
    kv = eng.kv(2, 256)
    ora = O.Model(hp, 2, 256, GPU_MODE)
    ora.set_layer(0, t)
    x = rng.standard_normal((2, 200, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [0, 1], x, [0, 0])
    ref = ora.forward([0, 1], x, [0, 0])
    err = rel_err(got, ref)
    print("prefill rel err", err)
    assert err < 5e-3
    # the cache it left behind serves a decode step that matches too
    x1 = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
    g1 = eng.forward(kv, [0, 1], x1, [200, 200])
    r1 = ora.forward([0, 1], x1, [200, 200])
    assert rel_err(g1, r1) < 5e-3


def test_prefill_golden_layer(vv, golden):
    """The reference's HF fixture (64 tokens) through the tensor-core path:
    f16 weights and activations bound the error at the FA-path level."""
    hp, t, x, y, pos = golden_layer(golden("qwen2_layer0.npz"))
    eng = vv.Engine(hp)
    eng.set_layer(0, t)
    kv = eng.kv(1, 80)
    got = eng.forward(kv, [0], x, [0])
    assert np.max(np.abs(got - y)) < 5e-3


@pytest.mark.parametrize("hd,std", [(64, 0.02), (64, 0.08), (128, 0.02), (128, 0.08)])
def test_prefill_flash_attention_vs_oracle(vv, hd, std):
    """Chunked prefill on the tcgen05 flash-attention path: 2 sequences with a
    100-position N(0,1) KV prefix, then 650 prompt tokens each (three chunks:
    later chunks attend to earlier ones, the last q tile is partial).  A
    larger weight scale gives sharp attention rows (scores of several units),
    which exercises the running-max rescale."""
    from fixtures_util import C4
    hp = dict(C1, n_layers=1) if hd == 64 else dict(C4, n_layers=1, ffn=2048)
    rng = np.random.default_rng(1000 + hd + int(std * 100))
    t = random_layer(rng, hp, O.Q8_0, std=std)
    eng = vv.Engine(hp)
    eng.set_layer(0, t)
    past, n = 100, 650
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
    print(f"hd {hd} std {std}: prefill rel err {err:.2e}")
    assert err < 5e-3
    # the K/V rows it appended serve the next decode step
    x1 = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
    g1 = eng.forward(kv, [0, 1], x1, [past + n, past + n])
    r1 = ora.forward([0, 1], x1, [past + n, past + n])
    assert rel_err(g1, r1) < 5e-3
