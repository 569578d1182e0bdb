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
