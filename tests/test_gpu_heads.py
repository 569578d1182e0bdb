"""The per-frame heads around the stack (src/vibevoice_tts.cpp:464-537):
SpeechConnector y = fc2(rms_norm(fc1 x + b1) * norm) + b2 and the EOS
classifier p = sigmoid(fc2(relu(fc1 x + b1)) + b2), through the C ABI on the
GPU, against the CPU oracle (exact mode: dequantized weights x f32
activations).  Tolerance: the north star's 2e-3 max relative error."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import f32_tensor, quant_tensor, rel_err

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _w(rng, rows, cols, qt, std=0.05):
    w = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
    return f32_tensor(w) if qt == O.F32 else quant_tensor(w, qt)


@pytest.mark.parametrize("qt", [O.F32, O.Q8_0])
@pytest.mark.parametrize("batch", [1, 2])
def test_speech_connector(vv, qt, batch):
    rng = np.random.default_rng(91 + batch + qt)
    hp = dict(hidden=896, n_heads=14, n_kv_heads=2, head_dim=64, ffn=512, n_layers=1, vocab=0)
    latent, H = 64, hp["hidden"]
    fc1, fc2 = _w(rng, H, latent, qt), _w(rng, H, H, qt)
    b1 = f32_tensor((rng.standard_normal(H) * 0.02).astype(np.float32))
    b2 = f32_tensor((rng.standard_normal(H) * 0.02).astype(np.float32))
    norm = f32_tensor((1.0 + rng.standard_normal(H) * 0.02).astype(np.float32))
    eng = vv.Engine(hp)
    eng.set_connector(fc1, b1, norm, fc2, b2)
    x = rng.standard_normal((batch, latent)).astype(np.float32)
    got = eng.connector(x)
    ref = O.connector(x, fc1, b1, norm, fc2, b2)
    assert got.shape == (batch, H)
    assert rel_err(got, ref) < TOL, rel_err(got, ref)


@pytest.mark.parametrize("qt", [O.F32, O.Q8_0])
@pytest.mark.parametrize("batch", [1, 2])
def test_eos_classifier(vv, qt, batch):
    rng = np.random.default_rng(77 + batch + qt)
    hp = dict(hidden=896, n_heads=14, n_kv_heads=2, head_dim=64, ffn=512, n_layers=1, vocab=0)
    H = hp["hidden"]
    fc1, fc2 = _w(rng, H, H, qt), _w(rng, 1, H, qt, std=0.2)
    b1 = f32_tensor((rng.standard_normal(H) * 0.02).astype(np.float32))
    b2 = f32_tensor(np.array([0.1], np.float32))
    eng = vv.Engine(hp)
    eng.set_eos(fc1, b1, fc2, b2)
    x = rng.standard_normal((batch, H)).astype(np.float32)
    got = eng.eos(x)
    ref = O.eos(x, fc1, b1, fc2, b2)
    assert got.shape == (batch,)
    assert np.max(np.abs(got - ref)) < 1e-4, (got, ref)


def test_heads_need_weights(vv):
    hp = dict(hidden=896, n_heads=14, n_kv_heads=2, head_dim=64, ffn=512, n_layers=1, vocab=0)
    eng = vv.Engine(hp)
    with pytest.raises(vv.VVQ2Error):
        eng.connector(np.zeros((1, 64), np.float32))
    with pytest.raises(vv.VVQ2Error):
        eng.eos(np.zeros((1, 896), np.float32))
