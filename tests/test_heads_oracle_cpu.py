"""CPU oracle of the per-frame heads (src/vibevoice_tts.cpp:464-537) against
a direct float64 numpy statement of the same formulas (F32 weights, so the
oracle's ggml-semantics matvec is plain f32 math).  No GPU."""
import numpy as np

import vvq2_oracle as O
from fixtures_util import f32_tensor


def test_connector_oracle_formula():
    rng = np.random.default_rng(11)
    latent, H = 64, 256
    W1 = (rng.standard_normal((H, latent)) * 0.05).astype(np.float32)
    W2 = (rng.standard_normal((H, H)) * 0.05).astype(np.float32)
    b1 = (rng.standard_normal(H) * 0.02).astype(np.float32)
    b2 = (rng.standard_normal(H) * 0.02).astype(np.float32)
    g = (1.0 + rng.standard_normal(H) * 0.02).astype(np.float32)
    x = rng.standard_normal((2, latent)).astype(np.float32)
    got = O.connector(x, f32_tensor(W1), f32_tensor(b1), f32_tensor(g), f32_tensor(W2), f32_tensor(b2))
    h = x.astype(np.float64) @ W1.T.astype(np.float64) + b1
    h = h / np.sqrt((h * h).mean(axis=1, keepdims=True) + 1e-6) * g
    ref = h @ W2.T.astype(np.float64) + b2
    assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) < 1e-5


def test_eos_oracle_formula():
    rng = np.random.default_rng(12)
    H = 256
    W1 = (rng.standard_normal((H, H)) * 0.05).astype(np.float32)
    W2 = (rng.standard_normal((1, H)) * 0.2).astype(np.float32)
    b1 = (rng.standard_normal(H) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, H)).astype(np.float32)
    got = O.eos(x, f32_tensor(W1), f32_tensor(b1), f32_tensor(W2), f32_tensor(np.array([0.1], np.float32)))
    h = np.maximum(x.astype(np.float64) @ W1.T.astype(np.float64) + b1, 0.0)
    z = (h @ W2.T.astype(np.float64)).ravel() + 0.1
    ref = 1.0 / (1.0 + np.exp(-z))
    assert got.shape == (3,) and np.max(np.abs(got - ref)) < 1e-6
