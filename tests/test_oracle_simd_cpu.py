"""The SIMD Q8_0 x Q8_0 dot of the CPU oracle (flag SIMD, used only by the
timed CPU baseline) against the generic one: the per-block integer sums are
the same, only the float summation order differs, so matvecs and a small
stack agree to float rounding."""
import numpy as np

import vvq2_oracle as O
from fixtures_util import rel_err


def test_simd_isa_reported():
    assert O.simd_isa() in ("avx512vnni", "avx2", "generic")


def test_simd_q8_0_matvec_matches_generic():
    import synth
    rng = np.random.default_rng(64)
    for rows, cols in ((37, 96), (128, 896), (64, 4864)):
        w = synth.q8_0_tensor(rng, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        gen = O.matvec(*w, x, O.ACT_GGML)
        simd = O.matvec(*w, x, O.ACT_GGML | O.SIMD)
        assert rel_err(simd, gen) < 1e-5, (rows, cols, rel_err(simd, gen))


def test_simd_small_stack_matches_generic():
    import synth
    hp = dict(hidden=128, n_heads=4, n_kv_heads=2, head_dim=32, ffn=256, n_layers=2, vocab=512,
              rope_theta=1.0e6, rms_eps=1.0e-6)
    model = synth.model_q8_0(5, hp)
    outs = []
    for flags in (O.GGML_CPU, O.GGML_CPU | O.SIMD):
        m = O.Model(hp, 2, 16, flags)
        for li, t in enumerate(model["layers"]):
            m.set_layer(li, t)
        m.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
        x = np.random.default_rng(9).standard_normal((2, 3, hp["hidden"])).astype(np.float32)
        outs.append(m.forward([0, 1], x, [0, 0], output_norm=True))
    # int8 activation quantization amplifies a last-bit difference only where
    # a value sits on a rounding boundary: allow a few times float noise
    assert rel_err(outs[1], outs[0]) < 1e-3, rel_err(outs[1], outs[0])
