"""How far the reference's own arithmetic sits from the exact math, on the
config-1 attention layer (batch 2, decode 1 token against 511 keys), measured
with the CPU oracle alone.

ggml's CPU backend rounds every activation row to int8 blocks before each
matrix product (vec_dot_type Q8_0 for Q8_0 weights) and accumulates flash
attention's V in f16.  The layer output in that arithmetic (oracle mode
GGML_CPU) differs from the exact math (f32 activations, f32 attention; the
mode the GPU path computes and is gated against at 2e-3) by about 3e-3 of
the output's max -- more than the 2e-3 gate itself.  So no implementation of
the exact layer can sit within 2e-3 of ggml's CPU output on these inputs; the
GPU path is held to 2e-3 against the exact mode and to this noise level
(1e-2) against the ggml mode (tests/test_gpu_parity.py).  The int8 part of
that noise is also what makes ggml's own SIMD and generic kernels disagree
after a few layers: a last-bit difference flips one int8 rounding, and the
next RMSNorm and re-quantization amplify it."""
import numpy as np

import vvq2_oracle as O
from fixtures_util import C1, random_layer, rel_err

EXACT = O.KV_F16 | O.Q_F16 | O.ROPE_GGML


def _layer_out(t, hp, flags, k, v, x):
    m = O.Model(hp, 2, 520, flags)
    m.set_layer(0, t)
    for s in range(2):
        m.kv_load(s, 0, k[s], v[s])
        m.set_past_len(s, 511)
    return m.forward([0, 1], x, [511, 511])


def test_ggml_cpu_numerics_vs_exact_on_c1():
    rng = np.random.default_rng(5)
    hp = dict(C1)
    w = hp["n_kv_heads"] * hp["head_dim"]
    worst = []
    for trial in range(3):
        t = random_layer(rng, hp, O.Q8_0)
        k = rng.standard_normal((2, 511, w)).astype(np.float32)
        v = rng.standard_normal((2, 511, w)).astype(np.float32)
        x = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
        exact = _layer_out(t, hp, EXACT, k, v, x)
        ggml = _layer_out(t, hp, O.GGML_CPU, k, v, x)
        ggml_int8_only = _layer_out(t, hp, O.GGML_CPU & ~O.FA_F16ACC, k, v, x)
        worst.append((rel_err(ggml, exact), rel_err(ggml_int8_only, exact)))
    print("C1 layer, ggml CPU arithmetic vs exact math (rel err: all ggml numerics, int8 activations only):",
          [(f"{a:.1e}", f"{b:.1e}") for a, b in worst])
    # the reference's own rounding noise is of the order of the 2e-3 gate
    assert all(1e-4 < a < 1e-2 for a, _ in worst)
