"""Parity of the sm_100a path (through the C ABI) against the CPU oracle and
the reference's golden vectors.  Mirrors vibevoice.cpp's tests/test_rope.cpp,
tests/test_qwen2_block.cpp and tests/test_qwen2_resident.cpp, and adds the
quantized / batch-2 / f16-KV cases no reference test covers.

Tolerance (the north star's): max |gpu - oracle| / max |oracle| <= 2e-3 on
layer outputs, fp32 accumulation.  The GPU path multiplies exactly dequantized
weights by f32 activations, so it is compared with the oracle's exact mode
(same f16 K/V and Q rounding, same ggml CPU RoPE recurrence); the reference
CPU backend's int8-activation numerics are checked separately, loosely."""

# what the GPU path computes: exact dequant x f32 activations, f16 K/V and Q,
# ggml CPU rope cache, f32 flash-attention accumulation
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C1, cos_sim, golden_layer, random_layer, rel_err

pytestmark = pytest.mark.gpu
GPU_MODE = O.KV_F16 | O.Q_F16 | O.ROPE_GGML
TOL = 2e-3


@pytest.mark.parametrize("name,qt", [("q8_0", O.Q8_0), ("q5_K", O.Q5_K), ("q6_K", O.Q6_K)])
def test_dequant_bit_exact_vs_gguf_py(vv, golden, name, qt):
    z = golden("dequant.npz")
    got = vv.dequantize(qt, z[f"{name}_blocks"], z[f"{name}_deq"].size)
    assert np.array_equal(got.view(np.uint32), z[f"{name}_deq"].view(np.uint32))


@pytest.mark.parametrize("case", ["d64", "d128"])
def test_rope_vs_reference_generator(vv, golden, case):
    z = golden("rope.npz")
    x, pos, y = z[f"{case}_x"], z[f"{case}_pos"], z[f"{case}_y"]
    got = vv.rope_neox(x, pos, 1.0e6)
    ora = np.stack([O.rope_neox(x[t], int(pos[t]), 1.0e6, O.ROPE_GGML) for t in range(x.shape[0])])
    assert np.max(np.abs(got - ora)) < 2e-6          # same f32 recurrence as ggml CPU
    tol = 5e-5 if case == "d64" else 2e-2             # tests/test_rope.cpp:97 at pos < 128
    assert np.max(np.abs(got - y)) < tol


def test_rms_norm_vs_oracle(vv):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 896)).astype(np.float32) * 3
    w = (1 + 0.02 * rng.standard_normal(896)).astype(np.float32)
    got = vv.rms_norm(x, w, 1e-6)
    ref = np.stack([O.rms_norm(x[i], w, 1e-6) for i in range(5)])
    assert rel_err(got, ref) < 1e-6


def _pair(vv, hp, layers, n_rows, max_seq, flags):
    eng = vv.Engine(hp)
    ora = O.Model(hp, n_rows, max_seq, flags)
    for li, t in enumerate(layers):
        eng.set_layer(li, t)
        ora.set_layer(li, t)
    kv = eng.kv(n_rows, max_seq)
    return eng, kv, ora


def test_qwen2_layer_f32_vs_hf_golden(vv, golden):
    """tests/test_qwen2_block.cpp's fixture through the GPU path (64 tokens,
    resident chunks).  K/V are stored f16, so the bound is the reference's
    flash-attention tolerance; against the oracle in the same numerics it is tight."""
    hp, t, x, y, pos = golden_layer(golden("qwen2_layer0.npz"))
    eng, kv, ora = _pair(vv, hp, [t], 1, 80, GPU_MODE)
    # 8-token resident chunks keep this on the exact (GEMV) path
    got = np.concatenate([eng.forward(kv, [0], x[:, i:i + 8], [i]) for i in range(0, x.shape[1], 8)], axis=1)
    ref = ora.forward([0], x, [0])
    assert rel_err(got, ref) < 1e-4
    assert np.max(np.abs(got - y)) < 1e-3
    assert cos_sim(got, y) >= 0.99999
    assert kv.past_len(0) == x.shape[1]


@pytest.mark.parametrize("kv_len", [512, 64, 1])
def test_c1_decode_layer_q8_0(vv, kv_len):
    """Config 1: 0.5B-shaped layer, Q8_0, batch 2 (CFG pair), decode 1 token
    against an f16 KV cache filled from N(0,1)."""
    rng = np.random.default_rng(20261201)
    hp = dict(C1)
    t = random_layer(rng, hp, O.Q8_0)
    eng, kv, ora = _pair(vv, hp, [t], 2, kv_len + 8, GPU_MODE)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(2):
        k = rng.standard_normal((kv_len - 1, w)).astype(np.float32) if kv_len > 1 else np.zeros((0, w), np.float32)
        v = rng.standard_normal(k.shape).astype(np.float32)
        if kv_len > 1:
            kv.load_prefix(s, 0, k, v)
            ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, kv_len - 1)
        ora.set_past_len(s, kv_len - 1)
    x = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [0, 1], x, [kv_len - 1, kv_len - 1])
    ref = ora.forward([0, 1], x, [kv_len - 1, kv_len - 1])
    assert rel_err(got, ref) < TOL, rel_err(got, ref)
    # the appended K/V row matches the oracle's (f16, allow 1 ulp flips)
    for s in range(2):
        kg, vg = kv.read(s, 0, kv_len)
        ko, vo = ora.kv_read(s, 0, kv_len)
        assert np.allclose(kg, ko, rtol=2e-3, atol=1e-3) and np.allclose(vg, vo, rtol=2e-3, atol=1e-3)


def test_c1_vs_ggml_cpu_fa_numerics(vv):
    """Against the reference CPU backend's own FA numerics (f16 V accumulator):
    the difference is the reference's rounding, bounded loosely."""
    rng = np.random.default_rng(5)
    hp = dict(C1)
    t = random_layer(rng, hp, O.Q8_0)
    eng, kv, ora = _pair(vv, hp, [t], 2, 520, O.GGML_CPU)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(2):
        k = rng.standard_normal((511, w)).astype(np.float32)
        v = rng.standard_normal((511, w)).astype(np.float32)
        kv.load_prefix(s, 0, k, v)
        ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, 511)
        ora.set_past_len(s, 511)
    x = rng.standard_normal((2, 1, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [0, 1], x, [511, 511])
    ref = ora.forward([0, 1], x, [511, 511])
    assert rel_err(got, ref) < 1e-2


@pytest.mark.parametrize("n_chunks", [2, 4])
def test_resident_chunking_matches_single_shot(vv, golden, n_chunks):
    """tests/test_qwen2_resident.cpp paths B/C/D on the GPU path."""
    hp, t, x, y, pos = golden_layer(golden("qwen2_layer0.npz"))
    eng = vv.Engine(hp)
    eng.set_layer(0, t)
    kv1 = eng.kv(1, 80)
    one = eng.forward(kv1, [0], x, [0])   # 64 rows: tensor-core path; chunks below too
    kv2 = eng.kv(1, 80)
    seq = x.shape[1]
    b = [seq * c // n_chunks for c in range(n_chunks + 1)]
    parts = [eng.forward(kv2, [0], x[:, lo:hi], [lo]) for lo, hi in zip(b[:-1], b[1:])]
    assert np.max(np.abs(np.concatenate(parts, axis=1) - one)) < 1e-5


def test_deep_chain_vs_oracle(vv, golden):
    """Path E: the fixture layer chained 28 deep (errors compounding)."""
    hp, t, x, y, pos = golden_layer(golden("qwen2_layer0.npz"))
    hp = dict(hp, n_layers=28)
    eng, kv, ora = _pair(vv, hp, [t] * 28, 1, 80, GPU_MODE)
    got = eng.forward(kv, [0], x[:, :16], [0])
    ref = ora.forward([0], x[:, :16], [0])
    assert rel_err(got, ref) < 1e-3


def test_kquant_layer_c4_shape(vv):
    """Config 4 shapes: hidden 1536, 12/2 heads, hd 128, Q5_K attention, Q6_K FFN."""
    rng = np.random.default_rng(44)
    hp = dict(hidden=1536, n_heads=12, n_kv_heads=2, head_dim=128, ffn=8960, n_layers=1, vocab=0,
              rope_theta=1.0e6, rms_eps=1.0e-6)
    t = random_layer(rng, hp, attn_type=O.Q5_K, ffn_type=O.Q6_K)
    eng, kv, ora = _pair(vv, hp, [t], 2, 300, GPU_MODE)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(2):
        k = rng.standard_normal((257, w)).astype(np.float32)
        v = rng.standard_normal((257, w)).astype(np.float32)
        kv.load_prefix(s, 0, k, v)
        ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, 257)
        ora.set_past_len(s, 257)
    x = rng.standard_normal((2, 3, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [0, 1], x, [257, 257])
    ref = ora.forward([0, 1], x, [257, 257])
    assert rel_err(got, ref) < TOL, rel_err(got, ref)


@pytest.mark.parametrize("rows,kv_len", [(1, 6001), (2, 3100), (2, 130)])
def test_long_context_decode_hd128(vv, rows, kv_len):
    """Decode of one token against long contexts with head_dim 128 and a GQA
    group of 7: many attention splits (the separate log-sum-exp merge), a
    partial last page, one and two rows."""
    rng = np.random.default_rng(7000 + kv_len)
    hp = dict(hidden=1792, n_heads=14, n_kv_heads=2, head_dim=128, ffn=1024, n_layers=1, vocab=0,
              rope_theta=1.0e6, rms_eps=1.0e-6)
    t = random_layer(rng, hp, O.Q8_0)
    eng, kv, ora = _pair(vv, hp, [t], rows, kv_len + 8, GPU_MODE)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(rows):
        k = rng.standard_normal((kv_len - 1, w)).astype(np.float32)
        v = rng.standard_normal((kv_len - 1, w)).astype(np.float32)
        kv.load_prefix(s, 0, k, v)
        ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, kv_len - 1)
        ora.set_past_len(s, kv_len - 1)
    x = rng.standard_normal((rows, 1, hp["hidden"])).astype(np.float32)
    seqs = list(range(rows))
    got = eng.forward(kv, seqs, x, [kv_len - 1] * rows)
    ref = ora.forward(seqs, x, [kv_len - 1] * rows)
    assert rel_err(got, ref) < TOL, rel_err(got, ref)


@pytest.mark.parametrize("rows", [1, 2])
def test_kquant_decode_c4_shape(vv, rows):
    """Config 4 decode: one token per row (the streaming GEMV for one or two
    rows) over Q5_K attention and Q6_K FFN weights, hd 128, KV 300."""
    rng = np.random.default_rng(4400 + rows)
    hp = dict(hidden=1536, n_heads=12, n_kv_heads=2, head_dim=128, ffn=8960, n_layers=1, vocab=0,
              rope_theta=1.0e6, rms_eps=1.0e-6)
    t = random_layer(rng, hp, attn_type=O.Q5_K, ffn_type=O.Q6_K)
    eng, kv, ora = _pair(vv, hp, [t], rows, 320, GPU_MODE)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(rows):
        k = rng.standard_normal((299, w)).astype(np.float32)
        v = rng.standard_normal((299, w)).astype(np.float32)
        kv.load_prefix(s, 0, k, v)
        ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, 299)
        ora.set_past_len(s, 299)
    x = rng.standard_normal((rows, 1, hp["hidden"])).astype(np.float32)
    seqs = list(range(rows))
    got = eng.forward(kv, seqs, x, [299] * rows)
    ref = ora.forward(seqs, x, [299] * rows)
    assert rel_err(got, ref) < TOL, rel_err(got, ref)


def test_ragged_sequences_and_last_only(vv):
    """Two sequences at different past lengths in one call; LAST_ONLY output."""
    import vvq2
    rng = np.random.default_rng(9)
    hp = dict(C1)
    t = random_layer(rng, hp, O.Q8_0)
    eng, kv, ora = _pair(vv, hp, [t], 3, 700, GPU_MODE)
    w = hp["n_kv_heads"] * hp["head_dim"]
    lens = [100, 0, 640]
    for s, L in enumerate(lens):
        if L:
            k = rng.standard_normal((L, w)).astype(np.float32)
            v = rng.standard_normal((L, w)).astype(np.float32)
            kv.load_prefix(s, 0, k, v)
            ora.kv_load(s, 0, k, v)
        kv.set_past_len(s, L)
        ora.set_past_len(s, L)
    x = rng.standard_normal((3, 2, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, [2, 0, 1], x, [640, 100, 0], flags=vvq2.ADVANCE | vvq2.LAST_ONLY)
    ref = ora.forward([2, 0, 1], x, [640, 100, 0])[:, -1]
    assert rel_err(got, ref) < TOL
    assert [kv.past_len(s) for s in range(3)] == [102, 2, 642]


def test_kv_overflow_is_an_error(vv):
    import vvq2
    rng = np.random.default_rng(1)
    hp = dict(C1)
    eng = vv.Engine(hp)
    eng.set_layer(0, random_layer(rng, hp, O.Q8_0))
    kv = eng.kv(1, 4)
    kv.set_past_len(0, 3)
    with pytest.raises(vvq2.VVQ2Error) as e:
        eng.forward(kv, [0], np.zeros((1, 2, hp["hidden"]), np.float32), [3])
    assert e.value.rc == -2
    assert kv.past_len(0) == 3
