"""Host-side checks of the random timing-model generators in
vibevoice.cpp_b200/synth.py: every block they emit is a valid GGUF block
whose dequantized values are finite and in the range of N(0, 0.02) weights
(the C4 bench feeds them to the engine).  No GPU."""
import numpy as np

import synth
import vvq2_oracle as O


def _deq(t):
    raw, qt, cols, rows = t
    return np.asarray(O.dequantize(qt, raw, cols * rows)).reshape(rows, cols)


def test_kquant_random_blocks_are_valid():
    rng = np.random.default_rng(3)
    for qt in (synth.Q5_K, synth.Q6_K):
        t = synth.kquant_random_tensor(rng, qt, 8, 1024)
        assert t[0].nbytes == 8 * 1024 // 256 * (176 if qt == synth.Q5_K else 210)
        w = _deq(t)
        assert np.isfinite(w).all()
        assert 0.002 < w.std() < 0.03 and np.abs(w).max() < 0.06


def test_q8_0_random_blocks_are_valid():
    rng = np.random.default_rng(4)
    t = synth.q8_0_random_tensor(rng, 8, 512)
    w = _deq(t)
    assert np.isfinite(w).all() and 0.005 < w.std() < 0.04


def test_layer_c4_fast_types():
    rng = np.random.default_rng(5)
    hp = dict(hidden=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn=512)
    L = synth.layer_c4_fast(rng, hp)
    assert L["attn_q"][1] == synth.Q5_K and L["attn_o"][1] == synth.Q5_K
    assert L["ffn_gate"][1] == synth.Q6_K and L["ffn_down"][1] == synth.Q6_K
    assert (L["attn_q"][2], L["attn_q"][3]) == (256, 256)
    assert (L["ffn_down"][2], L["ffn_down"][3]) == (512, 256)
