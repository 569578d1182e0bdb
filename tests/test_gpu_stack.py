"""Whole-LM decode on the GPU path vs the CPU oracle (config 2: 24-layer
0.5B-shaped Q8_0 stack, tied lm_head, batch 2 CFG, greedy decode from KV
lengths 128 / 1024 / 4096).

Greedy identity is checked free-running: the GPU is fed its OWN previous token
every step, exactly as a caller's decode loop runs, and the oracle follows the
GPU's token sequence, computing its argmax at every step.  A GPU argmax that
differs from the oracle's is only accepted when the two oracle logits are
within float-summation noise of each other (a near-tie); the run reports how
many tokens were identical and the first divergence.  A teacher-forced variant
(the oracle's token fed to both sides) is kept as a diagnostic."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C2, rel_err

pytestmark = pytest.mark.gpu

GPU_MODE = O.KV_F16 | O.Q_F16 | O.ROPE_GGML


def build(seed, hp, n_layers):
    import synth
    m = synth.model_q8_0(seed, dict(hp, n_layers=n_layers))
    return m


def make_pair(vv, hp, model, n_rows, max_seq):
    eng = vv.Engine(hp)
    ora = O.Model(hp, n_rows, max_seq, GPU_MODE)
    for li, t in enumerate(model["layers"]):
        eng.set_layer(li, t)
        ora.set_layer(li, t)
    eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    ora.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    return eng, eng.kv(n_rows, max_seq), ora


def fill_prefix(rng, hp, kv, ora, n_rows, L):
    w = hp["n_kv_heads"] * hp["head_dim"]
    for li in range(hp["n_layers"]):
        for s in range(n_rows):
            k = rng.standard_normal((L, w), dtype=np.float32)
            v = rng.standard_normal((L, w), dtype=np.float32)
            kv.load_prefix(s, li, k, v)
            ora.kv_load(s, li, k, v)
    for s in range(n_rows):
        kv.set_past_len(s, L)
        ora.set_past_len(s, L)


def greedy_compare(eng, kv, ora, hp, tok0, steps, follow="gpu"):
    """Greedy decode of both rows for `steps` steps.  follow="gpu": each side
    is fed the GPU's previous token (the GPU runs free); follow="oracle": the
    oracle's (teacher forcing).  Returns (identical, near_ties, first
    divergence (step, row) or None)."""
    tok = np.array(tok0, np.int32)
    identical, ties, first = 0, 0, None
    for step in range(steps):
        got = eng.decode_step(kv, [0, 1], tok)
        pos = [ora.past_len(0), ora.past_len(1)]
        h = ora.forward([0, 1], ora.embed(tok)[:, None, :], pos, output_norm=True)
        am, lg = ora.lm_head(h[:, 0], want_logits=True)
        for r in range(2):
            if got[r] == am[r]:
                identical += 1
            else:
                gap = abs(lg[r, am[r]] - lg[r, got[r]]) / np.max(np.abs(lg[r]))
                assert gap < 1e-5, (step, r, int(got[r]), int(am[r]), gap)
                ties += 1
                if first is None:
                    first = (step, r)
        tok = (got if follow == "gpu" else am).astype(np.int32)
    return identical, ties, first


def test_small_stack_decode_step_equals_forward(vv):
    """decode_step == embed -> forward(OUTPUT_NORM) -> lm_head."""
    import vvq2
    hp = dict(C2, n_layers=3, vocab=4096)
    model = build(11, hp, 3)
    eng, kv, ora = make_pair(vv, hp, model, 2, 64)
    tok = np.array([5, 4000], np.int32)
    x = eng.embed(tok)
    assert np.array_equal(x, ora.embed(tok))
    h = eng.forward(kv, [0, 1], x[:, None, :], [0, 0], flags=vvq2.OUTPUT_NORM)  # no advance
    am, lg = eng.lm_head(h[:, 0], want_logits=True)
    got = eng.decode_step(kv, [0, 1], tok)
    assert np.array_equal(am, got)
    hr = ora.forward([0, 1], ora.embed(tok)[:, None, :], [0, 0], output_norm=True)
    amr, lgr = ora.lm_head(hr[:, 0], want_logits=True)
    assert rel_err(h, hr) < 2e-3
    assert rel_err(lg, lgr) < 2e-3
    assert kv.past_len(0) == 1 and kv.past_len(1) == 1


@pytest.mark.parametrize("kv_len", [128, 1024, 4096])
def test_c2_greedy_256_steps(vv, kv_len):
    """Free-running: the GPU's own 256-token sequence, checked step by step."""
    hp = dict(C2)
    model = build(20261201, hp, hp["n_layers"])
    steps = 256
    eng, kv, ora = make_pair(vv, hp, model, 2, kv_len + steps + 1)
    rng = np.random.default_rng(kv_len)
    fill_prefix(rng, hp, kv, ora, 2, kv_len)
    tok0 = rng.integers(0, hp["vocab"], size=2).astype(np.int32)
    identical, ties, first = greedy_compare(eng, kv, ora, hp, tok0, steps, follow="gpu")
    print(f"kv {kv_len}: free-running, {identical}/{2 * steps} tokens identical, {ties} near-ties, "
          f"first divergence {first}")
    assert identical + ties == 2 * steps
    assert ties <= 2


def test_c2_greedy_teacher_forced_diagnostic(vv):
    """Diagnostic: the oracle's token fed to both sides (a near-tie cannot
    move the GPU onto another trajectory)."""
    hp = dict(C2)
    model = build(20261201, hp, hp["n_layers"])
    steps, kv_len = 128, 1024
    eng, kv, ora = make_pair(vv, hp, model, 2, kv_len + steps + 1)
    rng = np.random.default_rng(7 * kv_len)
    fill_prefix(rng, hp, kv, ora, 2, kv_len)
    tok0 = rng.integers(0, hp["vocab"], size=2).astype(np.int32)
    identical, ties, first = greedy_compare(eng, kv, ora, hp, tok0, steps, follow="oracle")
    print(f"kv {kv_len}: teacher-forced, {identical}/{2 * steps} identical, {ties} near-ties, first {first}")
    assert identical + ties == 2 * steps
    assert ties <= 2
