"""Many-stream decode (config 3's shape): one decode step for dozens of
independent sequences with ragged KV lengths, through the tensor-core path
(split-K decode attention per row, lm_head GEMM with an argmax epilogue),
against the CPU oracle."""
import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C2, rel_err

pytestmark = pytest.mark.gpu

GPU_MODE = O.KV_F16 | O.Q_F16 | O.ROPE_GGML


def setup(vv, n_streams, seed, lo=64, hi=300):
    import synth
    hp = dict(C2, n_layers=3, vocab=4096)
    model = synth.model_q8_0(seed, hp)
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n_streams)
    max_seq = int(lens.max()) + 16
    eng = vv.Engine(hp)
    ora = O.Model(hp, n_streams, max_seq, GPU_MODE)
    for li, t in enumerate(model["layers"]):
        eng.set_layer(li, t)
        ora.set_layer(li, t)
    eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    ora.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    kv = eng.kv(n_streams, max_seq)
    w = hp["n_kv_heads"] * hp["head_dim"]
    for s in range(n_streams):
        for li in range(hp["n_layers"]):
            k = rng.standard_normal((int(lens[s]), w), dtype=np.float32)
            v = rng.standard_normal((int(lens[s]), w), dtype=np.float32)
            kv.load_prefix(s, li, k, v)
            ora.kv_load(s, li, k, v)
        kv.set_past_len(s, int(lens[s]))
        ora.set_past_len(s, int(lens[s]))
    return hp, eng, kv, ora, rng


def test_batched_forward_ragged_vs_oracle(vv):
    """40 rows of one token each, KV lengths 64..300: hidden states."""
    n = 40
    hp, eng, kv, ora, rng = setup(vv, n, 31)
    seqs = list(range(n))
    pos = [ora.past_len(s) for s in seqs]
    x = rng.standard_normal((n, 1, hp["hidden"])).astype(np.float32)
    got = eng.forward(kv, seqs, x, pos)
    ref = ora.forward(seqs, x, pos)
    err = rel_err(got, ref)
    print("batched forward rel err", err)
    assert err < 5e-3


def test_batched_decode_steps_vs_oracle(vv):
    """48 streams, 4 greedy steps through vvq2_decode_step (oracle tokens fed
    to both).  The lm_head GEMM runs on f16 operands, so an argmax may differ
    from the exact oracle only where the two logits are within f16 rounding
    (gap < 2e-3 of the row's max |logit|)."""
    n = 48
    hp, eng, kv, ora, rng = setup(vv, n, 47)
    seqs = list(range(n))
    tok = rng.integers(0, hp["vocab"], size=n).astype(np.int32)
    identical = total = 0
    for step in range(4):
        got = eng.decode_step(kv, seqs, tok)
        pos = [ora.past_len(s) for s in seqs]
        h = ora.forward(seqs, ora.embed(tok)[:, None, :], pos, output_norm=True)
        am, lg = ora.lm_head(h[:, 0], want_logits=True)
        for r in range(n):
            total += 1
            if got[r] == am[r]:
                identical += 1
            else:
                gap = abs(lg[r, am[r]] - lg[r, got[r]]) / np.max(np.abs(lg[r]))
                assert gap < 2e-3, (step, r, int(got[r]), int(am[r]), gap)
        tok = am.astype(np.int32)
    print(f"batched decode: {identical}/{total} argmax identical")
    assert identical >= 0.9 * total
    assert all(kv.past_len(s) == ora.past_len(s) for s in seqs)
