"""Paged KV cache (vvq2_kv_init_paged): sequences take 64-position pages from
a shared pool as their writes need them and give them back when they are
shortened -- the per-sequence sizing of the reference's ResidentKV
(src/qwen2.cpp:207-246) for many ragged streams (config 3).

Two engines with the same weights, one on an identity-mapped cache and one
on a paged cache whose pool holds only the pages the streams need; ragged
prompts are fed in interleaved 64-token chunks so the streams' pages
interleave in the pool.  Every kernel reads K/V through the block table, so
prefill outputs and greedy tokens must be bit-identical.  Then a stream is
shortened to 0 (its pages return to the pool), refilled with a longer
prompt that takes pages others freed, and decoding continues; a write that
needs more pages than the pool has fails with VVQ2_ERR_OUT_OF_MEMORY and
changes nothing."""
import numpy as np
import pytest

from fixtures_util import C1

pytestmark = pytest.mark.gpu

PAGE = 64


def _pages(n):
    return (n + PAGE - 1) // PAGE


def test_paged_cache_matches_identity_cache(vv):
    import synth
    hp = dict(C1, n_layers=2, vocab=4096)
    model = synth.model_q8_0(20261207, hp)
    engs = [vv.Engine(hp), vv.Engine(hp)]
    for eng in engs:
        for li, t in enumerate(model["layers"]):
            eng.set_layer(li, t)
        eng.set_output(model["output_norm"], model["lm_head"], model["tok_embd"])
    lens = [130, 64, 1, 300, 65, 200]
    n, steps, max_seq = len(lens), 6, 1024
    pool = sum(_pages(l + 2 * steps + 1) for l in lens) + _pages(500) - _pages(300) + 1
    kv_id = engs[0].kv(n, max_seq)
    kv_pg = engs[1].kv(n, max_seq, pool_pages=pool)
    assert kv_pg.free_pages() == pool and kv_id.free_pages() == 0
    rng = np.random.default_rng(9)
    prompts = [rng.standard_normal((l, hp["hidden"])).astype(np.float32) for l in lens]

    def prefill(kv, eng, s, x):
        out = []
        for c0 in range(0, x.shape[0], PAGE):
            out.append(eng.forward(kv, [s], x[None, c0:c0 + PAGE], [c0])[0])
        return np.concatenate(out)

    # interleaved chunks: stream s's pages alternate with the others' in the pool
    outs = [[None] * n for _ in engs]
    for c0 in range(0, max(lens), PAGE):
        for s in range(n):
            if c0 < lens[s]:
                for e, (eng, kv) in enumerate(zip(engs, (kv_id, kv_pg))):
                    y = eng.forward(kv, [s], prompts[s][None, c0:c0 + PAGE], [c0])[0]
                    outs[e][s] = y if outs[e][s] is None else np.concatenate([outs[e][s], y])
    for s in range(n):
        assert np.array_equal(outs[0][s], outs[1][s]), s
    assert kv_pg.free_pages() == pool - sum(_pages(l) for l in lens)

    def decode(seqs, tok, k):
        got = []
        for _ in range(k):
            a = engs[0].decode_step(kv_id, seqs, tok)
            b = engs[1].decode_step(kv_pg, seqs, tok)
            assert np.array_equal(a, b)
            got.append(a)
            tok = a
        return tok

    tok = rng.integers(0, hp["vocab"], size=n).astype(np.int32)
    tok = decode(list(range(n)), tok, steps)                 # many-row step (tensor-core path)
    decode([0, 1], tok[:2], steps)                            # one CFG pair (persistent step)
    # stream 3 gives its pages back and takes a longer prompt
    before = kv_pg.free_pages()
    for kv in (kv_id, kv_pg):
        kv.set_past_len(3, 0)
    assert kv_pg.free_pages() == before + _pages(lens[3] + steps)
    x3 = rng.standard_normal((500, hp["hidden"])).astype(np.float32)
    y3 = [prefill(kv, eng, 3, x3) for eng, kv in zip(engs, (kv_id, kv_pg))]
    assert np.array_equal(y3[0], y3[1])
    decode([2, 3, 4], tok[2:5], steps)
    # a write beyond the pool fails and changes nothing
    free = kv_pg.free_pages()
    past = kv_pg.past_len(5)
    big = rng.standard_normal((1, (free + 2) * PAGE, hp["hidden"])).astype(np.float32)
    with pytest.raises(vv.VVQ2Error) as ei:
        engs[1].forward(kv_pg, [5], big, [past])
    assert ei.value.rc == -5
    assert kv_pg.free_pages() == free and kv_pg.past_len(5) == past
