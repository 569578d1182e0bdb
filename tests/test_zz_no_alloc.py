"""The allocation-free decode attention entry point
(vvq2_attention_decode_noalloc), for callers that cannot allocate device
memory themselves -- e.g. an engine whose memory pool owns the whole GPU, or a
real-time thread that must stay out of the driver's allocator.  Its scratch
lives in a fixed device array inside the library.

Checked against the existing entry point: a layer whose O-projection is the
identity and whose FFN is zero makes vvq2_forward's output minus its input
exactly the attention output; the allocation-free call, given the same Q and
the K/V pages that forward left behind, must match it within the tolerance of
the other parity tests, on two calls in a row (different lengths, so stale
scratch from the first call would show in the second).

A second test covers each kernel path the entry point can take -- one split,
the in-kernel merge by the last split (2-4 splits), the separate merge kernel
(more splits) -- at head_dim 32, 64 and 128 with a shuffled block table,
against a direct evaluation of the attention formula, and reads the error
word back through `err_out`: 0 on valid calls, 5 when a row is longer than
`max_kv` (its keys are then clamped, never read past the grid or the
block-table row)."""
import ctypes as C

import numpy as np
import pytest

import vvq2_oracle as O
from fixtures_util import C1, f32_tensor, random_layer, rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-3


def test_noalloc_attention_matches_forward(vv):
    import torch

    rng = np.random.default_rng(4242)
    hp = dict(C1)
    H, nq, nkv, hd, F = hp["hidden"], hp["n_heads"], hp["n_kv_heads"], hp["head_dim"], hp["ffn"]
    lay = random_layer(rng, hp, O.Q8_0)
    lay["attn_o"] = f32_tensor(np.eye(H, dtype=np.float32))
    lay["ffn_gate"] = f32_tensor(np.zeros((F, H), np.float32))
    lay["ffn_up"] = f32_tensor(np.zeros((F, H), np.float32))
    lay["ffn_down"] = f32_tensor(np.zeros((H, F), np.float32))
    eng = vv.Engine(hp)
    eng.set_layer(0, lay)
    L, max_seq = 300, 320
    kv = eng.kv(2, max_seq)
    w = nkv * hd
    for s in range(2):
        kv.load_prefix(s, 0, rng.standard_normal((L, w), dtype=np.float32),
                       rng.standard_normal((L, w), dtype=np.float32))
        kv.set_past_len(s, L)

    def q_of(x, pos):
        norm = np.frombuffer(lay["attn_norm"][0].tobytes(), np.float32)
        bias = np.frombuffer(lay["attn_q_bias"][0].tobytes(), np.float32)
        qs = []
        for r in range(2):
            xn = O.rms_norm(x[r, 0], norm, hp["rms_eps"])
            q = O.matvec(*lay["attn_q"], xn, 0) + bias
            qs.append(O.rope_neox(q.reshape(nq, hd), pos, hp["rope_theta"], O.ROPE_GGML).reshape(-1))
        return np.stack(qs).astype(np.float32)

    steps = []
    for pos in (L, L + 1):                       # two decode steps through the existing entry point
        x = rng.standard_normal((2, 1, H), dtype=np.float32)
        y = eng.forward(kv, [0, 1], x, [pos, pos])
        steps.append((pos, q_of(x, pos), (y - x)[:, 0]))

    # the K/V pages the forward calls wrote, as the caller's own device buffers
    max_pages = (max_seq + 63) // 64
    kp = np.zeros((2, max_pages, nkv, 64, hd), np.float16)
    vp = np.zeros_like(kp)
    n = L + 2
    for s in range(2):
        k, v = kv.read(s, 0, n)
        k = k.reshape(n, nkv, hd)
        v = v.reshape(n, nkv, hd)
        for j in range(n):
            kp[s, j // 64, :, j % 64] = k[j]
            vp[s, j // 64, :, j % 64] = v[j]
    dev = torch.device("cuda:0")
    k_d = torch.from_numpy(kp).to(dev)
    v_d = torch.from_numpy(vp).to(dev)
    bt = torch.arange(2 * max_pages, dtype=torch.int32, device=dev).reshape(2, max_pages)
    lib = vv.lib()
    for pos, q, ref in steps:                    # two allocation-free calls in a row
        meta = torch.tensor([[0, pos, pos, pos + 1], [1, pos, pos, pos + 1]], dtype=torch.int32, device=dev)
        q_d = torch.from_numpy(q).to(dev)
        out = torch.zeros((2, nq * hd), dtype=torch.float32, device=dev)
        err = torch.full((1,), -1, dtype=torch.int32, device=dev)
        rc = lib.vvq2_attention_decode_noalloc(q_d.data_ptr(), k_d.data_ptr(), v_d.data_ptr(), bt.data_ptr(),
                                               max_pages, meta.data_ptr(), 2, pos + 1, nq, nkv, hd,
                                               out.data_ptr(), err.data_ptr(), None)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert rel_err(got, ref) < TOL, (pos, rel_err(got, ref))

    # sizes beyond the fixed scratch are refused, not truncated
    rc = lib.vvq2_attention_decode_noalloc(q_d.data_ptr(), k_d.data_ptr(), v_d.data_ptr(), bt.data_ptr(),
                                           max_pages, meta.data_ptr(), 9, pos + 1, nq, nkv, hd,
                                           out.data_ptr(), None, None)
    assert rc == -2


def _attention_ref(q, kp, vp, bt, meta, nq, nkv, hd):
    """softmax(q_f16 . K^T / sqrt(hd)) V over keys j < min(pos + 1, kv_len), in f64
    (ggml's flash attention rounds Q to the f16 type of K)."""
    G = nq // nkv
    out = np.zeros((len(meta), nq * hd), np.float64)
    for r, (seq, pos, _, kvlen) in enumerate(meta):
        n = min(pos + 1, kvlen)
        for h in range(nq):
            g = h // G
            qh = q[r, h * hd:(h + 1) * hd].astype(np.float16).astype(np.float64)
            ks = np.stack([kp[bt[seq, j // 64], g, j % 64] for j in range(n)]).astype(np.float64)
            vs = np.stack([vp[bt[seq, j // 64], g, j % 64] for j in range(n)]).astype(np.float64)
            s = ks @ qh / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[r, h * hd:(h + 1) * hd] = (p / p.sum()) @ vs
    return out


# (head_dim, n_heads, n_kv_heads, max_kv, kv lengths of the two calls): one
# split (<= 64 keys), 2-4 splits merged by the last split, and > 4 splits
# merged by the separate kernel
PATHS = [
    (32, 8, 2, 60, ([60, 17, 33], [41, 60, 1])),
    (64, 14, 2, 250, ([250, 130, 65], [190, 250, 64])),
    (128, 12, 2, 700, ([700, 333], [512, 699])),
]


@pytest.mark.parametrize("hd,nq,nkv,max_kv,lens", PATHS, ids=["hd32-1split", "hd64-inline", "hd128-kernel"])
def test_noalloc_attention_paths_vs_formula(vv, hd, nq, nkv, max_kv, lens):
    import torch

    rng = np.random.default_rng(hd * 7 + max_kv)
    dev = torch.device("cuda:0")
    lib = vv.lib()
    n_seq = 3
    max_pages = (max_kv + 63) // 64 + 1
    n_pages = n_seq * max_pages
    kp = rng.standard_normal((n_pages, nkv, 64, hd)).astype(np.float16)
    vp = rng.standard_normal((n_pages, nkv, 64, hd)).astype(np.float16)
    bt = rng.permutation(n_pages).astype(np.int32).reshape(n_seq, max_pages)
    k_d = torch.from_numpy(kp).to(dev)
    v_d = torch.from_numpy(vp).to(dev)
    bt_d = torch.from_numpy(bt).to(dev)
    for call, lengths in enumerate(lens):          # two calls in a row, different lengths
        rows = len(lengths)
        meta = np.array([[(r + call) % n_seq, L - 1, L - 1, L] for r, L in enumerate(lengths)], np.int32)
        q = rng.standard_normal((rows, nq * hd)).astype(np.float32)
        out = torch.zeros((rows, nq * hd), dtype=torch.float32, device=dev)
        err = torch.full((1,), -1, dtype=torch.int32, device=dev)
        meta_d = torch.from_numpy(meta).to(dev)
        q_d = torch.from_numpy(q).to(dev)
        rc = lib.vvq2_attention_decode_noalloc(q_d.data_ptr(), k_d.data_ptr(), v_d.data_ptr(), bt_d.data_ptr(),
                                               max_pages, meta_d.data_ptr(), rows, max_kv, nq, nkv, hd,
                                               out.data_ptr(), err.data_ptr(), None)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert int(err.item()) == 0, int(err.item())
        ref = _attention_ref(q, kp, vp, bt, meta, nq, nkv, hd)
        e = rel_err(out.cpu().numpy(), ref)
        assert e < TOL, (call, e)

    # a row longer than max_kv: clamped to the keys the launch covers, error word 5
    L = max_kv + 64
    meta = np.array([[0, L - 1, L - 1, L]], np.int32)
    q = rng.standard_normal((1, nq * hd)).astype(np.float32)
    out = torch.zeros((1, nq * hd), dtype=torch.float32, device=dev)
    err = torch.full((1,), -1, dtype=torch.int32, device=dev)
    rc = lib.vvq2_attention_decode_noalloc(torch.from_numpy(q).to(dev).data_ptr(), k_d.data_ptr(), v_d.data_ptr(),
                                           bt_d.data_ptr(), max_pages, torch.from_numpy(meta).to(dev).data_ptr(),
                                           1, max_kv, nq, nkv, hd, out.data_ptr(), err.data_ptr(), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 5
    split = max(64, ((max_kv + 15) // 16 + 63) // 64 * 64)
    covered = min((max_kv + split - 1) // split * split, max_pages * 64)
    clamped = np.array([[0, covered - 1, covered - 1, covered]], np.int32)
    e = rel_err(out.cpu().numpy(), _attention_ref(q, kp, vp, bt, clamped, nq, nkv, hd))
    assert e < TOL, e
