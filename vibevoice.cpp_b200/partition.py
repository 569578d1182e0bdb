"""Attention partition plan for multi-GPU long-context decoding (config 5).

The same ownership rules the engine applies (vvq2_partition): `world` ranks
= head_groups x seq_parts; rank r holds KV-head group r // seq_parts (its q
heads, their QKV rows and attention) and sequence part r % seq_parts of
every sequence's keys.  The two parts interleave whole 64-position pages:
page p belongs to part (0, 1, 1, 0)[p % 4], so each part holds half of every
256-position span and a causal prompt of any length or chunking gives both
the same attention work; a part stores its positions in order.
Each rank's attention output is normalized over its own keys and carries its
log-sum-exp; two parts merge as o = sum_i e^(l_i - l) o_i / sum_i e^(l_i - l).
The FFN is split over all ranks: rank r holds intermediate features
[r F/world, (r+1) F/world) (gate/up rows, down columns); the partial down
projections are all-reduced.

Pure Python/numpy: the host side of the partition (plan, id exchange) and a
restatement of the merge used by the tests."""
from __future__ import annotations

import numpy as np

KV_PAGE = 64


ZZ = (0, 1, 1, 0)


def part_of(pos: int) -> int:
    """Sequence part that stores position pos."""
    return ZZ[(pos // KV_PAGE) % 4]


def part_count(part: int, n: int) -> int:
    """Positions below n that a part stores (= cache index of position n if it is the part's)."""
    full, rem = divmod(n, 4 * KV_PAGE)
    return full * 2 * KV_PAGE + sum(min(KV_PAGE, max(0, rem - j * KV_PAGE)) for j in range(4) if ZZ[j] == part)


def plan(rank: int, world: int, seq_parts: int, n_heads: int, n_kv_heads: int) -> dict:
    """Heads and sequence part of one rank."""
    if seq_parts not in (1, 2) or world % seq_parts or rank < 0 or rank >= world:
        raise ValueError("bad partition")
    groups = world // seq_parts
    if n_kv_heads % groups:
        raise ValueError(f"{n_kv_heads} KV heads over {groups} head groups")
    g, s = rank // seq_parts, rank % seq_parts
    nkv = n_kv_heads // groups
    nq = n_heads // groups
    return {"group": g, "part": s, "kv_heads": range(g * nkv, (g + 1) * nkv),
            "q_heads": range(g * nq, (g + 1) * nq), "groups": groups, "seq_parts": seq_parts}


def ffn_range(rank: int, world: int, ffn: int) -> range:
    """Intermediate FFN features one rank holds."""
    if ffn % (world * 64):
        raise ValueError(f"ffn {ffn} not a multiple of {world * 64}")
    f = ffn // world
    return range(rank * f, (rank + 1) * f)


def keys_of_part(part: int, seq_parts: int, n_keys: int) -> np.ndarray:
    """Absolute key positions a sequence part holds, in cache order."""
    pos = np.arange(n_keys, dtype=np.int64)
    if seq_parts == 1:
        return pos
    return pos[np.array([part_of(int(p)) == part for p in pos], dtype=bool)] if n_keys else pos


def lse_merge(o: np.ndarray, lse: np.ndarray) -> np.ndarray:
    """Merge normalized partial outputs o[i] ([..., hd]) with log-sum-exps
    lse[i] ([...]) over disjoint key sets; parts without keys have lse -inf."""
    m = np.max(lse, axis=0)
    safe = np.where(np.isfinite(m), m, 0.0)
    w = np.where(np.isfinite(lse), np.exp(lse - safe), 0.0)
    den = np.sum(w, axis=0)
    out = np.sum(w[..., None] * o, axis=0) / np.where(den > 0, den, 1.0)[..., None]
    return np.where((den > 0)[..., None], out, 0.0)


def partial_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, q_pos: np.ndarray, key_pos: np.ndarray,
                      scale: float):
    """Causal attention of q [T, hd] over keys (k, v [n, hd] at absolute
    positions key_pos): normalized output [T, hd] and log-sum-exp [T]."""
    s = (q @ k.T) * scale
    s = np.where(key_pos[None, :] <= q_pos[:, None], s, -np.inf)
    m = np.max(s, axis=1) if s.shape[1] else np.full(q.shape[0], -np.inf)
    ok = np.isfinite(m)
    p = np.exp(s - np.where(ok, m, 0.0)[:, None])
    p = np.where(np.isfinite(s), p, 0.0)
    den = p.sum(axis=1)
    out = (p @ v) / np.where(den > 0, den, 1.0)[:, None]
    lse = np.where(den > 0, np.where(ok, m, 0.0) + np.log(np.where(den > 0, den, 1.0)), -np.inf)
    return np.where((den > 0)[:, None], out, 0.0), lse
