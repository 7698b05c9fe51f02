"""The tile sequence of the single-kernel wide chains (mlp_gemm_chain.cuh), modelled on the CPU.

The device walks one sequence of tiles for all layers of a chain: step i holds layer s's tiles of
row block i - lag_s (and, for LayerNorm chains, the LayerNorm tile of row block i - lag_ln).
Pairs claim positions in order; a tile waits for the previous layer's tiles of its row block
(read after write) and, before overwriting a ring slot, for the consumers of the row block that
held it (write after read). This module restates that schedule (chain_step_tiles,
ChainCursor::advance, chain_decode, and the ring sizing of chain_schedule in wide_chains.cu) and
checks what the kernel relies on:
  - every position decodes to exactly one tile inside the chain, and a cursor that advances past
    the end stops at n_steps;
  - every dependency points to an earlier position (so claiming in order cannot deadlock);
  - a simulation of pairs claiming positions and waiting on dependencies always finishes.
"""
import heapq
import random

import pytest

BERT = dict(tiles=[16, 4], lags=[0, 16], ln=True, ln_lag=40, rings=[40, 40])
DLRM = dict(tiles=[4, 4, 2, 1], lags=[0, 20, 60, 100], ln=False, ln_lag=0, rings=[120, 120, 120, 0])


def make(nb, tiles, lags, ln, ln_lag, rings):
    """chain_schedule: total, n_steps and ring depths (at least the producer-consumer lag + 1,
    at most the row blocks)."""
    g = dict(nb=nb, tiles=list(tiles), lags=list(lags), ln=ln, ln_lag=ln_lag if ln else 0)
    g["total"] = sum(nb * t for t in tiles) + (nb if ln else 0)
    g["n_steps"] = max(list(lags) + [g["ln_lag"]]) + nb
    q = []
    for s in range(len(tiles)):
        if not (s + 1 < len(tiles) or ln):
            q.append(0)
            continue
        nxt = lags[s + 1] if s + 1 < len(tiles) else g["ln_lag"]
        q.append(min(max(rings[s], nxt - lags[s] + 1), nb))
    g["q"] = q
    return g


def step_tiles(g, i):
    n = sum(t for s, t in enumerate(g["tiles"]) if 0 <= i - g["lags"][s] < g["nb"])
    if g["ln"] and 0 <= i - g["ln_lag"] < g["nb"]:
        n += 1
    return n


def advance(g, cur, by):
    step, idx = cur
    idx += by
    while step < g["n_steps"]:
        n = step_tiles(g, step)
        if idx < n:
            return step, idx
        idx -= n
        step += 1
    return step, idx


def decode(g, cur):
    step, idx = cur
    for s, t in enumerate(g["tiles"]):
        r = step - g["lags"][s]
        if 0 <= r < g["nb"]:
            if idx < t:
                return s, r, idx
            idx -= t
    return len(g["tiles"]), step - g["ln_lag"], 0


def sequence(g):
    cur, prev, out = (0, 0), 0, []
    for t in range(g["total"]):
        cur = advance(g, cur, t - prev)
        prev = t
        assert cur[0] < g["n_steps"]
        out.append(decode(g, cur))
    assert advance(g, cur, 1)[0] == g["n_steps"]  # past the end: the walk stops
    return out


def deps(g, tile):
    S = len(g["tiles"])
    s, r, _ = tile
    d = []
    if 0 < s < S:
        d += [(s - 1, r, j) for j in range(g["tiles"][s - 1])]
    if s == S:
        d += [(S - 1, r, j) for j in range(g["tiles"][S - 1])]
    if s < S and g["q"][s] > 0 and r >= g["q"][s]:
        cs = s + 1
        d += [(cs, r - g["q"][s], j) for j in range(g["tiles"][cs])] if cs < S else [(S, r - g["q"][s], 0)]
    return d


def check(g, pairs, dur):
    seq = sequence(g)
    pos = {tile: t for t, tile in enumerate(seq)}
    assert len(pos) == g["total"]
    for tile in seq:
        s, r, _ = tile
        assert 0 <= r < g["nb"] and 0 <= s <= len(g["tiles"])
        for d in deps(g, tile):
            assert pos[d] < pos[tile], (tile, d)
    # pairs claim positions in order when free; a tile starts once its dependencies are done
    done, free = {}, [(0.0, p) for p in range(pairs)]
    for tile in seq:
        now, p = heapq.heappop(free)
        start = max([now] + [done[d] for d in deps(g, tile)])
        done[tile] = start + dur(tile)
        heapq.heappush(free, (done[tile], p))
    return max(done.values())


@pytest.mark.parametrize("nb", [1, 2, 3, 17, 36, 64, 65, 157])
@pytest.mark.parametrize("pairs", [1, 7, 74])
def test_default_schedules(nb, pairs):
    for cfg in (BERT, DLRM):
        check(make(nb, **cfg), pairs, lambda tile: 1.0)


def test_random_schedules():
    rnd = random.Random(7)
    for _ in range(200):
        S = rnd.randint(1, 4)
        lags = [0] + sorted(rnd.randint(1, 30) for _ in range(S - 1))
        ln = rnd.random() < 0.5
        g = make(rnd.randint(1, 80), [rnd.randint(1, 16) for _ in range(S)], lags, ln,
                 (lags[-1] + rnd.randint(1, 20)) if ln else 0, [rnd.randint(0, 30) for _ in range(S)])
        check(g, rnd.randint(1, 74), lambda tile: rnd.uniform(0.5, 4.0))


def test_dynamic_claims_balance_uneven_tiles():
    """BERT-large at M = 16,384: layer-1 tiles take ~4x a layer-0 tile. Claiming in order keeps
    74 pairs within ~10% of the ideal makespan."""
    g = make(64, **BERT)
    dur = {0: 1.0, 1: 4.0, 2: 0.3}
    span = check(g, 74, lambda tile: dur[tile[0]])
    ideal = 64 * (16 * 1.0 + 4 * 4.0 + 0.3) / 74
    assert span < 1.15 * ideal
