"""The expert-parallel engine's routing tables, on the CPU.

moe_ep_build_tables runs, on the host, the same table code the engine's
count kernel runs on the device after its count barrier (csrc/ep_exchange.cuh:
ep_wave_total, ep_owner_region, ep_slice, ep_recv_entry).  Checked two ways
over random world x E count tables (skewed, empty experts, negative and
oversized sizes, regions too small):

* against an independent Python restatement of the layout: per wave v an
  expert's rows are the sources' slices [c v / V, c (v+1) / V); an owner's
  landing region holds its experts in order, each expert's rows from sources
  o, o+1, ..., o-1 (mod world) in that order; everything is cut to the
  region and to M;
* across ranks, from one consistent count table: the slices every source
  computes tile each owner's region exactly (disjoint, owner's own rows
  first, sizes = the owner's group sizes), the owners' receive tables point
  back at the same rows, and every routed row of a source leaves exactly once.
"""

import ctypes

import numpy as np
import pytest

from src import _lib

I32P = ctypes.POINTER(ctypes.c_int32)


def build(counts, rank, el, waves, region_cap, max_rows, M, with_recv=True):
    W, E = counts.shape
    c = np.ascontiguousarray(counts, dtype=np.int32)
    slices = np.zeros((waves, E, 4), np.int32)
    wave_rows = np.zeros((waves, E + 1), np.int32)
    local_gs = np.zeros((waves, el), np.int32)
    recv = np.zeros((el, W, 4), np.int32) if with_recv else None
    st = _lib.lib().moe_ep_build_tables(
        c.ctypes.data_as(I32P), W, rank, el, waves, region_cap, max_rows, M,
        slices.ctypes.data_as(I32P), wave_rows.ctypes.data_as(I32P), local_gs.ctypes.data_as(I32P),
        recv.ctypes.data_as(I32P) if with_recv else None)
    assert st >= 0, _lib.lib().moe_last_error()
    return st, slices, wave_rows, local_gs, recv


def cut(c, v, V):
    return (int(c) * v) // V


def restate(counts, rank, el, V, cap, max_rows, M):
    """Independent restatement of the tables (see module doc)."""
    W, E = counts.shape
    status = 0
    own = []
    for x in counts[rank]:
        if x < 0:
            status |= 2
        own.append(min(max(int(x), 0), M))
    own_off, tot = [], 0
    for g in range(E):
        own_off.append(min(tot, M))
        tot = min(tot + own[g], M)
    for g in range(E):
        room = M - own_off[g]
        if own[g] > room:
            own[g] = room
            status |= 8
    cnt = np.array([[own[g] if s == rank else int(np.clip(counts[s, g], 0, max_rows)) for g in range(E)]
                    for s in range(W)], dtype=np.int64)
    wn = lambda s, g, v: cut(cnt[s, g], v + 1, V) - cut(cnt[s, g], v, V)  # noqa: E731
    start = np.zeros((V, E), np.int64)
    local = np.zeros((V, el), np.int64)
    for v in range(V):
        for p in range(W):
            run = 0
            for e in range(el):
                g = p * el + e
                n = min(sum(wn(s, g, v) for s in range(W)), cap - run)
                start[v, g] = run
                if p == rank:
                    local[v, e] = n
                run += n
    slices = np.zeros((V, E, 4), np.int64)
    for v in range(V):
        for g in range(E):
            o = g // el
            order = [(o + k) % W for k in range(W)]
            before = sum(wn(s, g, v) for s in order[:order.index(rank)])
            n = wn(rank, g, v)
            dst = start[v, g] + before
            if dst + n > cap:
                n = max(0, cap - dst)
                status |= 8
            slices[v, g] = (own_off[g] + cut(cnt[rank, g], v, V), n, dst, o)
    src_off = np.concatenate([np.zeros((W, 1), np.int64), np.cumsum(cnt, axis=1)[:, :-1]], axis=1)
    recv = np.zeros((el, W, 4), np.int64)
    for e in range(el):
        g = rank * el + e
        for sr in range(W):
            st = int(local[0, :e].sum()) + sum(int(cnt[s2, g]) for s2 in [(rank + k) % W for k in range(W)][
                :[(rank + k) % W for k in range(W)].index(sr)])
            n = int(cnt[sr, g])
            if st + n > cap:
                n = max(0, cap - st)
            recv[e, sr] = (st, n, src_off[sr, g], sr)
    wave_rows = np.zeros((V, E + 1), np.int64)
    for v in range(V):
        wave_rows[v, 1:] = np.cumsum(slices[v, :, 1])
    return status, slices, wave_rows, local, recv


def random_counts(rng, W, el, M):
    E = W * el
    out = np.zeros((W, E), np.int64)
    for s in range(W):
        w = rng.dirichlet(np.full(E, rng.choice([0.2, 1.0, 5.0])))
        w[rng.random(E) < 0.2] = 0                      # empty experts
        w = w / w.sum() if w.sum() > 0 else np.full(E, 1.0 / E)
        out[s] = rng.multinomial(rng.integers(0, M + 1), w)
    return out


@pytest.mark.parametrize("seed", range(40))
def test_tables_match_restatement(seed):
    rng = np.random.default_rng(seed)
    W = int(rng.integers(1, 9))
    el = int(rng.integers(1, 5))
    V = int(rng.integers(1, 4))
    M = int(rng.integers(1, 400))
    counts = random_counts(rng, W, el, M)
    rank = int(rng.integers(0, W))
    if seed % 5 == 0:
        counts[rank, 0] = -7                            # a negative size: counts as 0
    if seed % 7 == 0:
        counts[(rank + 1) % W, -1] = 10 ** 6            # a peer's size above max_rows
    cap = int(rng.integers(1, W * M + W * el + 2)) if seed % 3 == 0 else W * M // V + W * el + 8
    want = restate(counts, rank, el, V, cap, M, M)
    got = build(counts, rank, el, V, cap, M, M)
    assert got[0] == want[0]
    for a, b, name in zip(got[1:], want[1:], ("slices", "wave_rows", "local_gs", "recv")):
        np.testing.assert_array_equal(a, b, err_msg=name)


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("V", [1, 2, 3])
def test_tables_consistent_across_ranks(seed, V):
    rng = np.random.default_rng(100 + seed)
    W = int(rng.integers(2, 9))
    el = int(rng.integers(1, 4))
    E = W * el
    M = int(rng.integers(0, 300))
    counts = random_counts(rng, W, el, M)
    cap = (W * M + V - 1) // V + W * el                 # the engine's region size: nothing is cut
    tabs = [build(counts, r, el, V, cap, M, M) for r in range(W)]
    assert all(t[0] == 0 for t in tabs)
    for v in range(V):
        for o in range(W):
            local_gs = tabs[o][3][v]
            starts = np.concatenate([[0], np.cumsum(local_gs)])
            for e in range(el):
                g = o * el + e
                # the slices of every source into (owner o, expert g, wave v)
                got = sorted((tabs[s][1][v, g, 2], tabs[s][1][v, g, 1], s) for s in range(W))
                pos = starts[e]
                ordered = [x for x in got if x[1] > 0]
                for dst, n, s in ordered:
                    assert dst == pos, (v, o, g, s)     # contiguous and disjoint
                    pos += n
                assert pos == starts[e + 1]              # exactly the owner's group size
                if counts[o, g] // V or counts[o, g]:
                    first = [x for x in got if x[2] == o][0]
                    assert first[0] == starts[e]         # the owner's own rows lead
                assert all(tabs[s][1][v, g, 3] == o for s in range(W))
    if V == 1:
        for o in range(W):
            recv = tabs[o][4]
            for e in range(el):
                g = o * el + e
                for s in range(W):
                    sl = tabs[s][1][0, g]
                    assert tuple(recv[e, s]) == (sl[2], sl[1], sl[0], s)
    for s in range(W):                                   # every routed row of a source leaves once
        seen = np.zeros(M, np.int64)
        for v in range(V):
            for g in range(E):
                src, n = tabs[s][1][v, g, 0], tabs[s][1][v, g, 1]
                seen[src:src + n] += 1
        routed = min(int(counts[s].sum()), M)
        assert np.all(seen[:routed] == 1) and np.all(seen[routed:] == 0)
        assert tabs[s][2][:, -1].sum() == routed


def test_region_overflow_is_cut_and_reported():
    counts = np.array([[50, 50], [50, 50]], np.int64)
    st, slices, wr, local_gs, recv = build(counts, 0, 1, 1, region_cap=60, max_rows=100, M=100)
    assert st & 8
    assert local_gs[0, 0] == 60 and slices[0, 0, 1] == 50 and slices[0, 0, 2] == 0
    assert recv[0, 1, 1] == 10                           # only 10 of source 1's rows fit
    assert _lib.lib().moe_ep_build_tables(None, 2, 0, 1, 1, 60, 100, 100, None, None, None, None) == -1
