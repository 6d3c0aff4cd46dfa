"""Routing and permutation on the CPU: the oracle's restatement against
brute force, and the C ABI's argument checks (no GPU work)."""

import ctypes

import numpy as np

from oracle import moe_oracle as orc
from src import _lib


def test_route_topk_oracle_matches_brute_force_with_ties():
    rng = np.random.default_rng(0)
    logits = rng.integers(-3, 4, size=(200, 16)).astype(np.float32)   # many ties
    ids, w = orc.route_topk(logits, 4)
    for t in range(200):
        cand = sorted(range(16), key=lambda e: (-logits[t, e], e))[:4]
        assert ids[t].tolist() == cand
        sel = logits[t, cand].astype(np.float64)
        ref = np.exp(sel - sel.max()) / np.exp(sel - sel.max()).sum()
        np.testing.assert_allclose(w[t], ref, rtol=1e-12)


def test_permute_oracle_is_a_stable_sort_with_inverse():
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 10, size=(333, 3)).astype(np.int32)
    ids[5, 1] = -1
    ids[7, 2] = 10                       # outside [0, E): dropped
    gs, src, inv = orc.permute_by_expert(ids, 10)
    flat = ids.reshape(-1)
    assert gs.sum() == flat.size - 2 and src.size == flat.size - 2
    assert np.all(np.diff(flat[src]) >= 0)                   # sorted by expert
    for e in range(10):
        members = src[flat[src] == e]
        assert np.all(np.diff(members) > 0)                  # stable
    assert inv[5 * 3 + 1] == -1 and inv[7 * 3 + 2] == -1
    ok = inv >= 0
    assert np.array_equal(src[inv[ok]], np.nonzero(ok)[0])


def test_combine_oracle_weights_slots():
    ys = np.arange(12, dtype=np.float64).reshape(6, 2)
    inv = np.array([[0, 3], [5, -1]])
    w = np.array([[0.25, 0.75], [1.0, 9.0]])
    y = orc.combine_rows(ys, inv, w, 2)
    np.testing.assert_allclose(y, [[0.25 * ys[0] + 0.75 * ys[3]][0], ys[5]])


def test_routing_abi_validates_arguments():
    L = _lib.lib()
    vp = ctypes.c_void_p
    assert L.moe_route_topk(None, 10, 2000, 2, None, None, None) == -1      # E too large
    assert L.moe_route_topk(None, 10, 8, 9, None, None, None) == -1         # k > E
    assert L.moe_route_topk(None, 0, 8, 2, None, None, None) == 0           # nothing to do
    assert L.moe_permute(None, 100, 8, None, None, None, None, 0, None) == -1
    assert L.moe_permute(vp(16), 100, 8, vp(16), vp(16), vp(16), vp(256), 1, None) == -4
    assert L.moe_permute_workspace_size(1024, 8) >= 2 * 8 * 4
    assert L.moe_gather_rows(vp(16), vp(16), 4, 2, 100, vp(16), None) == -1  # row bytes not a multiple of 16
    assert L.moe_combine_rows(vp(16), vp(16), vp(16), 4, 2, 6, vp(16), None) == -1
