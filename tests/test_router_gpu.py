"""Routing and permutation kernels on the GPU against the oracle: expert ids,
group sizes, the permutation and gathered rows bit for bit; softmax weights
and the weighted combine within f32 rounding; a whole MoE layer (route ->
permute -> gather -> fused MLP -> combine) against the float64 oracle."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src import router
from src.routing import make_inputs_numpy

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("T,E,k", [(3000, 8, 2), (4099, 64, 6), (8192, 256, 8), (257, 1000, 16), (5, 3, 3)])
def test_route_topk_matches_oracle(T, E, k):
    rng = np.random.default_rng(T + E)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[::7] = np.round(logits[::7])            # rows with ties
    ids, w = router.route_topk(torch.from_numpy(logits).to(DEV), k)
    torch.cuda.synchronize()
    ref_ids, ref_w = orc.route_topk(logits, k)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=1e-5, atol=1e-7)   # fast exp


@pytest.mark.parametrize("T,k,E,kind", [(8192, 8, 256, "uniform"), (1000, 2, 8, "skewed"), (513, 3, 64, "bad"),
                                        (1, 1, 4, "uniform"), (20000, 4, 1024, "uniform")])
def test_permute_matches_oracle(T, k, E, kind):
    rng = np.random.default_rng(T)
    if kind == "skewed":
        ids = rng.choice([1, 5], size=(T, k), p=[0.9, 0.1]).astype(np.int32)   # most experts empty
    else:
        ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    if kind == "bad":
        ids[3, 0], ids[100, 2] = -1, E
    _lib.device_status(reset=True)
    gs, src, inv = router.permute(torch.from_numpy(ids).to(DEV), E)
    torch.cuda.synchronize()
    rgs, rsrc, rinv = orc.permute_by_expert(ids, E)
    assert np.array_equal(gs.cpu().numpy(), rgs)
    n = int(rgs.sum())
    assert np.array_equal(src.cpu().numpy()[:n], rsrc)
    assert np.array_equal(inv.cpu().numpy().reshape(-1), rinv)
    assert _lib.device_status(reset=True) == (16 if kind == "bad" else 0)


@pytest.mark.parametrize("dt,D", [(torch.bfloat16, 7168), (torch.float32, 128), (torch.bfloat16, 8), (torch.float32, 400)])
def test_gather_and_combine_match_oracle(dt, D):
    T, k, E = 777, 4, 32
    rng = np.random.default_rng(D)
    x = torch.randn((T, D), device=DEV).to(dt)
    ids = torch.from_numpy(rng.integers(0, E, size=(T, k)).astype(np.int32)).to(DEV)
    w = torch.rand((T, k), device=DEV)
    gs, src, inv = router.permute(ids, E)
    xs = router.gather_rows(x, src, k)
    torch.cuda.synchronize()
    assert torch.equal(xs, x[src.long() // k])                        # bit for bit
    if D % 4 == 0:
        ys = torch.randn((T * k, D), device=DEV)
        y = router.combine_rows(ys, inv, w)
        torch.cuda.synchronize()
        ref = orc.combine_rows(ys.cpu().numpy(), inv.cpu().numpy(), w.cpu().numpy(), k)
        np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dt,D,F,E,k", [("f32", 128, 512, 8, 2), ("bf16", 512, 1024, 16, 4)])
def test_moe_layer_end_to_end(dt, D, F, E, k):
    T = 1500
    _, wu, wd = make_inputs_numpy(8, D, F, E, seed=3)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((T, D)).astype(np.float32)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    xt, wut, wdt = (torch.from_numpy(a).to(DEV, tdt) for a in (x, wu, wd))
    y, gs = router.moe_layer(xt, torch.from_numpy(logits).to(DEV), wut, wdt, k)
    torch.cuda.synchronize()
    ids, w = orc.route_topk(logits, k)
    rgs, rsrc, rinv = orc.permute_by_expert(ids, E)
    xs = orc.gather_rows(xt.double().cpu().numpy(), rsrc, k)
    ys = orc.ref_ragged_mlp(xs, wut.double().cpu().numpy(), wdt.double().cpu().numpy(), rgs)
    ref = orc.combine_rows(ys, rinv, w, k)
    assert np.array_equal(gs.cpu().numpy(), rgs)
    err = orc.correctness_metrics(ref, y.cpu().numpy())["l2_relative_error"]
    assert err <= (1e-5 if dt == "f32" else 1e-2), err
    assert _lib.device_status(reset=True) == 0
