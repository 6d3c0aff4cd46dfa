"""SwiGLU experts on the GPU (bf16) against the float64 oracle on the
bf16-rounded inputs.  Tolerance: L2 relative error <= 1e-2, the bf16 bar of
the GELU path; the interleave is bit-exact."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src.kernel import fused_ragged_swiglu, swiglu_interleave
from src.routing import make_group_sizes, zipf_group_sizes

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0


def _weights(E, D, F, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    wg = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    wu = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    wd = (torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5).to(torch.bfloat16)
    return wg, wu, wd


def _x(M, D, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed + 1000)
    return torch.randn((M, D), generator=g, device=DEV).to(torch.bfloat16)


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("E,D,F", [(2, 256, 128), (3, 512, 384), (8, 4096, 14336)])
def test_interleave_bit_exact(E, D, F):
    wg, wu, _ = _weights(E, D, F, seed=E)
    w = swiglu_interleave(wg, wu)
    torch.cuda.synchronize()
    if E * D * F > 1 << 24:   # large: compare on the device, bit for bit
        ref = torch.stack([wg.view(E, D, F // 128, 128), wu.view(E, D, F // 128, 128)], dim=3).view(E, D, 2 * F)
        assert torch.equal(w.view(torch.int16), ref.view(torch.int16))
    else:
        ref = orc.swiglu_interleave(wg.view(torch.int16).cpu().numpy(), wu.view(torch.int16).cpu().numpy())
        np.testing.assert_array_equal(w.view(torch.int16).cpu().numpy(), ref)


@pytest.mark.parametrize("M,D,F,E", [(1024, 256, 128, 2), (2048, 512, 1024, 4), (1536, 768, 384, 3),
                                     (2048, 1024, 768, 2)])
def test_swiglu_full_oracle(M, D, F, E):
    gs = make_group_sizes(M, E)
    wg, wu, wd = _weights(E, D, F, seed=D)
    x = _x(M, D, seed=D)
    y = fused_ragged_swiglu(x, swiglu_interleave(wg, wu), wd, torch.from_numpy(gs).to(DEV))
    torch.cuda.synchronize()
    ref = orc.ref_ragged_swiglu(_np(x), _np(wg), _np(wu), _np(wd), gs)
    m = orc.correctness_metrics(ref, y.cpu().numpy())
    assert m["fused_is_finite"] and m["l2_relative_error"] <= TOL, m


@pytest.mark.parametrize("gs", [
    [0, 700, 0, 5],         # empty experts; one tiny expert
    [255, 257, 1, 511],     # 256-row block boundaries
    [300, 0, 0, 0],         # sum < M, trailing rows zero
    [0, 0, 0, 0],           # nothing routed
])
def test_swiglu_ragged_edges(gs):
    M, D, F, E = 1024, 512, 512, 4
    wg, wu, wd = _weights(E, D, F, seed=7)
    x = _x(M, D, seed=7)
    out = torch.full((M, D), float("nan"), device=DEV)
    y = fused_ragged_swiglu(x, swiglu_interleave(wg, wu), wd, torch.tensor(gs, dtype=torch.int32), out=out)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    tail = int(np.sum(gs))
    assert np.all(np.isfinite(y)) and np.all(y[tail:] == 0.0)
    if tail:
        ref = orc.ref_ragged_swiglu(_np(x), _np(wg), _np(wu), _np(wd), gs)
        m = orc.correctness_metrics(ref[:tail], y[:tail])
        assert m["l2_relative_error"] <= TOL, m


def test_swiglu_zipf_many_experts():
    M, D, F, E = 4096, 512, 1024, 16
    gs = zipf_group_sizes(M, E, np.random.default_rng(3))
    wg, wu, wd = _weights(E, D, F, seed=9)
    x = _x(M, D, seed=9)
    y = fused_ragged_swiglu(x, swiglu_interleave(wg, wu), wd, torch.from_numpy(gs).to(DEV))
    torch.cuda.synchronize()
    ref = orc.ref_ragged_swiglu(_np(x), _np(wg), _np(wu), _np(wd), gs)
    m = orc.correctness_metrics(ref, y.cpu().numpy())
    assert m["l2_relative_error"] <= TOL, m


def test_swiglu_mixtral_shape_sampled_rows():
    """Mixtral-8x7B experts (D=4096, F=14336, E=8), top-2 of 16384 tokens ->
    M=32768; the oracle checks 16 sampled rows per expert (a row depends only
    on its own X row and its expert's weights)."""
    M, D, F, E = 32768, 4096, 14336, 8
    gs = make_group_sizes(M, E)
    wg, wu, wd = _weights(E, D, F, seed=0)
    x = _x(M, D, seed=0)
    wgu = swiglu_interleave(wg, wu)
    y = fused_ragged_swiglu(x, wgu, wd, torch.from_numpy(gs).to(DEV))
    torch.cuda.synchronize()
    offs = orc.group_sizes_to_offsets(gs)
    rng = np.random.default_rng(1)
    refs, gots = [], []
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if b <= a:
            continue
        rows = np.unique(np.concatenate([rng.integers(a, b, 14), [a, b - 1]]))
        refs.append(orc.ref_ragged_swiglu(_np(x[rows]), _np(wg[e])[None], _np(wu[e])[None], _np(wd[e])[None],
                                          [len(rows)]))
        gots.append(y[rows].cpu().numpy())
    m = orc.correctness_metrics(np.concatenate(refs), np.concatenate(gots))
    assert m["fused_is_finite"] and m["l2_relative_error"] <= TOL, m
