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


# ----------------------------------------------------------------------------- e4m3 weights (DeepSeek-V3 format)
from src.kernel import swiglu_interleave_fp8  # noqa: E402
from src.routing import dequantize_e4m3_blockwise, quantize_e4m3_blockwise  # noqa: E402

FP8_TOL = 2e-2  # the FP8 bar of this library, against the dequantised weights


def _fp8_weights(E, D, F, seed):
    wg, wu, wd = _weights(E, D, F, seed)
    (qg, sg), (qu, su), (qd, sd) = (quantize_e4m3_blockwise(w.float()) for w in (wg, wu, wd))
    return (qg, sg), (qu, su), (qd, sd)


def test_fp8_interleave_bit_exact():
    E, D, F = 3, 256, 384
    (qg, sg), (qu, su), _ = _fp8_weights(E, D, F, seed=11)
    w, s = swiglu_interleave_fp8(qg, qu, sg, su)
    torch.cuda.synchronize()
    ref = orc.swiglu_interleave(qg.view(torch.uint8).cpu().numpy(), qu.view(torch.uint8).cpu().numpy())
    np.testing.assert_array_equal(w.view(torch.uint8).cpu().numpy(), ref)
    ref_s = orc.swiglu_interleave(np.repeat(sg.cpu().numpy(), 128, axis=2), np.repeat(su.cpu().numpy(), 128, axis=2))
    np.testing.assert_array_equal(s.cpu().numpy(), ref_s[:, :, ::128])


@pytest.mark.parametrize("M,D,F,E,gs", [(2048, 512, 512, 4, None), (1536, 768, 384, 3, None),
                                        (1024, 512, 256, 4, [0, 700, 0, 5]), (1024, 512, 256, 4, [300, 0, 0, 0])])
def test_fp8_swiglu_matches_oracle_on_dequantised_weights(M, D, F, E, gs):
    gs = make_group_sizes(M, E) if gs is None else np.asarray(gs, np.int32)
    (qg, sg), (qu, su), (qd, sd) = _fp8_weights(E, D, F, seed=M + F)
    wgu, sgu = swiglu_interleave_fp8(qg, qu, sg, su)
    x = _x(M, D, seed=F)
    out = torch.full((M, D), float("nan"), device=DEV)
    y = fused_ragged_swiglu(x, wgu, qd, torch.from_numpy(gs).to(DEV), w_gate_up_scale=sgu, w_down_scale=sd, out=out)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    n = int(gs.sum())
    assert np.all(np.isfinite(y)) and np.all(y[n:] == 0.0)
    deq = [dequantize_e4m3_blockwise(q, s).cpu().numpy() for q, s in ((qg, sg), (qu, su), (qd, sd))]
    ref = orc.ref_ragged_swiglu(_np(x), *deq, gs)
    if n:
        m = orc.correctness_metrics(ref[:n], y[:n])
        assert m["l2_relative_error"] <= FP8_TOL, m


def test_fp8_swiglu_deepseek_shape_sampled_rows():
    """DeepSeek-V3 expert shape (D=7168, F=2048) with 16 experts of a
    top-8-of-2048 routing (M=16384); 12 sampled rows per expert."""
    M, D, F, E = 16384, 7168, 2048, 16
    gs = make_group_sizes(M, E)
    (qg, sg), (qu, su), (qd, sd) = _fp8_weights(E, D, F, seed=5)
    wgu, sgu = swiglu_interleave_fp8(qg, qu, sg, su)
    x = _x(M, D, seed=5)
    y = fused_ragged_swiglu(x, wgu, qd, torch.from_numpy(gs).to(DEV), w_gate_up_scale=sgu, w_down_scale=sd)
    torch.cuda.synchronize()
    offs = orc.group_sizes_to_offsets(gs)
    rng = np.random.default_rng(2)
    refs, gots = [], []
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        rows = np.unique(np.concatenate([rng.integers(a, b, 10), [a, b - 1]]))
        deq = [dequantize_e4m3_blockwise(q[e:e + 1], s[e:e + 1]).cpu().numpy() for q, s in ((qg, sg), (qu, su), (qd, sd))]
        refs.append(orc.ref_ragged_swiglu(_np(x[rows]), *deq, [len(rows)]))
        gots.append(y[rows].cpu().numpy())
    m = orc.correctness_metrics(np.concatenate(refs), np.concatenate(gots))
    assert m["fused_is_finite"] and m["l2_relative_error"] <= FP8_TOL, m
