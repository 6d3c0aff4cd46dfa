"""Training kernels (bf16) against the float64 oracle on the bf16-rounded
inputs: the forward with the saved pre-activation, and the backward's dX,
dW_up and dW_down.  Tolerance: L2 relative error <= 1e-2 per gradient, the
bf16 bar of the forward (dY, dA and GELU(A) are rounded to bf16 for the
tensor cores)."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src.kernel import fused_ragged_mlp
from src.routing import make_group_sizes, zipf_group_sizes
from src.train import backward, forward_train, fused_ragged_mlp_train

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0


def _inputs(M, D, F, E, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn((M, D), generator=g, device=DEV).to(torch.bfloat16)
    wu = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    wd = (torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5).to(torch.bfloat16)
    dy = torch.randn((M, D), generator=g, device=DEV)
    return x, wu, wd, dy


def _np(t):
    return t.double().cpu().numpy()


def _rel(ref, got):
    ref, got = np.asarray(ref, np.float64), np.asarray(got, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def test_forward_train_matches_forward_and_saves_preactivation():
    M, D, F, E = 2048, 512, 1024, 4
    gs = make_group_sizes(M - 100, E)
    x, wu, wd, _ = _inputs(M, D, F, E, seed=1)
    gst = torch.from_numpy(gs).to(DEV)
    y, a = forward_train(x, wu, wd, gst)
    y_ref = fused_ragged_mlp(x, wu, wd, gst)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)  # same GEMMs and epilogue arithmetic
    n = int(gs.sum())
    pre = orc.ragged_dot(_np(x), _np(wu), gs, np.float64)
    assert _rel(pre[:n], _np(a[:n])) <= 4e-3  # bf16 rounding of A


@pytest.mark.parametrize("M,D,F,E,dy_dtype", [
    (1024, 256, 256, 2, torch.float32),
    (2048, 512, 1024, 4, torch.float32),
    (2048, 512, 1024, 4, torch.bfloat16),
    (1536, 768, 512, 3, torch.float32),
])
def test_backward_full_oracle(M, D, F, E, dy_dtype):
    gs = make_group_sizes(M, E)
    x, wu, wd, dy = _inputs(M, D, F, E, seed=D + F)
    dy = dy.to(dy_dtype)
    gst = torch.from_numpy(gs).to(DEV)
    _, a = forward_train(x, wu, wd, gst)
    dx, dwu, dwd = backward(x, wu, wd, gst, a, dy)
    torch.cuda.synchronize()
    rx, rwu, rwd = orc.ref_ragged_mlp_backward(_np(x), _np(wu), _np(wd), gs, _np(dy))
    for name, r, g in (("dx", rx, dx), ("dw_up", rwu, dwu), ("dw_down", rwd, dwd)):
        got = g.cpu().numpy()
        assert np.all(np.isfinite(got)), name
        assert _rel(r, got) <= TOL, (name, _rel(r, got))


@pytest.mark.parametrize("gs", [
    [0, 700, 0, 5],         # empty experts; one tiny expert
    [255, 257, 1, 511],     # 64- and 256-row boundaries
    [300, 0, 0, 0],         # sum < M: trailing rows carry no gradient
    [0, 0, 0, 0],           # nothing routed: every gradient is zero
])
def test_backward_ragged_edges(gs):
    M, D, F, E = 1024, 512, 512, 4
    x, wu, wd, dy = _inputs(M, D, F, E, seed=7)
    gst = torch.tensor(gs, dtype=torch.int32)
    _, a = forward_train(x, wu, wd, gst)
    dx, dwu, dwd = backward(x, wu, wd, gst, a, dy)
    torch.cuda.synchronize()
    dx, dwu, dwd = dx.cpu().numpy(), dwu.cpu().numpy(), dwd.cpu().numpy()
    n = int(np.sum(gs))
    assert np.all(dx[n:] == 0.0)
    for e, g in enumerate(gs):
        if g == 0:
            assert np.all(dwu[e] == 0.0) and np.all(dwd[e] == 0.0)
    if n:
        rx, rwu, rwd = orc.ref_ragged_mlp_backward(_np(x), _np(wu), _np(wd), gs, _np(dy))
        assert _rel(rx, dx) <= TOL and _rel(rwu, dwu) <= TOL and _rel(rwd, dwd) <= TOL


def test_backward_zipf_many_experts():
    M, D, F, E = 4096, 512, 768, 16
    gs = zipf_group_sizes(M, E, np.random.default_rng(3))
    x, wu, wd, dy = _inputs(M, D, F, E, seed=11)
    gst = torch.from_numpy(gs).to(DEV)
    _, a = forward_train(x, wu, wd, gst)
    dx, dwu, dwd = backward(x, wu, wd, gst, a, dy)
    torch.cuda.synchronize()
    rx, rwu, rwd = orc.ref_ragged_mlp_backward(_np(x), _np(wu), _np(wd), gs, _np(dy))
    assert _rel(rx, dx.cpu().numpy()) <= TOL
    assert _rel(rwu, dwu.cpu().numpy()) <= TOL
    assert _rel(rwd, dwd.cpu().numpy()) <= TOL


def test_autograd_function_matches_torch_autograd():
    M, D, F, E = 1024, 256, 512, 3
    gs = make_group_sizes(M - 30, E)
    x, wu, wd, dy = _inputs(M, D, F, E, seed=5)
    xs, wus, wds = (t.clone().requires_grad_(True) for t in (x, wu, wd))
    y = fused_ragged_mlp_train(xs, wus, wds, torch.from_numpy(gs).to(DEV))
    y.backward(dy)
    xr, wur, wdr = (t.float().clone().requires_grad_(True) for t in (x, wu, wd))
    offs = np.concatenate([[0], np.cumsum(gs)])
    parts = [torch.nn.functional.gelu(xr[offs[e]:offs[e + 1]] @ wur[e], approximate="tanh") @ wdr[e]
             for e in range(E)]
    yr = torch.cat(parts + [torch.zeros((M - int(offs[-1]), D), device=DEV)])
    yr.backward(dy)
    for g, r in ((xs.grad, xr.grad), (wus.grad, wur.grad), (wds.grad, wdr.grad)):
        assert g.dtype == torch.bfloat16
        assert _rel(r.double().cpu().numpy(), g.double().cpu().numpy()) <= 2e-2


def test_backward_mixtral_shape_sampled():
    """Mixtral-8x7B experts (D=4096, F=14336, E=8), top-2 of 16384 tokens ->
    M=32768.  dX is checked on 12 sampled rows per expert (a row's gradient
    depends only on its own X and dY rows); dW_up[:, f] and dW_down[f, :] on
    8 sampled hidden units per expert (a unit's weight gradients depend only
    on its own weights), each against the oracle on that slice."""
    M, D, F, E = 32768, 4096, 14336, 8
    gs = make_group_sizes(M, E)
    x, wu, wd, dy = _inputs(M, D, F, E, seed=0)
    gst = torch.from_numpy(gs).to(DEV)
    _, a = forward_train(x, wu, wd, gst)
    dx, dwu, dwd = backward(x, wu, wd, gst, a, dy)
    torch.cuda.synchronize()
    del a
    offs = orc.group_sizes_to_offsets(gs)
    rng = np.random.default_rng(1)
    ref_x, got_x, ref_w, got_w = [], [], [], []
    f32 = np.float32
    for e in range(E):
        lo, hi = int(offs[e]), int(offs[e + 1])
        rows = np.unique(np.concatenate([rng.integers(lo, hi, 10), [lo, hi - 1]]))
        wue, wde = wu[e].float().cpu().numpy(), wd[e].float().cpu().numpy()
        rx, _, _ = orc.ref_ragged_mlp_backward(x[rows].float().cpu().numpy(), wue[None], wde[None], [len(rows)],
                                               dy[rows].cpu().numpy(), acc_dtype=f32)
        ref_x.append(rx)
        got_x.append(dx[rows].cpu().numpy())
        cols = np.sort(rng.choice(F, 8, replace=False))
        xe, dye = x[lo:hi].float().cpu().numpy(), dy[lo:hi].cpu().numpy()
        _, rwu, rwd = orc.ref_ragged_mlp_backward(xe, wue[:, cols][None], wde[cols, :][None], [hi - lo], dye,
                                                  acc_dtype=f32)
        ref_w += [rwu[0], rwd[0].T]
        got_w += [dwu[e][:, cols].cpu().numpy(), dwd[e][cols, :].cpu().numpy().T]
    assert _rel(np.concatenate(ref_x), np.concatenate(got_x)) <= TOL
    assert _rel(np.concatenate(ref_w), np.concatenate(got_w)) <= TOL


# ----------------------------------------------------------------------------- SwiGLU experts
from src.kernel import fused_ragged_swiglu, swiglu_interleave  # noqa: E402
from src.train import fused_ragged_swiglu_train, swiglu_backward, swiglu_forward_train  # noqa: E402


def _swiglu_inputs(M, D, F, E, seed):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn((M, D), generator=g, device=DEV).to(torch.bfloat16)
    wg = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    wu = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(torch.bfloat16)
    wd = (torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5).to(torch.bfloat16)
    dy = torch.randn((M, D), generator=g, device=DEV)
    return x, wg, wu, wd, dy


def test_swiglu_forward_train_matches_forward_and_saves_gate_up():
    M, D, F, E = 2048, 512, 512, 4
    gs = make_group_sizes(M - 64, E)
    x, wg, wu, wd, _ = _swiglu_inputs(M, D, F, E, seed=3)
    wgu = swiglu_interleave(wg, wu)
    gst = torch.from_numpy(gs).to(DEV)
    y, gu = swiglu_forward_train(x, wgu, wd, gst)
    y_ref = fused_ragged_swiglu(x, wgu, wd, gst)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    n = int(gs.sum())
    pre = orc.ragged_dot(_np(x), orc.swiglu_interleave(_np(wg), _np(wu)), gs, np.float64)
    assert _rel(pre[:n], _np(gu[:n])) <= 4e-3


@pytest.mark.parametrize("M,D,F,E,gs", [
    (2048, 512, 512, 4, None),
    (1536, 768, 256, 3, None),
    (1024, 512, 512, 4, [0, 700, 0, 5]),
    (1024, 512, 512, 4, [300, 0, 0, 0]),
])
def test_swiglu_backward_full_oracle(M, D, F, E, gs):
    gs = make_group_sizes(M, E) if gs is None else np.asarray(gs, np.int32)
    x, wg, wu, wd, dy = _swiglu_inputs(M, D, F, E, seed=M + F)
    wgu = swiglu_interleave(wg, wu)
    gst = torch.from_numpy(gs).to(DEV)
    _, gu = swiglu_forward_train(x, wgu, wd, gst)
    dx, dwgu, dwd = swiglu_backward(x, wgu, wd, gst, gu, dy)
    torch.cuda.synchronize()
    rx, rwg, rwu, rwd = orc.ref_ragged_swiglu_backward(_np(x), _np(wg), _np(wu), _np(wd), gs, _np(dy))
    n = int(gs.sum())
    dx = dx.cpu().numpy()
    assert np.all(dx[n:] == 0.0)
    for e, g in enumerate(gs):
        if g == 0:
            assert torch.all(dwgu[e] == 0) and torch.all(dwd[e] == 0)
    assert _rel(rx, dx) <= TOL
    assert _rel(orc.swiglu_interleave(rwg, rwu), dwgu.cpu().numpy()) <= TOL
    assert _rel(rwd, dwd.cpu().numpy()) <= TOL


def test_swiglu_autograd_matches_torch_autograd():
    M, D, F, E = 1024, 256, 256, 3
    gs = make_group_sizes(M - 40, E)
    x, wg, wu, wd, dy = _swiglu_inputs(M, D, F, E, seed=21)
    wgu = swiglu_interleave(wg, wu)
    xs, wgus, wds = (t.clone().requires_grad_(True) for t in (x, wgu, wd))
    fused_ragged_swiglu_train(xs, wgus, wds, torch.from_numpy(gs).to(DEV)).backward(dy)
    xr, wgr, wur, wdr = (t.float().clone().requires_grad_(True) for t in (x, wg, wu, wd))
    offs = np.concatenate([[0], np.cumsum(gs)])
    parts = [(torch.nn.functional.silu(xr[offs[e]:offs[e + 1]] @ wgr[e]) * (xr[offs[e]:offs[e + 1]] @ wur[e])) @ wdr[e]
             for e in range(E)]
    torch.cat(parts + [torch.zeros((M - int(offs[-1]), D), device=DEV)]).backward(dy)
    assert _rel(xr.grad.double().cpu().numpy(), xs.grad.double().cpu().numpy()) <= 2e-2
    ref_gu = swiglu_interleave(wgr.grad.bfloat16(), wur.grad.bfloat16())
    assert _rel(ref_gu.double().cpu().numpy(), wgus.grad.double().cpu().numpy()) <= 2e-2
    assert _rel(wdr.grad.double().cpu().numpy(), wds.grad.double().cpu().numpy()) <= 2e-2
