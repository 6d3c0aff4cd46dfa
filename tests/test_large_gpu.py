"""Parity of the large-D path (two grouped GEMMs on CTA pairs, bf16) against
the CPU oracle.  Tolerance: L2 relative error <= 1e-2 against the float64
oracle on the bf16-rounded inputs, the bf16 bar of this library."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src.kernel import fused_ragged_mlp
from src.routing import CONFIGS, config_group_sizes, make_inputs_numpy, with_shape, zipf_group_sizes

import parity_checks

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    for key in (1, 2, 4):
        _lib.set_tuning(key, 0)
    assert _lib.device_status(reset=True) == 0


def _run_bf16(x, wu, wd, gs, out=None):
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    wut = torch.from_numpy(wu).to(dev).to(torch.bfloat16)
    wdt = torch.from_numpy(wd).to(dev).to(torch.bfloat16)
    y = fused_ragged_mlp(xt, wut, wdt, torch.as_tensor(np.asarray(gs, np.int32)), out=out)
    torch.cuda.synchronize()
    return y.cpu().numpy(), xt.float().cpu().numpy(), wut.float().cpu().numpy(), wdt.float().cpu().numpy()


@pytest.mark.parametrize("M,D,F,E", [(2048, 512, 1024, 4), (1536, 768, 512, 3), (2048, 1024, 768, 2)])
def test_large_d_full_oracle(M, D, F, E):
    gs = config_group_sizes(CONFIGS["c1"].__class__("t", M, D, F, E, "bf16", "multinomial"), seed=M + D)
    x, wu, wd = make_inputs_numpy(M, D, F, E, seed=D)
    y, x, wu, wd = _run_bf16(x, wu, wd, gs)
    ref = orc.ref_ragged_mlp(x, wu, wd, gs)
    m = orc.correctness_metrics(ref, y)
    assert m["fused_is_finite"] and m["l2_relative_error"] <= TOL, m


@pytest.mark.parametrize("gs", [
    [0, 700, 0, 5],         # empty experts; one tiny expert
    [255, 257, 1, 511],     # 256-row block boundaries
    [300, 0, 0, 0],         # sum < M, trailing rows zero
    [0, 0, 0, 0],           # nothing routed
])
def test_large_d_ragged_edges(gs):
    M, D, F, E = 1024, 512, 512, 4
    x, wu, wd = make_inputs_numpy(M, D, F, E, seed=5)
    out = torch.full((M, D), float("nan"), device="cuda:0")
    y, x, wu, wd = _run_bf16(x, wu, wd, gs, out=out)
    tail = int(np.sum(gs))
    assert np.all(np.isfinite(y))
    assert np.all(y[tail:] == 0.0)
    if tail:
        ref = orc.ref_ragged_mlp(x, wu, wd, gs)
        m = orc.correctness_metrics(ref[:tail], y[:tail])
        assert m["l2_relative_error"] <= TOL, m


def test_large_d_zipf_many_experts():
    M, D, F, E = 4096, 512, 1024, 16
    gs = zipf_group_sizes(M, E, np.random.default_rng(3))
    x, wu, wd = make_inputs_numpy(M, D, F, E, seed=9)
    y, x, wu, wd = _run_bf16(x, wu, wd, gs)
    ref = orc.ref_ragged_mlp(x, wu, wd, gs)
    m = orc.correctness_metrics(ref, y)
    assert m["l2_relative_error"] <= TOL, m


def _mixtral_inputs(cfg, seed):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((cfg.M, cfg.D), generator=g, device=dev).to(torch.bfloat16)
    wu = (torch.randn((cfg.E, cfg.D, cfg.F), generator=g, device=dev) / cfg.D ** 0.5).to(torch.bfloat16)
    wd = (torch.randn((cfg.E, cfg.F, cfg.D), generator=g, device=dev) / cfg.F ** 0.5).to(torch.bfloat16)
    return x, wu, wd


@pytest.mark.parametrize("tokens", [16384, 32768])
def test_mixtral_shape_every_expert_every_block(tokens):
    """The C4 shape (D=4096, F=14336, E=8, top-2 router) at 16384 tokens
    (M = 32768, the benchmarked configuration) and 32768 tokens (M = 65536,
    the bf16 target point of at least 64K routed rows).  Inputs are generated
    on the device.  The float64 oracle checks, per row, every expert's first
    and last row and one row in each of its 128-row blocks; an fp32 torch
    recomputation screens every row, per 128-row block."""
    cfg = with_shape(CONFIGS["c4"], M=2 * tokens, tokens=tokens)
    gs = config_group_sizes(cfg, seed=0)
    assert gs.sum() == cfg.M
    x, wu, wd = _mixtral_inputs(cfg, seed=tokens)
    dev = x.device
    out = torch.full((cfg.M, cfg.D), float("nan"), device=dev)
    y = fused_ragged_mlp(x, wu, wd, torch.from_numpy(gs).to(dev), out=out)
    torch.cuda.synchronize()
    o = parity_checks.oracle_rows_check(x, lambda e: wu[e], lambda e: wd[e], gs, y, TOL, seed=tokens)
    assert o["experts"] == int(np.count_nonzero(gs))
    assert o["rows"] >= cfg.M // 128
    s = parity_checks.torch_screen(x, lambda e: wu[e], lambda e: wd[e], gs, y, TOL)
    assert s["blocks"] >= cfg.M // 128
