"""FP8 e4m3 block-scaled weights (bf16 X, 128x128 f32 block scales) through
the large-D grouped GEMMs.  Tolerance: L2 relative error <= 2e-2 against the
float64 oracle on the dequantised weights, the FP8 bar of this library."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src.kernel import fused_ragged_mlp
from src.routing import CONFIGS, config_group_sizes, dequantize_e4m3_blockwise, quantize_e4m3_blockwise

import parity_checks

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0


def _make(M, D, F, E, seed):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((M, D), generator=g, device=dev).to(torch.bfloat16)
    wu = torch.randn((E, D, F), generator=g, device=dev) / D ** 0.5
    wd = torch.randn((E, F, D), generator=g, device=dev) / F ** 0.5
    wu_q, wu_s = quantize_e4m3_blockwise(wu)
    wd_q, wd_s = quantize_e4m3_blockwise(wd)
    return x, wu_q, wu_s, wd_q, wd_s


def test_quantizer_round_trip():
    w = torch.randn((2, 256, 384)) * 0.05
    q, s = quantize_e4m3_blockwise(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (2, 2, 3)
    back = dequantize_e4m3_blockwise(q, s)
    assert float((back - w).norm() / w.norm()) < 0.05
    # the oracle's own e4m3 decoding agrees with torch's
    codes = q.view(torch.uint8).numpy()
    deq = orc.dequant_block(orc.e4m3_decode(codes), s.numpy())
    np.testing.assert_allclose(deq, back.double().numpy(), rtol=1e-6, atol=1e-12)


@pytest.fixture(params=[1, 2], ids=["row_tiles", "expert_super_tiles"])
def fp8_kernel(request):
    """Both e4m3-weight kernels: row-tiled pair tiles and expert super-tiles."""
    _lib.set_tuning(7, request.param)
    yield request.param
    _lib.set_tuning(7, 0)


@pytest.mark.parametrize("M,D,F,E,gs", [
    (1024, 512, 512, 4, [300, 0, 500, 200]),
    (768, 256, 768, 3, [255, 257, 1]),        # D = 256 also takes this path for FP8
    (512, 512, 256, 2, [0, 0]),
])
def test_fp8_full_oracle(M, D, F, E, gs, fp8_kernel):
    x, wu_q, wu_s, wd_q, wd_s = _make(M, D, F, E, seed=M + D)
    out = torch.full((M, D), float("nan"), device="cuda:0")
    y = fused_ragged_mlp(x, wu_q, wd_q, torch.tensor(gs, dtype=torch.int32), w_up_scale=wu_s,
                         w_down_scale=wd_s, out=out)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    tail = sum(gs)
    assert np.all(np.isfinite(y)) and np.all(y[tail:] == 0)
    if tail:
        ref = orc.ref_ragged_mlp(x.float().cpu().numpy(), dequantize_e4m3_blockwise(wu_q, wu_s).cpu().numpy(),
                                 dequantize_e4m3_blockwise(wd_q, wd_s).cpu().numpy(), gs)
        m = orc.correctness_metrics(ref[:tail], y[:tail])
        assert m["l2_relative_error"] <= TOL, m


@pytest.mark.parametrize("gs", [
    [1, 31, 32, 33, 64, 96, 127, 128],         # chunk sizes around the 32-token MMA step
    [255, 256, 257, 383, 384, 385, 0, 0],      # chunk 0 / chunk 1 / next super-tile boundaries
    [700, 0, 0, 0, 0, 0, 0, 1069],             # several super-tiles per expert; sum < M
    [0, 0, 0, 0, 0, 0, 0, 0],                  # nothing routed
])
def test_fp8_super_tile_edges(gs, fp8_kernel):
    """Expert sizes at every chunk and super-tile boundary of the expert
    super-tile kernel (and the same cases through the row-tiled kernel), with
    a feature count that leaves a partial 256-feature block (F = 448) and a
    NaN-poisoned output: rows past sum(gs) must come back as zeros."""
    M, D, F, E = 2048, 384, 448, 8
    x, wu_q, wu_s, wd_q, wd_s = _make(M, D, F, E, seed=sum(gs) + 1)
    out = torch.full((M, D), float("nan"), device="cuda:0")
    y = fused_ragged_mlp(x, wu_q, wd_q, torch.tensor(gs, dtype=torch.int32), w_up_scale=wu_s,
                         w_down_scale=wd_s, out=out)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    tail = sum(gs)
    assert np.all(np.isfinite(y)) and np.all(y[tail:] == 0)
    if tail:
        ref = orc.ref_ragged_mlp(x.float().cpu().numpy(), dequantize_e4m3_blockwise(wu_q, wu_s).cpu().numpy(),
                                 dequantize_e4m3_blockwise(wd_q, wd_s).cpu().numpy(), gs)
        errs = [orc.correctness_metrics(ref[a:b], y[a:b])["l2_relative_error"]
                for a, b in zip(np.cumsum([0] + gs[:-1]), np.cumsum(gs)) if b > a]
        assert max(errs) <= TOL, errs


def test_c5_deepseek_shape_every_expert_every_block():
    """Full C5 shape: D=7168, F=2048, E=256, top-8 softmax router over 8192
    tokens -> M=65536 routed rows (the automatic kernel choice: expert
    super-tiles).  The float64 oracle (on the dequantised
    weights) checks, per row, every expert's first and last row and one row
    in each of its 128-row blocks; an fp32 torch recomputation screens every
    row, per 128-row block."""
    cfg = CONFIGS["c5"]
    gs = config_group_sizes(cfg, seed=0)
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x = torch.randn((cfg.M, cfg.D), generator=g, device=dev).to(torch.bfloat16)
    wu_q = torch.empty((cfg.E, cfg.D, cfg.F), dtype=torch.float8_e4m3fn, device=dev)
    wd_q = torch.empty((cfg.E, cfg.F, cfg.D), dtype=torch.float8_e4m3fn, device=dev)
    wu_s = torch.empty((cfg.E, cfg.D // 128, cfg.F // 128), device=dev)
    wd_s = torch.empty((cfg.E, cfg.F // 128, cfg.D // 128), device=dev)
    for e in range(cfg.E):
        wu_q[e], wu_s[e] = quantize_e4m3_blockwise(torch.randn((cfg.D, cfg.F), generator=g, device=dev) / cfg.D ** 0.5)
        wd_q[e], wd_s[e] = quantize_e4m3_blockwise(torch.randn((cfg.F, cfg.D), generator=g, device=dev) / cfg.F ** 0.5)
    out = torch.full((cfg.M, cfg.D), float("nan"), device=dev)
    y = fused_ragged_mlp(x, wu_q, wd_q, torch.from_numpy(gs).to(dev), w_up_scale=wu_s, w_down_scale=wd_s, out=out)
    torch.cuda.synchronize()
    wu_f = lambda e: dequantize_e4m3_blockwise(wu_q[e], wu_s[e])  # noqa: E731
    wd_f = lambda e: dequantize_e4m3_blockwise(wd_q[e], wd_s[e])  # noqa: E731
    o = parity_checks.oracle_rows_check(x, wu_f, wd_f, gs, y, TOL, seed=2)
    assert o["experts"] == int(np.count_nonzero(gs))
    assert o["rows"] >= cfg.M // 128
    s = parity_checks.torch_screen(x, wu_f, wd_f, gs, y, TOL)
    assert s["blocks"] >= cfg.M // 128
