"""Shapes outside the fused small-D kernels: the grouped-GEMM path with
partial tiles, for every precision.

The reference's entry point accepts any D (it asserts only D == D2, M % BM
and F % BF, ``src/kernel.py:97-102``) and its published sweep runs f32 at
D = 512 and 1024 (``results/structured_float32/config.json:12-18``).  Here:

* f32 with D outside {64, 128, 256} (or F % 64 != 0) runs the two grouped
  GEMMs in 3xTF32 (kind::tf32, hi/lo planes): L2 relative error <= 1e-5
  against the float64 oracle, plus the reference's own gate;
* bf16 and e4m3-weight shapes whose D or F is not a multiple of the 256-wide
  tiles (N tails masked at the store, K tails read as zeros through 3-D
  weight maps): <= 1e-2 and <= 2e-2;
* the ragged edges (empty experts, block boundaries, sum(gs) < M into a
  NaN-poisoned output, nothing routed) and the prepared-weights form.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src.kernel import fused_ragged_mlp
from src.routing import dequantize_e4m3_blockwise, make_inputs_numpy, multinomial_group_sizes, quantize_e4m3_blockwise

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2}


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0


def _run(M, D, F, E, gs, dtype, seed, out=None):
    x, wu, wd = make_inputs_numpy(M, D, F, E, seed=seed)
    xt, wut, wdt = (torch.from_numpy(a).to(DEV, dtype) for a in (x, wu, wd))
    y = fused_ragged_mlp(xt, wut, wdt, torch.as_tensor(np.asarray(gs, np.int32)), out=out)
    torch.cuda.synchronize()
    return y.cpu().numpy(), *(t.double().cpu().numpy() for t in (xt, wut, wdt))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,D,F,E", [
    (2048, 320, 448, 4),     # D and F not multiples of 64: N and K tails in both GEMMs
    (2048, 512, 512, 4),     # the reference sweep's D = 512 (f32 failed here before)
    (1024, 1024, 512, 2),    # D = 1024
    (1536, 128, 200, 3),     # small D whose F the fused kernel does not take
    (1024, 192, 1000, 2),    # K = F = 1000 in the down GEMM: a 40-column K tail
    (768, 40, 24, 3),        # tiny D and F: one partial tile each way
])
def test_generic_shapes_full_oracle(M, D, F, E, dtype):
    gs = multinomial_group_sizes(M, E, np.random.default_rng(M + D + F))
    y, x, wu, wd = _run(M, D, F, E, gs, dtype, seed=D + F)
    ref = orc.ref_ragged_mlp(x, wu, wd, gs)
    m = orc.correctness_metrics(ref, y)
    assert m["fused_is_finite"] and m["l2_relative_error"] <= TOL[dtype], m
    if dtype == torch.float32:  # the reference's own gate as well (src/benchmark.py:250-256)
        assert m["l2_relative_error"] < 1e-4 and m["normalized_max_error"] < 1e-3, m


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("gs", [
    [0, 700, 0, 5],          # empty experts; one tiny expert
    [255, 257, 1, 511],      # 256-row block boundaries
    [300, 0, 0, 0],          # sum < M: trailing rows zero
    [0, 0, 0, 0],            # nothing routed
])
def test_generic_shapes_ragged_edges(gs, dtype):
    M, D, F, E = 1024, 320, 448, 4
    out = torch.full((M, D), float("nan"), device=DEV)
    y, x, wu, wd = _run(M, D, F, E, gs, dtype, seed=11, out=out)
    tail = int(np.sum(gs))
    assert np.all(np.isfinite(y)) and np.all(y[tail:] == 0.0)
    if tail:
        ref = orc.ref_ragged_mlp(x, wu, wd, gs)
        m = orc.correctness_metrics(ref[:tail], y[:tail])
        assert m["l2_relative_error"] <= TOL[dtype], m


def test_f32_large_d_prepared_weights_bit_identical():
    """moe_prepare_weights + moe_fused_mlp_prepared (the tf32 planes built
    once) gives exactly the per-call result of moe_fused_mlp."""
    M, D, F, E = 1024, 512, 384, 3
    x, wu, wd = (torch.from_numpy(a).to(DEV) for a in make_inputs_numpy(M, D, F, E, seed=3))
    gs = torch.from_numpy(multinomial_group_sizes(M - 9, E, np.random.default_rng(3))).to(DEV)
    L = _lib.lib()
    nbytes = int(L.moe_fused_mlp_workspace_size(M, D, F, E, _lib.MOE_DTYPE_F32))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    vp = ctypes.c_void_p
    args = (vp(x.data_ptr()), vp(wu.data_ptr()), vp(wd.data_ptr()), vp(gs.data_ptr()), vp(0), vp(0))
    y1 = torch.full((M, D), float("nan"), device=DEV)
    assert L.moe_fused_mlp(*args, vp(y1.data_ptr()), M, D, F, E, _lib.MOE_DTYPE_F32, vp(ws.data_ptr()), nbytes,
                           st) == 0, L.moe_last_error()
    ws.zero_()
    assert L.moe_prepare_weights(vp(wu.data_ptr()), vp(wd.data_ptr()), vp(0), vp(0), D, F, E, _lib.MOE_DTYPE_F32,
                                 vp(ws.data_ptr()), nbytes, st) == 0, L.moe_last_error()
    y2 = torch.full((M, D), float("nan"), device=DEV)
    assert L.moe_fused_mlp_prepared(*args, vp(y2.data_ptr()), M, D, F, E, _lib.MOE_DTYPE_F32, vp(ws.data_ptr()),
                                    nbytes, st) == 0, L.moe_last_error()
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert int(L.moe_fused_mlp_launch_count(M, D, F, E, _lib.MOE_DTYPE_F32)) == 3


@pytest.mark.parametrize("M,D,F,E,gs", [
    (1024, 320, 448, 4, [300, 0, 500, 200]),   # partial 128-blocks of scales in K and N
    (768, 7168 // 4, 2048 // 4 + 64, 3, [255, 257, 1]),
    (512, 208, 144, 2, [0, 0]),                # nothing routed
])
def test_fp8_generic_shapes(M, D, F, E, gs):
    g = torch.Generator(device=DEV)
    g.manual_seed(M + D)
    x = torch.randn((M, D), generator=g, device=DEV).to(torch.bfloat16)
    wu_q, wu_s = quantize_e4m3_blockwise(torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5)
    wd_q, wd_s = quantize_e4m3_blockwise(torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5)
    assert wu_s.shape == (E, -(-D // 128), -(-F // 128))
    out = torch.full((M, D), float("nan"), device=DEV)
    y = fused_ragged_mlp(x, wu_q, wd_q, torch.tensor(gs, dtype=torch.int32), w_up_scale=wu_s,
                         w_down_scale=wd_s, out=out)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    tail = sum(gs)
    assert np.all(np.isfinite(y)) and np.all(y[tail:] == 0)
    if tail:
        ref = orc.ref_ragged_mlp(x.double().cpu().numpy(), dequantize_e4m3_blockwise(wu_q, wu_s).double().cpu().numpy(),
                                 dequantize_e4m3_blockwise(wd_q, wd_s).double().cpu().numpy(), gs)
        m = orc.correctness_metrics(ref[:tail], y[:tail])
        assert m["l2_relative_error"] <= 2e-2, m


def test_sweep_cases_that_had_no_kernel():
    """The structured sweep's D = 512 and D = 1024 shapes (M=16384, F=512,
    E=4) under all four routing patterns, through the sweep's own case runner
    (drop-in call, the reference algorithm in f32 torch on the GPU, the
    reference's gate): every case passes."""
    from src import sweep
    for D in (512, 1024):
        for pattern in ("balanced", "mild", "skewed", "one_dominant"):
            row = sweep.run_case(16384, D, 512, 4, pattern, seed=0, warmup=1, iterations=2, device=DEV)
            assert row["numerically_acceptable"], (D, pattern, row["l2_relative_error"], row["normalized_max_error"])
