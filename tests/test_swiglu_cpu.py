"""SwiGLU experts on the CPU: the oracle's restatement and interleave layout,
and the C-ABI's argument checks (no device work)."""

import ctypes

import numpy as np
import torch

from oracle import moe_oracle as orc
from src import _lib


def test_interleave_layout():
    rng = np.random.default_rng(0)
    E, D, F = 2, 3, 384
    g = rng.standard_normal((E, D, F)).astype(np.float32)
    u = rng.standard_normal((E, D, F)).astype(np.float32)
    w = orc.swiglu_interleave(g, u)
    assert w.shape == (E, D, 2 * F)
    for j in range(F // 128):
        np.testing.assert_array_equal(w[:, :, 256 * j:256 * j + 128], g[:, :, 128 * j:128 * (j + 1)])
        np.testing.assert_array_equal(w[:, :, 256 * j + 128:256 * (j + 1)], u[:, :, 128 * j:128 * (j + 1)])


def test_ref_ragged_swiglu_matches_torch_per_group():
    rng = np.random.default_rng(1)
    M, D, F, E = 40, 16, 24, 3
    gs = [10, 0, 25]                     # sum 35 < M: rows 35.. are zero
    x = rng.standard_normal((M, D))
    wg, wu = rng.standard_normal((E, D, F)), rng.standard_normal((E, D, F))
    wd = rng.standard_normal((E, F, D))
    y = orc.ref_ragged_swiglu(x, wg, wu, wd, gs)
    offs = np.cumsum([0] + gs)
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        xt = torch.from_numpy(x[a:b])
        h = torch.nn.functional.silu(xt @ torch.from_numpy(wg[e])) * (xt @ torch.from_numpy(wu[e]))
        np.testing.assert_allclose(y[a:b], (h @ torch.from_numpy(wd[e])).numpy(), rtol=1e-12, atol=1e-12)
    assert np.all(y[offs[-1]:] == 0)


def test_swiglu_abi_checks_before_device_work():
    L = _lib.lib()
    vp = ctypes.c_void_p
    null = vp(0)
    assert L.moe_fused_mlp_swiglu(null, null, null, null, null, -1, 4096, 14336, 8, null, 0, null) == -1
    assert b"bad sizes" in L.moe_last_error()
    # D not a multiple of 256, F not a multiple of 128 -> unsupported shape.
    assert L.moe_fused_mlp_swiglu(vp(16), vp(16), vp(16), vp(16), vp(16), 16, 384, 1024, 8, null, 0, null) == -2
    assert L.moe_fused_mlp_swiglu(vp(16), vp(16), vp(16), vp(16), vp(16), 16, 512, 1000, 8, null, 0, null) == -2
    # M == 0 is a no-op.
    assert L.moe_fused_mlp_swiglu(null, null, null, null, null, 0, 512, 1024, 8, null, 0, null) == 0
    assert L.moe_swiglu_interleave(vp(16), vp(16), vp(16), 8, 512, 1000, null) == -1
    assert L.moe_swiglu_interleave(null, vp(16), vp(16), 8, 512, 1024, null) == -1
    assert L.moe_swiglu_interleave(vp(8), vp(16), vp(16), 8, 512, 1024, null) == -7


def test_swiglu_workspace_size():
    L = _lib.lib()
    assert L.moe_fused_mlp_swiglu_workspace_size(32768, 4096, 14336) == 32768 * 14336 * 2
    assert L.moe_fused_mlp_swiglu_workspace_size(3, 256, 128) == 768
    assert L.moe_fused_mlp_swiglu_workspace_size(16, 384, 128) == 0
