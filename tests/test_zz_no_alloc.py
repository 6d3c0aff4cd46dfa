"""moe_fused_mlp_noalloc -- the allocation-free entry point for callers that
hold only their input and output buffers and have no way to get device
scratch (e.g. a runtime handing raw device pointers through an FFI without
an allocator, or a service that forbids allocation on its request path).

Both entry points are called through the C ABI.  The allocation-free one
must give the same Y as moe_fused_mlp with a caller workspace, within the
f32 (3xTF32) tolerance of the other tests, on consecutive calls whose shapes
differ (so the second call runs over the first call's leftover scratch), and
must refuse problems larger than its static scratch with an error instead of
touching memory.  This file is collected last so that a run stopping at the
first failure has already run every other test."""

import ctypes

import numpy as np
import pytest
import torch

from src import _lib
from src.routing import make_inputs_numpy, multinomial_group_sizes

pytestmark = pytest.mark.gpu
TOL = 1e-5  # f32 (3xTF32) tolerance used by the other parity tests

vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64


def _lib_bound():
    L = _lib.lib()
    L.moe_fused_mlp_noalloc.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, vp]
    L.moe_fused_mlp_noalloc.restype = ctypes.c_int
    return L


def _inputs(M, D, F, E, seed):
    dev = torch.device("cuda:0")
    x, wu, wd = make_inputs_numpy(M, D, F, E, seed=seed)
    gs = multinomial_group_sizes(M - 7, E, np.random.default_rng(seed))  # 7 unrouted rows
    return (torch.from_numpy(x).to(dev), torch.from_numpy(wu).to(dev), torch.from_numpy(wd).to(dev),
            torch.from_numpy(gs).to(dev))


def _stream():
    return vp(torch.cuda.current_stream().cuda_stream)


def _run_noalloc(L, x, wu, wd, gs, M, D, F, E):
    y = torch.full((M, D), float("nan"), device=x.device)
    rc = L.moe_fused_mlp_noalloc(vp(x.data_ptr()), vp(wu.data_ptr()), vp(wd.data_ptr()), vp(gs.data_ptr()),
                                 vp(y.data_ptr()), M, D, F, E, _stream())
    return rc, y


def _run_with_workspace(L, x, wu, wd, gs, M, D, F, E):
    y = torch.empty((M, D), device=x.device)
    nbytes = int(L.moe_fused_mlp_workspace_size(M, D, F, E, _lib.MOE_DTYPE_F32))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    rc = L.moe_fused_mlp(vp(x.data_ptr()), vp(wu.data_ptr()), vp(wd.data_ptr()), vp(gs.data_ptr()), vp(0), vp(0),
                         vp(y.data_ptr()), M, D, F, E, _lib.MOE_DTYPE_F32, vp(ws.data_ptr()), nbytes, _stream())
    return rc, y


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    L = _lib_bound()
    # Second call: other shape, other experts; it runs over the scratch the
    # first call left behind.
    for M, D, F, E, seed in [(4096, 128, 1024, 8, 0), (3000, 64, 512, 16, 1)]:
        x, wu, wd, gs = _inputs(M, D, F, E, seed)
        rc, y = _run_noalloc(L, x, wu, wd, gs, M, D, F, E)
        assert rc == 0, L.moe_last_error().decode()
        rc, y_ref = _run_with_workspace(L, x, wu, wd, gs, M, D, F, E)
        assert rc == 0, L.moe_last_error().decode()
        torch.cuda.synchronize()
        y, y_ref = y.cpu().double(), y_ref.cpu().double()
        assert torch.isfinite(y).all()
        rel = float(torch.linalg.norm(y - y_ref) / torch.linalg.norm(y_ref))
        assert rel <= TOL, rel
        assert torch.all(y[M - 7:] == 0)
    assert _lib.device_status(reset=True) == 0


def test_noalloc_refuses_problems_above_its_static_scratch():
    L = _lib_bound()
    M, D, F, E = 256, 128, 1024, 16          # E*D*F = 2,097,152 > 1,048,576
    x, wu, wd, gs = _inputs(M, D, F, E, 2)
    rc, y = _run_noalloc(L, x, wu, wd, gs, M, D, F, E)
    assert rc == -4                           # MOE_ERR_WORKSPACE_TOO_SMALL
    assert b"static buffer" in L.moe_last_error()
    torch.cuda.synchronize()
    assert torch.isnan(y).all()               # output untouched


def test_noalloc_warm_calls_leave_device_memory_unchanged():
    """After a first call (module load, scratch address look-up), further
    calls take no device memory: the free bytes the driver reports stay the
    same.  Inputs and outputs are created before the measurement."""
    L = _lib_bound()
    M, D, F, E = 2048, 128, 512, 8
    x, wu, wd, gs = _inputs(M, D, F, E, 3)
    y = torch.empty((M, D), device=x.device)
    args = (vp(x.data_ptr()), vp(wu.data_ptr()), vp(wd.data_ptr()), vp(gs.data_ptr()), vp(y.data_ptr()),
            M, D, F, E, _stream())
    assert L.moe_fused_mlp_noalloc(*args) == 0, L.moe_last_error().decode()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert L.moe_fused_mlp_noalloc(*args) == 0, L.moe_last_error().decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert _lib.device_status(reset=True) == 0
