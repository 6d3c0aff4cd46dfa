"""fused_ragged_dot_caller inside a CUDA graph: a call captured once and
replayed with new inputs (copied into the captured buffers) gives the Y of
the eager call -- equal up to the order of the reduce-adds of F-split
launches (float additions in another order), within 1e-5 relative.
Replaying removes the host-side cost of small calls."""

import numpy as np
import pytest
import torch

from src import _lib
from src.kernel import fused_ragged_dot_caller
from src.routing import make_group_sizes, zipf_group_sizes

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _status():
    _lib.device_status(reset=True)
    yield
    assert _lib.device_status(reset=True) == 0


@pytest.mark.parametrize("M,D,F,E,dt", [(512, 128, 512, 4, torch.float32), (1024, 512, 1024, 4, torch.bfloat16),
                                        (256, 256, 1024, 8, torch.bfloat16)])
def test_captured_call_matches_eager(M, D, F, E, dt):
    g = torch.Generator(device=DEV)
    g.manual_seed(M + D)
    x = torch.randn((M, D), generator=g, device=DEV).to(dt)
    wu = (torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5).to(dt)
    wd = (torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5).to(dt)
    gs = torch.from_numpy(make_group_sizes(M, E)).to(DEV)
    out = torch.empty((M, D), device=DEV)
    call = lambda: fused_ragged_dot_caller(x, wu, wd, gs, max_group_size=M, out=out)  # noqa: E731
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()                                     # first call on the device outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    rng = np.random.default_rng(M)
    for step in range(3):                          # new inputs each replay, same shapes
        x.copy_(torch.randn((M, D), generator=g, device=DEV).to(dt))
        new_gs = zipf_group_sizes(M - 16 * step, E, rng) if step else make_group_sizes(M - 7, E)
        gs.copy_(torch.from_numpy(new_gs))
        graph.replay()
        torch.cuda.synchronize()
        got = out.clone()
        want = fused_ragged_dot_caller(x, wu, wd, gs, max_group_size=M)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6, msg=f"replay {step}")
    del graph
