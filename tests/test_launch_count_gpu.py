"""moe_fused_mlp_launch_count (the bench's `gpu_launches`) and the launch
plan of moe_describe_plan (the analytic model's input) against the kernels a
call actually launches, recorded with torch's profiler."""

import pytest
import torch

from src import _lib
from src.kernel import fused_ragged_dot_caller
from src.routing import make_group_sizes, quantize_e4m3_blockwise

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _library_kernels(fn) -> list[str]:
    """Names of the library's kernels one call launches, in launch order."""
    from torch.profiler import ProfilerActivity, profile
    fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    events = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    if not events:
        pytest.skip("the profiler recorded no GPU activity on this box")
    events.sort(key=lambda e: e.time_range.start)
    return [e.name for e in events if "moe::" in e.name]


@pytest.mark.parametrize("M,D,F,E,dt", [
    (4096, 128, 1024, 8, "f32"),     # weight split + fused kernel
    (16384, 128, 512, 4, "bf16"),    # one wave of whole blocks: the fused kernel alone
    (512, 128, 512, 4, "bf16"),      # F split across CTAs: Y zeroed first
    (1024, 512, 1024, 4, "bf16"),    # two grouped GEMMs
    (1024, 512, 1024, 4, "fp8"),     # two grouped GEMMs (weights decoded in shared memory)
    (1024, 320, 448, 4, "f32"),      # tf32 split + two 3xTF32 grouped GEMMs
])
def test_launch_count_matches_launched_kernels(M, D, F, E, dt):
    g = torch.Generator(device=DEV)
    g.manual_seed(1)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    x = torch.randn((M, D), generator=g, device=DEV).to(tdt)
    wu = torch.randn((E, D, F), generator=g, device=DEV) / D ** 0.5
    wd = torch.randn((E, F, D), generator=g, device=DEV) / F ** 0.5
    kw = {}
    if dt == "fp8":
        (wu, su), (wd, sd) = quantize_e4m3_blockwise(wu), quantize_e4m3_blockwise(wd)
        kw = {"w_up_scale": su, "w_down_scale": sd}
    else:
        wu, wd = wu.to(tdt), wd.to(tdt)
    gs = torch.from_numpy(make_group_sizes(M, E)).to(DEV)
    out = torch.empty((M, D), device=DEV)
    code = {"f32": _lib.MOE_DTYPE_F32, "bf16": _lib.MOE_DTYPE_BF16, "fp8": _lib.MOE_DTYPE_FP8_E4M3_BLK128}[dt]
    claimed = _lib.lib().moe_fused_mlp_launch_count(M, D, F, E, code)
    names = _library_kernels(lambda: fused_ragged_dot_caller(x, wu, wd, gs, max_group_size=M, out=out, **kw))
    assert len(names) == claimed, (names, claimed)
    plan = _lib.describe_plan(M, D, F, E, code, sms=torch.cuda.get_device_properties(DEV).multi_processor_count)
    assert len(plan) == claimed
    for launched, planned in zip(names, plan):
        assert planned["kernel"].split()[0] in launched, (launched, planned["kernel"])
