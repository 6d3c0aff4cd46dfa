"""ctypes binding of ``libmoe_b200.so`` (declarations: include/moe_b200.h).

There is no fallback: if the library is missing or fails to load, every
entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libmoe_b200.so"

MOE_DTYPE_F32 = 0
MOE_DTYPE_BF16 = 1
MOE_DTYPE_FP8_E4M3_BLK128 = 2
MOE_EP_HANDLE_BYTES = 256

ERRORS = {
    -1: "MOE_ERR_INVALID_ARG",
    -2: "MOE_ERR_UNSUPPORTED_SHAPE",
    -3: "MOE_ERR_UNSUPPORTED_DTYPE",
    -4: "MOE_ERR_WORKSPACE_TOO_SMALL",
    -5: "MOE_ERR_CUDA",
    -6: "MOE_ERR_DEVICE_TIMEOUT",
    -7: "MOE_ERR_MISALIGNED",
}

MMA_KINDS = {0: "none", 1: "kind::f16 (bf16)", 2: "kind::f16 (bf16 from e4m3)", 3: "kind::tf32 x3",
             4: "kind::f16 (f16 from e4m3)"}


class LaunchDesc(ctypes.Structure):
    """``moe_launch_desc`` of include/moe_b200.h."""
    _fields_ = [("kernel", ctypes.c_char * 48)] + [(n, ctypes.c_int32) for n in (
        "grid", "threads", "smem_bytes", "tmem_cols", "cluster", "tile_m", "tile_n", "stage_k", "stages",
        "mma_kind", "gemm_n", "gemm_k", "f_splits", "accumulators", "reserved")]

    def as_dict(self) -> dict:
        d = {n: getattr(self, n) for n, _ in self._fields_ if n not in ("kernel", "reserved")}
        d["kernel"] = self.kernel.decode()
        d["mma"] = MMA_KINDS.get(self.mma_kind, str(self.mma_kind))
        return d


def describe_plan(M: int, D: int, F: int, E: int, dtype: int, sms: int = 148) -> list[dict]:
    """The library's launch plan for one moe_fused_mlp call (no device needed
    when ``sms`` > 0)."""
    arr = (LaunchDesc * 8)()
    n = lib().moe_describe_plan(M, D, F, E, dtype, sms, arr, 8)
    if n < 0:
        raise MoeError(n, lib().moe_last_error().decode())
    return [arr[i].as_dict() for i in range(n)]


_lib = None


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Loads the library once; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MOE_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(f"{path} not found: build it with `python __graft_entry__.py` or "
                           f"`python pallas-moe-kernel_b200/csrc/build.py`")
    L = ctypes.CDLL(str(path))
    vp, sz, i32, i64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_int64
    L.moe_fused_mlp.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp.restype = ctypes.c_int
    L.moe_fused_mlp_prepared.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_prepared.restype = ctypes.c_int
    L.moe_prepare_weights.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, vp, sz, vp]
    L.moe_prepare_weights.restype = ctypes.c_int
    L.moe_fused_mlp_workspace_size.argtypes = [i64, i32, i32, i32, i32]
    L.moe_fused_mlp_workspace_size.restype = sz
    L.moe_fused_mlp_launch_count.argtypes = [i64, i32, i32, i32, i32]
    L.moe_fused_mlp_launch_count.restype = ctypes.c_int
    L.moe_last_error.argtypes = []
    L.moe_last_error.restype = ctypes.c_char_p
    L.moe_device_status.argtypes = [ctypes.c_int]
    L.moe_device_status.restype = ctypes.c_int
    L.moe_describe_plan.argtypes = [i64, i32, i32, i32, i32, i32, ctypes.POINTER(LaunchDesc), i32]
    L.moe_describe_plan.restype = ctypes.c_int
    ip = ctypes.POINTER(ctypes.c_int32)
    L.moe_ep_build_tables.argtypes = [ip, i32, i32, i32, i32, i32, i32, i64, ip, ip, ip, ip]
    L.moe_ep_build_tables.restype = ctypes.c_int
    L.moe_sm_clock_sample.argtypes = [vp, i32, vp]
    L.moe_sm_clock_sample.restype = ctypes.c_int
    L.moe_version.argtypes = []
    L.moe_version.restype = ctypes.c_int
    L.moe_set_tuning.argtypes = [i32, i64]
    L.moe_set_tuning.restype = ctypes.c_int
    L.moe_ep_create.argtypes = [i32, i32, i32, i64, i32, i32, i32, i32, i32, ctypes.POINTER(vp)]
    L.moe_ep_create.restype = ctypes.c_int
    L.moe_ep_export.argtypes = [vp, vp]
    L.moe_ep_export.restype = ctypes.c_int
    L.moe_ep_connect.argtypes = [vp, vp]
    L.moe_ep_connect.restype = ctypes.c_int
    L.moe_ep_set_weights.argtypes = [vp, vp, vp, vp, vp, vp]
    L.moe_ep_set_weights.restype = ctypes.c_int
    L.moe_ep_forward.argtypes = [vp, vp, vp, vp, i64, vp]
    L.moe_ep_forward.restype = ctypes.c_int
    L.moe_ep_launches_per_forward.argtypes = [vp]
    L.moe_ep_launches_per_forward.restype = ctypes.c_int
    L.moe_ep_output.argtypes = [vp]
    L.moe_ep_output.restype = vp
    L.moe_route_topk.argtypes = [vp, i64, i32, i32, vp, vp, vp]
    L.moe_route_topk.restype = ctypes.c_int
    L.moe_permute_workspace_size.argtypes = [i64, i32]
    L.moe_permute_workspace_size.restype = sz
    L.moe_permute.argtypes = [vp, i64, i32, vp, vp, vp, vp, sz, vp]
    L.moe_permute.restype = ctypes.c_int
    L.moe_gather_rows.argtypes = [vp, vp, i64, i32, i32, vp, vp]
    L.moe_gather_rows.restype = ctypes.c_int
    L.moe_combine_rows.argtypes = [vp, vp, vp, i64, i32, i32, vp, vp]
    L.moe_combine_rows.restype = ctypes.c_int
    L.moe_swiglu_interleave.argtypes = [vp, vp, vp, i32, i32, i32, vp]
    L.moe_swiglu_interleave.restype = ctypes.c_int
    L.moe_fused_mlp_swiglu_workspace_size.argtypes = [i64, i32, i32]
    L.moe_fused_mlp_swiglu_workspace_size.restype = sz
    L.moe_fused_mlp_swiglu.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_swiglu.restype = ctypes.c_int
    L.moe_fused_mlp_forward_train_workspace_size.argtypes = [i64, i32, i32, i32]
    L.moe_fused_mlp_forward_train_workspace_size.restype = sz
    L.moe_fused_mlp_forward_train.argtypes = [vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_forward_train.restype = ctypes.c_int
    L.moe_fused_mlp_backward_workspace_size.argtypes = [i64, i32, i32, i32]
    L.moe_fused_mlp_backward_workspace_size.restype = sz
    L.moe_fused_mlp_backward.argtypes = [vp, vp, vp, vp, vp, vp, i32, vp, vp, vp, i64, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_backward.restype = ctypes.c_int
    L.moe_fused_mlp_swiglu_forward_train_workspace_size.argtypes = [i64, i32, i32, i32]
    L.moe_fused_mlp_swiglu_forward_train_workspace_size.restype = sz
    L.moe_fused_mlp_swiglu_forward_train.argtypes = [vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_swiglu_forward_train.restype = ctypes.c_int
    L.moe_fused_mlp_swiglu_backward_workspace_size.argtypes = [i64, i32, i32, i32]
    L.moe_fused_mlp_swiglu_backward_workspace_size.restype = sz
    L.moe_fused_mlp_swiglu_backward.argtypes = [vp, vp, vp, vp, vp, vp, i32, vp, vp, vp, i64, i32, i32, i32, vp, sz,
                                                vp]
    L.moe_fused_mlp_swiglu_backward.restype = ctypes.c_int
    L.moe_swiglu_interleave_fp8.argtypes = [vp, vp, vp, vp, vp, vp, i32, i32, i32, vp]
    L.moe_swiglu_interleave_fp8.restype = ctypes.c_int
    L.moe_fused_mlp_swiglu_fp8_workspace_size.argtypes = [i64, i32, i32]
    L.moe_fused_mlp_swiglu_fp8_workspace_size.restype = sz
    L.moe_fused_mlp_swiglu_fp8.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, vp, sz, vp]
    L.moe_fused_mlp_swiglu_fp8.restype = ctypes.c_int
    L.moe_ep_destroy.argtypes = [vp]
    L.moe_ep_destroy.restype = ctypes.c_int
    _lib = L
    return L


def check(code: int) -> None:
    if code != 0:
        raise MoeError(code, lib().moe_last_error().decode(errors="replace"))


def set_tuning(key: int, value: int) -> None:
    check(lib().moe_set_tuning(key, value))


def device_status(reset: bool = False) -> int:
    v = lib().moe_device_status(1 if reset else 0)
    if v < 0:
        check(v)
    return v
