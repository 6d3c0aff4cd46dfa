"""Fused MoE expert MLP on B200 -- drop-in for the reference's ``src/kernel.py``.

``fused_ragged_dot_caller`` keeps the signature and argument checks of the
reference entry point (Krushna-B/pallas-moe-kernel ``src/kernel.py:85-123``)
but runs the hand-written sm_100a kernels of ``libmoe_b200.so`` through its C
ABI on the current CUDA stream.  Arrays are torch CUDA tensors (JAX arrays in
the reference); the result is a new ``(M, D)`` float32 tensor.

Differences from the reference, by design:
  * ``BM``, ``BF`` and ``max_group_size`` are validated as the reference does
    (``M % BM == 0``, ``F % BF == 0``) but do not shape the launch: the kernel
    enumerates the real (expert, 128-row) blocks on the device from
    ``group_sizes``, so no host sync and no recompilation per routing.
  * Rows at or past ``sum(group_sizes)`` are zero, as in ``ragged_dot``; the
    Pallas kernel leaves them unwritten (``src/kernel.py:77-82``).
  * ``interpret=True`` (the Pallas CPU interpreter) has no counterpart: there
    is no CPU path, and the call raises.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

__all__ = [
    "fused_ragged_dot_caller",
    "fused_ragged_mlp",
    "group_sizes_to_offsets",
    "workspace_size",
    "ref_ragged_mlp",
    "ref_ragged_mlp_one_line",
]

_FP8 = getattr(torch, "float8_e4m3fn", None)


def _dtype_code(x: torch.Tensor, w_up: torch.Tensor) -> int:
    if x.dtype == torch.float32 and w_up.dtype == torch.float32:
        return _lib.MOE_DTYPE_F32
    if x.dtype == torch.bfloat16 and w_up.dtype == torch.bfloat16:
        return _lib.MOE_DTYPE_BF16
    if x.dtype == torch.bfloat16 and _FP8 is not None and w_up.dtype == _FP8:
        return _lib.MOE_DTYPE_FP8_E4M3_BLK128
    raise TypeError(f"unsupported dtypes x={x.dtype} w_up={w_up.dtype} "
                    f"(f32/f32, bf16/bf16 or bf16/float8_e4m3fn)")


def _weight_dtype_code(w_up: torch.Tensor) -> int:
    if w_up.dtype == torch.float32:
        return _lib.MOE_DTYPE_F32
    if w_up.dtype == torch.bfloat16:
        return _lib.MOE_DTYPE_BF16
    if _FP8 is not None and w_up.dtype == _FP8:
        return _lib.MOE_DTYPE_FP8_E4M3_BLK128
    raise TypeError(f"unsupported weight dtype {w_up.dtype}")


def workspace_size(M: int, D: int, F: int, E: int, dtype_code: int) -> int:
    return int(_lib.lib().moe_fused_mlp_workspace_size(M, D, F, E, dtype_code))


def _as_device_group_sizes(group_sizes, device) -> torch.Tensor:
    if (isinstance(group_sizes, torch.Tensor) and group_sizes.dtype == torch.int32
            and group_sizes.device == device and group_sizes.is_contiguous()):
        return group_sizes
    if not isinstance(group_sizes, torch.Tensor):
        group_sizes = torch.as_tensor(group_sizes)
    gs = group_sizes.to(device=device, dtype=torch.int32, non_blocking=True)
    return gs.contiguous()


_WORKSPACES: dict = {}
_WS_SIZES: dict = {}

_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(dev: torch.device) -> int:
    """cudaStream_t of torch's current stream on ``dev``."""
    if _raw_stream is not None:
        return _raw_stream(dev.index)
    return torch.cuda.current_stream(dev).cuda_stream


_WORKSPACE_CACHE_MAX = 64 << 20


def _stream_workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """A workspace of at least ``nbytes`` shared by the calls on one stream
    (they run in stream order, so none overlaps another's use of it); small
    calls are dominated by host time, and this saves an allocation each.
    Workspaces above 64 MiB, and every call while a CUDA graph is being
    captured (the graph's memory pool), get a fresh allocation."""
    if nbytes > _WORKSPACE_CACHE_MAX or torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, device=dev, dtype=torch.uint8)
    key = (dev.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
        _WORKSPACES[key] = ws
    return ws


def fused_ragged_mlp(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, group_sizes,
                     *, w_up_scale: Optional[torch.Tensor] = None,
                     w_down_scale: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None,
                     workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Core call: ``Y = ragged_dot(gelu_tanh(ragged_dot(X, W_up)), W_down)``.

    x (M, D) f32|bf16, w_up (E, D, F), w_down (E, F, D) of the same dtype
    (or float8_e4m3fn weights with f32 block scales (E, D/128, F/128) and
    (E, F/128, D/128)), group_sizes (E,) int -- all on one CUDA device.
    Stream-ordered on ``torch.cuda.current_stream()``.
    """
    if not x.is_cuda:
        raise ValueError("fused_ragged_mlp runs on CUDA tensors only (no CPU path)")
    M, D = x.shape
    E, D2, F = w_up.shape
    if D != D2 or tuple(w_down.shape) != (E, F, D):
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w_up={tuple(w_up.shape)} "
                         f"w_down={tuple(w_down.shape)}")
    code = _dtype_code(x, w_up)
    if w_down.dtype != w_up.dtype:
        raise TypeError("w_up and w_down must share a dtype")
    dev = x.device
    for t in (w_up, w_down):
        if t.device != dev:
            raise ValueError("all operands must be on the same device")
    x = x.contiguous()
    w_up = w_up.contiguous()
    w_down = w_down.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    if code == _lib.MOE_DTYPE_FP8_E4M3_BLK128:
        if w_up_scale is None or w_down_scale is None:
            raise ValueError("FP8 weights need w_up_scale and w_down_scale")
        w_up_scale = w_up_scale.to(device=dev, dtype=torch.float32).contiguous()
        w_down_scale = w_down_scale.to(device=dev, dtype=torch.float32).contiguous()
    if out is None:
        out = torch.empty((M, D), device=dev, dtype=torch.float32)
    elif out.shape != (M, D) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous (M, D) float32 tensor")
    L = _lib.lib()
    key = (M, D, F, E, code)
    ws_bytes = _WS_SIZES.get(key)
    if ws_bytes is None:
        if len(_WS_SIZES) > 4096:
            _WS_SIZES.clear()
        ws_bytes = _WS_SIZES.setdefault(key, int(L.moe_fused_mlp_workspace_size(M, D, F, E, code)))
    stream = _stream_handle(dev)
    if ws_bytes and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = _stream_workspace(dev, stream, ws_bytes)
    args = (x.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), gs.data_ptr(),
            w_up_scale.data_ptr() if w_up_scale is not None else None,
            w_down_scale.data_ptr() if w_down_scale is not None else None,
            out.data_ptr(), M, D, F, E, code, workspace.data_ptr() if ws_bytes else None, ws_bytes, stream)
    if dev.index == torch.cuda.current_device():
        rc = L.moe_fused_mlp(*args)
    else:
        with torch.cuda.device(dev):
            rc = L.moe_fused_mlp(*args)
    _lib.check(rc)
    return out


def swiglu_interleave(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """(E, D, F) bf16 gate and up weights -> the (E, D, 2F) operand of
    ``fused_ragged_swiglu``: blocks of 128 columns alternating gate, up."""
    if w_gate.shape != w_up.shape or w_gate.dim() != 3:
        raise ValueError(f"w_gate {tuple(w_gate.shape)} and w_up {tuple(w_up.shape)} must be the same (E, D, F)")
    if w_gate.dtype != torch.bfloat16 or w_up.dtype != torch.bfloat16:
        raise TypeError("SwiGLU weights are bf16")
    if not (w_gate.is_cuda and w_up.device == w_gate.device):
        raise ValueError("w_gate and w_up must be on one CUDA device")
    E, D, F = w_gate.shape
    w_gate, w_up = w_gate.contiguous(), w_up.contiguous()
    out = torch.empty((E, D, 2 * F), device=w_gate.device, dtype=torch.bfloat16)
    with torch.cuda.device(w_gate.device):
        rc = _lib.lib().moe_swiglu_interleave(
            ctypes.c_void_p(w_gate.data_ptr()), ctypes.c_void_p(w_up.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            E, D, F, ctypes.c_void_p(torch.cuda.current_stream(w_gate.device).cuda_stream))
    _lib.check(rc)
    return out


def swiglu_interleave_fp8(w_gate: torch.Tensor, w_up: torch.Tensor, s_gate: torch.Tensor, s_up: torch.Tensor):
    """e4m3 gate and up weights (E, D, F) with their 128 x 128 block scales
    (E, D/128, F/128) -> (w_gate_up (E, D, 2F), s_gate_up (E, D/128, 2F/128)),
    the operands of ``fused_ragged_swiglu`` with FP8 weights."""
    if w_gate.shape != w_up.shape or w_gate.dim() != 3 or s_gate.shape != s_up.shape:
        raise ValueError("gate and up weights (and scales) must have the same shapes")
    if _FP8 is None or w_gate.dtype != _FP8 or w_up.dtype != _FP8:
        raise TypeError("weights must be float8_e4m3fn")
    E, D, F = w_gate.shape
    if tuple(s_gate.shape) != (E, D // 128, F // 128):
        raise ValueError(f"scales must be (E, D/128, F/128) = {(E, D // 128, F // 128)}")
    dev = w_gate.device
    w_gate, w_up = w_gate.contiguous(), w_up.contiguous()
    s_gate = s_gate.to(device=dev, dtype=torch.float32).contiguous()
    s_up = s_up.to(device=dev, dtype=torch.float32).contiguous()
    w = torch.empty((E, D, 2 * F), device=dev, dtype=_FP8)
    sc = torch.empty((E, D // 128, 2 * F // 128), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        rc = _lib.lib().moe_swiglu_interleave_fp8(
            w_gate.data_ptr(), w_up.data_ptr(), s_gate.data_ptr(), s_up.data_ptr(), w.data_ptr(), sc.data_ptr(),
            E, D, F, _stream_handle(dev))
    _lib.check(rc)
    return w, sc


def fused_ragged_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, group_sizes,
                        *, w_gate_up_scale: Optional[torch.Tensor] = None,
                        w_down_scale: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None,
                        workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SwiGLU experts: ``Y = ragged_dot(silu(X W_gate) * (X W_up), W_down)``.

    x (M, D) bf16, w_gate_up (E, D, 2F) bf16 from ``swiglu_interleave``,
    w_down (E, F, D) bf16, group_sizes (E,) -> y (M, D) f32.  With
    float8_e4m3fn weights pass their block scales: w_gate_up_scale
    (E, D/128, 2F/128) from ``swiglu_interleave_fp8`` and w_down_scale
    (E, F/128, D/128).  Same ragged semantics as ``fused_ragged_mlp``; D a
    multiple of 256, F of 128.
    """
    if _FP8 is not None and w_gate_up.dtype == _FP8:
        return _fused_ragged_swiglu_fp8(x, w_gate_up, w_down, group_sizes, w_gate_up_scale, w_down_scale, out,
                                        workspace)
    if not x.is_cuda:
        raise ValueError("fused_ragged_swiglu runs on CUDA tensors only (no CPU path)")
    M, D = x.shape
    E, D2, F2 = w_gate_up.shape
    F = F2 // 2
    if D != D2 or F2 % 2 or tuple(w_down.shape) != (E, F, D):
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w_gate_up={tuple(w_gate_up.shape)} "
                         f"w_down={tuple(w_down.shape)}")
    for t in (x, w_gate_up, w_down):
        if t.dtype != torch.bfloat16:
            raise TypeError("SwiGLU experts take bf16 operands")
        if t.device != x.device:
            raise ValueError("all operands must be on the same device")
    dev = x.device
    x, w_gate_up, w_down = x.contiguous(), w_gate_up.contiguous(), w_down.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    if out is None:
        out = torch.empty((M, D), device=dev, dtype=torch.float32)
    elif out.shape != (M, D) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous (M, D) float32 tensor")
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_swiglu_workspace_size(M, D, F))
    if ws_bytes and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_swiglu(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w_gate_up.data_ptr()),
            ctypes.c_void_p(w_down.data_ptr()), ctypes.c_void_p(gs.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            M, D, F, E, ctypes.c_void_p(workspace.data_ptr() if ws_bytes else 0), ws_bytes,
            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc)
    return out


def _fused_ragged_swiglu_fp8(x, w_gate_up, w_down, group_sizes, s_gu, s_down, out, workspace):
    if not x.is_cuda:
        raise ValueError("fused_ragged_swiglu runs on CUDA tensors only (no CPU path)")
    if s_gu is None or s_down is None:
        raise ValueError("FP8 weights need w_gate_up_scale and w_down_scale")
    M, D = x.shape
    E, D2, F2 = w_gate_up.shape
    F = F2 // 2
    if D != D2 or F2 % 2 or tuple(w_down.shape) != (E, F, D) or x.dtype != torch.bfloat16 or w_down.dtype != _FP8:
        raise ValueError(f"expected bf16 x (M, D), e4m3 w_gate_up (E, D, 2F) and w_down (E, F, D); got "
                         f"{tuple(x.shape)} {x.dtype}, {tuple(w_gate_up.shape)}, {tuple(w_down.shape)} {w_down.dtype}")
    dev = x.device
    x, w_gate_up, w_down = x.contiguous(), w_gate_up.contiguous(), w_down.contiguous()
    s_gu = s_gu.to(device=dev, dtype=torch.float32).contiguous()
    s_down = s_down.to(device=dev, dtype=torch.float32).contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    if out is None:
        out = torch.empty((M, D), device=dev, dtype=torch.float32)
    elif out.shape != (M, D) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous (M, D) float32 tensor")
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_swiglu_fp8_workspace_size(M, D, F))
    if ws_bytes and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_swiglu_fp8(x.data_ptr(), w_gate_up.data_ptr(), w_down.data_ptr(), s_gu.data_ptr(),
                                        s_down.data_ptr(), gs.data_ptr(), out.data_ptr(), M, D, F, E,
                                        workspace.data_ptr() if ws_bytes else None, ws_bytes, _stream_handle(dev))
    _lib.check(rc)
    return out


class PreparedExperts:
    """Expert weights with their kernel-side operand layout built once
    (``moe_prepare_weights``), for repeated calls with fixed weights.

    ``max_tokens`` bounds M of later calls (it sizes the workspace)."""

    def __init__(self, w_up: torch.Tensor, w_down: torch.Tensor, *, max_tokens: int,
                 w_up_scale: Optional[torch.Tensor] = None, w_down_scale: Optional[torch.Tensor] = None):
        self.E, self.D, self.F = w_up.shape
        if tuple(w_down.shape) != (self.E, self.F, self.D):
            raise ValueError("w_down must be (E, F, D)")
        self.w_up = w_up.contiguous()
        self.w_down = w_down.contiguous()
        self.w_up_scale = None if w_up_scale is None else w_up_scale.float().contiguous()
        self.w_down_scale = None if w_down_scale is None else w_down_scale.float().contiguous()
        self.dtype_code = _weight_dtype_code(w_up)
        self.max_tokens = int(max_tokens)
        self.ws_bytes = workspace_size(self.max_tokens, self.D, self.F, self.E, self.dtype_code)
        self.workspace = torch.empty(max(self.ws_bytes, 1), device=w_up.device, dtype=torch.uint8)
        stream = torch.cuda.current_stream(w_up.device).cuda_stream
        with torch.cuda.device(w_up.device):
            rc = _lib.lib().moe_prepare_weights(
                ctypes.c_void_p(self.w_up.data_ptr()), ctypes.c_void_p(self.w_down.data_ptr()),
                ctypes.c_void_p(self.w_up_scale.data_ptr() if self.w_up_scale is not None else 0),
                ctypes.c_void_p(self.w_down_scale.data_ptr() if self.w_down_scale is not None else 0),
                self.D, self.F, self.E, self.dtype_code, ctypes.c_void_p(self.workspace.data_ptr()),
                self.ws_bytes, ctypes.c_void_p(stream))
        _lib.check(rc)

    def __call__(self, x: torch.Tensor, group_sizes, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M, D = x.shape
        if D != self.D:
            raise ValueError(f"x has D={D}, experts have D={self.D}")
        if M > self.max_tokens:
            raise ValueError(f"M={M} exceeds max_tokens={self.max_tokens}")
        dev = x.device
        gs = _as_device_group_sizes(group_sizes, dev)
        if out is None:
            out = torch.empty((M, D), device=dev, dtype=torch.float32)
        stream = _stream_handle(dev)
        args = (x.data_ptr(), self.w_up.data_ptr(), self.w_down.data_ptr(), gs.data_ptr(),
                self.w_up_scale.data_ptr() if self.w_up_scale is not None else None,
                self.w_down_scale.data_ptr() if self.w_down_scale is not None else None,
                out.data_ptr(), M, self.D, self.F, self.E, self.dtype_code, self.workspace.data_ptr(),
                self.ws_bytes, stream)
        if dev.index == torch.cuda.current_device():
            rc = _lib.lib().moe_fused_mlp_prepared(*args)
        else:
            with torch.cuda.device(dev):
                rc = _lib.lib().moe_fused_mlp_prepared(*args)
        _lib.check(rc)
        return out


def fused_ragged_dot_caller(x, w_up, w_down, group_sizes, *, BM: int = 16, BF: int = 64,
                            max_group_size: int, interpret: bool = False, **kwargs) -> torch.Tensor:
    """Reference entry point (``src/kernel.py:85-123``): same arguments and the
    same assertions; returns the f32 ``(M, D)`` output."""
    M, D = x.shape
    E, D2, F = w_up.shape
    assert D == D2
    assert tuple(w_down.shape) == (E, F, D)
    assert M % BM == 0
    assert F % BF == 0
    del max_group_size  # the device-side block walk covers every real block
    if interpret:
        raise NotImplementedError("interpret=True (Pallas CPU interpreter) has no counterpart: "
                                  "this library runs on the B200 only")
    return fused_ragged_mlp(x, w_up, w_down, group_sizes, **kwargs)


def group_sizes_to_offsets(group_sizes: torch.Tensor) -> torch.Tensor:
    """``[0, cumsum(group_sizes)]`` (``src/kernel.py:126-132``)."""
    gs = torch.as_tensor(group_sizes)
    return torch.cat([torch.zeros(1, dtype=gs.dtype, device=gs.device), torch.cumsum(gs, 0).to(gs.dtype)])


def _ref(x, w_up, w_down, group_sizes) -> torch.Tensor:
    gs = torch.as_tensor(group_sizes).to("cpu").tolist()
    M, D = x.shape
    y = torch.zeros((M, D), dtype=torch.float32, device=x.device)
    off = 0
    for e, g in enumerate(gs):
        g = max(int(g), 0)
        hi = min(off + g, M)
        if hi > off:
            h = x[off:hi].float() @ w_up[e].float()
            h = torch.nn.functional.gelu(h, approximate="tanh")
            y[off:hi] = h @ w_down[e].float()
        off = hi
    return y


def ref_ragged_mlp(x, w_up, w_down, group_sizes) -> torch.Tensor:
    """Unfused two-ragged-dot path (``src/kernel.py:152-175``) with torch ops on
    the tensors' own device: materialises H per expert.  For comparison only;
    it is not the fused path and is not used by it."""
    return _ref(x, w_up, w_down, group_sizes)


def ref_ragged_mlp_one_line(x, w_up, w_down, group_sizes) -> torch.Tensor:
    """Same as :func:`ref_ragged_mlp` (``src/kernel.py:137-149``)."""
    return _ref(x, w_up, w_down, group_sizes)
