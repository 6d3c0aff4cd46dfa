"""Training use of the fused expert MLP: forward with the pre-activation
saved, the backward kernels, and a ``torch.autograd.Function`` over both.

The reference is forward-only (``src/kernel.py:9-123``).  Here
``Y = ragged_dot(gelu_tanh(ragged_dot(X, W_up)), W_down)`` over
expert-sorted rows gets its gradients from ``libmoe_b200.so``:

  forward_train  the two grouped GEMMs of the bf16 path; the up GEMM's
                 epilogue also stores A = X W_up[e] (bf16, (M, F)).
  backward       dX, dW_up, dW_down (f32) from dY and A: the GEMMs
                 dY W_down^T (epilogue: dA = . * GELU'(A), H = GELU(A)),
                 dA W_up^T, X^T dA and H^T dY per expert.

bf16 operands, f32 accumulation; D and F multiples of 256.  There is no CPU
path: every call raises on non-CUDA tensors or a missing library.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from .kernel import _as_device_group_sizes

__all__ = ["forward_train", "backward", "FusedRaggedMLP", "fused_ragged_mlp_train", "swiglu_forward_train",
           "swiglu_backward", "FusedRaggedSwiGLU", "fused_ragged_swiglu_train"]


def _vp(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _check(x, w_up, w_down):
    if not x.is_cuda:
        raise ValueError("the training entry points run on CUDA tensors only (no CPU path)")
    M, D = x.shape
    E, D2, F = w_up.shape
    if D != D2 or tuple(w_down.shape) != (E, F, D):
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w_up={tuple(w_up.shape)} w_down={tuple(w_down.shape)}")
    for t in (x, w_up, w_down):
        if t.dtype != torch.bfloat16:
            raise TypeError("training takes bf16 x, w_up and w_down")
        if t.device != x.device:
            raise ValueError("all operands must be on the same device")
    return M, D, F, E


def _workspace(nbytes: int, dev, workspace: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if nbytes and (workspace is None or workspace.numel() * workspace.element_size() < nbytes):
        workspace = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    return workspace if nbytes else None


def forward_train(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, group_sizes, *,
                  out: Optional[torch.Tensor] = None, a_save: Optional[torch.Tensor] = None,
                  workspace: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Y (M, D) f32 and the saved pre-activation A (M, F) bf16."""
    M, D, F, E = _check(x, w_up, w_down)
    dev = x.device
    x, w_up, w_down = x.contiguous(), w_up.contiguous(), w_down.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    if out is None:
        out = torch.empty((M, D), device=dev, dtype=torch.float32)
    if a_save is None:
        a_save = torch.empty((M, F), device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_forward_train_workspace_size(M, D, F, E))
    workspace = _workspace(ws_bytes, dev, workspace)
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_forward_train(_vp(x), _vp(w_up), _vp(w_down), _vp(gs), _vp(out), _vp(a_save), M, D, F, E,
                                           _vp(workspace), ws_bytes,
                                           ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc)
    return out, a_save


def backward(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, group_sizes, a_saved: torch.Tensor,
             dy: torch.Tensor, *, workspace: Optional[torch.Tensor] = None
             ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dX (M, D), dW_up (E, D, F), dW_down (E, F, D)), all f32, for the
    upstream gradient dy (M, D) f32 or bf16."""
    M, D, F, E = _check(x, w_up, w_down)
    dev = x.device
    if dy.shape != (M, D) or dy.dtype not in (torch.float32, torch.bfloat16) or dy.device != dev:
        raise ValueError("dy must be an (M, D) float32 or bfloat16 tensor on the operands' device")
    if a_saved.shape != (M, F) or a_saved.dtype != torch.bfloat16 or a_saved.device != dev:
        raise ValueError("a_saved must be the (M, F) bfloat16 pre-activation from forward_train")
    x, w_up, w_down = x.contiguous(), w_up.contiguous(), w_down.contiguous()
    a_saved, dy = a_saved.contiguous(), dy.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    dx = torch.empty((M, D), device=dev, dtype=torch.float32)
    dwu = torch.empty((E, D, F), device=dev, dtype=torch.float32)
    dwd = torch.empty((E, F, D), device=dev, dtype=torch.float32)
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_backward_workspace_size(M, D, F, E))
    workspace = _workspace(ws_bytes, dev, workspace)
    code = _lib.MOE_DTYPE_F32 if dy.dtype == torch.float32 else _lib.MOE_DTYPE_BF16
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_backward(_vp(x), _vp(w_up), _vp(w_down), _vp(gs), _vp(a_saved), _vp(dy), code, _vp(dx),
                                      _vp(dwu), _vp(dwd), M, D, F, E, _vp(workspace), ws_bytes,
                                      ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc)
    return dx, dwu, dwd


class FusedRaggedMLP(torch.autograd.Function):
    """Autograd node of the expert MLP: Y (f32) from bf16 X and weights;
    gradients come back in the inputs' dtype (bf16)."""

    @staticmethod
    def forward(ctx, x, w_up, w_down, group_sizes):
        y, a = forward_train(x, w_up, w_down, group_sizes)
        ctx.save_for_backward(x, w_up, w_down, group_sizes if isinstance(group_sizes, torch.Tensor)
                              else torch.as_tensor(group_sizes), a)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w_up, w_down, gs, a = ctx.saved_tensors
        dx, dwu, dwd = backward(x, w_up, w_down, gs, a, dy)
        return dx.to(x.dtype), dwu.to(w_up.dtype), dwd.to(w_down.dtype), None


def fused_ragged_mlp_train(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, group_sizes) -> torch.Tensor:
    """Differentiable ``Y = ragged_dot(gelu_tanh(ragged_dot(X, W_up)), W_down)``."""
    return FusedRaggedMLP.apply(x, w_up, w_down, group_sizes)


# ----------------------------------------------------------------------------- SwiGLU experts
def _check_swiglu(x, w_gate_up, w_down):
    if not x.is_cuda:
        raise ValueError("the training entry points run on CUDA tensors only (no CPU path)")
    M, D = x.shape
    E, D2, F2 = w_gate_up.shape
    F = F2 // 2
    if D != D2 or F2 % 2 or tuple(w_down.shape) != (E, F, D):
        raise ValueError(f"shape mismatch x={tuple(x.shape)} w_gate_up={tuple(w_gate_up.shape)} "
                         f"w_down={tuple(w_down.shape)}")
    for t in (x, w_gate_up, w_down):
        if t.dtype != torch.bfloat16:
            raise TypeError("SwiGLU training takes bf16 x, w_gate_up and w_down")
        if t.device != x.device:
            raise ValueError("all operands must be on the same device")
    return M, D, F, E


def swiglu_forward_train(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, group_sizes, *,
                         out: Optional[torch.Tensor] = None, gu_save: Optional[torch.Tensor] = None,
                         workspace: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Y (M, D) f32 of the SwiGLU experts and the saved gate/up columns
    (M, 2F) bf16, interleaved like ``w_gate_up`` (from ``swiglu_interleave``)."""
    M, D, F, E = _check_swiglu(x, w_gate_up, w_down)
    dev = x.device
    x, w_gate_up, w_down = x.contiguous(), w_gate_up.contiguous(), w_down.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    if out is None:
        out = torch.empty((M, D), device=dev, dtype=torch.float32)
    if gu_save is None:
        gu_save = torch.empty((M, 2 * F), device=dev, dtype=torch.bfloat16)
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_swiglu_forward_train_workspace_size(M, D, F, E))
    workspace = _workspace(ws_bytes, dev, workspace)
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_swiglu_forward_train(_vp(x), _vp(w_gate_up), _vp(w_down), _vp(gs), _vp(out),
                                                  _vp(gu_save), M, D, F, E, _vp(workspace), ws_bytes,
                                                  ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc)
    return out, gu_save


def swiglu_backward(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor, group_sizes,
                    gu_saved: torch.Tensor, dy: torch.Tensor, *, workspace: Optional[torch.Tensor] = None
                    ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dX (M, D), dW_gate_up (E, D, 2F) interleaved like w_gate_up,
    dW_down (E, F, D)), all f32."""
    M, D, F, E = _check_swiglu(x, w_gate_up, w_down)
    dev = x.device
    if dy.shape != (M, D) or dy.dtype not in (torch.float32, torch.bfloat16) or dy.device != dev:
        raise ValueError("dy must be an (M, D) float32 or bfloat16 tensor on the operands' device")
    if gu_saved.shape != (M, 2 * F) or gu_saved.dtype != torch.bfloat16 or gu_saved.device != dev:
        raise ValueError("gu_saved must be the (M, 2F) bfloat16 gate/up columns from swiglu_forward_train")
    x, w_gate_up, w_down = x.contiguous(), w_gate_up.contiguous(), w_down.contiguous()
    gu_saved, dy = gu_saved.contiguous(), dy.contiguous()
    gs = _as_device_group_sizes(group_sizes, dev)
    if gs.numel() != E:
        raise ValueError(f"group_sizes has {gs.numel()} entries, expected E={E}")
    dx = torch.empty((M, D), device=dev, dtype=torch.float32)
    dwgu = torch.empty((E, D, 2 * F), device=dev, dtype=torch.float32)
    dwd = torch.empty((E, F, D), device=dev, dtype=torch.float32)
    L = _lib.lib()
    ws_bytes = int(L.moe_fused_mlp_swiglu_backward_workspace_size(M, D, F, E))
    workspace = _workspace(ws_bytes, dev, workspace)
    code = _lib.MOE_DTYPE_F32 if dy.dtype == torch.float32 else _lib.MOE_DTYPE_BF16
    with torch.cuda.device(dev):
        rc = L.moe_fused_mlp_swiglu_backward(_vp(x), _vp(w_gate_up), _vp(w_down), _vp(gs), _vp(gu_saved), _vp(dy),
                                             code, _vp(dx), _vp(dwgu), _vp(dwd), M, D, F, E, _vp(workspace),
                                             ws_bytes, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(rc)
    return dx, dwgu, dwd


class FusedRaggedSwiGLU(torch.autograd.Function):
    """Autograd node of the SwiGLU experts over interleaved gate/up weights:
    Y (f32) from bf16 X and weights; gradients in the inputs' dtype."""

    @staticmethod
    def forward(ctx, x, w_gate_up, w_down, group_sizes):
        y, gu = swiglu_forward_train(x, w_gate_up, w_down, group_sizes)
        ctx.save_for_backward(x, w_gate_up, w_down, group_sizes if isinstance(group_sizes, torch.Tensor)
                              else torch.as_tensor(group_sizes), gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w_gate_up, w_down, gs, gu = ctx.saved_tensors
        dx, dwgu, dwd = swiglu_backward(x, w_gate_up, w_down, gs, gu, dy)
        return dx.to(x.dtype), dwgu.to(w_gate_up.dtype), dwd.to(w_down.dtype), None


def fused_ragged_swiglu_train(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                              group_sizes) -> torch.Tensor:
    """Differentiable SwiGLU experts: ``ragged_dot(silu(X W_gate) * (X W_up), W_down)``
    with ``w_gate_up = swiglu_interleave(w_gate, w_up)``."""
    return FusedRaggedSwiGLU.apply(x, w_gate_up, w_down, group_sizes)
