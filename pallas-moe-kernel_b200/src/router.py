"""Routing and permutation around the fused expert MLP (torch CUDA tensors).

The reference's path starts from rows already sorted by expert plus their
``group_sizes`` (``src/kernel.py:85-95``; its benchmarks build the group
sizes directly).  These functions produce that input from router logits and
fold the expert outputs back per token, each one kernel of the library
(declared in ``include/moe_b200.h``):

    ids, w = route_topk(logits, k)                  # (T, k) experts and weights
    gs, src, inv = permute(ids, E)                  # stable sort of entries by expert
    xs = gather_rows(x, src, k)                     # X in expert order
    ys = fused_ragged_mlp(xs, w_up, w_down, gs)     # the reference's path
    y = combine_rows(ys, inv, w)                    # weighted sum per token

:func:`moe_layer` runs the five steps.  All calls are stream-ordered on the
current stream and never synchronise the host.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def route_topk(logits: torch.Tensor, k: int):
    """Top-k experts per token (larger logit first, ties to the lower expert
    id) and softmax weights over the selected logits.  ``logits`` (T, E)
    float32 on a CUDA device; returns (ids (T, k) int32, weights (T, k) f32)."""
    if not logits.is_cuda or logits.dim() != 2:
        raise ValueError("logits must be a 2-D CUDA tensor")
    logits = logits.float().contiguous()
    T, E = logits.shape
    ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    _lib.check(_lib.lib().moe_route_topk(logits.data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr(),
                                         _stream(logits.device)))
    return ids, w


def permute(ids: torch.Tensor, num_experts: int, workspace: Optional[torch.Tensor] = None):
    """Stable counting sort of the entries ``i = t * k + j`` of ``ids`` (T, k)
    by expert.  Returns (group_sizes (E,), sorted_src (N,) entry index of each
    row in expert order, inverse (T, k) row of each entry, -1 if dropped)."""
    ids = ids.to(torch.int32).contiguous()
    dev = ids.device
    N = ids.numel()
    L = _lib.lib()
    gs = torch.empty(num_experts, dtype=torch.int32, device=dev)
    src = torch.empty(N, dtype=torch.int32, device=dev)
    inv = torch.empty(ids.shape, dtype=torch.int32, device=dev)
    need = int(L.moe_permute_workspace_size(N, num_experts))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    _lib.check(L.moe_permute(ids.data_ptr(), N, num_experts, gs.data_ptr(), src.data_ptr(), inv.data_ptr(),
                             workspace.data_ptr(), workspace.numel(), _stream(dev)))
    return gs, src, inv


def gather_rows(x: torch.Tensor, sorted_src: torch.Tensor, k: int, out: Optional[torch.Tensor] = None):
    """Row r of the result is row ``sorted_src[r] // k`` of ``x`` (T, D)."""
    x = x.contiguous()
    rows = sorted_src.numel()
    if out is None:
        out = torch.empty((rows, x.shape[1]), dtype=x.dtype, device=x.device)
    row_bytes = x.shape[1] * x.element_size()
    _lib.check(_lib.lib().moe_gather_rows(x.data_ptr(), sorted_src.data_ptr(), rows, k, row_bytes, out.data_ptr(),
                                          _stream(x.device)))
    return out


def combine_rows(y_sorted: torch.Tensor, inverse: torch.Tensor, weights: torch.Tensor,
                 out: Optional[torch.Tensor] = None):
    """``y[t] = sum_j weights[t, j] * y_sorted[inverse[t, j]]`` (f32)."""
    T, k = inverse.shape
    D = y_sorted.shape[1]
    if out is None:
        out = torch.empty((T, D), dtype=torch.float32, device=y_sorted.device)
    _lib.check(_lib.lib().moe_combine_rows(y_sorted.contiguous().data_ptr(), inverse.contiguous().data_ptr(),
                                           weights.float().contiguous().data_ptr(), T, k, D, out.data_ptr(),
                                           _stream(y_sorted.device)))
    return out


def moe_layer(x: torch.Tensor, logits: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, k: int, *,
              w_up_scale: Optional[torch.Tensor] = None, w_down_scale: Optional[torch.Tensor] = None):
    """A whole MoE expert layer: top-k routing of ``x`` (T, D) by ``logits``
    (T, E), the fused expert MLP over the expert-sorted rows, and the
    weighted combine.  Returns (y (T, D) f32, group_sizes)."""
    from .kernel import fused_ragged_mlp
    E = w_up.shape[0]
    ids, w = route_topk(logits, k)
    gs, src, inv = permute(ids, E)
    xs = gather_rows(x, src, k)
    ys = fused_ragged_mlp(xs, w_up, w_down, gs, w_up_scale=w_up_scale, w_down_scale=w_down_scale)
    return combine_rows(ys, inv, w), gs
