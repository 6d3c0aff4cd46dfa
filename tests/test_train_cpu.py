"""Backward of the expert MLP on the CPU: the oracle's gradient formulas
against torch autograd (float64), and the C-ABI's argument checks."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib


def _torch_grads(x, wu, wd, gs, dy):
    xt, wut, wdt = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (x, wu, wd))
    M = x.shape[0]
    offs = np.minimum(np.concatenate([[0], np.cumsum(np.maximum(gs, 0))]), M)
    parts = []
    for e in range(len(gs)):
        a, b = int(offs[e]), int(offs[e + 1])
        h = torch.nn.functional.gelu(xt[a:b] @ wut[e], approximate="tanh")
        parts.append(h @ wdt[e])
    parts.append(torch.zeros((M - int(offs[-1]), x.shape[1]), dtype=torch.float64))
    y = torch.cat(parts)
    y.backward(torch.tensor(dy, dtype=torch.float64))
    return xt.grad.numpy(), wut.grad.numpy(), wdt.grad.numpy()


@pytest.mark.parametrize("gs", [[7, 0, 12], [0, 0, 0], [20, 3, 9], [5, 5, 2]])
def test_backward_oracle_matches_autograd(gs):
    rng = np.random.default_rng(sum(gs))
    M, D, F, E = 32, 6, 10, 3
    x = rng.standard_normal((M, D))
    wu = rng.standard_normal((E, D, F)) / 2
    wd = rng.standard_normal((E, F, D)) / 3
    dy = rng.standard_normal((M, D))
    dx, dwu, dwd = orc.ref_ragged_mlp_backward(x, wu, wd, gs, dy)
    tx, twu, twd = _torch_grads(x, wu, wd, np.array(gs), dy)
    np.testing.assert_allclose(dx, tx, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dwu, twu, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dwd, twd, rtol=1e-12, atol=1e-12)


def test_gelu_grad_matches_torch():
    x = torch.linspace(-12, 12, 4001, dtype=torch.float64, requires_grad=True)
    torch.nn.functional.gelu(x, approximate="tanh").sum().backward()
    np.testing.assert_allclose(orc.gelu_tanh_grad(x.detach().numpy()), x.grad.numpy(), rtol=1e-13, atol=1e-14)


def test_training_abi_checks_before_device_work():
    L = _lib.lib()
    vp = ctypes.c_void_p
    n = vp(0)
    s = vp(16)
    assert L.moe_fused_mlp_forward_train(n, n, n, n, n, n, -1, 512, 512, 4, n, 0, n) == -1
    assert b"bad sizes" in L.moe_last_error()
    assert L.moe_fused_mlp_forward_train(s, s, s, s, s, s, 16, 384, 512, 4, n, 0, n) == -2
    assert L.moe_fused_mlp_forward_train(s, s, s, s, s, s, 16, 512, 128, 4, n, 0, n) == -2
    assert L.moe_fused_mlp_forward_train(n, n, n, n, n, n, 0, 512, 512, 4, n, 0, n) == 0
    assert L.moe_fused_mlp_forward_train(s, s, s, s, vp(8), s, 16, 512, 512, 4, n, 0, n) == -7
    args = [s, s, s, s, s, s, 0, s, s, s, 16, 512, 512, 4, n, 0, n]
    assert L.moe_fused_mlp_backward(*args[:6], 2, *args[7:]) == -3        # dy must be f32 or bf16
    assert L.moe_fused_mlp_backward(*args[:6], 0, *args[7:10], -3, *args[11:]) == -1
    assert L.moe_fused_mlp_backward(*args[:6], 0, *args[7:10], 16, 512, 512, 5000, n, 0, n) == -2
    assert L.moe_fused_mlp_backward(*args[:5], n, 0, *args[7:]) == -1     # null dy


def test_training_workspace_sizes():
    L = _lib.lib()
    M, D, F, E = 32768, 4096, 14336, 8
    assert L.moe_fused_mlp_forward_train_workspace_size(M, D, F, E) == M * F * 2
    mp = M + 64 * E
    assert L.moe_fused_mlp_backward_workspace_size(M, D, F, E) == 2 * mp * D * 2 + 2 * mp * F * 2
    assert L.moe_fused_mlp_backward_workspace_size(M, 128, F, E) == 0


@pytest.mark.parametrize("gs", [[7, 0, 12], [20, 3, 9], [0, 0, 0]])
def test_swiglu_backward_oracle_matches_autograd(gs):
    rng = np.random.default_rng(50 + sum(gs))
    M, D, F, E = 32, 6, 10, 3
    x = rng.standard_normal((M, D))
    wg, wu = rng.standard_normal((E, D, F)) / 2, rng.standard_normal((E, D, F)) / 2
    wd = rng.standard_normal((E, F, D)) / 3
    dy = rng.standard_normal((M, D))
    dx, dwg, dwu, dwd = orc.ref_ragged_swiglu_backward(x, wg, wu, wd, gs, dy)
    xt, wgt, wut, wdt = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (x, wg, wu, wd))
    offs = np.concatenate([[0], np.cumsum(gs)])
    parts = [(torch.nn.functional.silu(xt[offs[e]:offs[e + 1]] @ wgt[e]) * (xt[offs[e]:offs[e + 1]] @ wut[e])) @ wdt[e]
             for e in range(E)]
    y = torch.cat(parts + [torch.zeros((M - int(offs[-1]), D), dtype=torch.float64)])
    y.backward(torch.tensor(dy))
    for got, ref in ((dx, xt.grad), (dwg, wgt.grad), (dwu, wut.grad), (dwd, wdt.grad)):
        np.testing.assert_allclose(got, ref.numpy(), rtol=1e-12, atol=1e-12)


def test_swiglu_training_abi_checks_before_device_work():
    L = _lib.lib()
    vp = ctypes.c_void_p
    n, s = vp(0), vp(16)
    assert L.moe_fused_mlp_swiglu_forward_train(n, n, n, n, n, n, -1, 512, 512, 4, n, 0, n) == -1
    assert L.moe_fused_mlp_swiglu_forward_train(s, s, s, s, s, s, 16, 512, 384, 4, n, 0, n) == -2
    assert L.moe_fused_mlp_swiglu_forward_train(n, n, n, n, n, n, 0, 512, 512, 4, n, 0, n) == 0
    args = [s, s, s, s, s, s, 0, s, s, s, 16, 512, 512, 4, n, 0, n]
    assert L.moe_fused_mlp_swiglu_backward(*args[:6], 2, *args[7:]) == -3
    assert L.moe_fused_mlp_swiglu_backward(*args[:5], n, 0, *args[7:]) == -1
    M, D, F, E = 32768, 4096, 14336, 8
    mp = M + 64 * E
    assert L.moe_fused_mlp_swiglu_backward_workspace_size(M, D, F, E) == 2 * mp * D * 2 + mp * 2 * F * 2 + mp * F * 2
    assert L.moe_fused_mlp_swiglu_forward_train_workspace_size(M, D, F, E) == M * F * 2
