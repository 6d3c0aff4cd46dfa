"""CPU oracle for the fused MoE expert MLP -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference path

    Y = ragged_dot(gelu_tanh(ragged_dot(X, W_up, gs)), W_down, gs)

as written in Krushna-B/pallas-moe-kernel ``src/kernel.py:137-175``
(``ref_ragged_mlp_one_line`` / ``ref_ragged_mlp``) and the masking rules of
the fused Pallas kernel ``src/kernel.py:9-82``.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and only as the checker or the timed CPU baseline; the product
(the CUDA library and its Python wrapper) never calls into it.

Parity status
-------------
* ``ragged_dot`` and ``gelu`` live in the third-party package JAX
  (``jax==0.8.0`` pinned by the reference's ``requirements.txt:1-2``; the
  published results used 0.7.2).  JAX is not installed in this environment,
  and the reference stores no output values (no golden vectors), so the MLP
  *values* are **parity unpinned**: the restatement follows JAX's documented
  semantics --
    - ``jax.lax.ragged_dot(lhs (M,K), rhs (G,K,N), group_sizes (G,))``:
      rows ``[off_g, off_{g+1})`` of ``lhs`` are multiplied by ``rhs[g]``;
      rows at or past ``sum(group_sizes)`` produce zeros;
    - ``jax.nn.gelu(x, approximate=True)`` =
      ``0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x**3)))``.
* The kernel's block/mask control flow (``src/kernel.py:9-82``) is restated
  in ``fused_kernel_blocks`` and checked against ``ref_ragged_mlp`` (tests);
  it is not executed from the reference's source.
* The host-side group-size generators are pinned against the reference's
  own functions executed here and against the group sizes recorded in the
  reference's ``results/structured_float32/results.csv``.
"""

from __future__ import annotations

import math
from typing import Sequence

import numpy as np

SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def group_sizes_to_offsets(group_sizes: Sequence[int]) -> np.ndarray:
    """``[0, cumsum(gs)]`` -- ``src/kernel.py:126-132``."""
    gs = np.asarray(group_sizes, dtype=np.int64)
    return np.concatenate([np.zeros(1, dtype=np.int64), np.cumsum(gs)])


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """tanh-form GELU, the form ``jax.nn.gelu`` uses by default
    (``approximate=True``), as called at ``src/kernel.py:67``,
    ``src/kernel.py:140-147`` and ``src/ragged_moe_speedup_experiment.py:203-206``.
    Computed in the dtype of ``x``."""
    c = x.dtype.type(SQRT_2_OVER_PI)
    k = x.dtype.type(0.044715)
    half = x.dtype.type(0.5)
    one = x.dtype.type(1.0)
    return half * x * (one + np.tanh(c * (x + k * x * x * x)))


def ragged_dot(lhs: np.ndarray, rhs: np.ndarray, group_sizes: Sequence[int],
               acc_dtype=np.float64) -> np.ndarray:
    """``jax.lax.ragged_dot`` semantics with ``preferred_element_type=acc_dtype``.

    lhs (M, K), rhs (G, K, N), group_sizes (G,) -> (M, N).  Rows past
    ``sum(group_sizes)`` are zero (call sites ``src/kernel.py:137-175``).
    Offsets are clamped to M, matching a well-formed JAX call where
    ``sum(group_sizes) <= M``.
    """
    M = lhs.shape[0]
    G, K, N = rhs.shape
    assert lhs.shape[1] == K, (lhs.shape, rhs.shape)
    out = np.zeros((M, N), dtype=acc_dtype)
    offs = np.minimum(group_sizes_to_offsets(np.maximum(np.asarray(group_sizes), 0)), M)
    for g in range(G):
        a, b = int(offs[g]), int(offs[g + 1])
        if b > a:
            out[a:b] = lhs[a:b].astype(acc_dtype) @ rhs[g].astype(acc_dtype)
    return out


def ref_ragged_mlp(x: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
                   group_sizes: Sequence[int], acc_dtype=np.float64) -> np.ndarray:
    """Two ragged dots with tanh-GELU between -- ``src/kernel.py:152-175``.

    With ``acc_dtype=np.float64`` this is the ground truth the tolerances
    are stated against; with ``np.float32`` it mirrors the reference's
    ``preferred_element_type=jnp.float32`` accumulation.
    """
    h = ragged_dot(x, w_up, group_sizes, acc_dtype)
    h = gelu_tanh(h)
    return ragged_dot(h, w_down, group_sizes, acc_dtype)


def ref_ragged_mlp_fp8(x: np.ndarray, w_up_q: np.ndarray, w_up_scale: np.ndarray,
                       w_down_q: np.ndarray, w_down_scale: np.ndarray,
                       group_sizes: Sequence[int], block: int = 128) -> np.ndarray:
    """The dequantised reference for FP8 block-scaled weights.

    ``W[e, i, j] = float(W_q[e, i, j]) * scale[e, i // block, j // block]``,
    then the same two-ragged-dot path.  ``w_*_q`` are float arrays holding
    the e4m3 values exactly (see :func:`e4m3_decode`).
    """
    return ref_ragged_mlp(x, dequant_block(w_up_q, w_up_scale, block),
                          dequant_block(w_down_q, w_down_scale, block),
                          group_sizes)


def dequant_block(wq: np.ndarray, scale: np.ndarray, block: int = 128) -> np.ndarray:
    E, R, C = wq.shape
    s = np.repeat(np.repeat(scale.astype(np.float64), block, axis=1), block, axis=2)
    return wq.astype(np.float64) * s[:, :R, :C]


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    """Decode OCP FP8 e4m3fn bytes (bias 7, no inf, 0x7f/0xff = NaN)."""
    c = codes.astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return s * val


def fused_kernel_blocks(x: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
                        group_sizes: Sequence[int], *, BM: int, BF: int,
                        max_group_size: int, fill=np.nan) -> np.ndarray:
    """Block-structured restatement of the Pallas kernel ``src/kernel.py:9-82``.

    Grid ``(E, cdiv(max_group_size, BM))`` (``:104-107``); program
    ``(e, pid_m)`` covers rows ``[off_e + pid_m*BM, ...)`` masked to
    ``< off_{e+1}`` (``:18-24``) and retires when ``m_start >= expert_end``
    (``:20``); it streams F in ``BF`` chunks (``:74``), accumulating
    ``gelu(x @ w_up_chunk) @ w_down_chunk`` in f32 (``:38``, ``:67-70``), and
    stores only masked rows (``:77-82``).  Rows never written keep ``fill``
    (the Pallas output buffer is uninitialised there, while ``ragged_dot``
    returns zeros).  Float32 arithmetic throughout, like the kernel.
    """
    M, D = x.shape
    E, _, F = w_up.shape
    assert F % BF == 0 and M % BM == 0
    y = np.full((M, D), fill, dtype=np.float32)
    offs = group_sizes_to_offsets(group_sizes)
    n_pid = -(-max_group_size // BM)
    for e in range(E):
        start, end = int(offs[e]), int(offs[e + 1])
        for pid_m in range(n_pid):
            m_start = start + pid_m * BM
            if not m_start < end:
                continue
            rows = np.arange(m_start, m_start + BM)
            mask = rows < end
            xb = np.zeros((BM, D), np.float32)
            valid = rows[mask]
            valid = valid[valid < M]
            xb[: len(valid)] = x[valid].astype(np.float32)
            acc = np.zeros((BM, D), np.float32)
            for fb in range(F // BF):
                wu = w_up[e, :, fb * BF:(fb + 1) * BF].astype(np.float32)
                wd = w_down[e, fb * BF:(fb + 1) * BF, :].astype(np.float32)
                acc += gelu_tanh(xb @ wu) @ wd
            y[valid] = acc[: len(valid)]
    return y


def correctness_metrics(y_ref: np.ndarray, y: np.ndarray) -> dict:
    """The reference's numerical gate quantities --
    ``src/ragged_moe_speedup_experiment.py:536-580`` and
    ``src/benchmark.py:226-256``."""
    y_ref = np.asarray(y_ref, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    diff = y - y_ref
    absd = np.abs(diff)
    ref_norm = float(np.linalg.norm(y_ref))
    return {
        "max_absolute_error": float(absd.max()) if absd.size else 0.0,
        "mean_absolute_error": float(absd.mean()) if absd.size else 0.0,
        "l2_relative_error": float(np.linalg.norm(diff) / max(ref_norm, 1e-12)),
        "normalized_max_error": float((absd.max() if absd.size else 0.0)
                                      / max(float(np.abs(y_ref).max()) if y_ref.size else 0.0, 1e-12)),
        "reference_is_finite": bool(np.all(np.isfinite(y_ref))),
        "fused_is_finite": bool(np.all(np.isfinite(y))),
    }


def time_cpu_reference(x: np.ndarray, w_up, w_down, group_sizes: Sequence[int]) -> np.ndarray:
    """The reference's unfused path on host cores, in float32 like
    ``ref_ragged_mlp`` (``preferred_element_type=f32``): per-group sgemm
    (BLAS, all threads), tanh-GELU, per-group sgemm.  Used as the timed CPU
    baseline.  ``w_up[e]`` / ``w_down[e]`` may be any per-expert indexable
    (an (E, D, F) array or a list); experts with no rows are not touched."""
    M, D = x.shape
    E = len(group_sizes)
    y = np.zeros((M, D), np.float32)
    offs = np.minimum(group_sizes_to_offsets(np.maximum(np.asarray(group_sizes), 0)), M)
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if b <= a:
            continue
        h = x[a:b].astype(np.float32, copy=False) @ w_up[e].astype(np.float32, copy=False)
        h = gelu_tanh(h)
        y[a:b] = h @ w_down[e].astype(np.float32, copy=False)
    return y


# ----------------------------------------------------------------------------- routing and permutation
# The reference has no router: its benchmarks build `group_sizes` directly
# and feed rows already sorted by expert (README.md:13).  These restate the
# steps on either side of its path that the library's routing kernels
# perform, with numpy's stable sort as the definition of the order.

def route_topk(logits: np.ndarray, k: int):
    """Top-k experts per token (larger logit first, ties to the lower expert
    id) and their weights: the softmax over all experts renormalised to the
    selected ones, which equals the softmax over the selected logits.
    Returns (ids (T, k) int32, weights (T, k) float64)."""
    lg = np.asarray(logits, dtype=np.float64)
    order = np.argsort(-lg, axis=1, kind="stable")[:, :k]
    sel = np.take_along_axis(lg, order, axis=1)
    w = np.exp(sel - sel[:, :1])
    w /= w.sum(axis=1, keepdims=True)
    return order.astype(np.int32), w


def permute_by_expert(ids: np.ndarray, num_experts: int):
    """Stable counting sort of the (token, slot) entries i = t * k + j by
    expert.  Returns (group_sizes (E,), sorted_src (N,) with the entry index
    of each sorted row, inverse (N,) with the sorted row of each entry or -1
    for an id outside [0, E))."""
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    valid = (flat >= 0) & (flat < num_experts)
    idx = np.nonzero(valid)[0]
    order = idx[np.argsort(flat[idx], kind="stable")]
    group_sizes = np.bincount(flat[idx], minlength=num_experts).astype(np.int32)
    inverse = np.full(flat.shape, -1, dtype=np.int64)
    inverse[order] = np.arange(order.size)
    return group_sizes, order.astype(np.int32), inverse.astype(np.int32)


def gather_rows(x: np.ndarray, sorted_src: np.ndarray, k: int) -> np.ndarray:
    """Row r of the result is row sorted_src[r] // k of x."""
    return np.asarray(x)[np.asarray(sorted_src, dtype=np.int64) // k]


def combine_rows(y_sorted: np.ndarray, inverse: np.ndarray, weights: np.ndarray, k: int) -> np.ndarray:
    """y[t] = sum_j weights[t, j] * y_sorted[inverse[t * k + j]] (slots with
    inverse -1 contribute nothing), in float64."""
    inv = np.asarray(inverse, dtype=np.int64).reshape(-1, k)
    w = np.asarray(weights, dtype=np.float64).reshape(-1, k)
    ys = np.asarray(y_sorted, dtype=np.float64)
    y = np.zeros((inv.shape[0], ys.shape[1]))
    for j in range(k):
        ok = inv[:, j] >= 0
        y[ok] += w[ok, j:j + 1] * ys[inv[ok, j]]
    return y


# ----------------------------------------------------------------------------- SwiGLU experts
# The reference's expert MLP is GELU-tanh only (src/kernel.py:46-63).  The
# SwiGLU variant keeps its ragged layout and group_sizes semantics and swaps
# the activation for the gated one of Mixtral / DeepSeek-style experts.

def silu(x: np.ndarray) -> np.ndarray:
    """x * sigmoid(x), in the input's precision."""
    return x / (1.0 + np.exp(-x))


def ref_ragged_swiglu(x: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
                      group_sizes: Sequence[int], acc_dtype=np.float64) -> np.ndarray:
    """Y = ragged_dot(silu(ragged_dot(X, W_gate)) * ragged_dot(X, W_up), W_down);
    rows past sum(group_sizes) are zero, as in ``ref_ragged_mlp``."""
    g = ragged_dot(x, w_gate, group_sizes, acc_dtype)
    u = ragged_dot(x, w_up, group_sizes, acc_dtype)
    return ragged_dot(silu(g) * u, w_down, group_sizes, acc_dtype)


def swiglu_interleave(w_gate: np.ndarray, w_up: np.ndarray, period: int = 128) -> np.ndarray:
    """(E, D, F) gate and up -> (E, D, 2F) with blocks of ``period`` columns
    alternating gate, up, gate, up, ..."""
    E, D, F = w_gate.shape
    g = w_gate.reshape(E, D, F // period, 1, period)
    u = w_up.reshape(E, D, F // period, 1, period)
    return np.concatenate([g, u], axis=3).reshape(E, D, 2 * F)


# ----------------------------------------------------------------------------- backward
# The reference is forward-only (src/kernel.py:9-123).  The gradients of its
# expert MLP, Y = ragged_dot(gelu_tanh(ragged_dot(X, W_up)), W_down), follow
# from the chain rule per expert; rows past sum(group_sizes) take no part.

def gelu_tanh_grad(x: np.ndarray) -> np.ndarray:
    """d/dx of ``gelu_tanh``: 0.5 (1 + t) + 0.5 x (1 - t^2) k0 (1 + 3 k1 x^2),
    t = tanh(k0 (x + k1 x^3))."""
    k0 = np.sqrt(2.0 / np.pi)
    k1 = 0.044715
    t = np.tanh(k0 * (x + k1 * x ** 3))
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * k0 * (1.0 + 3.0 * k1 * x * x)


def ref_ragged_mlp_backward(x: np.ndarray, w_up: np.ndarray, w_down: np.ndarray, group_sizes: Sequence[int],
                            dy: np.ndarray, acc_dtype=np.float64):
    """(dX (M, D), dW_up (E, D, F), dW_down (E, F, D)) of ``ref_ragged_mlp``
    for the upstream gradient dy (M, D): per expert e with rows R,
    A = X_R W_up[e], dA = (dy_R W_down[e]^T) * gelu'(A), dX_R = dA W_up[e]^T,
    dW_up[e] = X_R^T dA, dW_down[e] = gelu(A)^T dy_R.  Rows past
    sum(group_sizes) get dX = 0; experts without rows get zero dW."""
    M, D = x.shape
    E, _, F = w_up.shape
    dx = np.zeros((M, D), acc_dtype)
    dwu = np.zeros((E, D, F), acc_dtype)
    dwd = np.zeros((E, F, D), acc_dtype)
    offs = np.minimum(group_sizes_to_offsets(np.maximum(np.asarray(group_sizes), 0)), M)
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if b <= a:
            continue
        xe = x[a:b].astype(acc_dtype)
        ye = dy[a:b].astype(acc_dtype)
        wu = w_up[e].astype(acc_dtype)
        wd = w_down[e].astype(acc_dtype)
        pre = xe @ wu
        da = (ye @ wd.T) * gelu_tanh_grad(pre)
        dx[a:b] = da @ wu.T
        dwu[e] = xe.T @ da
        dwd[e] = gelu_tanh(pre).T @ ye
    return dx, dwu, dwd


def ref_ragged_swiglu_backward(x: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray,
                               group_sizes: Sequence[int], dy: np.ndarray, acc_dtype=np.float64):
    """(dX, dW_gate, dW_up, dW_down) of ``ref_ragged_swiglu`` for the upstream
    gradient dy: per expert e with rows R, G = X_R W_gate[e], U = X_R W_up[e],
    s = sigmoid(G), dH = dy_R W_down[e]^T, dG = dH U s (1 + G (1 - s)),
    dU = dH G s, dX_R = dG W_gate[e]^T + dU W_up[e]^T, dW_gate[e] = X_R^T dG,
    dW_up[e] = X_R^T dU, dW_down[e] = (G s U)^T dy_R."""
    M, D = x.shape
    E, _, F = w_gate.shape
    dx = np.zeros((M, D), acc_dtype)
    dwg = np.zeros((E, D, F), acc_dtype)
    dwu = np.zeros((E, D, F), acc_dtype)
    dwd = np.zeros((E, F, D), acc_dtype)
    offs = np.minimum(group_sizes_to_offsets(np.maximum(np.asarray(group_sizes), 0)), M)
    for e in range(E):
        a, b = int(offs[e]), int(offs[e + 1])
        if b <= a:
            continue
        xe = x[a:b].astype(acc_dtype)
        ye = dy[a:b].astype(acc_dtype)
        wg, wu, wd = (w[e].astype(acc_dtype) for w in (w_gate, w_up, w_down))
        g = xe @ wg
        u = xe @ wu
        s = 1.0 / (1.0 + np.exp(-g))
        dh = ye @ wd.T
        dg = dh * u * s * (1.0 + g * (1.0 - s))
        du = dh * g * s
        dx[a:b] = dg @ wg.T + du @ wu.T
        dwg[e] = xe.T @ dg
        dwu[e] = xe.T @ du
        dwd[e] = (g * s * u).T @ ye
    return dx, dwg, dwu, dwd
