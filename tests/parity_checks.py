"""Shared checks for the full-size parity tests (C4, C5 and the bf16 M=65536
point), where the float64 oracle cannot run over every row in seconds.

Two layers:

* ``oracle_rows_check`` -- the tolerance authority.  For EVERY expert with
  rows it picks the expert's first and last row and one random row inside
  every 128-row block of the expert (the kernels' row tiles start at the
  expert's first row and are 128 rows per CTA), runs the float64 oracle on
  those rows, and asserts the L2 relative error of EACH row, so a fault
  confined to one row tile of one expert cannot hide in an average.
* ``torch_screen`` -- a coarse screen over ALL rows: per expert, the same
  two matmuls with the tanh GELU in fp32 torch on the GPU (TF32 off), and
  the L2 relative error of every 128-row block of every expert against the
  kernel's output.  It is a screen only (fp32 rounding), the oracle above
  stays the authority.

A row of Y depends only on its own row of X and its expert's weights, which
is what makes checking sampled rows against the oracle exact.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as orc

BLOCK = 128


def block_rows(a: int, b: int, rng: np.random.Generator, block: int = BLOCK) -> np.ndarray:
    """First and last row of [a, b) and one random row in every ``block``-row
    block counted from ``a``."""
    rows = [a, b - 1]
    for s in range(a, b, block):
        rows.append(int(rng.integers(s, min(s + block, b))))
    return np.unique(np.asarray(rows, dtype=np.int64))


def oracle_rows_check(x, w_up_f32, w_down_f32, gs, y, tol: float, seed: int = 0, experts=None) -> dict:
    """Float64 oracle on sampled rows of every expert (see module doc).

    ``x`` (M, D) and ``y`` (M, D) are device tensors; ``w_up_f32(e)`` /
    ``w_down_f32(e)`` return expert e's weights as (D, F) / (F, D) tensors of
    the values the kernel multiplies (bf16-rounded or dequantised).  Returns
    the worst row error and the number of rows and experts checked."""
    offs = orc.group_sizes_to_offsets(gs)
    rng = np.random.default_rng(seed)
    worst, nrows, nexp = 0.0, 0, 0
    todo = range(len(gs)) if experts is None else experts
    for e in todo:
        a, b = int(offs[e]), int(offs[e + 1])
        if b <= a:
            continue
        rows = block_rows(a, b, rng)
        idx = torch.from_numpy(rows).to(x.device)
        xe = x.index_select(0, idx).double().cpu().numpy()
        wue = w_up_f32(e).double().cpu().numpy()
        wde = w_down_f32(e).double().cpu().numpy()
        ref = orc.gelu_tanh(xe @ wue) @ wde
        got = y.index_select(0, idx).double().cpu().numpy()
        assert np.all(np.isfinite(got)), f"expert {e}: non-finite output"
        err = np.linalg.norm(got - ref, axis=1) / np.maximum(np.linalg.norm(ref, axis=1), 1e-30)
        bad = np.nonzero(err > tol)[0]
        assert bad.size == 0, f"expert {e}: rows {rows[bad][:8].tolist()} L2 rel {err[bad][:8].tolist()} > {tol}"
        worst = max(worst, float(err.max()))
        nrows += rows.size
        nexp += 1
    return {"worst_row_l2_rel": worst, "rows": nrows, "experts": nexp}


def torch_screen(x, w_up_f32, w_down_f32, gs, y, tol: float) -> dict:
    """fp32 torch recomputation of every row, compared per 128-row block of
    every expert (see module doc).  Also checks that rows at or past
    sum(gs) are zero."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        offs = orc.group_sizes_to_offsets(gs)
        worst, nblocks = 0.0, 0
        for e in range(len(gs)):
            a, b = int(offs[e]), int(offs[e + 1])
            if b <= a:
                continue
            h = torch.nn.functional.gelu(x[a:b].float() @ w_up_f32(e).float(), approximate="tanh")
            ref = h @ w_down_f32(e).float()
            got = y[a:b].float()
            assert torch.isfinite(got).all(), f"expert {e}: non-finite output"
            for s in range(0, b - a, BLOCK):
                r, g = ref[s:s + BLOCK], got[s:s + BLOCK]
                err = float(torch.linalg.norm(g - r) / torch.linalg.norm(r).clamp_min(1e-30))
                assert err <= tol, f"expert {e} rows [{a + s}, {min(a + s + BLOCK, b)}): L2 rel {err} > {tol}"
                worst = max(worst, err)
                nblocks += 1
        tail = int(offs[-1])
        assert torch.all(y[tail:] == 0), "rows past sum(group_sizes) must be zero"
        return {"worst_block_l2_rel": worst, "blocks": nblocks}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
