"""Structured sweep of the fused expert MLP on B200, with the reference's
tables, for a case-by-case comparison with its published L4 sweep.

Mirrors the reference's ``SweepConfig(mode="structured")`` run
(``src/ragged_moe_speedup_experiment.py:417-444``, ``run_experiment``
``:844-1217``; grid recorded in its ``results/structured_float32/config.json``):
the baseline shape M=16384, D=128, F=512, E=4, one axis varied at a time over
its values, each shape under the four routing patterns, group sizes from
``make_group_sizes_pattern`` (``:475-493``), f32 inputs, 3 warm-up and 10
timed calls, median.

Per case it times the drop-in ``fused_ragged_dot_caller`` (weights passed raw
every call, as the reference's jitted call receives them) and the unfused
reference algorithm -- two ragged matmuls with the tanh GELU between them,
``ref_ragged_mlp`` (``src/kernel.py:152-175``) -- as f32 torch/cuBLAS on the
same GPU, checks the reference's numerical gate (``:536-580``), adds the
reference's theoretical traffic and padding model (``:583-700``, with this
kernel's 128-row blocks in place of BM), and writes ``results.csv`` /
``failures.csv`` plus the tables of ``src/analyze_results.py`` (speedup by M,
cost vs E, padding buckets, roofline) and ``comparison_l4.csv`` against the
reference's published L4 medians (``data/l4_structured_float32.json``).

Differences, on purpose: there is one row per shape (the kernel has no BM/BF
tile parameters -- its blocks are 128 rows by 64 hidden columns); times are
CUDA events on the device rather than wall clock around
``block_until_ready``.  Usage: ``python -m src.sweep --out <dir>``.
"""

from __future__ import annotations

import argparse
import json
import math
import statistics
import time
from pathlib import Path

import numpy as np

GRID = {  # the reference's structured grid
    "M_values": [128, 256, 512, 1024, 4096, 16384, 65536, 131072],
    "D_values": [64, 128, 256, 512, 1024],
    "F_values": [256, 512, 1024, 2048, 4096],
    "E_values": [1, 2, 4, 8, 16],
    "group_patterns": ["balanced", "mild", "skewed", "one_dominant"],
    "baseline": {"M": 16384, "D": 128, "F": 512, "E": 4},
}
ROW_BLOCK = 128   # rows per work unit of the f32 kernel
HIDDEN_CHUNK = 64


def structured_shapes(grid=GRID):
    """The baseline plus every one-axis variation, in a fixed order."""
    b = grid["baseline"]
    shapes = []
    for axis, values in (("M", grid["M_values"]), ("D", grid["D_values"]), ("F", grid["F_values"]),
                         ("E", grid["E_values"])):
        for v in values:
            s = dict(b)
            s[axis] = v
            t = (s["M"], s["D"], s["F"], s["E"])
            if t not in shapes:
                shapes.append(t)
    return shapes


def theoretical_metrics(M: int, D: int, F: int, E: int, group_sizes, dtype_bytes: int = 4) -> dict:
    """The reference's traffic / padding model (its ``theoretical_metrics``)
    with this kernel's 128-row blocks as the row tile; the fused minimum
    counts the weights of non-empty experts only (the same as the
    reference's whenever every expert has rows, as in all its cases)."""
    gs = [max(int(g), 0) for g in group_sizes]
    blocks = sum(math.ceil(g / ROW_BLOCK) for g in gs)
    slots = blocks * ROW_BLOCK
    useful = 4 * M * D * F
    out_b = 4
    ref_bytes = dtype_bytes * M * D + 2 * dtype_bytes * E * D * F + 2 * out_b * M * F + out_b * M * D
    active = sum(1 for g in gs if g > 0)
    fused_bytes = dtype_bytes * M * D + 2 * dtype_bytes * active * D * F + out_b * M * D
    return {
        "max_group_size": max(gs) if gs else 0, "row_blocks": blocks, "processed_token_slots": slots,
        "padded_rows": slots - M, "row_utilization": M / slots if slots else 0.0,
        "padding_overhead_percent": 100.0 * (slots - M) / M,
        "useful_flops": useful, "actual_fused_flops": 4 * slots * D * F,
        "reference_min_bytes": ref_bytes, "fused_min_bytes": fused_bytes,
        "hidden_activation_bytes": out_b * M * F,
        "ideal_memory_speedup": ref_bytes / fused_bytes,
        "reference_ideal_ai_flops_per_byte": useful / ref_bytes,
        "fused_ideal_ai_flops_per_byte": useful / fused_bytes,
    }


def correctness(ref, y) -> dict:
    """The reference's gate quantities (its ``compute_correctness``)."""
    import torch
    ref64, y64 = ref.double(), y.double()
    diff = (y64 - ref64).abs()
    scale = ref64.abs().max().item()
    m = {
        "max_absolute_error": diff.max().item(),
        "mean_absolute_error": diff.mean().item(),
        "l2_relative_error": (torch.linalg.norm(y64 - ref64) / max(torch.linalg.norm(ref64).item(), 1e-30)).item(),
        "normalized_max_error": diff.max().item() / max(scale, 1e-30),
        "fused_is_finite": bool(torch.isfinite(y).all().item()),
        "reference_is_finite": bool(torch.isfinite(ref).all().item()),
    }
    m["numerically_acceptable"] = (m["fused_is_finite"] and m["reference_is_finite"]
                                   and m["l2_relative_error"] < 1e-4 and m["normalized_max_error"] < 1e-3)
    return m


def _time(fn, warmup: int, iterations: int):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iterations):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    return {"median_ms": statistics.median(ts), "min_ms": ts[0], "max_ms": ts[-1],
            "p10_ms": ts[max(0, int(0.1 * len(ts)) - 0)], "p90_ms": ts[min(len(ts) - 1, int(0.9 * len(ts)))]}


def run_case(M, D, F, E, pattern, seed, warmup, iterations, device):
    import torch
    from .kernel import fused_ragged_dot_caller, ref_ragged_mlp
    from .routing import make_group_sizes_pattern
    gs = make_group_sizes_pattern(M, E, pattern)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((M, D), generator=g, device=device)
    w_up = torch.randn((E, D, F), generator=g, device=device) / math.sqrt(D)
    w_down = torch.randn((E, F, D), generator=g, device=device) / math.sqrt(F)
    gs_dev = torch.from_numpy(gs).to(device)
    gs_host = gs.tolist()
    fused = lambda: fused_ragged_dot_caller(x, w_up, w_down, gs_dev, BM=ROW_BLOCK, BF=HIDDEN_CHUNK,  # noqa: E731
                                            max_group_size=int(gs.max()))
    ref = lambda: ref_ragged_mlp(x, w_up, w_down, gs_host)  # noqa: E731
    tf = _time(fused, warmup, iterations)
    tr = _time(ref, warmup, iterations)
    row = {"M": M, "D": D, "F": F, "E": E, "group_pattern": pattern, "group_sizes": json.dumps(gs.tolist()),
           "input_dtype": "float32", "backend": "b200"}
    row.update(theoretical_metrics(M, D, F, E, gs))
    row.update(correctness(ref(), fused()))
    row.update({f"fused_{k}": v for k, v in tf.items()})
    row.update({f"ref_{k}": v for k, v in tr.items()})
    row["speedup_ref_over_fused"] = tr["median_ms"] / tf["median_ms"]
    row["speedup_percent_of_ideal"] = 100.0 * row["speedup_ref_over_fused"] / row["ideal_memory_speedup"]
    row["fused_useful_tflops"] = row["useful_flops"] / (tf["median_ms"] / 1e3) / 1e12
    row["fused_routed_tokens_per_s"] = M / (tf["median_ms"] / 1e3)
    return row


# --------------------------------------------------------------------- tables (the reference's analyze_results)
def speedup_vs_tokens(df):
    return df.groupby("M").agg(cases=("M", "size"), median_speedup=("speedup_ref_over_fused", "median"),
                               max_speedup=("speedup_ref_over_fused", "max"),
                               median_ideal=("ideal_memory_speedup", "median"),
                               percent_of_ideal=("speedup_percent_of_ideal", "median"))


def cost_vs_experts(df, M=16384, D=128, F=512):
    sub = df[(df.M == M) & (df.D == D) & (df.F == F)]
    t = sub.groupby("E").agg(reference_ms=("ref_median_ms", "median"), fused_ms=("fused_median_ms", "median"),
                             useful_gflops=("useful_flops", "median"))
    t["useful_gflops"] /= 1e9
    t["speedup"] = t.reference_ms / t.fused_ms
    return t


def padding_effect(df):
    import pandas as pd
    b = df.copy()
    b["padding_bucket"] = pd.cut(b.padding_overhead_percent, [-1, 1, 10, 50, 10_000],
                                 labels=["<1%", "1-10%", "10-50%", ">50%"])
    return b.groupby("padding_bucket", observed=True).agg(cases=("M", "size"),
                                                          median_speedup=("speedup_ref_over_fused", "median"),
                                                          median_M=("M", "median"))


def roofline(df, tensor_tflops: float, hbm_gbs: float):
    """Fused time against max(useful FLOPs / the 3xTF32 tensor ceiling,
    fused minimum bytes / HBM bandwidth)."""
    f = df.copy()
    c = f.useful_flops / (tensor_tflops * 1e12)
    m = f.fused_min_bytes / (hbm_gbs * 1e9)
    f["fused_roofline_ms"] = 1e3 * np.maximum(c, m)
    f["fused_efficiency"] = f.fused_roofline_ms / f.fused_median_ms
    f["fused_limiter"] = np.where(c >= m, "compute", "memory")
    return f[["M", "D", "F", "E", "group_pattern", "fused_median_ms", "fused_roofline_ms", "fused_efficiency",
              "fused_limiter"]]


def compare_l4(df):
    import pandas as pd
    l4 = json.loads((Path(__file__).resolve().parent / "data" / "l4_structured_float32.json").read_text())
    ref = pd.DataFrame(l4["shapes"]).rename(columns={"pattern": "group_pattern", "fused_median_ms": "l4_fused_ms",
                                                     "ref_median_ms": "l4_ref_ms", "BM": "l4_best_BM",
                                                     "BF": "l4_best_BF"})
    j = df.merge(ref[["M", "D", "F", "E", "group_pattern", "l4_fused_ms", "l4_best_BM", "l4_best_BF", "l4_ref_ms"]],
                 on=["M", "D", "F", "E", "group_pattern"], how="left")
    j["b200_over_l4_fused_speedup"] = j.l4_fused_ms / j.fused_median_ms
    return j[["M", "D", "F", "E", "group_pattern", "l4_fused_ms", "l4_best_BM", "l4_best_BF", "fused_median_ms",
              "b200_over_l4_fused_speedup", "l4_ref_ms", "ref_median_ms", "speedup_ref_over_fused"]]


def run_sweep(out: Path, seed: int = 0, warmup: int = 3, iterations: int = 10, quick: bool = False) -> dict:
    import pandas as pd
    import torch
    from . import _lib
    device = torch.device("cuda", torch.cuda.current_device())
    out.mkdir(parents=True, exist_ok=True)
    rows, failures = [], []
    shapes = structured_shapes()
    if quick:
        shapes = shapes[:3]
    for i, (M, D, F, E) in enumerate(shapes):
        for j, pattern in enumerate(GRID["group_patterns"]):
            try:
                rows.append(run_case(M, D, F, E, pattern, seed * 1000 + 4 * i + j, warmup, iterations, device))
            except _lib.MoeError as e:   # a shape without a kernel, recorded like the reference's failures.csv
                failures.append({"M": M, "D": D, "F": F, "E": E, "group_pattern": pattern, "error": str(e)})
            torch.cuda.empty_cache()
    status = _lib.device_status(reset=True)
    df = pd.DataFrame(rows)
    df.to_csv(out / "results.csv", index=False)
    pd.DataFrame(failures, columns=["M", "D", "F", "E", "group_pattern", "error"]).to_csv(out / "failures.csv",
                                                                                       index=False)
    speedup_vs_tokens(df).to_csv(out / "summary_by_M.csv")
    cost_vs_experts(df).to_csv(out / "cost_vs_E.csv")
    padding_effect(df).to_csv(out / "padding_effect.csv")
    peaks_path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {}
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    roofline(df, bf16 / 6.0, hbm).to_csv(out / "roofline.csv", index=False)
    compare_l4(df).to_csv(out / "comparison_l4.csv", index=False)
    meta = {"cases": len(rows), "failures": len(failures), "device_status": status,
            "all_numerically_acceptable": bool(df.numerically_acceptable.all()) if len(df) else False,
            "median_speedup_ref_over_fused": float(df.speedup_ref_over_fused.median()) if len(df) else None,
            "device": torch.cuda.get_device_name(device), "warmup": warmup, "iterations": iterations,
            "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}
    (out / "summary.json").write_text(json.dumps(meta, indent=1))
    return meta


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", default="results/b200_structured_float32")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--quick", action="store_true", help="first three shapes only")
    a = ap.parse_args()
    print(json.dumps(run_sweep(Path(a.out), seed=a.seed, quick=a.quick)))


if __name__ == "__main__":
    main()
