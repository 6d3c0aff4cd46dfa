"""Generates the fixtures that pin the host-side routing generators and the
structured sweep's comparison table.

Reads a checkout of the reference (Krushna-B/pallas-moe-kernel), given as the
first argument or in the environment variable ``MOE_REFERENCE_DIR``; only the
fixtures it writes are committed and travel, the reference does not:

* executes ``make_group_sizes`` (src/benchmark.py:42-91) and
  ``routing_weights`` / ``make_group_sizes`` (src/ragged_moe_speedup_experiment.py:455-493)
  -- plain numpy functions, extracted with ``ast`` because their modules
  import JAX at the top -- on a grid of inputs;
* collects the group sizes the reference recorded in
  results/structured_float32/results.csv (M, E, routing pattern -> sizes);
* writes ``analysis_columns.json``: a sample of the published sweep's cases
  with the analysis columns the reference's model recorded for them;
* writes ``pallas-moe-kernel_b200/src/data/l4_structured_float32.json``: per
  shape of that published sweep (measured on an NVIDIA L4), the fused
  kernel's best median over the swept (BM, BF) tiles and the median of the
  unfused ``ragged_dot`` reference, which ``src/sweep.py`` compares against.

Run:  python tests/golden/make_golden.py <reference checkout>
"""

import ast
import csv
import json
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
L4_TABLE = OUT.parent.parent / "pallas-moe-kernel_b200" / "src" / "data" / "l4_structured_float32.json"


def _reference_dir() -> Path:
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MOE_REFERENCE_DIR")
    if not arg:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set MOE_REFERENCE_DIR)")
    ref = Path(arg)
    if not (ref / "src" / "benchmark.py").exists():
        raise SystemExit(f"{ref} does not look like a checkout of the reference (no src/benchmark.py)")
    return ref


def _load_functions(path, names):
    tree = ast.parse(path.read_text())
    fns = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    mod = ast.Module(body=fns, type_ignores=[])
    ns = {"np": np}
    exec(compile(mod, str(path), "exec"), ns)
    return ns


def write_l4_table(ref: Path) -> int:
    """Per-shape summary of the reference's published L4 sweep."""
    import pandas as pd

    src = ref / "results" / "structured_float32"
    r = pd.read_csv(src / "results.csv")
    rows = []
    for (M, D, F, E, pat), g in r.groupby(["M", "D", "F", "E", "group_pattern"]):
        best = g.loc[g.fused_median_ms.idxmin()]
        rows.append({"M": int(M), "D": int(D), "F": int(F), "E": int(E), "pattern": pat,
                     "fused_median_ms": float(best.fused_median_ms), "BM": int(best.BM), "BF": int(best.BF),
                     "ref_median_ms": float(g.ref_median_ms.median()), "tiles": int(len(g)),
                     "group_sizes": json.loads(best.group_sizes), "useful_flops": int(best.useful_flops),
                     "reference_min_bytes": int(best.reference_min_bytes),
                     "ideal_memory_speedup": float(best.ideal_memory_speedup)})
    cfg = json.loads((src / "config.json").read_text())
    env = json.loads((src / "environment.json").read_text()) if (src / "environment.json").exists() else {}
    L4_TABLE.write_text(json.dumps({"source": "Krushna-B/pallas-moe-kernel results/structured_float32",
                                    "hardware": (env.get("devices") or [{}])[0].get("device_kind", "NVIDIA L4"),
                                    "warmup": cfg.get("warmup"), "iterations": cfg.get("iterations"),
                                    "shapes": rows}, indent=1, default=str))
    return len(rows)


ANALYSIS_COLUMNS = [
    "max_group_size", "programs_per_expert", "active_programs_Q", "launched_programs", "inactive_programs",
    "grid_utilization", "processed_token_slots", "padded_rows", "row_utilization", "padding_overhead_fraction",
    "padding_overhead_percent", "padding_overcompute_factor", "hidden_chunks_F_over_BF", "useful_flops",
    "actual_fused_flops", "padding_extra_flops", "reference_min_bytes", "fused_min_bytes",
    "hidden_activation_bytes", "hidden_intermediate_mib", "hidden_write_read_saved_bytes",
    "memory_saved_fraction", "memory_saved_percent", "fused_no_cache_bytes", "fused_tile_upper_bytes",
    "minimum_weight_bytes", "no_cache_weight_bytes", "weight_reread_factor_no_cache",
    "reference_ideal_ai_flops_per_byte", "fused_ideal_effective_ai_flops_per_byte",
    "fused_ideal_actual_ai_flops_per_byte", "fused_no_cache_actual_ai_flops_per_byte",
    "fused_per_program_ai_flops_per_byte", "fused_large_F_ai_approximation", "expansion_ratio_F_over_D",
    "token_to_expert_hidden_ratio_M_over_EF", "fraction_of_asymptotic_benefit",
    "fraction_of_asymptotic_benefit_percent", "asymptotic_max_memory_speedup", "ideal_memory_speedup",
    "logical_tile_shared_bytes", "inferred_one_extra_stage_shared_bytes",
]


def write_analysis_columns(ref: Path) -> int:
    """Every 7th row of the reference's published sweep: the case's inputs
    and the analysis columns it recorded (the values its model produced)."""
    rows = []
    with open(ref / "results" / "structured_float32" / "results.csv") as f:
        for i, row in enumerate(csv.DictReader(f)):
            if i % 7:
                continue
            case = {k: int(row[k]) for k in ("M", "D", "F", "E", "BM", "BF")}
            case["group_sizes"] = json.loads(row["group_sizes"].replace("(", "[").replace(")", "]"))
            case["dtype_bytes"] = 4
            case["recorded"] = {c: (json.loads(row[c]) if c == "programs_per_expert" else float(row[c]))
                                for c in ANALYSIS_COLUMNS}
            rows.append(case)
    (OUT / "analysis_columns.json").write_text(json.dumps({
        "source": "results/structured_float32/results.csv of the reference (every 7th row)",
        "cases": rows}, indent=0))
    return len(rows)


def main():
    REF = _reference_dir()
    bench = _load_functions(REF / "src/benchmark.py", {"make_group_sizes"})
    exp = _load_functions(REF / "src/ragged_moe_speedup_experiment.py", {"routing_weights", "make_group_sizes"})

    cases_bench = []
    for M in (4, 16, 100, 1000, 2048, 4096, 65536, 131072):
        for E in (1, 2, 3, 4, 7, 8, 16):
            if M < E:
                continue
            cases_bench.append({"M": M, "E": E, "fractions": None,
                                "sizes": bench["make_group_sizes"](M, E).tolist()})
    for M, E, fr in ((2048, 4, [470, 530, 421, 627]), (1000, 3, [0.2, 0.3, 0.5]), (4097, 5, [1, 1, 1, 1, 1])):
        cases_bench.append({"M": M, "E": E, "fractions": fr,
                            "sizes": bench["make_group_sizes"](M, E, group_fractions=fr).tolist()})

    cases_exp = []
    for pattern in ("balanced", "mild", "skewed", "one_dominant"):
        for E in (1, 2, 4, 8, 16):
            w = exp["routing_weights"](E, pattern)
            for M in (16, 128, 1024, 16384, 131072):
                if M < E:
                    continue
                cases_exp.append({"M": M, "E": E, "pattern": pattern, "weights": w.tolist(),
                                  "sizes": exp["make_group_sizes"](M, E, pattern).tolist()})

    recorded = {}
    with open(REF / "results/structured_float32/results.csv") as f:
        for row in csv.DictReader(f):
            key = (int(row["M"]), int(row["E"]), row["group_pattern"])
            sizes = json.loads(row["group_sizes"].replace("(", "[").replace(")", "]"))
            recorded[key] = sizes
    recorded_list = [{"M": k[0], "E": k[1], "pattern": k[2], "sizes": v} for k, v in sorted(recorded.items())]

    (OUT / "group_sizes.json").write_text(json.dumps({
        "source": "reference functions executed from src/benchmark.py and src/ragged_moe_speedup_experiment.py; "
                  "recorded sizes from results/structured_float32/results.csv",
        "benchmark_make_group_sizes": cases_bench,
        "experiment_make_group_sizes": cases_exp,
        "results_csv_recorded": recorded_list,
    }, indent=0))
    print(len(cases_bench), len(cases_exp), len(recorded_list), write_l4_table(REF), write_analysis_columns(REF))


if __name__ == "__main__":
    main()
