"""Generates the golden fixtures that pin the host-side routing generators.

Reads the reference's own sources from /root/reference (this container only;
the fixtures travel, the reference does not):

* executes ``make_group_sizes`` (src/benchmark.py:42-91) and
  ``routing_weights`` / ``make_group_sizes`` (src/ragged_moe_speedup_experiment.py:455-493)
  -- plain numpy functions, extracted with ``ast`` because their modules
  import JAX at the top -- on a grid of inputs;
* collects the group sizes the reference recorded in
  results/structured_float32/results.csv (M, E, routing pattern -> sizes).

Run:  python tests/golden/make_golden.py
"""

import ast
import csv
import json
from pathlib import Path

import numpy as np

REF = Path("/root/reference")
OUT = Path(__file__).resolve().parent


def _load_functions(path, names):
    tree = ast.parse(path.read_text())
    fns = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    mod = ast.Module(body=fns, type_ignores=[])
    ns = {"np": np}
    exec(compile(mod, str(path), "exec"), ns)
    return ns


def main():
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
    print(len(cases_bench), len(cases_exp), len(recorded_list))


if __name__ == "__main__":
    main()
