"""Writes ``l4_structured_float32.json``: per shape of the reference's
published structured sweep (its ``results/structured_float32/results.csv``,
measured on an NVIDIA L4), the fused kernel's best median over the swept
(BM, BF) tiles and the median of the unfused ``ragged_dot`` reference.  Run
in a checkout that has the reference under ``/root/reference``; the sweep in
``src/sweep.py`` reads only the JSON it writes."""

import json
from pathlib import Path

import pandas as pd

SRC = Path("/root/reference/results/structured_float32")
OUT = Path(__file__).resolve().parent / "l4_structured_float32.json"


def main() -> None:
    r = pd.read_csv(SRC / "results.csv")
    rows = []
    for (M, D, F, E, pat), g in r.groupby(["M", "D", "F", "E", "group_pattern"]):
        best = g.loc[g.fused_median_ms.idxmin()]
        rows.append({"M": int(M), "D": int(D), "F": int(F), "E": int(E), "pattern": pat,
                     "fused_median_ms": float(best.fused_median_ms), "BM": int(best.BM), "BF": int(best.BF),
                     "ref_median_ms": float(g.ref_median_ms.median()), "tiles": int(len(g)),
                     "group_sizes": json.loads(best.group_sizes), "useful_flops": int(best.useful_flops),
                     "reference_min_bytes": int(best.reference_min_bytes),
                     "ideal_memory_speedup": float(best.ideal_memory_speedup)})
    cfg = json.loads((SRC / "config.json").read_text())
    env = json.loads((SRC / "environment.json").read_text()) if (SRC / "environment.json").exists() else {}
    OUT.write_text(json.dumps({"source": "Krushna-B/pallas-moe-kernel results/structured_float32",
                               "hardware": (env.get("devices") or [{}])[0].get("device_kind", "NVIDIA L4"),
                               "warmup": cfg.get("warmup"), "iterations": cfg.get("iterations"),
                               "shapes": rows}, indent=1, default=str))
    print(OUT, len(rows))


if __name__ == "__main__":
    main()
