"""The structured sweep's case grid and traffic model against the
reference's own recorded sweep (the per-shape fixture that
``tests/golden/make_golden.py`` extracts from the reference's results.csv)."""

import json
from pathlib import Path

import numpy as np

from src import sweep
from src.routing import make_group_sizes_pattern

L4 = json.loads((Path(sweep.__file__).resolve().parent / "data" / "l4_structured_float32.json").read_text())


def test_structured_grid_covers_the_reference_sweep():
    shapes = sweep.structured_shapes()
    assert len(shapes) == 20                                 # 18 that ran on L4 + D = 512, 1024
    recorded = {(r["M"], r["D"], r["F"], r["E"]) for r in L4["shapes"]}
    assert recorded <= set(shapes) and len(recorded) == 18
    assert {(16384, 512, 512, 4), (16384, 1024, 512, 4)} == set(shapes) - recorded


def test_group_sizes_and_traffic_model_match_the_reference_rows():
    for r in L4["shapes"]:
        gs = make_group_sizes_pattern(r["M"], r["E"], r["pattern"])
        assert gs.tolist() == r["group_sizes"], r
        m = sweep.theoretical_metrics(r["M"], r["D"], r["F"], r["E"], gs)
        assert m["useful_flops"] == r["useful_flops"]
        assert m["reference_min_bytes"] == r["reference_min_bytes"]
        assert np.isclose(m["ideal_memory_speedup"], r["ideal_memory_speedup"], rtol=1e-12)
