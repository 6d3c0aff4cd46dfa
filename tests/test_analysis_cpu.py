"""The analytic model (src/analysis.py) on the CPU.

* Its reference layer reproduces the analysis columns the reference's model
  recorded for its published sweep (tests/golden/analysis_columns.json,
  every 7th case of results/structured_float32/results.csv).
* Its B200 layer reads the library's real launch plan (moe_describe_plan,
  no device needed) and turns group sizes into work units, padding, waves,
  issued tensor work and compulsory DRAM bytes; checked here on cases worked
  out by hand, against the library's launch counts, and against the DRAM
  bytes that ncu measured for the C4 grouped GEMMs (profiles/).
"""

import json
import math
from pathlib import Path

import pytest

from src import _lib, analysis
from src.routing import CONFIGS, config_group_sizes

GOLDEN = Path(__file__).resolve().parent / "golden" / "analysis_columns.json"
PROFILES = Path(__file__).resolve().parent.parent / "profiles"


def test_reference_layer_matches_recorded_sweep_columns():
    cases = json.loads(GOLDEN.read_text())["cases"]
    assert len(cases) >= 80
    for c in cases:
        got = analysis.reference_metrics(c["M"], c["E"], c["D"], c["F"], c["BM"], c["BF"], c["group_sizes"],
                                         c["dtype_bytes"])
        for k, want in c["recorded"].items():
            if isinstance(want, list):
                assert got[k] == want, (k, c["M"], c["D"], c["F"], c["E"])
            else:
                assert math.isclose(got[k], want, rel_tol=1e-12, abs_tol=1e-12), (k, got[k], want, c)


def test_reference_entry_point_sections():
    gs = [300, 0, 500, 224]
    r = analysis.analyze_ragged_moe(M=1024, E=4, D=128, F=512, BM=32, BF=32, group_sizes=gs, ref_ms=2.0,
                                    fused_ms=0.5, peak_compute_tflops=30.3, peak_bandwidth_gbps=300.0,
                                    compiled_shared_bytes=90000, shared_memory_limit_bytes=101376)
    assert r["active_programs_Q"] == 10 + 0 + 16 + 7
    assert r["launched_programs"] == 4 * 16 and r["inactive_programs"] == 64 - 33
    assert r["measured_speedup"] == 4.0
    assert r["fused_ideal_roofline_limiter"] in ("compute", "memory")
    assert r["compiled_shared_fits"] is True
    assert [p["padded_rows"] for p in r["per_expert"]] == [20, 0, 12, 0]
    with pytest.raises(ValueError):
        analysis.analyze_ragged_moe(M=1024, E=4, D=128, F=512, BM=32, BF=48, group_sizes=gs)
    with pytest.raises(ValueError):
        analysis.reference_metrics(1000, 4, 128, 512, 32, 32, gs, 4)   # sizes do not sum to M


def test_plan_matches_library_launch_counts():
    for name in ("c4", "c5"):
        cfg = CONFIGS[name]
        plan = _lib.describe_plan(cfg.M, cfg.D, cfg.F, cfg.E, analysis.DTYPE_CODES[cfg.dtype])
        assert len(plan) == _lib.lib().moe_fused_mlp_launch_count(cfg.M, cfg.D, cfg.F, cfg.E,
                                                                  analysis.DTYPE_CODES[cfg.dtype])
        for L in plan:
            assert L["smem_bytes"] <= analysis.SMEM_LIMIT and L["tmem_cols"] <= analysis.TMEM_COLS
    f32_large = _lib.describe_plan(2048, 512, 512, 4, 0)
    assert [L["kernel"] for L in f32_large] == ["small_prep_kernel", "grouped_gemm_pair_kernel (up)",
                                               "grouped_gemm_pair_kernel (down)"]
    assert all(L["mma"] == "kind::tf32 x3" and L["accumulators"] == 1 for L in f32_large[1:])
    small = _lib.describe_plan(65536, 128, 512, 8, 0)
    assert small[-1]["kernel"] == "fused_mlp_small_kernel" and small[-1]["tile_m"] == 128


def test_b200_layer_by_hand():
    gs = [255, 257, 1, 511]                   # pair tiles of 256 rows: 1 + 2 + 1 + 2 = 6 row blocks
    m = analysis.b200_model(1024, 512, 512, 4, gs, "bf16")
    up, down = m["launches"]
    assert up["units"] == 6 * 2 and down["units"] == 6 * 2   # 256-column tiles: 2 per row block
    _lib.set_tuning(8, 2)                     # the down GEMM's optional 512-column tiles
    try:
        wide = analysis.b200_model(1024, 512, 512, 4, gs, "bf16")["launches"][1]
    finally:
        _lib.set_tuning(8, 0)
    assert wide["units"] == 6 * 1 and wide["tile_n"] == 512 and wide["accumulators"] == 1
    assert up["rows_processed"] == 6 * 256 and up["padded_rows"] == 6 * 256 - 1024
    assert up["issued_f16_equiv_flops"] == 2 * 1536 * 512 * 512
    assert up["useful_flops"] == 2 * 1024 * 512 * 512
    assert up["waves"] == pytest.approx(12 / 74)
    # f32: three tf32 products at half the f16 rate = 6 bf16-equivalent
    m32 = analysis.b200_model(1024, 512, 512, 4, gs, "f32")
    assert m32["launches"][1]["issued_f16_equiv_flops"] == 6 * up["issued_f16_equiv_flops"]
    # negative sizes count as zero and the running total is cut at M
    assert analysis.clamp_group_sizes(100, [50, -3, 80, 10]) == [50, 0, 50, 0]


def test_roofline_is_the_bench_figure():
    import bench
    for name in ("c1", "c2", "c3", "c4", "c5"):
        cfg = CONFIGS[name]
        gs = config_group_sizes(cfg, 0)
        a = analysis.algorithmic_work(cfg.M, cfg.D, cfg.F, gs, cfg.dtype)
        b = bench.algorithmic(cfg, gs)
        assert a["flops"] == b["flops"] and a["bytes"] == b["bytes"], name
    r = analysis.roofline(32768, 4096, 14336, config_group_sizes(CONFIGS["c4"], 0), "bf16", kernel_ms=5.426,
                          peaks={"bf16_tflops": 1669.0, "hbm_gbs": 6547.2})
    assert r["bound"] == "tensor" and r["frac"] == pytest.approx(7696581394432 / 5.426e-3 / 1e12 / 1669.0)


def test_compulsory_bytes_bound_the_measured_c4_traffic():
    """ncu's DRAM bytes for the two grouped GEMMs of the C4 step (profiles/)
    are never below the model's compulsory bytes, and the table in the
    profile records how far above they are (weight and H re-reads)."""
    prof = json.loads((PROFILES / "traffic_c4_bf16_M32768_D4096_F14336_E8_top2.json").read_text())
    for case in prof["by_rows"]:
        M = case["M"]
        cfg = CONFIGS["c4"]
        gs = config_group_sizes(cfg.__class__(cfg.name, M, cfg.D, cfg.F, cfg.E, cfg.dtype, cfg.routing, M // 2), 0)
        model = analysis.b200_model(M, cfg.D, cfg.F, cfg.E, gs, "bf16")
        comp = {L["kernel"].split()[-1].strip("()"): L["compulsory_dram_bytes"] for L in model["launches"]}
        for k in ("up", "down"):
            measured = case[k]["read"] + case[k]["write"]
            assert measured >= 0.97 * comp[k], (M, k, measured, comp[k])
            assert measured / comp[k] == pytest.approx(case[k]["over_compulsory"], rel=1e-3)
