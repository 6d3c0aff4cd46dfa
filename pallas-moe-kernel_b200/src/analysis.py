"""Analytic model of the fused ragged MoE expert MLP: work, traffic, tiling
and roofline.

Two layers.

1. The reference's model (``src/analysis.py:51-474`` ``analyze_ragged_moe``
   and the sweep's ``theoretical_metrics``,
   ``src/ragged_moe_speedup_experiment.py:583-700``): for a Pallas grid of
   (E, ceil(max_group / BM)) programs of BM rows, the padding and grid
   utilisation, useful and padded FLOPs, the traffic bounds of the unfused
   and fused paths, arithmetic intensities, the ideal memory speedup and the
   source-level shared-memory tile estimate.  ``reference_metrics`` returns
   them under the reference's own column names, and the tests pin them to
   the values its published sweep recorded (``results.csv``).
   ``analyze_ragged_moe`` keeps the reference's signature (timing, roofline
   and shared-memory sections included).

2. The B200 model of this library (``b200_model``): the launch plan the
   library would run (``moe_describe_plan``: kernel, persistent grid,
   threads, shared memory, TMEM columns, cluster, tile shape, pipeline
   stages, tcgen05 MMA kind, F-splits), and per launch the work units the
   group sizes produce (256-row x 256-column pair tiles of the grouped GEMMs,
   expert super-tiles of up to 384 tokens x 256 features for small experts
   with e4m3 weights, 128-row blocks x F-splits of the fused small-D kernel),
   padded rows, waves
   over the persistent grid, tensor work issued (padding and the three
   products of 3xTF32 included, in bf16-equivalent FLOPs), compulsory DRAM
   bytes (every operand once, H's round trip on the two-GEMM path, the tf32
   operand planes), and the roofline times against the peaks measured on
   this pool's B200s (``MEASURED_PEAKS.json``).  ``roofline`` is the figure
   ``bench.py`` reports: useful FLOPs = 4 M D F (GELU excluded, as
   ``src/analysis.py:87-88``), algorithmic bytes = X + the non-empty
   experts' weights (+ FP8 block scales) + f32 Y.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Any, Optional, Sequence

DTYPE_CODES = {"f32": 0, "bf16": 1, "fp8": 2}
IN_BYTES = {"f32": 4, "bf16": 2, "fp8": 2}      # X as passed to the call (FP8 weights take bf16 X)
W_BYTES = {"f32": 4, "bf16": 2, "fp8": 1}
SMEM_LIMIT = 232448                               # bytes per CTA (227 KB opt-in)
TMEM_COLS = 512                                   # f32 columns x 128 lanes per SM
F16_FLOP_PER_CLK_SM = 8192                        # kind::f16: M=128, N=256, K=16 in 128 cycles
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ============================================================================ the reference's model
def reference_metrics(M: int, E: int, D: int, F: int, BM: int, BF: int, group_sizes: Sequence[int],
                      dtype_bytes: int = 4) -> dict[str, Any]:
    """The reference sweep's theoretical columns for one case (f32 outputs:
    H and Y count 4 bytes per element, inputs and weights ``dtype_bytes``)."""
    g = [int(v) for v in group_sizes]
    if len(g) != E or any(v < 0 for v in g) or sum(g) != M:
        raise ValueError(f"group sizes {g} do not describe M={M} rows over E={E} experts")
    b, ob = dtype_bytes, 4
    progs = [-(-v // BM) for v in g]
    Q = sum(progs)
    launched = E * -(-max(g) // BM)
    slots = Q * BM
    useful = 4 * M * D * F
    actual = 4 * slots * D * F
    ref_min = b * M * D + 2 * b * E * D * F + 2 * ob * M * F + ob * M * D
    fused_min = b * M * D + 2 * b * E * D * F + ob * M * D
    hidden = ob * M * F
    no_cache = b * M * D + 2 * b * Q * D * F + ob * M * D
    w_min, w_nc = 2 * b * E * D * F, 2 * b * Q * D * F
    frac_asym = M / (M + E * F)
    return {
        "max_group_size": max(g),
        "programs_per_expert": progs,
        "active_programs_Q": Q,
        "launched_programs": launched,
        "inactive_programs": launched - Q,
        "grid_utilization": Q / launched,
        "processed_token_slots": slots,
        "padded_rows": slots - M,
        "row_utilization": M / slots,
        "padding_overhead_fraction": (slots - M) / M,
        "padding_overhead_percent": 100.0 * (slots - M) / M,
        "padding_overcompute_factor": slots / M,
        "hidden_chunks_F_over_BF": F // BF,
        "useful_flops": useful,
        "actual_fused_flops": actual,
        "padding_extra_flops": actual - useful,
        "reference_min_bytes": ref_min,
        "fused_min_bytes": fused_min,
        "hidden_activation_bytes": hidden,
        "hidden_intermediate_mib": hidden / 2 ** 20,
        "hidden_write_read_saved_bytes": 2 * hidden,
        "memory_saved_fraction": 2 * hidden / ref_min,
        "memory_saved_percent": 100.0 * 2 * hidden / ref_min,
        "fused_no_cache_bytes": no_cache,
        "fused_tile_upper_bytes": Q * ((b + ob) * BM * D + 2 * b * D * F),
        "minimum_weight_bytes": w_min,
        "no_cache_weight_bytes": w_nc,
        "weight_reread_factor_no_cache": w_nc / w_min,
        "reference_ideal_ai_flops_per_byte": useful / ref_min,
        "fused_ideal_effective_ai_flops_per_byte": useful / fused_min,
        "fused_ideal_actual_ai_flops_per_byte": actual / fused_min,
        "fused_no_cache_actual_ai_flops_per_byte": actual / no_cache,
        "fused_per_program_ai_flops_per_byte": 4 * BM * F / (BM * (b + ob) + 2 * b * F),
        "fused_large_F_ai_approximation": 2 * BM / b,
        "expansion_ratio_F_over_D": F / D,
        "token_to_expert_hidden_ratio_M_over_EF": M / (E * F),
        "fraction_of_asymptotic_benefit": frac_asym,
        "fraction_of_asymptotic_benefit_percent": 100.0 * frac_asym,
        "asymptotic_max_memory_speedup": 1 + F / D,
        "ideal_memory_speedup": ref_min / fused_min,
        "logical_tile_shared_bytes": b * (2 * BM * D + 2 * D * BF + BM * BF),
        "inferred_one_extra_stage_shared_bytes": b * (2 * BM * D + 3 * D * BF + BM * BF),
    }


def analyze_ragged_moe(*, M: int, E: int, D: int, F: int, BM: int, BF: int, group_sizes: Sequence[int],
                       dtype_bytes: int = 4, ref_ms: Optional[float] = None, fused_ms: Optional[float] = None,
                       measured_speedup: Optional[float] = None, peak_compute_tflops: Optional[float] = None,
                       peak_bandwidth_gbps: Optional[float] = None, compiled_shared_bytes: Optional[int] = None,
                       shared_memory_limit_bytes: Optional[int] = None, print_results: bool = False) -> dict:
    """The reference's analysis entry point (same arguments): the theoretical
    columns, plus timing, roofline and shared-memory sections when their
    inputs are given.  ``print_results`` prints the result as JSON."""
    for name, v in (("M", M), ("E", E), ("D", D), ("F", F), ("BM", BM), ("BF", BF), ("dtype_bytes", dtype_bytes)):
        if not isinstance(v, int) or v <= 0:
            raise ValueError(f"{name} must be a positive integer, got {v!r}")
    if F % BF:
        raise ValueError(f"BF={BF} must divide F={F}")
    if (ref_ms is None) != (fused_ms is None):
        raise ValueError("give both ref_ms and fused_ms, or neither")
    out = reference_metrics(M, E, D, F, BM, BF, group_sizes, dtype_bytes)
    if ref_ms is not None:
        if ref_ms <= 0 or fused_ms <= 0:
            raise ValueError("latencies must be positive")
        s = ref_ms / fused_ms
        if measured_speedup is not None and abs(measured_speedup - s) > 1e-3:
            raise ValueError(f"measured_speedup {measured_speedup} disagrees with ref_ms / fused_ms = {s}")
        measured_speedup = s
        out.update({
            "ref_ms": ref_ms, "fused_ms": fused_ms, "measured_speedup": s,
            "ref_tokens_per_second": M / (ref_ms / 1e3), "fused_tokens_per_second": M / (fused_ms / 1e3),
            "ref_effective_tflops": out["useful_flops"] / (ref_ms / 1e3) / 1e12,
            "fused_effective_tflops": out["useful_flops"] / (fused_ms / 1e3) / 1e12,
            "fused_actual_tflops": out["actual_fused_flops"] / (fused_ms / 1e3) / 1e12,
            "ref_minimum_traffic_gbps": out["reference_min_bytes"] / (ref_ms / 1e3) / 1e9,
            "fused_minimum_traffic_gbps": out["fused_min_bytes"] / (fused_ms / 1e3) / 1e9,
            "fused_no_cache_traffic_gbps": out["fused_no_cache_bytes"] / (fused_ms / 1e3) / 1e9,
        })
    if measured_speedup is not None:
        ideal = out["ideal_memory_speedup"]
        out.update({
            "measured_speedup": measured_speedup,
            "speedup_as_fraction_of_ideal": measured_speedup / ideal,
            "speedup_percent_of_ideal": 100.0 * measured_speedup / ideal,
            "speedup_gap_from_ideal": ideal - measured_speedup,
            "speedup_gap_percent_of_ideal": 100.0 * (ideal - measured_speedup) / ideal,
            "incremental_fusion_benefit_fraction": (measured_speedup - 1) / (ideal - 1) if ideal > 1 else math.nan,
        })
    if peak_compute_tflops is not None and peak_bandwidth_gbps is not None:
        P, B = peak_compute_tflops * 1e12, peak_bandwidth_gbps * 1e9
        rc, rm = out["useful_flops"] / P, out["reference_min_bytes"] / B
        fc, fm, fn = out["actual_fused_flops"] / P, out["fused_min_bytes"] / B, out["fused_no_cache_bytes"] / B
        r_roof, f_roof, n_roof = max(rc, rm), max(fc, fm), max(fc, fn)
        out.update({
            "peak_compute_tflops": peak_compute_tflops, "peak_bandwidth_gbps": peak_bandwidth_gbps,
            "ridge_point_flops_per_byte": P / B,
            "reference_compute_bound_ms": rc * 1e3, "reference_memory_bound_ms": rm * 1e3,
            "reference_roofline_ms": r_roof * 1e3, "reference_roofline_limiter": "compute" if rc >= rm else "memory",
            "fused_compute_bound_ms": fc * 1e3, "fused_ideal_memory_bound_ms": fm * 1e3,
            "fused_ideal_roofline_ms": f_roof * 1e3, "fused_ideal_roofline_limiter": "compute" if fc >= fm else "memory",
            "fused_no_cache_memory_bound_ms": fn * 1e3, "fused_no_cache_roofline_ms": n_roof * 1e3,
            "fused_no_cache_roofline_limiter": "compute" if fc >= fn else "memory",
            "ideal_roofline_speedup": r_roof / f_roof, "no_cache_roofline_speedup": r_roof / n_roof,
        })
        if ref_ms is not None:
            rs, fs = ref_ms / 1e3, fused_ms / 1e3
            out.update({
                "reference_roofline_efficiency": r_roof / rs, "fused_ideal_roofline_efficiency": f_roof / fs,
                "fused_no_cache_roofline_efficiency": n_roof / fs,
                "reference_compute_utilization": out["useful_flops"] / rs / P,
                "fused_effective_compute_utilization": out["useful_flops"] / fs / P,
                "fused_actual_compute_utilization": out["actual_fused_flops"] / fs / P,
            })
    if compiled_shared_bytes is not None:
        out["compiled_shared_bytes"] = compiled_shared_bytes
    if shared_memory_limit_bytes is not None:
        lim = shared_memory_limit_bytes
        out["shared_memory_limit_bytes"] = lim
        out["logical_shared_fraction_of_limit"] = out["logical_tile_shared_bytes"] / lim
        out["inferred_shared_fraction_of_limit"] = out["inferred_one_extra_stage_shared_bytes"] / lim
        if compiled_shared_bytes is not None:
            out["compiled_shared_fraction_of_limit"] = compiled_shared_bytes / lim
            out["compiled_shared_fits"] = compiled_shared_bytes <= lim
    offs = [0]
    for v in group_sizes:
        offs.append(offs[-1] + int(v))
    out["per_expert"] = [{"expert_id": e, "start_offset": offs[e], "end_offset": offs[e + 1],
                          "group_size": int(group_sizes[e]), "active_programs": p, "processed_row_slots": p * BM,
                          "padded_rows": p * BM - int(group_sizes[e]),
                          "row_utilization": int(group_sizes[e]) / (p * BM) if p else None}
                         for e, p in enumerate(out["programs_per_expert"])]
    if print_results:
        print(json.dumps(out, indent=1, default=str))
    return out


# ============================================================================ the B200 model
def load_peaks(path: Optional[Path] = None) -> tuple[dict, str]:
    """Peaks measured on this pool's B200s (HBM copy GB/s, cuBLAS bf16
    TF/s burst and sustained), else the pool's earlier fallback figures."""
    p = Path(path) if path else Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


def clamp_group_sizes(M: int, group_sizes: Sequence[int]) -> list[int]:
    """The rows each expert actually gets from the kernels: negatives count
    as 0 and the running total is cut at M (the library's clamping)."""
    out, total = [], 0
    for v in group_sizes:
        g = max(int(v), 0)
        g = min(g, max(M - total, 0))
        out.append(g)
        total += g
    return out


def algorithmic_work(M: int, D: int, F: int, group_sizes: Sequence[int], dtype: str) -> dict:
    """Useful FLOPs (4 M D F, every routed row; GELU excluded) and
    algorithmic bytes: X + the non-empty experts' two weight matrices (+ the
    128x128 f32 block scales of e4m3 weights) + f32 Y."""
    g = clamp_group_sizes(M, group_sizes)
    routed = sum(g)
    active = sum(1 for v in g if v > 0)
    scales = 2 * math.ceil(D / 128) * math.ceil(F / 128) * 4 if dtype == "fp8" else 0
    byts = M * D * IN_BYTES[dtype] + active * (2 * D * F * W_BYTES[dtype] + scales) + M * D * 4
    return {"flops": 4 * routed * D * F, "bytes": byts, "routed_rows": routed, "active_experts": active}


def tensor_peak(dtype: str, peaks: dict) -> float:
    """Useful-FLOP tensor ceiling in TF/s: the measured bf16 rate, a sixth of
    it for 3xTF32 (kind::tf32 issues at half the f16 rate, three products per
    f32 product); e4m3 weights run on f16 operands at the bf16 rate."""
    bf16 = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    return bf16 / 6.0 if dtype == "f32" else bf16


def roofline(M: int, D: int, F: int, group_sizes: Sequence[int], dtype: str, kernel_ms: Optional[float] = None,
             peaks: Optional[dict] = None) -> dict:
    """The roofline figure bench.py reports: t_roof = max(useful FLOPs /
    tensor ceiling, algorithmic bytes / HBM), and with a measured time the
    achieved rate and its fraction of the ceiling of the bound resource."""
    if peaks is None:
        peaks, _ = load_peaks()
    w = algorithmic_work(M, D, F, group_sizes, dtype)
    P = tensor_peak(dtype, peaks)
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    t_c, t_m = w["flops"] / (P * 1e12), w["bytes"] / (hbm * 1e9)
    out = {"bound": "tensor" if t_c >= t_m else "hbm", "t_roof_ms": max(t_c, t_m) * 1e3,
           "t_tensor_ms": t_c * 1e3, "t_hbm_ms": t_m * 1e3, "tensor_peak_tflops": P, "hbm_gbs": hbm,
           "algorithmic_flops": w["flops"], "algorithmic_bytes": w["bytes"]}
    if kernel_ms:
        s = kernel_ms / 1e3
        if out["bound"] == "tensor":
            out.update(achieved=w["flops"] / s / 1e12, peak=P, unit="TFLOP/s")
        else:
            out.update(achieved=w["bytes"] / s / 1e9, peak=hbm, unit="GB/s")
        out["frac"] = out["achieved"] / out["peak"]
    return out


_PRODUCTS = {0: 0, 1: 1, 2: 1, 3: 6, 4: 1}  # bf16-equivalent MMA work per useful multiply-add, per MMA kind


def _launch_model(L: dict, M: int, D: int, F: int, E: int, g: list[int], dtype: str) -> dict:
    name = L["kernel"]
    out = dict(L)
    routed = sum(g)
    active = sum(1 for v in g if v > 0)
    if name.startswith("grouped_gemm_pair_kernel") or name.startswith("grouped_gemm_swap_kernel"):
        N, K = L["gemm_n"], L["gemm_k"]
        ncol = -(-N // L["tile_n"])
        if name.startswith("grouped_gemm_swap_kernel"):
            # expert super-tiles of tile_m tokens: chunks of <= 256 and <= 128
            # tokens, each an MMA with N = its tokens rounded up to 32
            st = [-(-v // L["tile_m"]) for v in g]
            tiles = sum(st) * ncol
            rows_pad = 0
            for v in g:
                for k in range(-(-v // L["tile_m"])):
                    rem = v - k * L["tile_m"]
                    n0 = min(rem, 256)
                    n1 = min(max(rem - 256, 0), 128)
                    rows_pad += -(-n0 // 32) * 32 + -(-n1 // 32) * 32
        else:
            rows_blocks = [-(-v // L["tile_m"]) for v in g]
            tiles = sum(rows_blocks) * ncol
            rows_pad = sum(rows_blocks) * L["tile_m"]
        workers = L["grid"] // L["cluster"]
        up = name.endswith("(up)")
        k_pad = -(-K // L["stage_k"]) * L["stage_k"]
        issued = 2 * rows_pad * ncol * L["tile_n"] * k_pad * _PRODUCTS[L["mma_kind"]]
        a_b = {"bf16": 2, "fp8": 2, "f32": 8}[dtype]          # A (X or H) as the GEMM reads it (tf32: hi + lo)
        b_b = {"bf16": 2, "fp8": 1, "f32": 8}[dtype]          # weights as read (tf32: hi + lo planes)
        c_b = (2 if dtype != "f32" else 8) if up else 4       # H (bf16/f16, or tf32 planes) or Y f32
        scales = math.ceil(K / 128) * math.ceil(N / 128) * 4 if dtype == "fp8" else 0
        dram = routed * K * a_b + active * (K * N * b_b + scales) + routed * N * c_b
        if not up:
            dram += (M - routed) * N * 4                      # Y rows past sum(gs) are zeroed
        out.update(units=tiles, rows_processed=rows_pad, padded_rows=rows_pad - routed,
                   waves=tiles / workers if workers else 0.0,
                   wave_efficiency=tiles / (math.ceil(tiles / workers) * workers) if tiles else 1.0,
                   useful_flops=2 * routed * N * K, issued_f16_equiv_flops=issued, compulsory_dram_bytes=dram)
    elif name == "fused_mlp_small_kernel":
        blocks = [-(-v // L["tile_m"]) for v in g]
        units = sum(blocks) * L["f_splits"]
        rows_pad = sum(blocks) * L["tile_m"]
        issued = 4 * rows_pad * D * F * _PRODUCTS[L["mma_kind"]]
        wplanes = 8 if dtype == "f32" else 2                  # tf32 hi + lo planes, or bf16 weights
        xb = IN_BYTES[dtype] * (2 if dtype == "f32" and D > 128 else 1)  # D = 256 f32 streams X hi + lo planes
        ybytes = M * D * 4 * (2 if L["f_splits"] > 1 else 1)  # F-split CTAs add into Y (read + write)
        dram = routed * D * xb + active * 2 * D * F * wplanes + ybytes
        # A last partial wave of at most grid / 2 units runs as half units
        # (two CTAs per unit, half of its hidden chunks each): the makespan
        # is the full waves plus half a unit.
        G = L["grid"]
        full = (units // G) * G if G else units
        tail = units - full
        nch = F // L["tile_n"] // max(L["f_splits"], 1) if L["tile_n"] else 0
        halves = 2 if tail > 0 and 2 * tail <= G and nch % 2 == 0 else 1
        makespan = full // G + (0.5 if halves == 2 else (1 if tail else 0)) if G else 0
        out.update(units=full + tail * halves, half_units=tail * halves if halves == 2 else 0,
                   rows_processed=rows_pad, padded_rows=rows_pad - routed,
                   waves=units / G if G else 0.0,
                   wave_efficiency=units / G / makespan if units and makespan else 1.0,
                   useful_flops=4 * routed * D * F, issued_f16_equiv_flops=issued, compulsory_dram_bytes=dram)
    elif name == "small_prep_kernel":
        wsplit = L["grid"] > 0 and dtype == "f32"
        # weight split of the experts with rows: read W, write hi + lo (12 B per element)
        out.update(units=L["grid"], useful_flops=0, issued_f16_equiv_flops=0,
                   compulsory_dram_bytes=(active * 2 * D * F * 12 if wsplit else 0))
    out["smem_fraction"] = L["smem_bytes"] / SMEM_LIMIT
    out["tmem_fraction"] = L["tmem_cols"] / TMEM_COLS
    return out


def b200_model(M: int, D: int, F: int, E: int, group_sizes: Sequence[int], dtype: str, sms: int = 148,
               peaks: Optional[dict] = None, measured_ms: Optional[float] = None) -> dict:
    """This library's kernels for one call (see the module doc): the launch
    plan with per-launch work units, padding, waves, issued tensor work and
    compulsory DRAM bytes, the modelled time per launch (the slower of its
    tensor time at the measured bf16 rate and its DRAM time at the measured
    copy bandwidth), and the roofline figure of the call."""
    from . import _lib

    if peaks is None:
        peaks, src = load_peaks()
    else:
        src = "given"
    g = clamp_group_sizes(M, group_sizes)
    plan = _lib.describe_plan(M, D, F, E, DTYPE_CODES[dtype], sms)
    bf16 = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])) * 1e12
    hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])) * 1e9
    launches = []
    for L in plan:
        m = _launch_model(L, M, D, F, E, g, dtype)
        m["t_tensor_ms"] = m["issued_f16_equiv_flops"] / bf16 * 1e3
        m["t_dram_ms"] = m["compulsory_dram_bytes"] / hbm * 1e3
        m["t_model_ms"] = max(m["t_tensor_ms"], m["t_dram_ms"])
        m["limiter"] = "tensor" if m["t_tensor_ms"] >= m["t_dram_ms"] else "dram"
        launches.append(m)
    t_model = sum(m["t_model_ms"] for m in launches)
    rf = roofline(M, D, F, g, dtype, measured_ms, peaks)
    out = {"M": M, "D": D, "F": F, "E": E, "dtype": dtype, "sms": sms, "peaks_source": src,
           "path": "grouped GEMMs (H through HBM)" if any(m["kernel"].startswith("grouped") for m in launches)
           else "fused small-D kernel (H on chip)",
           "launches": launches, "t_model_ms": t_model,
           "padded_row_fraction": (sum(m.get("padded_rows", 0) for m in launches if m.get("rows_processed"))
                                   / max(1, sum(m.get("rows_processed", 0) for m in launches))),
           "compulsory_dram_bytes": sum(m["compulsory_dram_bytes"] for m in launches),
           "roofline": rf, "model_frac_of_roof": rf["t_roof_ms"] / t_model if t_model else None}
    if measured_ms:
        out["measured_ms"] = measured_ms
        out["measured_over_model"] = measured_ms / t_model if t_model else None
    return out


def main() -> None:
    import argparse
    ap = argparse.ArgumentParser(description="B200 analytic model of one fused expert-MLP call")
    ap.add_argument("--config", default="c4", help="c1 .. c5")
    ap.add_argument("--measured-ms", type=float, default=None)
    ap.add_argument("--sms", type=int, default=148)
    a = ap.parse_args()
    from .routing import CONFIGS, config_group_sizes
    cfg = CONFIGS[a.config]
    print(json.dumps(b200_model(cfg.M, cfg.D, cfg.F, cfg.E, config_group_sizes(cfg, 0), cfg.dtype, a.sms,
                                measured_ms=a.measured_ms), indent=1))


if __name__ == "__main__":
    main()
