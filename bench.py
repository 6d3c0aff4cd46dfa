"""Benchmark of the B200 fused MoE expert MLP (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A step is one forward of the expert MLP over one batch of synthetic routed
tokens (seeded; shapes, inits and routing of the named configuration).
``value`` is routed tokens/s over the whole job with inputs resident in HBM,
device-timed with CUDA events, L2 flushed before every step; ``e2e`` is the
same metric through the public call with every step's inputs copied from
pinned host memory and its result read back into pinned host memory inside
the timed region (consecutive steps pipelined over three streams, as a
serving loop runs them).

At N > 1 (torchrun, one rank per GPU) the expert-parallel layer runs: every
rank owns E/N experts and its own batch of tokens; tokens travel to their
expert's rank and back through the library's NVLink exchange kernels
(``--transport peer``, default) or NCCL send/recv (``--transport nccl``);
weak scaling.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "pallas-moe-kernel_b200"
for _p in (str(PKG), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20  # twice the 126 MB L2


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every ~10 ms."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples: list[tuple[float, int, int]] = []
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = device_index
            if vis:
                parts = [v for v in vis.split(",") if v.strip()]
                if device_index < len(parts) and parts[device_index].strip().isdigit():
                    idx = int(parts[device_index])
            self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:
                pass
            time.sleep(0.01)

    def start(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self, t0: float, t1: float) -> dict:
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win and self.samples:  # very short timed region: nearest samples
            win = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        if not win:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        reasons = set()
        for _, _, rs in win:
            for bit, name in self.REASONS.items():
                if rs & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for _, m, _ in win), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(win)}


class DeviceClock:
    """SM clock measured on the device: one-thread blocks record (SM id,
    clock64, globaltimer) before and after a region on the launching stream;
    per SM, cycles / nanoseconds is the clock averaged over the region (the
    cycle counter is per SM, so only SMs seen in both samples count).  Unlike
    NVML's sampled clock it covers the whole region and nothing else."""

    def __init__(self, device):
        import torch
        from src import _lib
        self.L = _lib.lib()
        self.device = device
        self.blocks = min(1024, 2 * torch.cuda.get_device_properties(device).multi_processor_count)

    def sample(self, stream):
        import ctypes
        import torch
        buf = torch.zeros(3 * self.blocks, dtype=torch.int64, device=self.device)
        rc = self.L.moe_sm_clock_sample(ctypes.c_void_p(buf.data_ptr()), self.blocks,
                                        ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(self.L.moe_last_error().decode())
        return buf

    @staticmethod
    def mhz(a, b) -> dict:
        first = {}
        for sm, cyc, ns in a.cpu().view(-1, 3).tolist():
            first.setdefault(sm, (cyc, ns))
        rates = []
        seen = set()
        for sm, cyc, ns in b.cpu().view(-1, 3).tolist():
            if sm in first and sm not in seen and ns > first[sm][1]:
                seen.add(sm)
                rates.append((cyc - first[sm][0]) / (ns - first[sm][1]) * 1e3)
        if not rates:
            return {"sm_mhz": None, "sms": 0}
        return {"sm_mhz": statistics.median(rates), "sm_mhz_min": min(rates), "sm_mhz_max": max(rates),
                "sms": len(rates)}


def bind_to_gpu_numa_node(device_index: int) -> dict:
    """Restricts this process to the CPUs NVML reports as closest to the GPU
    (its NUMA node), so that the pinned host buffers allocated afterwards --
    first touched by this process -- live in that node's memory and the
    host<->device copies do not cross the CPU interconnect.  Returns what
    was done; leaves the affinity alone when NVML cannot tell."""
    try:
        import pynvml
        pynvml.nvmlInit()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = device_index
        if vis:
            parts = [v for v in vis.split(",") if v.strip()]
            if device_index < len(parts) and parts[device_index].strip().isdigit():
                idx = int(parts[device_index])
        h = pynvml.nvmlDeviceGetHandleByIndex(idx)
        ncpu = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        if not cpus:
            return {"numa_bound": False, "reason": "no CPU of the GPU's node available to this process"}
        os.sched_setaffinity(0, cpus)
        return {"numa_bound": True, "cpus": len(cpus)}
    except Exception as e:  # pragma: no cover - NVML missing or no affinity information
        return {"numa_bound": False, "reason": type(e).__name__}


# dense kind::f16 MMA rate per SM and clock cycle (M=128, N=256, K=16 in 128 cycles)
F16_FLOP_PER_CLK_SM = 8192


# --------------------------------------------------------------------- workload
def make_workload(cfg, device, seed: int = 0, experts=None):
    """Seeded synthetic inputs on the device: X ~ N(0,1) (M, D) and the routed
    group sizes of this batch (seed = rank), plus W_up ~ N(0, 1/D) (E', D, F)
    and W_down ~ N(0, 1/F) (E', F, D) for the experts in ``experts`` (all by
    default); each expert's weights come from its own seed, so the shards of
    an expert-parallel job form one consistent model."""
    import torch
    from src.routing import config_group_sizes

    from src.routing import quantize_e4m3_blockwise

    gs = config_group_sizes(cfg, seed=seed)
    tdt = torch.float32 if cfg.dtype == "f32" else torch.bfloat16
    wdt = torch.float8_e4m3fn if cfg.dtype == "fp8" else tdt
    g = torch.Generator(device=device)
    g.manual_seed(1234 + seed)
    x = torch.randn((cfg.M, cfg.D), generator=g, device=device, dtype=torch.float32).to(tdt)
    e0, e1 = experts if experts is not None else (0, cfg.E)
    w_up = torch.empty((e1 - e0, cfg.D, cfg.F), device=device, dtype=wdt)
    w_down = torch.empty((e1 - e0, cfg.F, cfg.D), device=device, dtype=wdt)
    scales = None
    if cfg.dtype == "fp8":   # e4m3 weights with 128x128 f32 block scales (amax / 448)
        db, fb = -(-cfg.D // 128), -(-cfg.F // 128)   # partial 128-blocks at the ends
        scales = (torch.empty((e1 - e0, db, fb), device=device), torch.empty((e1 - e0, fb, db), device=device))
    for i, e in enumerate(range(e0, e1)):
        g.manual_seed(99991 * (e + 1))
        wu = torch.randn((cfg.D, cfg.F), generator=g, device=device) / math.sqrt(cfg.D)
        wd = torch.randn((cfg.F, cfg.D), generator=g, device=device) / math.sqrt(cfg.F)
        if scales is None:
            w_up[i], w_down[i] = wu.to(tdt), wd.to(tdt)
        else:
            (w_up[i], scales[0][i]), (w_down[i], scales[1][i]) = quantize_e4m3_blockwise(wu), quantize_e4m3_blockwise(wd)
    return x, w_up, w_down, gs, scales


def algorithmic(cfg, gs) -> dict:
    """FLOPs = 4 M D F (GELU excluded); bytes = X + non-empty experts' weights
    (+ FP8 block scales) + Y -- the analytic model's figures."""
    from src import analysis
    w = analysis.algorithmic_work(cfg.M, cfg.D, cfg.F, gs, cfg.dtype)
    return {"flops": w["flops"], "bytes": w["bytes"]}


def tensor_peak(cfg, peaks) -> tuple[float, str]:
    from src import analysis
    p = analysis.tensor_peak(cfg.dtype, peaks)
    if cfg.dtype == "f32":
        return p, (f"bf16 {6 * p:.1f} TF/s / 6: kind::tf32 issues at half the f16 rate and "
                   f"3xTF32 spends 3 products per f32 product")
    return p, f"bf16 {p:.1f} TF/s"


def sustained_frac(achieved: float, peak: float, peaks: dict):
    """achieved / peak scaled to the power-capped (seconds-long) tensor peak."""
    burst, sust = peaks.get("bf16_tflops"), peaks.get("bf16_tflops_sustained")
    if not burst or not sust:
        return None
    return achieved / (peak * float(sust) / float(burst))


# --------------------------------------------------------------------- our arm
def run_ours(args, cfg, rank, world, device) -> dict | None:
    import torch
    import torch.distributed as dist
    from src import _lib
    from src.kernel import PreparedExperts, fused_ragged_dot_caller

    if world > 1 and cfg.E % world:
        raise SystemExit(f"E={cfg.E} experts do not shard over {world} ranks")
    el = cfg.E // world
    x, w_up, w_down, gs_np, scales = make_workload(cfg, device, seed=rank, experts=(rank * el, (rank + 1) * el))
    sc = {} if scales is None else {"w_up_scale": scales[0], "w_down_scale": scales[1]}
    gs_dev = torch.from_numpy(gs_np).to(device)
    if world > 1:
        from src.ep import ExpertParallelMLP, PeerExpertParallelMLP
        if args.transport == "peer":
            layer = PeerExpertParallelMLP(w_up, w_down, rank=rank, world=world, max_tokens=cfg.M,
                                          waves=args.waves, comm_ctas=args.reserve_sms, **sc)
            launches_per_step = layer.launches_per_forward
        else:
            layer = ExpertParallelMLP(w_up, w_down, rank=rank, world=world, max_tokens=cfg.M,
                                      waves=args.waves, reserve_sms=args.reserve_sms, **sc)
            launches_per_step = None
        step_fn = lambda: layer(x, gs_dev)  # noqa: E731
        kern_fn = None
    else:
        experts = PreparedExperts(w_up, w_down, max_tokens=cfg.M, **sc)
        y = torch.empty((cfg.M, cfg.D), device=device, dtype=torch.float32)
        ws = torch.empty(max(experts.ws_bytes, 1), device=device, dtype=torch.uint8)

        def step_fn():  # the reference entry point: raw weights in, Y out
            return fused_ragged_dot_caller(x, w_up, w_down, gs_dev, BM=16, BF=64, max_group_size=cfg.M,
                                           out=y, workspace=ws, **sc)

        def kern_fn():  # the dominant kernel alone (weights already prepared)
            return experts(x, gs_dev, out=y)
        code = {"f32": _lib.MOE_DTYPE_F32, "bf16": _lib.MOE_DTYPE_BF16, "fp8": _lib.MOE_DTYPE_FP8_E4M3_BLK128}[cfg.dtype]
        launches_per_step = _lib.lib().moe_fused_mlp_launch_count(cfg.M, cfg.D, cfg.F, cfg.E, code)

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        torch.cuda.synchronize(device)
        return [a.elapsed_time(b) for a, b in ev]

    for _ in range(args.warmup):
        step_fn()
        if kern_fn:
            kern_fn()
    torch.cuda.synchronize(device)
    _lib.device_status(reset=True)

    dclk = DeviceClock(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.05)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    c_a = dclk.sample(stream)   # outside the step events: not part of any step's time
    step_ms = timed(step_fn, args.steps)
    c_b = dclk.sample(stream)
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks.stop()
    total_ms = float(sum(step_ms))
    step_clock = DeviceClock.mhz(c_a, c_b)
    if launches_per_step is None:
        launches_per_step = layer.last_launches
    rl = None
    # When the step's launches are exactly the dominant kernels (the two
    # grouped GEMMs of bf16 and e4m3 experts: no preparation launch), the
    # kernel time is the step time of the timed region itself, at its clock.
    step_is_kernels = bool(kern_fn) and all(
        L["kernel"].startswith("grouped_gemm") for L in _lib.describe_plan(cfg.M, cfg.D, cfg.F, cfg.E, code))
    if step_is_kernels:
        rl = {"kern_ms": list(step_ms), "step_ms": list(step_ms), "clock": step_clock, "same_region": True}
    elif kern_fn:
        # Roofline leg: the dominant kernel(s) alone (weights prepared) and
        # the whole step, alternated launch by launch in one region so both
        # run at the same clock; the region's clock is measured on the device.
        k_ev, s_ev = [], []
        r_a = dclk.sample(stream)
        for _ in range(args.steps):
            for fn, evs in ((step_fn, s_ev), (kern_fn, k_ev)):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                evs.append((a, b))
        r_b = dclk.sample(stream)
        torch.cuda.synchronize(device)
        rl = {"kern_ms": [a.elapsed_time(b) for a, b in k_ev], "step_ms": [a.elapsed_time(b) for a, b in s_ev],
              "clock": DeviceClock.mhz(r_a, r_b), "same_region": False}
    status = _lib.device_status(reset=True)
    if status:
        raise RuntimeError(f"device status {status} after the timed region")

    # Expert parallelism: what sets the step.  Each rank's landing rows (its
    # experts' rows from every source, from the gathered group sizes) and a
    # compute-only leg -- this rank's experts on that many rows through the
    # single-GPU grouped GEMMs, no exchange -- timed the same way as the step.
    ep_rank = None
    if world > 1:
        gs_all = torch.empty((world, cfg.E), dtype=torch.int64, device=device)
        dist.all_gather_into_tensor(gs_all, gs_dev.to(torch.int64))
        lgs = gs_all[:, rank * el:(rank + 1) * el].clamp(min=0).sum(dim=0)
        land = int(lgs.sum())
        local = PreparedExperts(w_up, w_down, max_tokens=max(land, 1), **sc)
        gl = torch.Generator(device=device)
        gl.manual_seed(4321 + rank)
        x_land = torch.randn((max(land, 1), cfg.D), generator=gl, device=device, dtype=torch.float32).to(x.dtype)
        y_land = torch.empty((max(land, 1), cfg.D), device=device, dtype=torch.float32)
        lgs32 = lgs.to(torch.int32)
        for _ in range(2):
            local(x_land, lgs32, out=y_land)
        comp_ms = timed(lambda: local(x_land, lgs32, out=y_land), args.steps)
        del local, x_land, y_land
        mine = torch.tensor([statistics.mean(step_ms), statistics.mean(comp_ms), float(land),
                             float(step_clock.get("sm_mhz") or 0.0)], dtype=torch.float64, device=device)
        ep_rank = torch.empty((world, 4), dtype=torch.float64, device=device)
        dist.all_gather_into_tensor(ep_rank, mine)
        ep_rank = ep_rank.cpu().tolist()
        if _lib.device_status(reset=True):
            raise RuntimeError("device status set by the compute-only leg")

    # e2e: every step copies its inputs from pinned host memory, runs the
    # public call and reads Y back into pinned host memory.  Consecutive steps
    # are pipelined on three streams (copy in, compute, copy out) over two
    # device and two host buffer slots, as a serving loop runs them: H2D of
    # step i+1 and D2H of step i-1 overlap the compute of step i.
    # Pinned host buffers on the GPU's NUMA node (first touch after binding);
    # the original affinity comes back after the host-copy legs, so that the
    # CPU baseline keeps every host thread.
    affinity = os.sched_getaffinity(0)
    numa = (bind_to_gpu_numa_node(device.index) if args.numa_bind == "on"
            else {"numa_bound": False, "reason": "--numa-bind off"})
    xh = x.cpu().pin_memory()
    gsh = torch.from_numpy(gs_np).pin_memory()
    yh = [torch.empty((cfg.M, cfg.D), dtype=torch.float32).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(x) for _ in range(2)]
    gsd = [torch.empty_like(gs_dev) for _ in range(2)]
    yd = [torch.empty((cfg.M, cfg.D), dtype=torch.float32, device=device) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in, ev_cmp, ev_out = ([torch.cuda.Event() for _ in range(2)] for _ in range(3))

    def e2e_run(n):
        for i in range(n):
            b = i & 1
            s_in.wait_event(ev_cmp[b])              # step i-2 no longer reads slot b's inputs
            with torch.cuda.stream(s_in):
                xd[b].copy_(xh, non_blocking=True)
                gsd[b].copy_(gsh, non_blocking=True)
            ev_in[b].record(s_in)
            stream.wait_event(ev_in[b])
            stream.wait_event(ev_out[b])            # step i-2's Y has left slot b
            if world > 1:
                out = layer(xd[b], gsd[b], out=yd[b]) if hasattr(layer, "close") else layer(xd[b], gsd[b])
                if out is not yd[b]:
                    yd[b].copy_(out)
            else:
                fused_ragged_dot_caller(xd[b], w_up, w_down, gsd[b], BM=16, BF=64, max_group_size=cfg.M,
                                        out=yd[b], workspace=ws, **sc)
            ev_cmp[b].record(stream)
            s_out.wait_event(ev_cmp[b])
            with torch.cuda.stream(s_out):
                yh[b].copy_(yd[b], non_blocking=True)
            ev_out[b].record(s_out)
        stream.wait_event(ev_out[(n - 1) & 1])

    e2e_run(max(2, args.warmup))
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1)

    # The host link alone: the same copies (X in, Y out, two slots, the copy
    # streams of the e2e loop) with no compute, on every rank at once -- the
    # ceiling the e2e figure runs into when the copies outlast the compute.
    def copies_only(n):
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(s_in):
                xd[b].copy_(xh, non_blocking=True)
            with torch.cuda.stream(s_out):
                yh[b].copy_(yd[b], non_blocking=True)
    copies_only(2)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    s_in.wait_event(c0)
    s_out.wait_event(c0)
    copies_only(args.steps)
    stream.wait_stream(s_in)
    stream.wait_stream(s_out)
    c1.record(stream)
    torch.cuda.synchronize(device)
    copy_ms = c0.elapsed_time(c1)
    os.sched_setaffinity(0, affinity)

    vals = torch.tensor([total_ms, e2e_ms, copy_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        if hasattr(layer, "close"):
            layer.close()
    total_ms, e2e_ms, copy_ms = vals.tolist()
    if rank != 0:
        return None

    peaks, peak_src = load_peaks()
    alg = algorithmic(cfg, gs_np)
    ms_per_step = total_ms / args.steps
    value = world * cfg.M * args.steps / (total_ms / 1e3)
    line = {
        "metric": "routed_tokens_per_s",
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": {"f32": "f32 (3xTF32)", "bf16": "bf16", "fp8": "fp8e4m3 weights, bf16 x"}[cfg.dtype],
        "data": "synthetic (seeded; the configuration's shapes, N(0,1)/N(0,1/D)/N(0,1/F) init)",
        "config": {"workload": cfg.name, "M_per_gpu": cfg.M, "D": cfg.D, "F": cfg.F, "E": cfg.E,
                   "routing": cfg.routing, "parallelism": f"ep{world}" if world > 1 else "single",
                   **({"waves": getattr(layer, "waves", args.waves), "transport": args.transport}
                      if world > 1 else {}),
                   "l2": "flushed before every step (256 MiB write)"},
        "useful_tflops": alg["flops"] * world / (ms_per_step / 1e3) / 1e12,
        "gpu_launches": launches_per_step * args.steps,
        # per-step event times of the timed region (this rank's when N > 1), as the
        # reference's sweep reports them: median with p10 / p90
        "step_ms_percentiles": _percentiles(step_ms),
    }
    if rl is not None:
        k_avg = statistics.mean(rl["kern_ms"])
        s_avg = statistics.mean(rl["step_ms"])
        peak, basis = tensor_peak(cfg, peaks)
        achieved = alg["flops"] / (k_avg / 1e3) / 1e12
        t_mem = alg["bytes"] / (float(peaks["hbm_gbs"]) * 1e9)
        t_cmp = alg["flops"] / (peak * 1e12)
        kname = " + ".join(L["kernel"] for L in _lib.describe_plan(cfg.M, cfg.D, cfg.F, cfg.E, code)
                           if L["mma_kind"] != 0)
        mhz = rl["clock"].get("sm_mhz")
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        # The tensor peak at the clock the region ran at (kind::f16 rate; the
        # 3xTF32 path: a sixth of it).
        clk_peak = (F16_FLOP_PER_CLK_SM * sms * mhz * 1e6 / 1e12 / (6.0 if cfg.dtype == "f32" else 1.0)
                    if mhz else None)
        line["roofline"] = {
            "bound": "tensor" if t_cmp >= t_mem else "hbm",
            "kernel": kname,
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peak_src}: {basis}",
            "frac_of_sustained": sustained_frac(achieved, peak, peaks),
            "kernel_ms": k_avg, "algorithmic_flops": alg["flops"], "algorithmic_bytes": alg["bytes"],
            "hbm_frac": (alg["bytes"] / (k_avg / 1e3)) / (float(peaks["hbm_gbs"]) * 1e9),
            "traffic": None,
            "timing": ("the step is exactly the two grouped-GEMM launches: kernel time = step time of the "
                       "timed region" if rl["same_region"] else
                       "kernel leg and whole step alternated launch by launch in one region "
                       f"({args.steps} each, L2 flushed before each)"),
            "step_ms_same_region": s_avg,
            "kernel_le_step": bool(k_avg <= s_avg * 1.005),
            "sm_mhz_device": mhz,
            "tensor_peak_at_clock": clk_peak,
            "frac_at_clock": achieved / clk_peak if clk_peak else None,
        }
        if not line["roofline"]["kernel_le_step"]:
            print(f"warning: kernel leg {k_avg:.3f} ms > step {s_avg:.3f} ms in the same region", file=sys.stderr)
        prof = REPO / "profiles" / f"traffic_{cfg.name}.json"
        if prof.exists():
            try:
                line["roofline"]["traffic"] = json.loads(prof.read_text()).get("traffic_bytes_per_launch")
            except Exception:
                pass
    if ep_rank is not None:
        st_ms = [r[0] for r in ep_rank]
        cp_ms = [r[1] for r in ep_rank]
        rows = [int(r[2]) for r in ep_rank]
        slow = max(range(world), key=lambda r: st_ms[r])
        heavy = max(range(world), key=lambda r: cp_ms[r])
        line["ep"] = {
            "rank_step_ms": [round(v, 4) for v in st_ms],
            "rank_compute_only_ms": [round(v, 4) for v in cp_ms],
            "rank_landing_rows": rows,
            "rank_sm_mhz_device": [round(r[3]) for r in ep_rank],
            "rows_imbalance": max(rows) / (sum(rows) / world) if sum(rows) else None,
            "exchange_overhead_ms": max(st_ms) - max(cp_ms),
            "sets_the_step": (f"rank {heavy}'s expert GEMMs on its {rows[heavy]} landing rows take "
                              f"{cp_ms[heavy]:.3f} ms of the slowest rank's (rank {slow}) "
                              f"{st_ms[slow]:.3f} ms step; the rest ({max(st_ms) - max(cp_ms):.3f} ms) is the "
                              f"exchange beyond the overlap"),
            "compute_only": "this rank's experts on a landing-sized input through the single-GPU grouped GEMMs, "
                            "no exchange, timed like the step (L2 flushed)",
        }
    line["clocks"] = clocks.summary(t0, t1)
    line["clocks"]["sm_mhz_device"] = step_clock.get("sm_mhz")
    line["clocks"]["device_sms_sampled"] = step_clock.get("sms")
    h2d = cfg.M * cfg.D * x.element_size() + gs_np.nbytes
    line["e2e"] = {"value": world * cfg.M * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": cfg.M * cfg.D * 4,
                   "pipelining": "copy-in, compute and copy-out of consecutive steps on three streams, "
                                 "two buffer slots",
                   "host_copy_gbs_per_gpu": (h2d + cfg.M * cfg.D * 4) * args.steps / (e2e_ms / 1e3) / 1e9,
                   "host_copy_ceiling_gbs_per_gpu": (cfg.M * cfg.D * x.element_size() + cfg.M * cfg.D * 4)
                   * args.steps / (copy_ms / 1e3) / 1e9,
                   "host_copy_ceiling": "the same H2D + D2H copies with no compute, every rank at once, "
                                        "max over ranks",
                   "host_buffers": numa}
    return line



# --------------------------------------------------------------------- whole MoE layer (routing stage)
def _percentiles(ms: list) -> dict:
    """p10 / median / p90 (nearest rank), min and max of per-step times."""
    v = sorted(ms)
    if not v:
        return {}
    q = lambda f: v[min(len(v) - 1, max(0, math.ceil(f * len(v)) - 1))]  # noqa: E731
    return {"p10": q(0.1), "p50": statistics.median(v), "p90": q(0.9), "min": v[0], "max": v[-1], "n": len(v)}


def quick_config(cfg, steps: int, warmup: int, device) -> dict:
    """Device-resident figures of one more configuration on this GPU: the
    reference entry point (raw weights in, Y out) and the fused kernel(s)
    alone (weights prepared), alternated launch by launch with L2 flushed
    before each, with the device clock of that region.  No e2e leg and no
    CPU baseline: these ride along the headline line as evidence."""
    import torch
    from src import _lib, analysis
    from src.kernel import PreparedExperts, fused_ragged_dot_caller

    x, w_up, w_down, gs_np, scales = make_workload(cfg, device)
    sc = {} if scales is None else {"w_up_scale": scales[0], "w_down_scale": scales[1]}
    gs_dev = torch.from_numpy(gs_np).to(device)
    experts = PreparedExperts(w_up, w_down, max_tokens=cfg.M, **sc)
    y = torch.empty((cfg.M, cfg.D), device=device, dtype=torch.float32)
    ws = torch.empty(max(experts.ws_bytes, 1), device=device, dtype=torch.uint8)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step_fn():
        return fused_ragged_dot_caller(x, w_up, w_down, gs_dev, BM=16, BF=64, max_group_size=cfg.M,
                                       out=y, workspace=ws, **sc)

    def kern_fn():
        return experts(x, gs_dev, out=y)

    for _ in range(warmup):
        step_fn()
        kern_fn()
    torch.cuda.synchronize(device)
    _lib.device_status(reset=True)
    dclk = DeviceClock(device)
    s_ev, k_ev = [], []
    c_a = dclk.sample(stream)
    for _ in range(steps):
        for fn, evs in ((step_fn, s_ev), (kern_fn, k_ev)):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            evs.append((a, b))
    c_b = dclk.sample(stream)
    torch.cuda.synchronize(device)
    if _lib.device_status(reset=True):
        raise RuntimeError(f"device status set while timing {cfg.name}")
    s_all = [a.elapsed_time(b) for a, b in s_ev]
    k_all = [a.elapsed_time(b) for a, b in k_ev]
    # bf16 and e4m3 experts: both legs launch exactly the two grouped GEMMs
    # (no preparation launch), so their samples are pooled for both figures.
    code = {"f32": _lib.MOE_DTYPE_F32, "bf16": _lib.MOE_DTYPE_BF16, "fp8": _lib.MOE_DTYPE_FP8_E4M3_BLK128}[cfg.dtype]
    step_is_kernels = all(L["kernel"].startswith("grouped_gemm")
                          for L in _lib.describe_plan(cfg.M, cfg.D, cfg.F, cfg.E, code))
    if step_is_kernels:
        s_all = k_all = s_all + k_all
    s_ms = statistics.mean(s_all)
    k_ms = statistics.mean(k_all)
    mhz = DeviceClock.mhz(c_a, c_b).get("sm_mhz")
    peaks, _ = load_peaks()
    r = analysis.roofline(cfg.M, cfg.D, cfg.F, gs_np.tolist(), cfg.dtype, kernel_ms=k_ms, peaks=peaks)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    clk_peak = (F16_FLOP_PER_CLK_SM * sms * mhz * 1e6 / 1e12 / (6.0 if cfg.dtype == "f32" else 1.0)
                if mhz else None)
    out = {"workload": cfg.name, "value": cfg.M / (s_ms / 1e3), "unit": "tokens/s", "ms_per_step": s_ms,
           "kernel_ms": k_ms, "bound": r["bound"], "achieved": r["achieved"], "roofline_unit": r["unit"],
           "frac": r["frac"], "sm_mhz_device": mhz,
           "frac_at_clock": (r["achieved"] / clk_peak if clk_peak and r["bound"] == "tensor" else None),
           "steps": steps, "warmup": warmup,
           "step_ms_percentiles": _percentiles(s_all), "same_launches": step_is_kernels}
    del x, w_up, w_down, experts, y, ws, flush
    torch.cuda.empty_cache()
    return out


def run_layer(args, cfg, device) -> dict:
    """Routing stage around the expert MLP on one GPU: top-k routing of
    ``tokens`` router inputs over E experts, stable permutation by expert, row
    gather, and the weighted combine (HBM-bound kernels, timed alone), plus
    the whole layer (routing + the fused expert MLP)."""
    import torch
    from src import router
    from src.kernel import PreparedExperts

    k = {"top2": 2, "top8_softmax": 8}.get(cfg.routing)
    if not k:
        raise SystemExit("--stage layer needs a top-k configuration (c4 or c5)")
    T = cfg.M // k
    g = torch.Generator(device=device)
    g.manual_seed(7)
    tdt = torch.float32 if cfg.dtype == "f32" else torch.bfloat16
    x = torch.randn((T, cfg.D), generator=g, device=device).to(tdt)
    logits = torch.randn((T, cfg.E), generator=g, device=device)
    ys = torch.randn((T * k, cfg.D), generator=g, device=device)
    _, w_up, w_down, _, scales = make_workload(cfg, device)
    sc = {} if scales is None else {"w_up_scale": scales[0], "w_down_scale": scales[1]}
    experts = PreparedExperts(w_up, w_down, max_tokens=T * k, **sc)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    st = torch.cuda.current_stream(device)

    def routing():
        ids, w = router.route_topk(logits, k)
        gs, src, inv = router.permute(ids, cfg.E, workspace=ws)
        xs = router.gather_rows(x, src, k)
        return router.combine_rows(ys, inv, w), xs, gs

    def layer():
        ids, w = router.route_topk(logits, k)
        gs, src, inv = router.permute(ids, cfg.E, workspace=ws)
        xs = router.gather_rows(x, src, k)
        return router.combine_rows(experts(xs, gs), inv, w)

    def timed(fn, n):
        out = []
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            fn()
            b.record(st)
            torch.cuda.synchronize(device)
            out.append(a.elapsed_time(b))
        return statistics.median(out)

    for _ in range(args.warmup):
        routing()
        layer()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.05)
    t0 = time.perf_counter()
    r_ms = timed(routing, args.steps)
    l_ms = timed(layer, args.steps)
    t1 = time.perf_counter()
    clocks.stop()
    if _lib_status():
        raise RuntimeError("device status set after the layer stage")
    peaks, peak_src = load_peaks()
    N = T * k
    sx = x.element_size()
    # logits in, ids + weights out; ids read by 2 permutation passes, src + inverse out;
    # X read once and written in expert order; expert outputs read and per-token Y written.
    alg = (T * cfg.E * 4 + 2 * N * 4) + (2 * N * 4 + 2 * N * 4) + (T * cfg.D * sx + N * cfg.D * sx) \
        + (N * cfg.D * 4 + T * cfg.D * 4)
    hbm = float(peaks["hbm_gbs"])
    achieved = alg / (r_ms / 1e3) / 1e9
    # CPU baseline: the oracle's numpy routing + permutation + gather + combine on a sample.
    from oracle import moe_oracle as orc
    ns = min(T, 512)
    lg, xh, ysh = logits[:ns].cpu().numpy(), x[:ns].float().cpu().numpy(), ys[:ns * k].cpu().numpy()
    c0 = time.perf_counter()
    reps = 0
    while True:
        ids_h, w_h = orc.route_topk(lg, k)
        gs_h, src_h, inv_h = orc.permute_by_expert(ids_h, cfg.E)
        orc.gather_rows(xh, src_h, k)
        orc.combine_rows(ysh, inv_h, w_h, k)
        reps += 1
        if time.perf_counter() - c0 > 5.0:
            break
    cpu_tps = reps * ns / (time.perf_counter() - c0)
    return {
        "metric": "moe_layer_tokens_per_s", "value": T / (l_ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": l_ms, "higher_is_better": True,
        "dtype": str(tdt).replace("torch.", ""), "data": "synthetic (seeded N(0,1) tokens and router logits)",
        "config": {"workload": f"{cfg.name}_layer", "tokens": T, "k": k, "E": cfg.E, "D": cfg.D, "F": cfg.F,
                   "l2": "flushed before every step (256 MiB write)"},
        "routing": {"ms": r_ms, "tokens_per_s": T / (r_ms / 1e3), "kernels": 6,
                    "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                                 "frac": achieved / hbm, "algorithmic_bytes": alg,
                                 "peak_source": f"{peak_src}: hbm_gbs"}},
        "expert_mlp_ms": l_ms - r_ms,
        "clocks": clocks.summary(t0, t1),
        "cpu_baseline": {"value": cpu_tps, "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": f"oracle routing + permutation + gather + combine of {ns} tokens, repeated 5 s"},
    }


def run_train(args, cfg, device) -> dict:
    """Training step of the expert MLP (bf16) on one GPU: forward with the
    pre-activation saved, then the backward (dX, dW_up, dW_down) for a given
    dY; inputs resident in HBM, L2 flushed before every step.  FLOPs = 12 M D F
    (forward 4, backward 8); launches per step: 2 forward + 5 backward."""
    import torch
    from src import _lib
    from src.train import backward, forward_train, swiglu_backward, swiglu_forward_train

    if cfg.dtype != "bf16":
        cfg = with_shape_dtype(cfg, "bf16")
    x, w_up, w_down, gs, _ = make_workload(cfg, device)
    gs_dev = torch.from_numpy(gs).to(device)
    swiglu = args.act == "swiglu"
    if swiglu:  # gate and up weights, interleaved for the up GEMM
        from src.kernel import swiglu_interleave
        g0 = torch.Generator(device=device)
        g0.manual_seed(777)
        w_gate = (torch.randn(w_up.shape, generator=g0, device=device) / math.sqrt(cfg.D)).to(torch.bfloat16)
        w_up = swiglu_interleave(w_gate, w_up)
        del w_gate
    g = torch.Generator(device=device)
    g.manual_seed(4321)
    dy = torch.randn((cfg.M, cfg.D), generator=g, device=device)
    y = torch.empty((cfg.M, cfg.D), device=device)
    a = torch.empty((cfg.M, 2 * cfg.F if swiglu else cfg.F), device=device, dtype=torch.bfloat16)
    L = _lib.lib()
    if swiglu:
        f_bytes = L.moe_fused_mlp_swiglu_forward_train_workspace_size(cfg.M, cfg.D, cfg.F, cfg.E)
        b_bytes = L.moe_fused_mlp_swiglu_backward_workspace_size(cfg.M, cfg.D, cfg.F, cfg.E)
        fwd_fn = lambda ws: swiglu_forward_train(x, w_up, w_down, gs_dev, out=y, gu_save=a, workspace=ws)  # noqa: E731
        bwd_fn = lambda ws: swiglu_backward(x, w_up, w_down, gs_dev, a, dy, workspace=ws)  # noqa: E731
    else:
        f_bytes = L.moe_fused_mlp_forward_train_workspace_size(cfg.M, cfg.D, cfg.F, cfg.E)
        b_bytes = L.moe_fused_mlp_backward_workspace_size(cfg.M, cfg.D, cfg.F, cfg.E)
        fwd_fn = lambda ws: forward_train(x, w_up, w_down, gs_dev, out=y, a_save=a, workspace=ws)  # noqa: E731
        bwd_fn = lambda ws: backward(x, w_up, w_down, gs_dev, a, dy, workspace=ws)  # noqa: E731
    ws_f = torch.empty(int(f_bytes), dtype=torch.uint8, device=device)
    ws_b = torch.empty(int(b_bytes), dtype=torch.uint8, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    st = torch.cuda.current_stream(device)

    def step():
        fwd_fn(ws_f)
        return bwd_fn(ws_b)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.05)
    t0 = time.perf_counter()
    fwd, tot = [], []
    for _ in range(args.steps):
        flush.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(st)
        fwd_fn(ws_f)
        ev[1].record(st)
        bwd_fn(ws_b)
        ev[2].record(st)
        torch.cuda.synchronize(device)
        fwd.append(ev[0].elapsed_time(ev[1]))
        tot.append(ev[0].elapsed_time(ev[2]))
    t1 = time.perf_counter()
    clocks.stop()
    if _lib_status():
        raise RuntimeError("device status set after the training stage")
    ms = sum(tot) / len(tot)
    f_ms = sum(fwd) / len(fwd)
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    mdf = cfg.M * cfg.D * cfg.F
    f_fl, b_fl = (6, 12) if swiglu else (4, 8)  # forward / backward FLOPs in units of M D F
    achieved = (f_fl + b_fl) * mdf / (ms / 1e3) / 1e12
    return {
        "metric": "routed_tokens_per_s", "value": cfg.M / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) X and dY, N(0,1/D) / N(0,1/F) weights)",
        "config": {"workload": f"{cfg.name}_train" + ("_swiglu" if swiglu else ""), "M": cfg.M, "D": cfg.D,
                   "F": cfg.F, "E": cfg.E, "activation": args.act,
                   "step": "forward (pre-activation saved) + backward (dX and the weight gradients, f32)",
                   "l2": "flushed before every step (256 MiB write)"},
        "gpu_launches": 7 * args.steps,
        "forward_ms": f_ms, "backward_ms": ms - f_ms,
        "backward_tflops": b_fl * mdf / ((ms - f_ms) / 1e3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "algorithmic_flops": (f_fl + b_fl) * mdf,
                     "peak_source": f"{peak_src}: bf16_tflops",
                     "kernels": "forward 2 grouped GEMMs + backward pad + 4 grouped GEMMs, timed together"},
        "clocks": clocks.summary(t0, t1),
    }


def with_shape_dtype(cfg, dtype):
    from src.routing import with_shape
    return with_shape(cfg, dtype=dtype, name=f"{cfg.name}_as_{dtype}")


def run_swiglu(args, cfg, device) -> dict:
    """SwiGLU experts (bf16) on the configuration's shape and routing on one
    GPU: the up GEMM over the interleaved gate/up weights with the SiLU-gate
    epilogue, then the down GEMM; inputs resident in HBM, L2 flushed before
    every step.  FLOPs = 6 M D F; algorithmic bytes = X + the non-empty
    experts' three weight matrices + Y (H is an intermediate)."""
    import torch
    from src import _lib
    from src.kernel import fused_ragged_swiglu, swiglu_interleave, swiglu_interleave_fp8
    from src.routing import config_group_sizes, quantize_e4m3_blockwise

    gs = config_group_sizes(cfg, seed=0)
    g = torch.Generator(device=device)
    g.manual_seed(1234)
    x = torch.randn((cfg.M, cfg.D), generator=g, device=device).to(torch.bfloat16)
    fp8 = cfg.dtype == "fp8"
    sc = {}
    if fp8:  # e4m3 weights with 128 x 128 block scales, built one expert at a time
        E, D, F = cfg.E, cfg.D, cfg.F
        q = [torch.empty(shape, device=device, dtype=torch.float8_e4m3fn) for shape in ((E, D, F), (E, D, F), (E, F, D))]
        s = [torch.empty(shape, device=device) for shape in ((E, D // 128, F // 128), (E, D // 128, F // 128),
                                                            (E, F // 128, D // 128))]
        for e in range(E):
            for i, (r, c, fan) in enumerate(((D, F, D), (D, F, D), (F, D, F))):
                q[i][e], s[i][e] = quantize_e4m3_blockwise(torch.randn((r, c), generator=g, device=device)
                                                           / math.sqrt(fan))
        w_gu, s_gu = swiglu_interleave_fp8(q[0], q[1], s[0], s[1])
        w_down = q[2]
        sc = {"w_gate_up_scale": s_gu, "w_down_scale": s[2]}
        del q[0:2], s[0:2]
        ws_bytes = _lib.lib().moe_fused_mlp_swiglu_fp8_workspace_size(cfg.M, cfg.D, cfg.F)
    else:
        w_gate = (torch.randn((cfg.E, cfg.D, cfg.F), generator=g, device=device) / math.sqrt(cfg.D)).to(torch.bfloat16)
        w_up = (torch.randn((cfg.E, cfg.D, cfg.F), generator=g, device=device) / math.sqrt(cfg.D)).to(torch.bfloat16)
        w_down = (torch.randn((cfg.E, cfg.F, cfg.D), generator=g, device=device) / math.sqrt(cfg.F)).to(torch.bfloat16)
        w_gu = swiglu_interleave(w_gate, w_up)
        del w_gate, w_up
        ws_bytes = _lib.lib().moe_fused_mlp_swiglu_workspace_size(cfg.M, cfg.D, cfg.F)
    gs_dev = torch.from_numpy(gs).to(device)
    y = torch.empty((cfg.M, cfg.D), device=device)
    ws = torch.empty(int(ws_bytes), dtype=torch.uint8, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    st = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        fused_ragged_swiglu(x, w_gu, w_down, gs_dev, out=y, workspace=ws, **sc)
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.05)
    t0 = time.perf_counter()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fused_ragged_swiglu(x, w_gu, w_down, gs_dev, out=y, workspace=ws, **sc)
        b.record(st)
        torch.cuda.synchronize(device)
        times.append(a.elapsed_time(b))
    t1 = time.perf_counter()
    clocks.stop()
    if _lib_status():
        raise RuntimeError("device status set after the SwiGLU stage")
    ms = sum(times) / len(times)
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    flops = 6 * cfg.M * cfg.D * cfg.F
    active = int(np.count_nonzero(gs > 0))
    wbytes = 1 if fp8 else 2
    byts = cfg.M * cfg.D * 2 + active * 3 * cfg.D * cfg.F * wbytes + cfg.M * cfg.D * 4
    achieved = flops / (ms / 1e3) / 1e12
    return {
        "metric": "routed_tokens_per_s", "value": cfg.M / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "fp8 e4m3 weights, f16 operands" if fp8 else "bf16",
        "data": "synthetic (seeded N(0,1) X, N(0,1/D) / N(0,1/F) weights)",
        "config": {"workload": f"{cfg.name}_swiglu", "M": cfg.M, "D": cfg.D, "F": cfg.F, "E": cfg.E,
                   "activation": "swiglu", "l2": "flushed before every step (256 MiB write)"},
        "gpu_launches": (3 if fp8 else 2) * args.steps,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": None, "algorithmic_flops": flops,
                     "algorithmic_bytes": byts, "peak_source": f"{peak_src}: bf16_tflops",
                     "kernels": "up GEMM (SiLU-gate epilogue) + down GEMM, timed together"},
        "clocks": clocks.summary(t0, t1),
    }


def _lib_status() -> int:
    from src import _lib
    return _lib.device_status(reset=True)

# --------------------------------------------------------------------- CPU baseline
def cpu_reference(cfg, budget_s: float, seed: int = 0) -> dict:
    """The reference's unfused path (two ragged dots with tanh-GELU, f32) on
    host cores, timed on a bounded sample of the workload's rows."""
    from oracle import moe_oracle as orc
    from src.routing import config_group_sizes

    gs = config_group_sizes(cfg, seed=seed)
    # Bounded sample: the first routed rows in expert order, always whole
    # experts and at least one (so BLAS runs at the expert's real M), up to
    # about 30 GFLOP per timed call when one expert is smaller than that.
    rng = np.random.default_rng(seed)
    per_row_flops = 4 * cfg.D * cfg.F
    offs = np.concatenate([[0], np.cumsum(gs)])
    target = min(cfg.M, 3e10 / per_row_flops)
    rows = 0
    for e in range(cfg.E):
        rows = int(offs[e + 1])
        if rows >= target and rows > 0:
            break
    rows = max(1, min(rows, cfg.M))
    gs_s = np.clip(np.minimum(offs[1:], rows) - np.minimum(offs[:-1], rows), 0, None).astype(np.int32)
    active = np.nonzero(gs_s)[0]
    x = rng.standard_normal((rows, cfg.D), dtype=np.float32)
    # Only the experts the sample touches are materialised.
    w_up = [None] * cfg.E
    w_down = [None] * cfg.E
    for e in active:
        w_up[e] = rng.standard_normal((cfg.D, cfg.F), dtype=np.float32) / np.float32(math.sqrt(cfg.D))
        w_down[e] = rng.standard_normal((cfg.F, cfg.D), dtype=np.float32) / np.float32(math.sqrt(cfg.F))
    cores = len(os.sched_getaffinity(0))
    try:  # torchrun sets OMP_NUM_THREADS=1; the baseline uses every host thread
        from threadpoolctl import threadpool_limits
        limiter = threadpool_limits(limits=cores)
    except Exception:  # pragma: no cover
        limiter = None
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t = time.perf_counter()
        orc.time_cpu_reference(x, w_up, w_down, gs_s)
        times.append(time.perf_counter() - t)
        if time.perf_counter() > t_end or len(times) >= 50:
            break
    med = statistics.median(times)
    if limiter is not None:
        limiter.restore_original_limits()
    return {"value": rows / med, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of {cfg.M} routed rows ({len(active)} whole experts), f32 numpy/BLAS, "
                      f"median of {len(times)} calls; tokens/s = rows / seconds per call",
            "seconds_per_call": med}


def run_reference(args, cfg, rank, world) -> dict | None:
    if rank != 0:
        return None
    base = cpu_reference(cfg, budget_s=args.ref_budget)
    steps_t = base["seconds_per_call"]
    return {
        "impl": "reference", "metric": "routed_tokens_per_s", "value": base["value"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": steps_t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)", "config": {"workload": cfg.name, "M_per_gpu": cfg.M, "D": cfg.D,
                                                  "F": cfg.F, "E": cfg.E},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------- main
def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c4",
                    help="c1..c5 (default c4: bf16 Mixtral-shaped M=32768 D=4096 F=14336 E=8, top-2)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--act", default="gelu", choices=["gelu", "swiglu"],
                    help="expert activation: gelu (the reference's GELU-tanh MLP) or swiglu "
                         "(SiLU-gated experts, bf16, one GPU)")
    ap.add_argument("--stage", default="mlp", choices=["mlp", "layer", "train"],
                    help="mlp: the expert MLP (the reference's path); layer: routing + permutation + expert MLP "
                         "+ combine of a whole MoE layer on one GPU (top-k configurations); train: forward with "
                         "the pre-activation saved + backward of the expert MLP (bf16, one GPU)")
    ap.add_argument("--ref-budget", type=float, default=10.0, help="seconds of CPU baseline timing")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=0, help="override M (routed rows per GPU)")
    ap.add_argument("--dtype", default="", choices=["", "f32", "bf16", "fp8"],
                    help="override the configuration's precision path (same shapes and routing)")
    ap.add_argument("--experts", type=int, default=0,
                    help="override E (with --tokens: a smaller case with the same rows per expert)")
    ap.add_argument("--dmodel", type=int, default=0, help="override D (the model dimension)")
    ap.add_argument("--dff", type=int, default=0, help="override F (the expert hidden dimension)")
    ap.add_argument("--waves", type=int, default=2,
                    help="N>1: token waves per step (dispatch/combine of one wave overlap the experts of the next)")
    ap.add_argument("--reserve-sms", type=int, default=0,
                    help="N>1: SMs left free of the persistent expert kernels for the exchange kernels "
                         "(0: the engine's default of 16 with --transport peer, none with nccl)")
    ap.add_argument("--transport", default="peer", choices=["peer", "nccl"],
                    help="N>1: token exchange by the library's kernels over NVLink peer memory (peer) "
                         "or by NCCL send/recv from Python (nccl)")
    ap.add_argument("--numa-bind", default="on", choices=["on", "off"],
                    help="bind the process to the GPU's NUMA node before pinning the e2e host buffers")
    ap.add_argument("--no-other-configs", dest="other_configs", action="store_false",
                    help="N=1: skip the device-resident figures of the other configurations (c1..c5) that "
                         "otherwise ride along the line under other_configs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    from src.routing import CONFIGS, with_shape
    cfg = CONFIGS[args.config]
    if args.tokens:
        # Top-k configs route `tokens` router inputs to M = k * tokens rows.
        k = {"top2": 2, "top8_softmax": 8}.get(cfg.routing, 0)
        if k and args.tokens % k:
            raise SystemExit(f"--tokens must be a multiple of {k} for {cfg.routing} routing")
        cfg = with_shape(cfg, M=args.tokens, tokens=args.tokens // k if k else 0, name=f"{cfg.name}_M{args.tokens}")
    if args.experts:
        cfg = with_shape(cfg, E=args.experts, name=f"{cfg.name}_E{args.experts}")
    if args.dmodel or args.dff:
        D, F = args.dmodel or cfg.D, args.dff or cfg.F
        cfg = with_shape(cfg, D=D, F=F, name=f"{cfg.name}_D{D}_F{F}")
    if args.dtype and args.dtype != cfg.dtype:
        cfg = with_shape(cfg, dtype=args.dtype, name=f"{cfg.name}_as_{args.dtype}")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, cfg, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    import torch
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    if args.act == "swiglu" and args.stage != "train":
        if world > 1:
            raise SystemExit("--act swiglu runs on one GPU")
        print(json.dumps(run_swiglu(args, cfg, device)), flush=True)
        return 0
    if args.stage == "layer":
        print(json.dumps(run_layer(args, cfg, device)), flush=True)
        return 0
    if args.stage == "train":
        if world > 1:
            raise SystemExit("--stage train runs on one GPU")
        print(json.dumps(run_train(args, cfg, device)), flush=True)
        return 0
    try:
        line = run_ours(args, cfg, rank, world, device)
        if line is not None:
            if not args.no_cpu_baseline and world == 1:
                base = cpu_reference(cfg, budget_s=args.ref_budget)
                line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
            if world == 1 and args.other_configs and not (args.tokens or args.experts or args.dmodel
                                                          or args.dff or args.dtype):
                others = {}
                for name in ("c1", "c2", "c3", "c5"):
                    if name == args.config:
                        continue
                    try:
                        others[name] = quick_config(CONFIGS[name], steps=min(args.steps, 20), warmup=3,
                                                    device=device)
                    except Exception as exc:  # reported, never hides the headline line
                        others[name] = {"error": f"{type(exc).__name__}: {exc}"}
                line["other_configs"] = others
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
