"""Device expert-parallel engine (``moe_ep_*``, src.ep.PeerExpertParallelMLP).

world = 1 runs on one GPU: the count exchange, wave slicing, landing
regions, the experts over each region and the pull back into Y all run, with
every wait for a peer trivially satisfied (a rank never waits on itself).
The per-row arithmetic of the expert kernels does not depend on which rows
share a tile, so for the bf16 grouped-GEMM path the engine's Y must equal
moe_fused_mlp's Y bit for bit; the f32 path is checked against the oracle.

world = 2 (skipped with fewer GPUs) checks the NVLink exchange proper:
every rank's Y against the single-process oracle over all experts, for
several steps with different routings."""

import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import moe_oracle as orc
from src import _lib
from src.ep import PeerExpertParallelMLP
from src.kernel import fused_ragged_mlp
from src.routing import make_inputs_numpy, multinomial_group_sizes, zipf_group_sizes

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent
DEV = torch.device("cuda", 0)


def _weights(E, D, F, dt, seed=0):
    _, wu, wd = make_inputs_numpy(8, D, F, E, seed=seed)
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dt]
    return torch.from_numpy(wu).to(DEV, tdt), torch.from_numpy(wd).to(DEV, tdt)


def _routing(kind, M, E, rng):
    if kind == "uniform":
        return multinomial_group_sizes(M - 5, E, rng)                 # 5 unrouted rows
    if kind == "zipf":
        return zipf_group_sizes(M, E, rng, min_empty=min(3, E - 1))
    if kind == "one":
        gs = np.zeros(E, np.int32)
        gs[E // 2] = M
        return gs
    raise ValueError(kind)


@pytest.mark.parametrize("dt,D,F,E,waves", [("f32", 128, 512, 4, 1), ("f32", 128, 512, 4, 3),
                                             ("bf16", 512, 1024, 4, 2), ("bf16", 512, 1024, 6, 4)])
def test_engine_world1_matches_single_gpu(dt, D, F, E, waves):
    wu, wd = _weights(E, D, F, dt)
    M_max = 3000
    layer = PeerExpertParallelMLP(wu, wd, rank=0, world=1, max_tokens=M_max, waves=waves)
    tol = 1e-5 if dt == "f32" else 1e-2
    rng = np.random.default_rng(5)
    try:
        for step, (kind, M) in enumerate([("uniform", 3000), ("zipf", 2048), ("one", 777), ("uniform", 8)]):
            gs = _routing(kind, M, E, rng)
            x = torch.randn((M, D), device=DEV).to(wu.dtype)
            y = layer(x, torch.from_numpy(gs))
            ref = fused_ragged_mlp(x, wu, wd, torch.from_numpy(gs).to(DEV))
            torch.cuda.synchronize()
            if dt == "bf16":
                assert torch.equal(y, ref), (step, kind)
            exact = orc.ref_ragged_mlp(x.double().cpu().numpy(), wu.double().cpu().numpy(),
                                       wd.double().cpu().numpy(), gs)
            m = orc.correctness_metrics(exact, y.cpu().numpy())
            assert m["l2_relative_error"] <= tol, (step, kind, m)
            routed = int(gs.sum())
            assert torch.all(y[routed:] == 0)
            if dt == "bf16":
                # Two-GEMM engines return a view of their own output buffer;
                # with `out` the same rows are copied into the caller's array.
                y2 = torch.full((M, D), float("nan"), device=DEV)
                assert layer(x, torch.from_numpy(gs), out=y2) is y2
                torch.cuda.synchronize()
                assert torch.equal(y2, ref), (step, kind)
        assert _lib.device_status(reset=True) == 0
    finally:
        layer.close()


def test_engine_world1_fp8_matches_single_gpu():
    """e4m3 block-scaled weights through the engine (combine fused into the
    down GEMM): bit-identical to moe_fused_mlp on the same rows."""
    from src.routing import quantize_e4m3_blockwise
    D, F, E = 512, 1024, 4
    wu, wd = _weights(E, D, F, "f32")
    (wq_u, su), (wq_d, sd) = quantize_e4m3_blockwise(wu), quantize_e4m3_blockwise(wd)
    layer = PeerExpertParallelMLP(wq_u, wq_d, rank=0, world=1, max_tokens=2048, w_up_scale=su, w_down_scale=sd)
    rng = np.random.default_rng(9)
    try:
        for kind, M in [("uniform", 2048), ("zipf", 1000)]:
            gs = _routing(kind, M, E, rng)
            x = torch.randn((M, D), device=DEV).to(torch.bfloat16)
            y = layer(x, torch.from_numpy(gs)).clone()
            ref = fused_ragged_mlp(x, wq_u, wq_d, torch.from_numpy(gs).to(DEV), w_up_scale=su, w_down_scale=sd)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), kind
        assert _lib.device_status(reset=True) == 0
    finally:
        layer.close()


def test_engine_world1_clamps_bad_group_sizes_and_empty_batch():
    D, F, E = 128, 512, 4
    wu, wd = _weights(E, D, F, "f32")
    layer = PeerExpertParallelMLP(wu, wd, rank=0, world=1, max_tokens=1024, waves=2)
    try:
        M = 1000
        x = torch.randn((M, D), device=DEV)
        # Negative entry counts as zero; the running total past M is cut.
        gs = np.array([300, -7, 500, 400], np.int32)
        y = layer(x, torch.from_numpy(gs))
        torch.cuda.synchronize()
        clamped = np.array([300, 0, 500, 200], np.int32)
        exact = orc.ref_ragged_mlp(x.double().cpu().numpy(), wu.double().cpu().numpy(), wd.double().cpu().numpy(),
                                   clamped)
        assert orc.correctness_metrics(exact, y.cpu().numpy())["l2_relative_error"] <= 1e-5
        assert _lib.device_status(reset=True) == 2 | 8
        # An empty batch still takes part in the step.
        y0 = layer(torch.empty((0, D), device=DEV), torch.zeros(E, dtype=torch.int32))
        torch.cuda.synchronize()
        assert y0.shape == (0, D)
        assert _lib.device_status(reset=True) == 0
        with pytest.raises(ValueError):
            layer(torch.randn((10, D + 1), device=DEV), torch.zeros(E, dtype=torch.int32))
        with pytest.raises(_lib.MoeError):                      # above max_tokens
            layer(torch.randn((2048, D), device=DEV), torch.zeros(E, dtype=torch.int32))
    finally:
        layer.close()


# ----------------------------------------------------------------------------- two GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    try:
        sys.path[:0] = [str(REPO / "pallas-moe-kernel_b200"), str(REPO)]
        import datetime
        import torch.distributed as dist
        from oracle import moe_oracle as orc
        from src import _lib
        from src.ep import PeerExpertParallelMLP
        from src.routing import (dequantize_e4m3_blockwise, multinomial_group_sizes, quantize_e4m3_blockwise,
                                 zipf_group_sizes)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        M, D, F, E, dt, waves = case
        rng = np.random.default_rng(7)
        wu = (rng.standard_normal((E, D, F)) / np.sqrt(D)).astype(np.float32)
        wd = (rng.standard_normal((E, F, D)) / np.sqrt(F)).astype(np.float32)
        tdt = torch.float32 if dt == "f32" else torch.bfloat16
        El = E // world
        own = slice(rank * El, (rank + 1) * El)
        if dt == "fp8":   # e4m3 weights with 128 x 128 block scales; the oracle sees them dequantised
            (qu, su), (qd, sd) = (quantize_e4m3_blockwise(torch.from_numpy(w).to(dev)) for w in (wu, wd))
            wu_t, wd_t = dequantize_e4m3_blockwise(qu, su), dequantize_e4m3_blockwise(qd, sd)
            layer = PeerExpertParallelMLP(qu[own], qd[own], rank=rank, world=world, max_tokens=M, waves=waves,
                                          w_up_scale=su[own], w_down_scale=sd[own])
        else:
            wu_t = torch.from_numpy(wu).to(dev, tdt)
            wd_t = torch.from_numpy(wd).to(dev, tdt)
            layer = PeerExpertParallelMLP(wu_t[own], wd_t[own], rank=rank, world=world, max_tokens=M, waves=waves)
        errs = []
        r2 = np.random.default_rng(100 + rank)
        for step in range(3):
            if step == 1:   # skewed with empty experts, different on each rank
                gs = zipf_group_sizes(M, E, r2, min_empty=2)
            else:
                gs = multinomial_group_sizes(M - 5 * (step + 1), E, r2)
            x = torch.from_numpy(r2.standard_normal((M, D)).astype(np.float32)).to(dev, tdt)
            y = layer(x, torch.from_numpy(gs).to(dev))
            torch.cuda.synchronize()
            ref = orc.ref_ragged_mlp(x.double().cpu().numpy(), wu_t.double().cpu().numpy(),
                                     wd_t.double().cpu().numpy(), gs)
            errs.append(orc.correctness_metrics(ref, y.cpu().numpy())["l2_relative_error"])
            assert bool(torch.all(y[int(gs.sum()):] == 0))
        status = _lib.device_status(reset=True)
        layer.close()
        q.put((rank, "ok", max(errs), status))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc(limit=6), -1))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case,tol", [((2048, 128, 512, 4, "f32", 1), 1e-5), ((2048, 128, 512, 4, "f32", 3), 1e-5),
                                      ((2048, 512, 1024, 4, "bf16", 2), 1e-2), ((1024, 512, 1024, 8, "bf16", 1), 1e-2),
                                      ((2048, 512, 1024, 8, "fp8", 1), 2e-2)])
def test_engine_two_gpus(case, tol):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, status, err, dev_status in res:
        assert status == "ok", res
        assert err <= tol and dev_status == 0, res


def _timeout_worker(rank, world, port, q):
    """Rank 1 skips a step (between steps: none of its kernels in flight);
    rank 0's count barrier must give up within its bound, report status bit
    4 and leave the device usable."""
    try:
        sys.path[:0] = [str(REPO / "pallas-moe-kernel_b200"), str(REPO)]
        import datetime
        import time
        import torch.distributed as dist
        from src import _lib
        from src.ep import PeerExpertParallelMLP
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        D, F, El = 128, 512, 2
        wu = torch.randn((El, D, F), device=dev) / D ** 0.5
        wd = torch.randn((El, F, D), device=dev) / F ** 0.5
        layer = PeerExpertParallelMLP(wu, wd, rank=rank, world=world, max_tokens=256, waves=1)
        x = torch.randn((256, D), device=dev)
        gs = torch.full((El * world,), 64, dtype=torch.int32, device=dev)
        layer(x, gs)                                   # one good step on both ranks
        torch.cuda.synchronize()
        good = _lib.device_status(reset=True)
        t = 0.0
        if rank == 0:                                  # rank 1 does not take part in this step
            t0 = time.time()
            layer(x, gs)
            torch.cuda.synchronize()
            t = time.time() - t0
        status = _lib.device_status(reset=True)
        ok_after = float(torch.ones(4, device=dev).sum())   # the context still works
        layer.close()
        q.put((rank, "ok", (good, status, t, ok_after)))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc(limit=6)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_engine_peer_wait_times_out_with_status():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict((r, (s, v)) for r, s, v in (q.get(timeout=300) for _ in range(2)))
    for p in ps:
        p.join(timeout=60)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    good0, status0, t0, after0 = res[0][1]
    assert good0 == 0 and res[1][1][0] == 0
    assert status0 & 4, res           # the count barrier gave up
    assert 1.5 < t0 < 30.0, res       # after its 2 s bound, not forever
    assert after0 == 4.0 and res[1][1][1] == 0
