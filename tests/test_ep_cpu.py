"""Expert-parallel dispatch / combine on CPU ranks (gloo), checked against the
single-process oracle.  The local expert function is the oracle itself, so
these tests cover the routing, count exchange and reverse exchange logic of
``src.ep.ExpertParallelMLP`` without a GPU."""

import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(E, D, F):
    rng = np.random.default_rng(1234)
    wu = rng.standard_normal((E, D, F)) / np.sqrt(D)
    wd = rng.standard_normal((E, F, D)) / np.sqrt(F)
    return wu, wd


def _rank_inputs(rank, M, D, E, mode):
    rng = np.random.default_rng(100 + rank)
    x = rng.standard_normal((M, D))
    if mode == "uniform":
        gs = rng.multinomial(M - 3, np.full(E, 1.0 / E))      # 3 unrouted trailing rows
    else:                                                     # skewed, with empty experts
        w = np.zeros(E)
        w[rank % E] = 1.0
        gs = rng.multinomial(M, w)
    return x, gs.astype(np.int32)


def _worker(rank, world, port, E, D, F, M, modes, q, fail_rank=-1, waves=1):
    try:
        sys.path[:0] = [str(REPO / "pallas-moe-kernel_b200"), str(REPO)]
        import datetime
        import torch.distributed as dist
        from oracle import moe_oracle as orc
        from src.ep import ExpertParallelMLP
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        wu, wd = _weights(E, D, F)
        El = E // world
        wu_l, wd_l = wu[rank * El:(rank + 1) * El], wd[rank * El:(rank + 1) * El]

        def expert_fn(xr, gs):
            return torch.from_numpy(orc.ref_ragged_mlp(xr.numpy(), wu_l, wd_l, gs.numpy()))

        layer = ExpertParallelMLP(None, None, rank=rank, world=world, num_local_experts=El, max_tokens=M,
                                  expert_fn=expert_fn, out_dtype=torch.float64, waves=waves)
        if rank == fail_rank:
            raise SystemExit(3)          # this rank leaves before the exchange
        err = 0.0
        for mode in modes:
            x, gs = _rank_inputs(rank, M, D, E, mode)
            y = layer(torch.from_numpy(x), torch.from_numpy(gs)).numpy()
            ref = orc.ref_ragged_mlp(x, wu, wd, gs)
            err = max(err, float(np.abs(y - ref).max()))
        q.put((rank, "ok", err))
        dist.destroy_process_group()
    except SystemExit:
        q.put((rank, "left", 0.0))
    except Exception:
        q.put((rank, "error", traceback.format_exc(limit=3)))


def _run(world, E, D, F, M, modes, fail_rank=-1, timeout=120, waves=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, E, D, F, M, modes, q, fail_rank, waves)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, status, val = q.get(timeout=timeout)
        out[r] = (status, val)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("world,E,waves", [(2, 4, 1), (4, 4, 1), (2, 4, 3), (4, 8, 2)])
def test_ep_matches_single_process_oracle(world, E, waves):
    """Uniform routing with unrouted trailing rows, then one-expert-per-rank
    skew (most experts empty on every rank), through the same layer; with
    waves > 1 the groups are cut into slices (some empty: groups smaller than
    the wave count) whose exchanges overlap."""
    out = _run(world, E, D=16, F=24, M=40, modes=("uniform", "skewed", "uniform"), waves=waves)
    for r in range(world):
        status, err = out[r]
        assert status == "ok", out
        assert err < 1e-10, out


def test_ep_rank_failure_is_reported_not_hung():
    """A rank that leaves before the exchange: the survivor's collective ends
    with an error within the process-group timeout (host-side detection)."""
    out = _run(2, 4, D=8, F=8, M=16, modes=("uniform",), fail_rank=1, timeout=90)
    assert out[1][0] == "left"
    assert out[0][0] == "error", out


def test_wave_cuts_partition_every_group():
    from importlib import import_module
    sys.path[:0] = [str(REPO / "pallas-moe-kernel_b200")]
    ep = import_module("src.ep")
    counts = torch.tensor([[0, 1, 2, 7], [5, 3, 100, 64]])
    for v in (1, 2, 3, 4, 8):
        cut = ep.ExpertParallelMLP.wave_cuts(counts, v)
        assert cut.shape == (2, 4, v + 1)
        assert torch.equal(cut[..., 0], torch.zeros_like(counts)) and torch.equal(cut[..., -1], counts)
        d = cut.diff(dim=-1)
        assert bool((d >= 0).all()) and bool((d.max(-1).values - d.min(-1).values <= 1).all())
