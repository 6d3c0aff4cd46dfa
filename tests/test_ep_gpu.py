"""Expert-parallel layer on 2 GPUs (NCCL) with the B200 kernels as the local
experts, checked against the single-process CPU oracle.  Skipped when fewer
than two GPUs are visible."""

import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


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
        from src.ep import ExpertParallelMLP
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
        wu_t = torch.from_numpy(wu).to(dev, tdt)
        wd_t = torch.from_numpy(wd).to(dev, tdt)
        El = E // world
        layer = ExpertParallelMLP(wu_t[rank * El:(rank + 1) * El], wd_t[rank * El:(rank + 1) * El],
                                  rank=rank, world=world, max_tokens=M, waves=waves)
        r2 = np.random.default_rng(100 + rank)
        x = torch.from_numpy(r2.standard_normal((M, D)).astype(np.float32)).to(dev, tdt)
        gs = r2.multinomial(M - 5, np.full(E, 1.0 / E)).astype(np.int32)
        y = layer(x, torch.from_numpy(gs).to(dev))
        torch.cuda.synchronize()
        ref = orc.ref_ragged_mlp(x.float().cpu().numpy(), wu_t.float().cpu().numpy(), wd_t.float().cpu().numpy(), gs)
        m = orc.correctness_metrics(ref, y.cpu().numpy())
        q.put((rank, "ok", m["l2_relative_error"], bool(np.all(y[M - 5:].cpu().numpy() == 0))))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc(limit=4), False))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("case,tol", [((2048, 128, 512, 4, "f32", 1), 1e-5), ((1024, 512, 1024, 4, "bf16", 1), 1e-2),
                                      ((2048, 128, 512, 4, "f32", 3), 1e-5), ((2048, 512, 1024, 4, "bf16", 2), 1e-2)])
def test_ep_two_gpus(case, tol):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, status, err, tail_zero in res:
        assert status == "ok", res
        assert err <= tol and tail_zero, res
