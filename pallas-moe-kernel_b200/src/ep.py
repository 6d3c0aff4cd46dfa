"""Expert-parallel fused expert MLP over ``torch.distributed`` (NCCL on B200).

The reference is single-device (there is no parallelism beyond its kernel
grid); this layer shards the experts over the ranks of a process group:

* rank ``r`` owns experts ``[r*E_local, (r+1)*E_local)`` and their weights;
* each rank holds its own batch of routed rows ``x`` (M_r, D) sorted by
  global expert id with per-expert ``group_sizes`` (E,), as the fused
  kernel expects (``src/kernel.py:85-95`` of the reference);
* counts: one ``all_to_all_single`` of (world, E_local) int32 counts tells
  every rank how many rows each source sends for each of its experts;
* dispatch: rows for (destination, expert) are contiguous in the sorted
  batch, so they go out as one grouped send/recv batch (NCCL group) and land
  expert-major on the receiver -- no permutation kernel.  Messages carry a
  per-expert tag (NCCL orders messages per peer pair anyway; gloo needs the
  tags to match several messages between the same two ranks);
* the local fused MLP runs once over the received rows (E_local groups);
* combine: the exact reverse exchange returns each row's f32 output to the
  rank and position it came from.

The expert function is injectable (``expert_fn``) so that the dispatch and
combine logic can be exercised on CPU ranks with the gloo backend; by
default it is the B200 fused kernel (:class:`src.kernel.PreparedExperts`).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class ExpertParallelMLP:
    def __init__(self, w_up_local: Optional[torch.Tensor], w_down_local: Optional[torch.Tensor], *,
                 rank: int, world: int, num_local_experts: Optional[int] = None, max_tokens: int,
                 group=None, expert_fn: Optional[Callable[[torch.Tensor, torch.Tensor], torch.Tensor]] = None,
                 out_dtype=torch.float32, w_up_scale: Optional[torch.Tensor] = None,
                 w_down_scale: Optional[torch.Tensor] = None):
        self.rank, self.world, self.group = rank, world, group
        if w_up_local is not None:
            self.e_local = w_up_local.shape[0]
            self.d = w_up_local.shape[1]
        else:
            self.e_local = int(num_local_experts)
            self.d = None
        self.num_experts = self.e_local * world
        self.out_dtype = out_dtype
        if expert_fn is None:
            from .kernel import PreparedExperts
            # A rank can receive up to world * max_tokens rows in the worst routing.
            self._experts = PreparedExperts(w_up_local, w_down_local, max_tokens=world * max_tokens,
                                            w_up_scale=w_up_scale, w_down_scale=w_down_scale)
            expert_fn = lambda xr, gs: self._experts(xr, gs)  # noqa: E731
            self.launches_per_step = 2 if w_up_local.shape[1] > 256 else 1
        else:
            self.launches_per_step = 0
        self.expert_fn = expert_fn
        self.last_recv_rows = 0

    # ------------------------------------------------------------------ helpers
    def _exchange_counts(self, group_sizes: torch.Tensor, device) -> torch.Tensor:
        send = group_sizes.to(device=device, dtype=torch.int32).reshape(self.world, self.e_local).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv  # recv[s, e]: rows from source s for local expert e

    def _p2p(self, ops):
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()

    # ------------------------------------------------------------------ forward
    def __call__(self, x: torch.Tensor, group_sizes) -> torch.Tensor:
        W, El, r = self.world, self.e_local, self.rank
        dev = x.device
        gs = torch.as_tensor(group_sizes).to(torch.int64)
        if gs.numel() != self.num_experts:
            raise ValueError(f"group_sizes has {gs.numel()} entries, expected {self.num_experts}")
        recv_counts = self._exchange_counts(gs, dev)
        gs_h = gs.cpu().clamp(min=0)
        rc_h = recv_counts.cpu().to(torch.int64).clamp(min=0)       # (W, El), host sync
        send_off = torch.zeros(self.num_experts + 1, dtype=torch.int64)
        send_off[1:] = torch.cumsum(gs_h, 0)
        # Expert-major receive layout: for local expert e, sources in rank order.
        recv_sizes = rc_h.t().reshape(-1)                             # (El*W) in (e, s) order
        recv_off = torch.zeros(El * W + 1, dtype=torch.int64)
        recv_off[1:] = torch.cumsum(recv_sizes, 0)
        n_recv = int(recv_off[-1])
        self.last_recv_rows = n_recv
        x_recv = torch.empty((n_recv, x.shape[1]), dtype=x.dtype, device=dev)

        def send_slice(dest, e):   # my rows for global expert dest*El + e
            g = dest * El + e
            return int(send_off[g]), int(gs_h[g])

        def recv_slice(src, e):    # rows from src for my local expert e
            k = e * W + src
            return int(recv_off[k]), int(recv_sizes[k])

        # ---- dispatch
        ops = []
        for peer in range(W):
            for e in range(El):
                if peer == r:
                    a, n = send_slice(r, e)
                    b, m = recv_slice(r, e)
                    if n:
                        x_recv[b:b + m].copy_(x[a:a + n])
                    continue
                a, n = send_slice(peer, e)
                if n:
                    ops.append(dist.P2POp(dist.isend, x[a:a + n].contiguous(), peer, group=self.group, tag=1 + e))
                b, m = recv_slice(peer, e)
                if m:
                    ops.append(dist.P2POp(dist.irecv, x_recv[b:b + m], peer, group=self.group, tag=1 + e))
        self._p2p(ops)

        # ---- local experts
        local_gs = rc_h.sum(0).to(torch.int32)                        # (El,)
        if n_recv:
            y_recv = self.expert_fn(x_recv, local_gs).to(self.out_dtype)
        else:   # every rank must agree on the combine dtype, even with nothing to compute
            y_recv = torch.empty((0, x.shape[1]), dtype=self.out_dtype, device=dev)

        # ---- combine (reverse exchange)
        M = x.shape[0]
        y = torch.empty((M, x.shape[1]), dtype=y_recv.dtype, device=dev)
        routed = int(min(int(send_off[-1]), M))
        if routed < M:
            y[routed:].zero_()          # rows past sum(group_sizes) are zero (ragged_dot)
        ops = []
        for peer in range(W):
            for e in range(El):
                if peer == r:
                    a, n = send_slice(r, e)
                    b, m = recv_slice(r, e)
                    if n:
                        y[a:a + n].copy_(y_recv[b:b + m])
                    continue
                b, m = recv_slice(peer, e)
                if m:
                    ops.append(dist.P2POp(dist.isend, y_recv[b:b + m].contiguous(), peer, group=self.group,
                                          tag=1 + El + e))
                a, n = send_slice(peer, e)
                if n:
                    ops.append(dist.P2POp(dist.irecv, y[a:a + n], peer, group=self.group, tag=1 + El + e))
        self._p2p(ops)
        return y
