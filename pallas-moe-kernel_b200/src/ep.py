"""Expert-parallel fused expert MLP: experts sharded over the GPUs of a node.

Two transports for the same layer contract:

* :class:`PeerExpertParallelMLP` -- the product path on B200: the library's
  device engine (``moe_ep_*`` in the C ABI) moves rows with its own kernels
  over NVLink peer memory, exchanges group sizes on the device (no host
  synchronisation per step) and overlaps the exchange of one wave with the
  experts of the next;
* :class:`ExpertParallelMLP` -- the same exchange as NCCL (or gloo) grouped
  send/recv issued from Python, with a host synchronisation on the counts;
  it also runs on CPU ranks, which is how the exchange logic is tested
  without GPUs.

The reference is single-device (there is no parallelism beyond its kernel
grid); both layers shard the experts over the ranks of a process group:

* rank ``r`` owns experts ``[r*E_local, (r+1)*E_local)`` and their weights;
* each rank holds its own batch of routed rows ``x`` (M_r, D) sorted by
  global expert id with per-expert ``group_sizes`` (E,), as the fused
  kernel expects (``src/kernel.py:85-95`` of the reference);
* counts: one ``all_to_all_single`` of (world, E_local) int32 counts tells
  every rank how many rows each source sends for each of its experts (the one
  host synchronisation of a step: message sizes must be known on the host);
* waves: the batch is cut into ``waves`` slices, wave w taking rows
  ``[c*w//V, c*(w+1)//V)`` of every expert group of ``c`` rows, so that each
  wave is itself a routed batch over all experts;
* dispatch: per wave, the rows for (destination, expert) are contiguous in
  the sorted batch, so they go out as one grouped send/recv batch (an NCCL
  group) and land expert-major on the receiver -- no permutation kernel.
  Messages carry a per-expert tag (NCCL orders messages per peer pair anyway;
  gloo needs the tags to match several messages between the same two ranks);
* the local fused MLP runs over each wave's received rows (E_local groups);
* combine: the exact reverse exchange returns each row's output to the rank
  and position it came from.

Overlap: the dispatch of wave w+1 and the combine of wave w-1 are in flight
on NCCL's stream while the experts of wave w compute, so with V waves only
the first dispatch and the last combine are exposed.  ``reserve_sms`` keeps
that many SMs free of the persistent expert kernels so NCCL's kernels can run
beside them.

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
                 w_down_scale: Optional[torch.Tensor] = None, waves: int = 1, reserve_sms: int = 0):
        self.rank, self.world, self.group = rank, world, group
        if w_up_local is not None:
            self.e_local = w_up_local.shape[0]
        else:
            self.e_local = int(num_local_experts)
        self.num_experts = self.e_local * world
        self.out_dtype = out_dtype
        self.waves = max(1, int(waves))
        self.reserve_sms = max(0, int(reserve_sms))
        if expert_fn is None:
            from . import _lib
            from .kernel import PreparedExperts
            # A rank can receive up to world * max_tokens rows in the worst routing.
            self._experts = PreparedExperts(w_up_local, w_down_local, max_tokens=world * max_tokens,
                                            w_up_scale=w_up_scale, w_down_scale=w_down_scale)
            ctas = 0
            if self.reserve_sms:
                sms = torch.cuda.get_device_properties(w_up_local.device).multi_processor_count
                ctas = max(2, sms - self.reserve_sms)

            def expert_fn(xr, gs):
                # Persistent CTAs per launch capped for this layer's launches only.
                if not ctas:
                    return self._experts(xr, gs)
                _lib.set_tuning(2, ctas)
                try:
                    return self._experts(xr, gs)
                finally:
                    _lib.set_tuning(2, 0)
            self.launches_per_wave = 2 if w_up_local.shape[1] > 256 else 1
        else:
            self.launches_per_wave = 0
        self.expert_fn = expert_fn
        self.last_recv_rows = 0
        self.last_launches = 0

    # ------------------------------------------------------------------ helpers
    def _exchange_counts(self, group_sizes: torch.Tensor, device) -> torch.Tensor:
        send = group_sizes.to(device=device, dtype=torch.int32).reshape(self.world, self.e_local).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv  # recv[s, e]: rows from source s for local expert e

    @staticmethod
    def wave_cuts(counts: torch.Tensor, waves: int) -> torch.Tensor:
        """Row offsets inside each group at the wave boundaries:
        ``cut[..., w] = counts * w // waves``, shape (..., waves + 1)."""
        w = torch.arange(waves + 1, dtype=torch.int64)
        return (counts.to(torch.int64).unsqueeze(-1) * w) // waves

    @staticmethod
    def _start(ops):
        return dist.batch_isend_irecv(ops) if ops else []

    @staticmethod
    def _wait(reqs):
        for q in reqs:
            q.wait()

    # ------------------------------------------------------------------ forward
    def __call__(self, x: torch.Tensor, group_sizes) -> torch.Tensor:
        W, El, r, V = self.world, self.e_local, self.rank, self.waves
        dev, M, D = x.device, x.shape[0], x.shape[1]
        gs = torch.as_tensor(group_sizes).to(torch.int64)
        if gs.numel() != self.num_experts:
            raise ValueError(f"group_sizes has {gs.numel()} entries, expected {self.num_experts}")
        recv_counts = self._exchange_counts(gs, dev)
        gs_h = gs.cpu().clamp(min=0)
        rc_h = recv_counts.cpu().to(torch.int64).clamp(min=0)        # (W, El), host sync
        send_off = torch.zeros(self.num_experts + 1, dtype=torch.int64)
        send_off[1:] = torch.cumsum(gs_h, 0)
        send_cut = self.wave_cuts(gs_h, V).tolist()                   # (E, V+1)
        recv_cut = self.wave_cuts(rc_h, V).tolist()                   # (W, El, V+1)
        send_off = send_off.tolist()

        y = torch.empty((M, D), dtype=self.out_dtype, device=dev)
        routed = min(send_off[-1], M)
        if routed < M:
            y[routed:].zero_()          # rows past sum(group_sizes) are zero (ragged_dot)

        def plan(v):
            """Wave v: my sends (peer, e) -> rows [a, a+n) of x and y, my
            receives (peer, e) -> rows [b, b+m) of this wave's expert-major
            buffer, the buffer's row count and its per-expert group sizes."""
            sends, recvs, pos, local = {}, {}, 0, []
            for peer in range(W):
                for e in range(El):
                    g = peer * El + e
                    sends[(peer, e)] = (send_off[g] + send_cut[g][v], send_cut[g][v + 1] - send_cut[g][v])
            for e in range(El):
                start = pos
                for src in range(W):
                    m = recv_cut[src][e][v + 1] - recv_cut[src][e][v]
                    recvs[(src, e)] = (pos, m)
                    pos += m
                local.append(pos - start)
            return sends, recvs, pos, torch.tensor(local, dtype=torch.int32)

        plans = [plan(v) for v in range(V)]
        self.last_recv_rows = sum(p[2] for p in plans)

        def dispatch(v):
            sends, recvs, n_recv, _ = plans[v]
            xr = torch.empty((n_recv, D), dtype=x.dtype, device=dev)
            ops = []
            for peer in range(W):
                for e in range(El):
                    a, n = sends[(peer, e)]
                    b, m = recvs[(peer, e)]
                    if peer == r:
                        if n:
                            xr[b:b + m].copy_(x[a:a + n])
                        continue
                    if n:
                        ops.append(dist.P2POp(dist.isend, x[a:a + n], peer, group=self.group, tag=1 + e))
                    if m:
                        ops.append(dist.P2POp(dist.irecv, xr[b:b + m], peer, group=self.group, tag=1 + e))
            return xr, self._start(ops)

        def combine(v, yr):
            sends, recvs, _, _ = plans[v]
            ops = []
            for peer in range(W):
                for e in range(El):
                    a, n = sends[(peer, e)]
                    b, m = recvs[(peer, e)]
                    if peer == r:
                        if n:
                            y[a:a + n].copy_(yr[b:b + m])
                        continue
                    if m:
                        ops.append(dist.P2POp(dist.isend, yr[b:b + m], peer, group=self.group, tag=1 + El + e))
                    if n:
                        ops.append(dist.P2POp(dist.irecv, y[a:a + n], peer, group=self.group, tag=1 + El + e))
            return self._start(ops)

        # Software pipeline over the waves.  Every rank issues the same
        # sequence of grouped exchanges (dispatch 0, then per wave: dispatch
        # v+1, combine v), so the NCCL groups pair up across ranks.
        launches = 0
        combines = []
        xr_next, req_next = dispatch(0)
        for v in range(V):
            xr, req = xr_next, req_next
            if v + 1 < V:
                xr_next, req_next = dispatch(v + 1)
            self._wait(req)                             # wave v's rows have landed
            n_recv, local_gs = plans[v][2], plans[v][3]
            if n_recv:
                yr = self.expert_fn(xr, local_gs).to(self.out_dtype)
                launches += self.launches_per_wave
            else:   # every rank must agree on the combine dtype, even with nothing to compute
                yr = torch.empty((0, D), dtype=self.out_dtype, device=dev)
            combines.append(combine(v, yr))
        for reqs in combines:
            self._wait(reqs)
        self.last_launches = launches
        return y


class PeerExpertParallelMLP:
    """Expert-parallel fused MLP on the device engine of the C ABI
    (``moe_ep_*``): the token exchange is done by the library's own kernels
    over NVLink peer memory instead of NCCL messages, group sizes are
    exchanged on the device (no host synchronisation per step), and the
    exchange of one wave overlaps the experts of the next.

    Same contract as :class:`ExpertParallelMLP`: rank ``r`` owns experts
    ``[r*E_local, (r+1)*E_local)``; ``__call__(x, group_sizes)`` takes this
    rank's rows sorted by global expert and returns their f32 outputs in the
    same order.  Every rank calls it the same number of times (it is a
    collective) and calls :meth:`close` at the end.  With ``world == 1`` no
    process group is needed.
    """

    def __init__(self, w_up_local: torch.Tensor, w_down_local: torch.Tensor, *, rank: int, world: int,
                 max_tokens: int, group=None, w_up_scale: Optional[torch.Tensor] = None,
                 w_down_scale: Optional[torch.Tensor] = None, waves: int = 2, comm_ctas: int = 0):
        import ctypes

        from . import _lib
        self._L = L = _lib.lib()
        self._check = _lib.check
        self.rank, self.world, self.group = rank, world, group
        self.device = w_up_local.device
        self.e_local, D, F = w_up_local.shape
        self.num_experts = self.e_local * world
        self.d, self.max_tokens = D, int(max_tokens)
        self.dtype_code = {torch.float32: _lib.MOE_DTYPE_F32, torch.bfloat16: _lib.MOE_DTYPE_BF16,
                           torch.float8_e4m3fn: _lib.MOE_DTYPE_FP8_E4M3_BLK128}[w_up_local.dtype]
        self.x_dtype = torch.float32 if self.dtype_code == _lib.MOE_DTYPE_F32 else torch.bfloat16
        # Keep every buffer the engine reads by pointer alive with the engine.
        self._weights = [t.contiguous() for t in (w_up_local, w_down_local)]
        self._scales = [None if t is None else t.to(device=self.device, dtype=torch.float32).contiguous()
                        for t in (w_up_scale, w_down_scale)]
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            self._check(L.moe_ep_create(rank, world, self.e_local, self.max_tokens, D, F, self.dtype_code,
                                        int(waves), int(comm_ctas), ctypes.byref(h)))
            self._ep = h
            blob = (ctypes.c_uint8 * _lib.MOE_EP_HANDLE_BYTES)()
            self._check(L.moe_ep_export(self._ep, blob))
            mine = torch.tensor(bytearray(blob), dtype=torch.uint8, device=self.device)
            if world > 1:
                every = torch.empty(world * _lib.MOE_EP_HANDLE_BYTES, dtype=torch.uint8, device=self.device)
                dist.all_gather_into_tensor(every, mine, group=group)
            else:
                every = mine
            self._check(L.moe_ep_connect(self._ep, bytes(every.cpu().numpy().tobytes())))
            stream = torch.cuda.current_stream(self.device).cuda_stream
            self._check(L.moe_ep_set_weights(self._ep, self._weights[0].data_ptr(), self._weights[1].data_ptr(),
                                              0 if self._scales[0] is None else self._scales[0].data_ptr(),
                                              0 if self._scales[1] is None else self._scales[1].data_ptr(),
                                              stream))
            torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)
        self.launches_per_forward = L.moe_ep_launches_per_forward(self._ep)
        # D > 256 engines store Y rows straight into their own buffer; without
        # `out` the result is a view of it (valid until the next call).
        self._own_y = L.moe_ep_output(self._ep)
        self.waves = 1 if self._own_y else int(waves)   # two-GEMM engines run one wave

    def _own_view(self, M: int) -> torch.Tensor:
        iface = {"shape": (M, self.d), "typestr": "<f4", "version": 3,
                 "data": (int(self._own_y), False), "strides": None}
        view = type("_EngineY", (), {"__cuda_array_interface__": iface})()
        return torch.as_tensor(view, device=self.device)

    def __call__(self, x: torch.Tensor, group_sizes, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self._ep is None:
            raise RuntimeError("engine closed")
        if x.dim() != 2 or x.shape[1] != self.d or x.dtype != self.x_dtype or x.device != self.device:
            raise ValueError(f"x must be ({'M'}, {self.d}) {self.x_dtype} on {self.device}")
        M = x.shape[0]
        x = x.contiguous()
        gs = torch.as_tensor(group_sizes).to(device=self.device, dtype=torch.int32, non_blocking=True).contiguous()
        if gs.numel() != self.num_experts:
            raise ValueError(f"group_sizes has {gs.numel()} entries, expected {self.num_experts}")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if out is None and self._own_y and M > 0:
            self._check(self._L.moe_ep_forward(self._ep, x.data_ptr(), gs.data_ptr(), None, M, stream))
            return self._own_view(M)
        y = out if out is not None else torch.empty((M, self.d), dtype=torch.float32, device=self.device)
        if y.shape != (M, self.d) or y.dtype != torch.float32 or not y.is_contiguous():
            raise ValueError("out must be a contiguous (M, D) float32 tensor")
        self._check(self._L.moe_ep_forward(self._ep, x.data_ptr(), gs.data_ptr(), y.data_ptr(), M, stream))
        return y

    def close(self) -> None:
        """Collective: waits for this rank's work, meets the other ranks and
        frees the engine (no rank may still read another's buffer)."""
        if self._ep is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._check(self._L.moe_ep_destroy(self._ep))
        self._ep = None
