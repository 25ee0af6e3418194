"""Expert parallelism on B200: the same public surface as the reference's
``miniep.ep`` (Placement, Comm, EPStats, EPMoEBackend), with the layer step
running as sm_100a kernels behind libminiep_b200's C ABI.

Differences a caller of the reference sees:
  * ``Comm`` needs the layer shape up front (it allocates the symmetric
    receive/landing buffers every rank can store into) and opens every peer's
    buffers over CUDA IPC; the counts exchange and both all-to-alls are peer
    stores issued by the kernels, with no host synchronisation in the step.
  * Placement tables, the round-robin state and the routing statistics live on
    the device (one context per rank); ``Placement.dest_ranks``/``reset_rr``
    and ``EPStats.snapshot`` read or update that state.
  * Every tensor argument is a CUDA tensor. There is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._lib import MEPError, check, ptr

_DTYPES = {torch.float32: _lib.MEP_F32, torch.bfloat16: _lib.MEP_BF16}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class Placement:
    """owners[layer][expert] = ranks holding that expert (>= 1, sorted, distinct).

    Same constructors and queries as the reference (miniep/ep.py:20-96). The
    round-robin dispatch over replicas runs on the device of the ``Comm`` the
    placement is installed on.
    """

    def __init__(self, owners: list[list[list[int]]]):
        self.owners = [[list(o) for o in layer] for layer in owners]
        self.num_layers = len(self.owners)
        self.num_experts = len(self.owners[0])
        for l, layer in enumerate(self.owners):
            if len(layer) != self.num_experts:
                raise ValueError(f"layer {l}: {len(layer)} experts, expected {self.num_experts}")
            for e, o in enumerate(layer):
                if not o or len(set(o)) != len(o) or min(o) < 0:
                    raise ValueError(f"layer {l} expert {e}: bad owner list {o}")
        self._comm = None

    @staticmethod
    def naive(num_layers: int, num_experts: int, world: int) -> "Placement":
        if num_experts % world:
            raise ValueError("num_experts must be divisible by world")
        per = num_experts // world
        return Placement([[[e // per] for e in range(num_experts)] for _ in range(num_layers)])

    @staticmethod
    def from_plan(plan: dict) -> "Placement":
        owners_by_layer = plan["owners"]
        return Placement([
            [sorted(owners_by_layer[str(l)][str(e)]) for e in range(len(owners_by_layer[str(l)]))]
            for l in range(len(owners_by_layer))
        ])

    def to_plan(self) -> dict:
        return {"owners": {
            str(l): {str(e): self.owners[l][e] for e in range(self.num_experts)}
            for l in range(self.num_layers)}}

    def experts_of_rank(self, rank: int) -> dict[int, list[int]]:
        return {l: sorted(e for e in range(self.num_experts) if rank in self.owners[l][e])
                for l in range(self.num_layers)}

    def table(self, layer: int):
        """(E, rmax) int64 table and (E,) int64 replica counts of one layer."""
        own = self.owners[layer]
        rmax = max(len(o) for o in own)
        table = torch.zeros(self.num_experts, rmax, dtype=torch.int64)
        n_rep = torch.zeros(self.num_experts, dtype=torch.int64)
        for e, o in enumerate(own):
            table[e, :len(o)] = torch.tensor(o)
            n_rep[e] = len(o)
        return table, n_rep

    def _bound(self) -> "Comm":
        if self._comm is None:
            raise MEPError("placement is not installed on a Comm (call comm.install(placement))")
        return self._comm

    def reset_rr(self):
        comm = self._bound()
        check(_lib.lib().mep_reset_rr(comm._ctx, _stream()), comm._ctx, "mep_reset_rr")

    def dest_ranks(self, layer: int, expert_ids: torch.Tensor) -> torch.Tensor:
        """Destination rank of each entry (i-th occurrence of expert e goes to
        replica (rr[e] + i) % n_rep[e]; then rr[e] += count[e])."""
        comm = self._bound()
        ids = expert_ids.to(device=comm.device, dtype=torch.int64).contiguous()
        out = torch.empty_like(ids)
        check(_lib.lib().mep_dest_ranks(comm._ctx, layer, ptr(ids), ids.numel(), ptr(out),
                                        _stream()), comm._ctx, "mep_dest_ranks")
        return out


class Comm:
    """Per-rank device context: symmetric buffers reachable by every rank,
    placement tables, round-robin state and routing statistics.

    ``group``: torch.distributed group whose ranks are the expert-parallel
    ranks (default: the world, or a single rank when torch.distributed is not
    initialised). Shape arguments describe the MoE layers that will run.
    """

    def __init__(self, group=None, *, num_layers: int, num_experts: int, topk: int,
                 hidden: int, inter: int, max_tokens: int, dtype=torch.bfloat16,
                 device=None, recv_capacity_rows: int = 0, timeout_ms: int = 10000,
                 single_process: bool = False):
        if dtype not in _DTYPES:
            raise ValueError(f"dtype must be one of {list(_DTYPES)}")
        self.group = group
        if single_process or not (dist.is_available() and dist.is_initialized()):
            self.rank, self.world = 0, 1
        else:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device if isinstance(device, int) else
                                   torch.device(device).index or 0)
        self.dtype = dtype
        self.num_layers, self.num_experts, self.topk = num_layers, num_experts, topk
        self.hidden, self.inter, self.max_tokens = hidden, inter, max_tokens
        self.native = True
        L = _lib.lib()
        ctx = C.c_void_p()
        check(L.mep_ctx_create(self.rank, self.world, self.device.index, num_layers, num_experts,
                               topk, hidden, inter, max_tokens, _DTYPES[dtype],
                               recv_capacity_rows, C.byref(ctx)), None, "mep_ctx_create")
        self._ctx = ctx
        check(L.mep_set_option(ctx, b"timeout_ms", timeout_ms), ctx, "mep_set_option")
        if self.world > 1:
            self._open_peers()
        self.placement = None
        self.stats = None

    def _open_peers(self):
        L = _lib.lib()
        buf = C.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        check(L.mep_ipc_handle(self._ctx, buf), self._ctx, "mep_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(buf.raw), group=self.group)
        for peer, h in enumerate(handles):
            if peer != self.rank:
                hb = C.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
                check(L.mep_ipc_open(self._ctx, peer, hb), self._ctx, "mep_ipc_open")
        if dist.get_backend(self.group) == "nccl":
            dist.barrier(group=self.group, device_ids=[self.device.index])
        else:
            dist.barrier(group=self.group)

    def install(self, placement: Placement):
        """Upload every layer's dispatch table (same tables on every rank)."""
        if placement.num_layers != self.num_layers or placement.num_experts != self.num_experts:
            raise ValueError("placement shape does not match the Comm")
        L = _lib.lib()
        for layer in range(placement.num_layers):
            table, n_rep = placement.table(layer)
            check(L.mep_set_placement(self._ctx, layer, table.data_ptr(), n_rep.data_ptr(),
                                      table.shape[1]), self._ctx, "mep_set_placement")
        placement._comm = self
        self.placement = placement

    def barrier(self):
        """Rank barrier on the device (mep_barrier): enqueued on the current
        stream; every rank's stream continues once all ranks have reached it.
        Every rank must call it the same number of times."""
        check(_lib.lib().mep_barrier(self._ctx, _stream()), self._ctx, "mep_barrier")

    def set_option(self, name: str, value: int):
        check(_lib.lib().mep_set_option(self._ctx, name.encode(), int(value)), self._ctx,
              "mep_set_option")

    def check(self):
        """Raise if a kernel recorded a device-side error (synchronises)."""
        torch.cuda.current_stream(self.device).synchronize()
        check(_lib.lib().mep_check(self._ctx), self._ctx, "device")

    def read_timeline(self) -> dict:
        """Stamps of the last layer step recorded with the "timeline" option
        (synchronises, then clears them): {stage: (start_us, end_us)} and
        {mark: t_us}, in microseconds after this rank's last device barrier
        (or after the step's first stamp when no barrier ran). Stages that did
        not run are left out."""
        buf = (C.c_uint64 * _lib.TL_SLOTS)()
        check(_lib.lib().mep_read_timeline(self._ctx, buf, _stream()), self._ctx,
              "mep_read_timeline")
        raw = list(buf)
        t0 = raw[_lib.TL_MARKS["barrier_end"]] or min((v for v in raw if v), default=0)
        us = lambda v: (v - t0) / 1e3  # noqa: E731
        out = {}
        for name, s in _lib.TL_STAGES.items():
            if raw[s] and raw[s + 1]:
                out[name] = (us(raw[s]), us(raw[s + 1]))
        for name, s in _lib.TL_MARKS.items():
            if raw[s] and name != "barrier_end":
                out[name] = us(raw[s])
        return out

    def last_recv_rows(self) -> int:
        v = C.c_int64()
        check(_lib.lib().mep_last_recv_rows(self._ctx, C.byref(v), _stream()), self._ctx)
        return v.value

    def close(self):
        if getattr(self, "_ctx", None):
            _lib.lib().mep_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class EPStats:
    """Per-rank counters for one run; same fields and snapshot schema as the
    reference (miniep/ep.py:164-183). Counts are kept on the device by the
    kernels; times (seconds) come from CUDA events around the stages."""

    def __init__(self, num_layers: int, num_experts: int, timing: bool = True):
        self.num_layers, self.num_experts = num_layers, num_experts
        self.timing = timing
        self.compute_time = 0.0
        self.a2a_time = 0.0
        self.steps = 0
        self._comm = None
        self._pending = []
        self._route_counts = torch.zeros(num_layers, num_experts, dtype=torch.long)
        self._recv = torch.zeros(num_layers, dtype=torch.long)

    def _bind(self, comm: Comm):
        if self._comm is comm:
            return
        if comm.stats is not None and comm.stats is not self:
            raise MEPError("this Comm already reports into another EPStats")
        check(_lib.lib().mep_reset_stats(comm._ctx, _stream()), comm._ctx, "mep_reset_stats")
        self._comm = comm
        comm.stats = self

    def _refresh(self):
        if self._comm is None:
            return
        rc = torch.zeros(self.num_layers, self.num_experts, dtype=torch.long)
        rv = torch.zeros(self.num_layers, dtype=torch.long)
        check(_lib.lib().mep_read_stats(self._comm._ctx, rc.data_ptr(), rv.data_ptr(),
                                        _stream()), self._comm._ctx, "mep_read_stats")
        self._route_counts, self._recv = rc, rv
        for e0, e1, e2, e3 in self._pending:
            self.a2a_time += (e0.elapsed_time(e1) + e2.elapsed_time(e3)) / 1e3
            self.compute_time += e1.elapsed_time(e2) / 1e3
        self._pending.clear()

    @property
    def route_counts(self) -> torch.Tensor:
        self._refresh()
        return self._route_counts

    @property
    def recv_tokens_per_layer(self) -> torch.Tensor:
        self._refresh()
        return self._recv

    @property
    def recv_tokens(self) -> int:
        return int(self.recv_tokens_per_layer.sum())

    def snapshot(self) -> dict:
        self._refresh()
        return {
            "recv_tokens": int(self._recv.sum()),
            "recv_tokens_per_layer": self._recv.tolist(),
            "compute_time": self.compute_time,
            "a2a_time": self.a2a_time,
            "route_counts": self._route_counts.tolist(),
            "steps": self.steps,
        }


def _as_valid(valid_mask, n, device):
    if valid_mask is None:
        return None
    v = valid_mask.reshape(-1)
    if v.numel() != n:
        raise ValueError("valid_mask must have one entry per token")
    return v.to(device=device, dtype=torch.uint8).contiguous()


class EPMoEBackend:
    """Drop-in for the reference's EPMoEBackend / LocalMoEBackend: same
    constructor and ``__call__`` contract (miniep/ep.py:186-249).

    local_experts: sorted global expert ids resident on this rank for this
    layer; w_in (E_l, 2I, H) / w_out (E_l, H, I) are the matching stacked
    slices, as CUDA tensors of the Comm's dtype.
    """

    def __init__(self, layer, comm: Comm, placement: Placement, local_experts: list[int],
                 w_in, w_out, stats: EPStats):
        self.layer = layer
        self.comm = comm
        self.placement = placement
        self.w_in = w_in
        self.w_out = w_out
        self.stats = stats
        self._update_map(local_experts)

    def _update_map(self, local_experts):
        self.local_experts = list(local_experts)

    def _prepare(self, x_flat):
        comm = self.comm
        if comm.placement is not self.placement:
            comm.install(self.placement)
        if self.stats is not None:
            self.stats._bind(comm)
        want = self.placement.experts_of_rank(comm.rank)[self.layer]
        if self.local_experts != want:
            raise MEPError(f"layer {self.layer}: local_experts {self.local_experts} do not match "
                           f"the placement's experts of rank {comm.rank}: {want}")
        for name, t in (("x_flat", x_flat), ("w_in", self.w_in), ("w_out", self.w_out)):
            if not t.is_cuda or t.dtype != comm.dtype:
                raise MEPError(f"{name} must be a CUDA {comm.dtype} tensor")
        n_local = len(self.local_experts)
        if tuple(self.w_in.shape) != (n_local, 2 * comm.inter, comm.hidden) or \
                tuple(self.w_out.shape) != (n_local, comm.hidden, comm.inter):
            raise MEPError(f"layer {self.layer}: expert weight shapes {tuple(self.w_in.shape)} / "
                           f"{tuple(self.w_out.shape)} do not match {n_local} local experts")
        return n_local

    def __call__(self, x_flat, topk_idx, topk_gate, valid_mask=None):
        comm = self.comm
        n_local = self._prepare(x_flat)
        n, k = topk_idx.shape
        x = x_flat.contiguous()
        idx = topk_idx.to(torch.int64).contiguous()
        gate = topk_gate.to(comm.dtype).contiguous()
        valid = _as_valid(valid_mask, n, x.device)
        w_in, w_out = self.w_in.contiguous(), self.w_out.contiguous()
        out = torch.empty_like(x)
        L, ctx, st = _lib.lib(), comm._ctx, _stream()
        timing = self.stats is not None and self.stats.timing
        if not timing:
            check(L.mep_moe_forward(ctx, self.layer, ptr(x), ptr(idx), ptr(gate), ptr(valid), n,
                                    ptr(w_in), ptr(w_out), n_local, ptr(out), st), ctx,
                  "mep_moe_forward")
        else:
            # the reference's three timed phases (ep.py:223-235), as CUDA events
            # for EPStats and as NVTX ranges for a profiler's timeline
            nvtx = torch.cuda.nvtx
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            ev[0].record()
            nvtx.range_push(f"moe L{self.layer}: counts + dispatch")
            check(L.mep_route(ctx, self.layer, ptr(idx), ptr(valid), n, n_local, st), ctx,
                  "mep_route")
            check(L.mep_dispatch(ctx, ptr(x), ptr(idx), n, st), ctx, "mep_dispatch")
            nvtx.range_pop()
            ev[1].record()
            nvtx.range_push(f"moe L{self.layer}: experts")
            check(L.mep_expert_ffn(ctx, ptr(w_in), ptr(w_out), n_local, st), ctx,
                  "mep_expert_ffn")
            nvtx.range_pop()
            ev[2].record()
            nvtx.range_push(f"moe L{self.layer}: combine")
            check(L.mep_combine(ctx, ptr(gate), ptr(valid), n, None, 0.0, ptr(out), None, st),
                  ctx, "mep_combine")
            nvtx.range_pop()
            ev[3].record()
            self.stats._pending.append(tuple(ev))
        return out

    def moe_block(self, h, x_flat, router_w, residual_multiplier: float, bias=None,
                  valid_mask=None):
        """Router + this backend + residual in one call: the MoE half of
        ``Block.forward`` (miniep/modeling.py:192-197). Returns
        (h + moe(x) * residual_multiplier, topk_idx, topk_gate)."""
        comm = self.comm
        n_local = self._prepare(x_flat)
        n = x_flat.shape[0]
        x = x_flat.contiguous()
        hh = h.reshape(n, -1).contiguous()
        rw = router_w.to(comm.dtype).contiguous()
        b = None if bias is None else bias.to(device=x.device, dtype=torch.float32).contiguous()
        valid = _as_valid(valid_mask, n, x.device)
        idx = torch.empty(n, comm.topk, dtype=torch.int64, device=x.device)
        gate = torch.empty(n, comm.topk, dtype=comm.dtype, device=x.device)
        h_out = torch.empty_like(hh)
        w_in, w_out = self.w_in.contiguous(), self.w_out.contiguous()
        check(_lib.lib().mep_moe_block(comm._ctx, self.layer, ptr(hh), ptr(x), ptr(rw), ptr(b),
                                       ptr(valid), n, ptr(w_in), ptr(w_out), n_local,
                                       float(residual_multiplier), ptr(h_out), ptr(idx),
                                       ptr(gate), _stream()), comm._ctx, "mep_moe_block")
        return h_out.view_as(h), idx, gate

    def moe_block_from_h(self, h, norm_w, eps: float, router_w, residual_multiplier: float,
                         bias=None, valid_mask=None):
        """The MoE half of ``Block.forward`` from the residual stream alone
        (miniep/modeling.py:192-197): post-attention RMSNorm, router, this
        backend, residual, in one call. Returns (h_out, topk_idx, topk_gate, x)."""
        comm = self.comm
        n = h.reshape(-1, comm.hidden).shape[0]
        hh = h.reshape(n, -1).contiguous()
        n_local = self._prepare(hh)
        nw = norm_w.to(device=hh.device, dtype=comm.dtype).contiguous()
        rw = router_w.to(comm.dtype).contiguous()
        b = None if bias is None else bias.to(device=hh.device, dtype=torch.float32).contiguous()
        valid = _as_valid(valid_mask, n, hh.device)
        x = torch.empty_like(hh)
        idx = torch.empty(n, comm.topk, dtype=torch.int64, device=hh.device)
        gate = torch.empty(n, comm.topk, dtype=comm.dtype, device=hh.device)
        h_out = torch.empty_like(hh)
        w_in, w_out = self.w_in.contiguous(), self.w_out.contiguous()
        check(_lib.lib().mep_moe_block_from_h(
            comm._ctx, self.layer, ptr(hh), ptr(nw), float(eps), ptr(rw), ptr(b), ptr(valid), n,
            ptr(w_in), ptr(w_out), n_local, float(residual_multiplier), ptr(h_out), ptr(x),
            ptr(idx), ptr(gate), _stream()), comm._ctx, "mep_moe_block_from_h")
        return h_out.view_as(h), idx, gate, x


def _captured_state(backend: "EPMoEBackend") -> tuple:
    """What a captured layer step bakes into its CUDA graph from the backend:
    the expert weight addresses, the resident-expert list and the placement
    object (the tables the graph's kernels read are uploaded per placement)."""
    return (backend.w_in.data_ptr(), backend.w_out.data_ptr(), tuple(backend.local_experts),
            id(backend.placement))


def _check_replay(backend: "EPMoEBackend", captured: tuple):
    """Refuse to replay a graph whose backend changed since capture (a
    re-placement swaps the weight tensors, the expert list and the tables;
    the graph would read freed weights with a stale expert count)."""
    if _captured_state(backend) != captured:
        raise MEPError(f"layer {backend.layer}: the backend's placement or expert weights "
                       "changed since this graphed block was captured (a re-placement); "
                       "build a new GraphedMoEBlock / StreamedMoEBlock")


class GraphedMoEBlock:
    """The MoE half of ``Block.forward`` (router + expert-parallel layer +
    residual, miniep/modeling.py:192-197) for a fixed token count, captured once
    into a CUDA graph over static device buffers and replayed per step: one
    launch per layer step instead of seven to nine, no host work in between.

    The step's sequence number lives on the device, so replays stay in lockstep
    with the other ranks exactly like eager calls. Every rank must construct
    its GraphedMoEBlock at the same point (construction runs one warm-up step)
    and then replay the same number of times.
    """

    def __init__(self, backend: "EPMoEBackend", n_tokens: int, router_w,
                 residual_multiplier: float, bias=None, norm_w=None, eps: float = 1e-6):
        comm = backend.comm
        self.backend, self.n = backend, n_tokens
        dev = backend.w_in.device
        H, k = comm.hidden, comm.topk
        self.x = torch.zeros(n_tokens, H, dtype=comm.dtype, device=dev)
        self.h = torch.zeros(n_tokens, H, dtype=comm.dtype, device=dev)
        self.h_out = torch.empty_like(self.h)
        self.idx = torch.empty(n_tokens, k, dtype=torch.int64, device=dev)
        self.gate = torch.empty(n_tokens, k, dtype=comm.dtype, device=dev)
        self.router_w = router_w.to(comm.dtype).contiguous()
        self.bias = None if bias is None else bias.to(device=dev, dtype=torch.float32).contiguous()
        self.rm = float(residual_multiplier)
        # with the post-attention norm weight the block starts from h alone:
        # x is computed on the device (modeling.py:192)
        self.norm_w = None if norm_w is None else \
            norm_w.to(device=dev, dtype=comm.dtype).contiguous()
        self.eps = float(eps)
        self.n_local = backend._prepare(self.x)
        self._step()  # warm-up outside capture (resolves driver entry points, kernel attributes)
        torch.cuda.current_stream().synchronize()
        comm.check()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self.captured = _captured_state(backend)

    def _step(self):
        be, comm = self.backend, self.backend.comm
        L, ctx, st, n = _lib.lib(), comm._ctx, _stream(), self.n
        if self.norm_w is not None:
            check(L.mep_rmsnorm(ctx, ptr(self.h), ptr(self.norm_w), self.eps, n, ptr(self.x), st),
                  ctx, "mep_rmsnorm")
        check(L.mep_router_topk(ctx, ptr(self.x), ptr(self.router_w), ptr(self.bias), n,
                                ptr(self.idx), ptr(self.gate), None, st), ctx, "mep_router_topk")
        check(L.mep_route(ctx, be.layer, ptr(self.idx), None, n, self.n_local, st), ctx, "mep_route")
        check(L.mep_dispatch(ctx, ptr(self.x), ptr(self.idx), n, st), ctx, "mep_dispatch")
        check(L.mep_expert_ffn(ctx, ptr(be.w_in), ptr(be.w_out), self.n_local, st), ctx,
              "mep_expert_ffn")
        check(L.mep_combine(ctx, ptr(self.gate), None, n, ptr(self.h), self.rm, None,
                            ptr(self.h_out), st), ctx, "mep_combine")

    def __call__(self, x=None, h=None):
        """Copy x / h (device or pinned host tensors) into the static inputs
        when given, replay the step, return the static output h + moe(x) * rm.
        With the norm weight the step computes x from h; pass h only."""
        if x is not None and self.norm_w is not None:
            raise ValueError("this block computes x from h (norm_w given): pass h only")
        if x is not None:
            self.x.copy_(x, non_blocking=True)
        if h is not None:
            self.h.copy_(h, non_blocking=True)
        _check_replay(self.backend, self.captured)
        self.graph.replay()
        return self.h_out


class StreamedMoEBlock:
    """``GraphedMoEBlock`` for token batches that live in (pinned) host memory.

    Each call copies the batch from the host, runs the captured layer step and
    copies the result back. The host-to-device copies run on one stream, the
    steps on the caller's stream and the device-to-host copies on a third, so
    the two copy directions (which PCIe carries at the same time) overlap each
    other and the steps:

    * ``depth`` sets of device buffers (each with its own captured step) are
      used round-robin by consecutive calls, so call j+1's input copy and call
      j-1's output copy run while call j's step computes (default 2);
    * ``chunks`` cuts each batch into pieces with their own captured steps, so
      that the pieces of one call overlap each other too (each piece is one
      layer call of the reference's contract: routing, replica round-robin and
      stats advance per piece exactly as for consecutive eager calls, and
      every output row is bit-identical to the unchunked step's).

    ``__call__(..., wait_output=True)`` makes the caller's stream wait for
    this call's output copy (``out_host`` is complete once the stream reaches
    that point). With ``wait_output=False`` it does not: the next call's step
    can then overlap this call's output copy, and the caller must wait on
    ``self.done`` (the last call's output copy) before reading ``out_host`` or
    changing ``h_host`` / ``x_host``. Every rank must use the same ``chunks``
    and ``depth`` and call in lockstep. ``capture`` records one call's whole
    pipeline for fixed pinned buffers into one CUDA graph (consecutive calls
    then no longer overlap each other, only the pieces of one call do).
    """

    class _Set:
        def __init__(self, blocks):
            self.blocks = blocks
            ev = lambda: [torch.cuda.Event() for _ in blocks]  # noqa: E731
            self.loaded, self.stepped, self.inputs_free, self.output_free = ev(), ev(), ev(), ev()

    def __init__(self, backend: "EPMoEBackend", n_tokens: int, router_w,
                 residual_multiplier: float, bias=None, chunks: int = 1, norm_w=None,
                 eps: float = 1e-6, depth: int = 2):
        if n_tokens < 1 or chunks < 1 or depth < 1:
            raise ValueError("StreamedMoEBlock: n_tokens, chunks and depth must be positive")
        chunks = min(chunks, n_tokens)
        base, extra = divmod(n_tokens, chunks)
        self.sizes = [base + (1 if i < extra else 0) for i in range(chunks)]
        self.n = n_tokens
        self.from_h = norm_w is not None
        self.sets = [self._Set([GraphedMoEBlock(backend, m, router_w, residual_multiplier,
                                                bias=bias, norm_w=norm_w, eps=eps)
                                for m in self.sizes])
                     for _ in range(depth)]
        self.blocks = self.sets[0].blocks
        self.copy_in = torch.cuda.Stream()
        self.copy_out = torch.cuda.Stream()
        self.done = torch.cuda.Event()
        self.calls = 0

    def _check(self, x_host, h_host, out_host):
        if (x_host is None) != self.from_h:
            raise ValueError("StreamedMoEBlock: pass x_host exactly when the block has no norm_w")
        if (x_host is not None and x_host.shape[0] != self.n) or h_host.shape[0] != self.n or \
                out_host.shape[0] != self.n:
            raise ValueError(f"StreamedMoEBlock: expected {self.n} tokens")

    def _enqueue(self, st, x_host, h_host, out_host, capturing: bool, wait_output: bool):
        cur = torch.cuda.current_stream()
        if capturing:  # the side streams join the capture
            self.copy_in.wait_stream(cur)
            self.copy_out.wait_stream(cur)
        off = 0
        for i, (blk, m) in enumerate(zip(st.blocks, self.sizes)):
            rows = slice(off, off + m)
            off += m
            with torch.cuda.stream(self.copy_in):
                if not capturing:
                    self.copy_in.wait_event(st.inputs_free[i])  # this set's last step read blk.x / blk.h
                if x_host is not None:
                    blk.x.copy_(x_host[rows], non_blocking=True)
                blk.h.copy_(h_host[rows], non_blocking=True)
                st.loaded[i].record(self.copy_in)
            cur.wait_event(st.loaded[i])
            if capturing:
                blk._step()
            else:
                cur.wait_event(st.output_free[i])  # this set's last copy-out of blk.h_out is done
                _check_replay(blk.backend, blk.captured)
                blk.graph.replay()
                st.inputs_free[i].record(cur)
            st.stepped[i].record(cur)
            with torch.cuda.stream(self.copy_out):
                self.copy_out.wait_event(st.stepped[i])
                out_host[rows].copy_(blk.h_out, non_blocking=True)
                if not capturing:
                    st.output_free[i].record(self.copy_out)
        if capturing:
            cur.wait_stream(self.copy_in)
            cur.wait_stream(self.copy_out)
            return
        self.done.record(self.copy_out)
        if wait_output:
            cur.wait_stream(self.copy_out)

    def capture(self, x_host, h_host, out_host):
        """Record the whole per-call pipeline (copies in, the pieces' layer
        steps, copies out, and their cross-stream order) into one CUDA graph
        for these pinned host buffers; later calls with the same buffers
        replay it: one launch per call instead of a few dozen. Every rank
        captures at the same point."""
        self._check(x_host, h_host, out_host)
        self(x_host, h_host, out_host)  # one eager call first
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._enqueue(self.sets[0], x_host, h_host, out_host, capturing=True,
                          wait_output=True)
        self.graph = g
        self.bound = (None if x_host is None else x_host.data_ptr(), h_host.data_ptr(),
                      out_host.data_ptr())

    def __call__(self, x_host, h_host, out_host, wait_output: bool = True):
        """Enqueue ``out_host = h_host + moe(x_host) * rm`` (see the class
        notes for ``wait_output``). The host tensors must be pinned for the
        copies to overlap."""
        self._check(x_host, h_host, out_host)
        if getattr(self, "graph", None) is not None and self.bound == (
                None if x_host is None else x_host.data_ptr(), h_host.data_ptr(),
                out_host.data_ptr()):
            for blk in self.sets[0].blocks:
                _check_replay(blk.backend, blk.captured)
            self.graph.replay()
            return out_host
        st = self.sets[self.calls % len(self.sets)]
        self.calls += 1
        self._enqueue(st, x_host, h_host, out_host, capturing=False, wait_output=wait_output)
        return out_host


def rms_norm(comm: Comm, h, weight, eps: float):
    """Post-attention RMSNorm on the device (miniep/modeling.py:51-52) with the
    reference's rounding points in the model dtype."""
    hh = h.reshape(-1, comm.hidden).contiguous()
    w = weight.to(device=hh.device, dtype=comm.dtype).contiguous()
    x = torch.empty_like(hh)
    check(_lib.lib().mep_rmsnorm(comm._ctx, ptr(hh), ptr(w), float(eps), hh.shape[0], ptr(x),
                                 _stream()), comm._ctx, "mep_rmsnorm")
    return x.view_as(h)


def router_topk(comm: Comm, x_flat, router_w, bias=None, return_logits: bool = False):
    """Router of ``Block.forward`` (miniep/modeling.py:193-195) on the device:
    (topk_idx int64, topk_gate model dtype[, logits fp32])."""
    n = x_flat.shape[0]
    x = x_flat.contiguous()
    rw = router_w.to(comm.dtype).contiguous()
    b = None if bias is None else bias.to(device=x.device, dtype=torch.float32).contiguous()
    idx = torch.empty(n, comm.topk, dtype=torch.int64, device=x.device)
    gate = torch.empty(n, comm.topk, dtype=comm.dtype, device=x.device)
    logits = torch.empty(n, comm.num_experts, dtype=torch.float32, device=x.device) \
        if return_logits else None
    check(_lib.lib().mep_router_topk(comm._ctx, ptr(x), ptr(rw), ptr(b), n, ptr(idx), ptr(gate),
                                     ptr(logits), _stream()), comm._ctx, "mep_router_topk")
    return (idx, gate, logits) if return_logits else (idx, gate)


class LocalMoEBackend(EPMoEBackend):
    """All experts on this GPU (the reference's LocalMoEBackend,
    miniep/modeling.py:131-145): a one-rank expert-parallel step."""

    def __init__(self, w_in, w_out, max_tokens: int, topk: int, stats: EPStats | None = None):
        num_experts, two_i, hidden = w_in.shape
        comm = Comm(num_layers=1, num_experts=num_experts, topk=topk, hidden=hidden,
                    inter=two_i // 2, max_tokens=max_tokens, dtype=w_in.dtype,
                    device=w_in.device.index, single_process=True)
        placement = Placement.naive(1, num_experts, 1)
        comm.install(placement)
        super().__init__(0, comm, placement, list(range(num_experts)), w_in, w_out, stats)
