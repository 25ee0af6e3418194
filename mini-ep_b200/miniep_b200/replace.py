"""Live re-placement of experts: the reference's /rebalance path
(miniep/server.py:166-183, apply_placement :49-61), with the expert weights
moved between ranks instead of re-read from the checkpoint.

The reference all-reduces the source-side route counts, plans on rank 0,
broadcasts the plan and has every rank load the weights of the experts it now
owns from disk. Here every rank already holds the weights of its old experts,
so each newly owned expert is sent by one of its old owners (P2P over NCCL on
GPUs, NVLink inside a box; over gloo the tensors are staged through host
memory). Every rank derives the same transfer schedule from the old and new
placements, so the sends and receives pair up without any extra exchange.
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from .balancer import plan_balanced
from .ep import EPMoEBackend, EPStats, Placement


def global_route_counts(stats: EPStats, group=None) -> torch.Tensor:
    """(L, E) entries routed to each expert, summed over ranks
    (server.py:168-169: source-side counts all-reduced)."""
    counts = stats.route_counts.clone().to(torch.int64)
    if dist.is_available() and dist.is_initialized():
        dev = torch.device("cuda", torch.cuda.current_device()) \
            if dist.get_backend(group) == "nccl" else torch.device("cpu")
        buf = counts.to(dev)
        dist.all_reduce(buf, group=group)
        counts = buf.cpu()
    return counts


def transfer_schedule(old: Placement, new: Placement, world: int) -> list[tuple[int, int, int, int]]:
    """(layer, expert, src, dst) for every expert a rank owns under `new` but
    did not own under `old`. The sender is one of the expert's old owners,
    chosen by the receiving rank (old_owners[dst % n]) so that a hot expert's
    new replicas are fed by different old owners."""
    if old.num_layers != new.num_layers or old.num_experts != new.num_experts:
        raise ValueError("placements of different shapes")
    old_mine = [old.experts_of_rank(r) for r in range(world)]
    new_mine = [new.experts_of_rank(r) for r in range(world)]
    out = []
    for layer in range(new.num_layers):
        for dst in range(world):
            have = set(old_mine[dst][layer])
            for e in new_mine[dst][layer]:
                if e in have:
                    continue
                owners = sorted(old.owners[layer][e])
                out.append((layer, e, owners[dst % len(owners)], dst))
    return out


def apply_placement(backends: list[EPMoEBackend], new: Placement, group=None) -> dict:
    """Swap every layer's backend to `new` in place: keep the weights of the
    experts this rank still owns, receive the newly owned ones from their old
    owners, drop the rest, then upload the new tables and reset the
    round-robin state (a fresh placement, as the reference's apply_placement
    makes)."""
    if not backends:
        return {"moved_experts": 0, "bytes_received": 0}
    comm = backends[0].comm
    rank, world = comm.rank, comm.world
    old = backends[0].placement
    sched = transfer_schedule(old, new, world)
    gloo = dist.is_available() and dist.is_initialized() and dist.get_backend(group) == "gloo"
    new_w, ops, staged = [], [], []
    received = 0

    def wire(t: torch.Tensor) -> torch.Tensor:
        # gloo moves host tensors only
        return t.cpu().contiguous() if gloo and t.is_cuda else t.contiguous()

    for layer, be in enumerate(backends):
        old_mine = list(be.local_experts)
        mine = new.experts_of_rank(rank)[layer]
        w_in = be.w_in.new_empty((len(mine),) + tuple(be.w_in.shape[1:]))
        w_out = be.w_out.new_empty((len(mine),) + tuple(be.w_out.shape[1:]))
        for j, e in enumerate(mine):
            if e in old_mine:
                i = old_mine.index(e)
                w_in[j].copy_(be.w_in[i])
                w_out[j].copy_(be.w_out[i])
        for (l, e, src, dst) in sched:
            if l != layer or src == dst:
                continue
            if src == rank:
                i = old_mine.index(e)
                for t in (be.w_in[i], be.w_out[i]):
                    ops.append(dist.P2POp(dist.isend, wire(t), dst, group=group))
            if dst == rank:
                j = mine.index(e)
                for t in (w_in[j], w_out[j]):
                    buf = torch.empty(t.shape, dtype=t.dtype) if gloo and t.is_cuda else t
                    ops.append(dist.P2POp(dist.irecv, buf, src, group=group))
                    if buf is not t:
                        staged.append((buf, t))
                    received += t.numel() * t.element_size()
        new_w.append((mine, w_in, w_out))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    for buf, t in staged:
        t.copy_(buf)
    for be, (mine, w_in, w_out) in zip(backends, new_w):
        be.placement = new
        be.w_in, be.w_out = w_in, w_out
        be._update_map(mine)
    comm.install(new)
    new.reset_rr()
    moved = sum(1 for s in sched if s[2] != s[3])
    return {"moved_experts": moved, "bytes_received": received}


def rebalance(backends: list[EPMoEBackend], stats: EPStats, slots_per_rank: int = 2,
              group=None) -> dict:
    """The reference's /rebalance on the live engine: global counts ->
    plan_balanced -> rank 0's plan to every rank -> apply. Every rank calls it.
    Returns the reference's payload (replicas added, predicted imbalance
    before/after, apply seconds) plus what moved."""
    comm = backends[0].comm
    counts = global_route_counts(stats, group)
    placement, report = plan_balanced(counts, comm.world, slots_per_rank=slots_per_rank)
    plan = placement.to_plan()
    if dist.is_available() and dist.is_initialized():
        box = [plan if comm.rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        plan = box[0]
    t0 = time.perf_counter()
    moved = apply_placement(backends, Placement.from_plan(plan), group)
    ib = [l["imbalance_before"] for l in report["layers"]]
    ia = [l["imbalance_after"] for l in report["layers"]]
    return {
        "replicas_added": report["replicas_total"],
        "predicted_imbalance_before_avg": round(sum(ib) / len(ib), 3),
        "predicted_imbalance_after_avg": round(sum(ia) / len(ia), 3),
        "apply_seconds": round(time.perf_counter() - t0, 2),
        "plan": plan,
        **moved,
    }
