"""Hot-expert replication planner (host side).

Same contract and the same greedy steps as the reference planner
(miniep/balancer.py:17-89), so a plan made here is byte-identical to the
reference's for the same counts: start from the naive contiguous placement;
while the busiest rank of a layer carries more than ``target_ratio`` x the
mean load, add the single (expert, rank) replica that lowers the layer's
maximum rank load the most, subject to ``slots_per_rank`` extra copies per
rank. A replicated expert's load is split evenly over its copies (the
dispatch round-robins over them). Candidates are scanned expert-major,
rank-minor and only a strictly better maximum replaces the current best, and
rank loads are summed in expert order, so ties resolve exactly as the
reference resolves them.

The planner is milliseconds of host work per plan and runs off the hot path;
it is not a GPU kernel.
"""
from __future__ import annotations

from .ep import Placement


def rank_loads(loads: list[float], owners: list[list[int]], world: int) -> list[float]:
    """Load per rank when each expert's load is split evenly over its owners."""
    acc = [0.0] * world
    for load, own in zip(loads, owners):
        share = load / len(own)
        for r in own:
            acc[r] += share
    return acc


def _best_addition(loads, owners, world, budget):
    peak = max(rank_loads(loads, owners, world))
    best = None
    for e, own in enumerate(owners):
        if loads[e] / len(own) == 0:
            continue
        for r in range(world):
            if r in own or budget[r] <= 0:
                continue
            trial = list(owners)
            trial[e] = sorted(own + [r])
            m = max(rank_loads(loads, trial, world))
            if m < peak and (best is None or m < best[0]):
                best = (m, e, r)
    return best


def plan_layer(loads: list[float], world: int, slots_per_rank: int, target_ratio: float):
    """Owner lists for one layer plus the rank loads before and after."""
    per = len(loads) // world
    owners = [[e // per] for e in range(len(loads))]
    budget = [slots_per_rank] * world
    before = rank_loads(loads, owners, world)
    mean = sum(before) / world
    while mean and max(rank_loads(loads, owners, world)) / mean > target_ratio:
        best = _best_addition(loads, owners, world, budget)
        if best is None:
            break
        _, e, r = best
        owners[e] = sorted(owners[e] + [r])
        budget[r] -= 1
    return owners, before, rank_loads(loads, owners, world)


def plan_balanced(counts, world: int, slots_per_rank: int = 2, target_ratio: float = 1.05):
    """counts: (num_layers, num_experts) global routing counts (tensor or nested list).

    Returns (Placement, report) with report = {"layers": [{layer,
    imbalance_before, imbalance_after, replicas}], "replicas_total"}.
    """
    rows = counts.tolist() if hasattr(counts, "tolist") else counts
    num_experts = len(rows[0])
    all_owners = []
    report = {"layers": [], "replicas_total": 0}
    for layer, row in enumerate(rows):
        loads = [float(v) for v in row]
        owners, before, after = plan_layer(loads, world, slots_per_rank, target_ratio)
        mean = sum(before) / world
        replicas = sum(len(o) for o in owners) - num_experts
        report["replicas_total"] += replicas
        report["layers"].append({
            "layer": layer,
            "imbalance_before": max(before) / mean if mean else 1.0,
            "imbalance_after": max(after) / mean if mean else 1.0,
            "replicas": replicas,
        })
        all_owners.append(owners)
    return Placement(all_owners), report


def _lpt_layer(loads: list[float], nrep: list[int], world: int, cap: int):
    """Longest-processing-time-first placement of the expert copies: expert e
    is cut into nrep[e] equal pieces (its round-robin shares), pieces are
    taken largest first (ties: lower expert id) and each goes to the least
    loaded rank (ties: fewer experts, then lower rank) that has a free slot
    and no copy of e yet. None when some piece finds no rank."""
    pieces = sorted(((loads[e] / nrep[e], e) for e in range(len(loads)) for _ in range(nrep[e])),
                    key=lambda p: (-p[0], p[1]))
    acc, used = [0.0] * world, [0] * world
    owners = [[] for _ in loads]
    for share, e in pieces:
        cands = [r for r in range(world) if used[r] < cap and r not in owners[e]]
        if not cands:
            return None
        r = min(cands, key=lambda r: (acc[r], used[r], r))
        acc[r] += share
        used[r] += 1
        owners[e].append(r)
    return [sorted(o) for o in owners], acc


def plan_lpt(counts, world: int, slots_per_rank: int = 2, target_ratio: float = 1.05):
    """A load-aware placement in the same plan format, for skews that the
    replica-only planner above cannot balance.

    ``plan_balanced`` keeps every expert on its naive rank and only adds
    copies, so a rank whose own experts are all hot stays hot: under the
    Zipf(1.2) router of the layer benchmarks its plan stops at 1.17x the mean
    load at 4 ranks and 1.24x at 8 (no slot budget gets 8 ranks below 1.14x).
    This planner instead re-places the experts themselves: every rank holds
    at most E / world + ``slots_per_rank`` expert copies (the same memory
    budget), the copies are placed longest-first onto the least loaded rank
    (``_lpt_layer``), and while the busiest rank exceeds ``target_ratio`` x
    the mean and slots remain, the expert with the largest per-copy load gets
    one more copy. The best placement seen is kept. Deterministic: the same
    counts give the same plan on every rank. Moving to such a plan moves
    experts between ranks (``replace.apply_placement`` does that for a live
    model). Returns (Placement, report) like ``plan_balanced``.
    """
    rows = counts.tolist() if hasattr(counts, "tolist") else counts
    num_experts = len(rows[0])
    if num_experts % world:
        raise ValueError("num_experts must be divisible by world")
    cap = num_experts // world + slots_per_rank
    all_owners = []
    report = {"layers": [], "replicas_total": 0}
    for layer, row in enumerate(rows):
        loads = [float(v) for v in row]
        naive = [[e // (num_experts // world)] for e in range(num_experts)]
        before = rank_loads(loads, naive, world)
        mean = sum(loads) / world
        nrep = [1] * num_experts
        best = None
        while True:
            got = _lpt_layer(loads, nrep, world, cap)
            if got is None:
                break
            owners, acc = got
            if best is None or max(acc) < max(best[1]):
                best = (owners, acc)
            if not mean or max(acc) / mean <= target_ratio or sum(nrep) >= world * cap:
                break
            grow = [e for e in range(num_experts) if nrep[e] < world and loads[e] > 0]
            if not grow:
                break
            e = max(grow, key=lambda e: (loads[e] / nrep[e], -e))
            nrep[e] += 1
        owners, after = best
        replicas = sum(len(o) for o in owners) - num_experts
        report["replicas_total"] += replicas
        report["layers"].append({
            "layer": layer,
            "imbalance_before": max(before) / mean if mean else 1.0,
            "imbalance_after": max(after) / mean if mean else 1.0,
            "replicas": replicas,
        })
        all_owners.append(owners)
    return Placement(all_owners), report


def straggler_overhead(recv_tokens_per_layer) -> float:
    """sum_l max_r load / sum_l mean_r load - 1, over per-rank per-layer entry
    counts (W x L); the load-based straggler figure of the reference's results."""
    per_rank = [list(map(float, r)) for r in recv_tokens_per_layer]
    layers = len(per_rank[0])
    world = len(per_rank)
    mx = sum(max(per_rank[r][l] for r in range(world)) for l in range(layers))
    mean = sum(sum(per_rank[r][l] for r in range(world)) / world for l in range(layers))
    return mx / mean - 1.0 if mean else 0.0


def layer_imbalance(recv_tokens_per_layer) -> list[float]:
    """max/mean rank load per layer (1.0 for an empty layer)."""
    per_rank = [list(map(float, r)) for r in recv_tokens_per_layer]
    world = len(per_rank)
    out = []
    for l in range(len(per_rank[0])):
        col = [per_rank[r][l] for r in range(world)]
        mean = sum(col) / world
        out.append(max(col) / mean if mean else 1.0)
    return out
