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
