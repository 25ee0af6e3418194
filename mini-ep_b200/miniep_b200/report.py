"""Bench reports in the reference's results/bench_*.json layout.

The reference's bench mode gathers one payload per rank -- its rank, the
positions it processed and ``EPStats.snapshot()`` -- on rank 0 and writes
(miniep/worker.py:232-257)::

    {"world", "plan", "iters", "decode_steps", "wall_time", "iter_times",
     "positions_per_s", "total_positions", "ranks": [{"rank", "positions",
     "stats"}, ...]}

then prints the per-rank load summary (worker.py:258-267). The reference's
scripts/make_charts.py reads ``ranks[r]["stats"]["recv_tokens_per_layer"]``
and scripts/make_plan.py reads ``route_counts``, so a report written here
feeds them unchanged. For a layer bench, "positions" are the tokens a rank
pushed through the layer.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from .balancer import layer_imbalance, straggler_overhead

BENCH_KEYS = ("world", "plan", "iters", "decode_steps", "wall_time", "iter_times",
              "positions_per_s", "total_positions", "ranks")
RANK_KEYS = ("rank", "positions", "stats")


def rank_payload(rank: int, positions: int, snapshot: dict) -> dict:
    """One rank's entry (worker.py:232-236)."""
    return {"rank": int(rank), "positions": int(positions), "stats": dict(snapshot)}


def gather_payloads(payload: dict, group=None) -> list[dict] | None:
    """All ranks' payloads on rank 0 (``dist.gather_object``, as
    worker.py:237-238); None on the other ranks. Every rank must call it."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return [payload]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    out = [None] * world if rank == 0 else None
    dist.gather_object(payload, out, dst=0, group=group)
    return out


def bench_report(payloads: list[dict], plan: str | None, iters: int, wall_time: float,
                 iter_times: list[float], decode_steps: int = 0) -> dict:
    """The bench JSON of worker.py:244-257 from the gathered payloads."""
    ranks = sorted(payloads, key=lambda p: p["rank"])
    total = sum(p["positions"] for p in ranks)
    return {
        "world": len(ranks),
        "plan": plan or "naive",
        "iters": int(iters),
        "decode_steps": int(decode_steps),
        "wall_time": float(wall_time),
        "iter_times": [float(t) for t in iter_times],
        "positions_per_s": total / wall_time if wall_time > 0 else 0.0,
        "total_positions": total,
        "ranks": ranks,
    }


def load_summary(report: dict) -> dict:
    """Straggler overhead (sum_l max_r / sum_l mean_r - 1) and per-layer
    max/mean imbalance of the received entries, the figures the reference's
    README quotes for its bench files."""
    loads = [r["stats"]["recv_tokens_per_layer"] for r in report["ranks"]]  # (W, L)
    per_layer = layer_imbalance(loads)
    return {"straggler": straggler_overhead(loads),
            "imbalance_avg": sum(per_layer) / len(per_layer),
            "imbalance_worst": max(per_layer),
            "per_layer_imbalance": per_layer}


def summary_lines(report: dict) -> list[str]:
    """The per-rank summary the reference prints after a bench (worker.py:258-267)."""
    loads = [r["stats"]["recv_tokens"] for r in report["ranks"]]
    comp = [r["stats"]["compute_time"] for r in report["ranks"]]
    a2a = [r["stats"]["a2a_time"] for r in report["ranks"]]
    mean_load = sum(loads) / len(loads) if loads else 0.0
    imb = max(loads) / mean_load if mean_load else 1.0
    return [f"wall {report['wall_time']:.1f}s  positions/s {report['positions_per_s']:.1f}",
            f"per-rank expert entries: {loads}  imbalance max/mean: {imb:.2f}",
            f"per-rank compute_time: {[round(c, 1) for c in comp]}",
            f"per-rank a2a(+wait)  : {[round(a, 1) for a in a2a]}"]


def write_bench_report(path, report: dict) -> Path:
    """Write the report as the reference does (json, indent=1)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(report, indent=1))
    return path


def expert_counts(report: dict) -> torch.Tensor:
    """(L, E) routed entries summed over ranks, the counts make_plan.py feeds
    to the balancer."""
    rc = [torch.tensor(r["stats"]["route_counts"], dtype=torch.long) for r in report["ranks"]]
    return torch.stack(rc).sum(dim=0)
