"""Host-side logic that needs no GPU: placement objects and plan JSON, the
replication planner against the reference's known answers, straggler and
imbalance figures against the reference's published results."""
import json

import pytest

from miniep_b200 import Placement, layer_imbalance, plan_balanced, straggler_overhead
from oracle import moe_oracle as O


def test_placement_naive_and_plan_roundtrip():
    p = Placement.naive(3, 8, 4)
    assert p.owners[1][5] == [2]
    assert p.experts_of_rank(3) == {0: [6, 7], 1: [6, 7], 2: [6, 7]}
    q = Placement.from_plan(json.loads(json.dumps(p.to_plan())))
    assert q.owners == p.owners
    table, n_rep = q.table(0)
    assert table.shape == (8, 1) and n_rep.tolist() == [1] * 8
    assert O.naive_owners(3, 8, 4) == p.owners


def test_placement_from_plan_sorts_and_validates():
    plan = {"owners": {"0": {"0": [2, 0], "1": [1], "2": [1], "3": [2]}}}
    p = Placement.from_plan(plan)
    assert p.owners[0][0] == [0, 2]
    table, n_rep = p.table(0)
    assert table.tolist()[0] == [0, 2] and n_rep.tolist() == [2, 1, 1, 1]
    assert p.experts_of_rank(0) == {0: [0]}
    assert p.experts_of_rank(2) == {0: [0, 3]}
    with pytest.raises(ValueError):
        Placement([[[0, 0], [1]]])
    with pytest.raises(ValueError):
        Placement([[[]]])
    with pytest.raises(ValueError):
        Placement.naive(1, 6, 4)


def test_unbound_placement_has_no_cpu_path():
    from miniep_b200 import MEPError
    import torch
    p = Placement.naive(1, 4, 1)
    with pytest.raises(MEPError):
        p.dest_ranks(0, torch.tensor([0, 1]))


def test_planner_reproduces_reference_plans(golden):
    cases = json.loads((golden / "balancer.json").read_text())
    assert cases[0]["name"] == "shipped_bench_naive"
    for case in cases:
        placement, report = plan_balanced(case["counts"], case["world"],
                                          slots_per_rank=case["slots"])
        assert placement.to_plan() == case["plan"], case["name"]
        assert report["replicas_total"] == case["report"]["replicas_total"]
        for got, want in zip(report["layers"], case["report"]["layers"]):
            assert got["replicas"] == want["replicas"]
            assert got["imbalance_before"] == pytest.approx(want["imbalance_before"], rel=1e-12)
            assert got["imbalance_after"] == pytest.approx(want["imbalance_after"], rel=1e-12)
    assert cases[0]["report"]["replicas_total"] == 71


def test_straggler_figures_match_published_results(golden):
    s = json.loads((golden / "stats_schema.json").read_text())
    for name, published in (("naive", 0.266), ("balanced", 0.041)):
        loads = s[name]["recv_tokens_per_layer"]
        assert straggler_overhead(loads) == pytest.approx(s[name]["straggler"], rel=1e-12)
        assert round(straggler_overhead(loads), 3) == published
        imb = layer_imbalance(loads)
        assert sum(imb) / len(imb) == pytest.approx(s[name]["imbalance_avg"], rel=1e-12)
        assert max(imb) == pytest.approx(s[name]["imbalance_worst"], rel=1e-12)
        assert s[name]["snapshot_keys"] == sorted(
            ["recv_tokens", "recv_tokens_per_layer", "compute_time", "a2a_time",
             "route_counts", "steps"])
    assert s["route_counts_placement_invariant"]
