"""Bench reports in the reference's results/bench_*.json layout
(miniep/worker.py:232-267), checked against the key sets, loads and derived
figures recorded from the reference's shipped bench files
(tests/golden/stats_schema.json), and gathered over real gloo ranks."""
import json
import os
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

from miniep_b200 import EPStats, report

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def schema():
    return json.loads((REPO / "tests/golden/stats_schema.json").read_text())


def _payloads(case):
    out = []
    for r, (per_layer, total, pos) in enumerate(zip(case["recv_tokens_per_layer"],
                                                    case["recv_tokens"], case["positions"])):
        snap = {"recv_tokens": total, "recv_tokens_per_layer": per_layer, "compute_time": 1.0 + r,
                "a2a_time": 0.5, "route_counts": [[r] * 32] * len(per_layer), "steps": 3}
        out.append(report.rank_payload(r, pos, snap))
    return out


@pytest.mark.parametrize("name", ["naive", "balanced"])
def test_report_layout_and_figures_match_reference_files(schema, name):
    case = schema[name]
    payloads = _payloads(case)
    rep = report.bench_report(payloads[::-1], plan=name, iters=3, wall_time=case["wall_time"],
                              iter_times=[1.0, 2.0, 3.0], decode_steps=16)
    assert list(rep.keys()) == case["bench_keys"] == list(report.BENCH_KEYS)
    assert [list(r.keys()) for r in rep["ranks"]] == [case["rank_keys"]] * case["world"]
    assert [r["rank"] for r in rep["ranks"]] == list(range(case["world"]))
    assert sorted(rep["ranks"][0]["stats"].keys()) == case["snapshot_keys"]
    assert rep["world"] == case["world"]
    assert rep["positions_per_s"] == pytest.approx(case["positions_per_s"], rel=1e-12)
    s = report.load_summary(rep)
    assert s["straggler"] == pytest.approx(case["straggler"], rel=1e-12)
    assert s["imbalance_avg"] == pytest.approx(case["imbalance_avg"], rel=1e-12)
    assert s["imbalance_worst"] == pytest.approx(case["imbalance_worst"], rel=1e-12)
    lines = report.summary_lines(rep)
    assert lines[1].startswith(f"per-rank expert entries: {case['recv_tokens']}")
    # make_plan.py's input: route counts summed over ranks
    assert report.expert_counts(rep).tolist()[0] == [sum(range(case["world"]))] * 32


def test_report_round_trips_through_json(tmp_path, schema):
    rep = report.bench_report(_payloads(schema["balanced"]), plan="plan.json", iters=1,
                              wall_time=2.0, iter_times=[2.0])
    path = report.write_bench_report(tmp_path / "out" / "bench.json", rep)
    assert json.loads(path.read_text()) == rep


def test_epstats_snapshot_has_the_reference_keys(schema):
    snap = EPStats(3, 32).snapshot()  # no device counters bound: zeros
    assert sorted(snap.keys()) == schema["naive"]["snapshot_keys"]
    assert snap["recv_tokens_per_layer"] == [0, 0, 0]


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(REPO / "mini-ep_b200"), str(REPO)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from miniep_b200 import report as rp
    dist.init_process_group("gloo", rank=rank, world_size=world)
    snap = {"recv_tokens": 10 * (rank + 1), "recv_tokens_per_layer": [10 * (rank + 1)],
            "compute_time": 0.1, "a2a_time": 0.2, "route_counts": [[rank, 1]], "steps": 1}
    got = rp.gather_payloads(rp.rank_payload(rank, 100 + rank, snap))
    if rank == 0:
        rep = rp.bench_report(got, plan=None, iters=1, wall_time=1.0, iter_times=[1.0])
        rp.write_bench_report(Path(out_dir, "bench.json"), rep)
    else:
        assert got is None
    dist.destroy_process_group()


def test_payloads_gathered_over_gloo_ranks(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, 29811, str(tmp_path)), nprocs=world, join=True)
    rep = json.loads((tmp_path / "bench.json").read_text())
    assert rep["world"] == 2 and rep["plan"] == "naive"
    assert [r["positions"] for r in rep["ranks"]] == [100, 101]
    assert rep["total_positions"] == 201
    assert report.load_summary(rep)["straggler"] == pytest.approx(20 / 15 - 1)
    assert report.expert_counts(rep).tolist() == [[1, 2]]
