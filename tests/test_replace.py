"""Live re-placement (the reference's /rebalance, miniep/server.py:166-183 and
apply_placement :49-61) on CPU: the transfer schedule on its own, and the
whole rebalance over two gloo ranks with expert weights moved rank to rank.
The device calls (table upload, round-robin reset) go to a recording
stand-in."""
import json
import os
import sys
from pathlib import Path

import torch
import torch.multiprocessing as mp

from miniep_b200 import Placement, plan_balanced
from miniep_b200.replace import transfer_schedule

REPO = Path(__file__).resolve().parents[1]


def test_transfer_schedule_feeds_every_new_replica_from_an_old_owner():
    old = Placement.naive(2, 8, 4)
    counts = torch.tensor([[900, 5, 5, 5, 5, 5, 5, 300], [5, 5, 700, 5, 5, 400, 5, 5]])
    new, _ = plan_balanced(counts, 4, slots_per_rank=2)
    sched = transfer_schedule(old, new, 4)
    want = set()
    for l in range(2):
        for r in range(4):
            for e in new.experts_of_rank(r)[l]:
                if e not in old.experts_of_rank(r)[l]:
                    want.add((l, e, r))
    assert {(l, e, d) for (l, e, s, d) in sched} == want
    for (l, e, s, d) in sched:
        assert s in old.owners[l][e] and d in new.owners[l][e] and d not in old.owners[l][e]
    assert transfer_schedule(old, old, 4) == []


class _FakeLib:
    def __init__(self):
        self.tables, self.resets = [], 0

    def mep_set_placement(self, ctx, layer, table_ptr, nrep_ptr, rmax):
        self.tables.append(layer)
        return 0

    def mep_reset_rr(self, ctx, stream):
        self.resets += 1
        return 0

    def mep_last_error(self, ctx):
        return b""


def _worker(rank, world, port, out_dir):
    sys.path[:0] = [str(REPO / "mini-ep_b200"), str(REPO)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from miniep_b200 import EPMoEBackend, EPStats, _lib, ep
    from miniep_b200.replace import rebalance
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = _FakeLib()
    _lib._lib = fake
    ep._stream = lambda: 0
    L, E, H, I = 2, 8, 16, 8
    g = torch.Generator().manual_seed(0)
    w_in_all = torch.randn(L, E, 2 * I, H, generator=g)
    w_out_all = torch.randn(L, E, H, I, generator=g)
    comm = object.__new__(ep.Comm)
    comm.group, comm.rank, comm.world, comm._ctx = None, rank, world, None
    comm.num_layers, comm.num_experts, comm.placement = L, E, None
    old = Placement.naive(L, E, world)
    comm.install(old)
    stats = EPStats(L, E)
    # skewed source-side counts, different on each rank
    rc = torch.full((L, E), 10, dtype=torch.long)
    rc[0, 1] = 500 + rank
    rc[1, 6] = 300 * (rank + 1)
    stats._route_counts = rc
    backends = []
    for l in range(L):
        mine = old.experts_of_rank(rank)[l]
        backends.append(EPMoEBackend(l, comm, old, mine, w_in_all[l][mine].clone(),
                                     w_out_all[l][mine].clone(), stats))
    caps = [ep._captured_state(be) for be in backends]  # what graphed blocks would hold
    res = rebalance(backends, stats, slots_per_rank=2)
    stale = []
    for be, cap in zip(backends, caps):
        try:
            ep._check_replay(be, cap)
            stale.append(False)
        except _lib.MEPError:
            stale.append(True)
    ep._check_replay(backends[0], ep._captured_state(backends[0]))  # a fresh capture replays
    new = backends[0].placement
    ok = []
    for l, be in enumerate(backends):
        mine = new.experts_of_rank(rank)[l]
        ok.append(be.local_experts == mine and torch.equal(be.w_in, w_in_all[l][mine])
                  and torch.equal(be.w_out, w_out_all[l][mine]))
    out = dict(plan=res["plan"], ok=ok, moved=res["moved_experts"], tables=fake.tables,
               resets=fake.resets, installed=comm.placement is new,
               replicas=res["replicas_added"], stale=stale)
    Path(out_dir, f"r{rank}.json").write_text(json.dumps(out))
    dist.destroy_process_group()


def test_rebalance_moves_weights_between_gloo_ranks(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, 29831, str(tmp_path)), nprocs=world, join=True)
    res = [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(world)]
    assert res[0]["plan"] == res[1]["plan"]
    # the plan is the balancer's on the counts summed over ranks
    counts = torch.full((2, 8), 20, dtype=torch.long)
    counts[0, 1] = 1001
    counts[1, 6] = 900
    want, _ = plan_balanced(counts, world, slots_per_rank=2)
    assert res[0]["plan"] == json.loads(json.dumps(want.to_plan()))
    assert res[0]["replicas"] > 0 and res[0]["moved"] > 0
    for r in res:
        assert all(r["ok"])
        assert r["installed"] and r["resets"] == 1
        assert r["tables"][-2:] == [0, 1]
        # graphs captured before the re-placement refuse to replay after it
        assert r["stale"] == [True, True]
