"""World-size-2 host logic on CPU (gloo): the peer-buffer handle exchange of
``Comm`` (every rank opens exactly every other rank's handle, and only after
all handles are known) and the plan upload that every rank must perform with
identical tables. The device calls are replaced by a recording stand-in."""
import os
import sys
from pathlib import Path

import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


class _FakeLib:
    def __init__(self, rank):
        self.rank = rank
        self.opened = []
        self.tables = []

    def mep_ipc_handle(self, ctx, buf):
        buf.raw = bytes([self.rank + 1]) * 64
        return 0

    def mep_ipc_open(self, ctx, peer, hb):
        self.opened.append((peer, hb.raw[0]))
        return 0

    def mep_set_placement(self, ctx, layer, table_ptr, nrep_ptr, rmax):
        import ctypes as C
        self.tables.append((layer, rmax))
        return 0

    def mep_last_error(self, ctx):
        return b""


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(REPO / "mini-ep_b200"))
    sys.path.insert(0, str(REPO))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from miniep_b200 import _lib, ep
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = _FakeLib(rank)
    _lib._lib = fake  # route the binding to the stand-in
    comm = object.__new__(ep.Comm)
    comm.group, comm.rank, comm.world, comm._ctx = None, rank, world, None
    comm.num_layers, comm.num_experts = 2, 4
    comm.placement = None
    comm._open_peers()
    placement = ep.Placement([[[0, 1], [0], [1], [1]], [[0], [0], [1], [0, 1]]])
    comm.install(placement)
    assert placement._comm is comm
    result = dict(opened=fake.opened, tables=fake.tables)
    gathered = [None] * world
    dist.all_gather_object(gathered, result)
    if rank == 0:
        import json
        Path(out_dir, "res.json").write_text(json.dumps(gathered))
    dist.destroy_process_group()


def test_handle_exchange_world2(tmp_path):
    mp.spawn(_worker, args=(2, 29655, str(tmp_path)), nprocs=2, join=True)
    import json
    res = json.loads((tmp_path / "res.json").read_text())
    assert res[0]["opened"] == [[1, 2]]  # rank 0 opened rank 1's handle (tagged 2)
    assert res[1]["opened"] == [[0, 1]]
    assert res[0]["tables"] == res[1]["tables"] == [[0, 2], [1, 2]]
