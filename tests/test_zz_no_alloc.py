"""mep_dest_ranks_noalloc, the destination scan for callers that cannot call
cudaMalloc (a serving process whose HBM is all handed to its own pool, or a
latency-critical path where an allocation would synchronise the device).

It must give the same destinations as the context-based mep_dest_ranks on
consecutive calls (the round-robin state carries over), without allocating.
This file is collected last so that a failure here, in a run that stops at the
first failure, comes after every other test has run.
"""
import json

import numpy as np
import pytest
import torch

from gpu_util import RawCtx, require_gpu, stream
from miniep_b200 import _lib
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


def test_noalloc_matches_context_entry_point_on_consecutive_calls(golden):
    require_gpu()
    g = np.load(golden / "dest_ranks.npz")
    owners = O.owners_from_plan(json.loads(str(g["plan"])))
    layer = max(range(len(owners)), key=lambda l: sum(len(o) for o in owners[l]))
    table, n_rep = O.build_table(owners[layer])
    E, rmax, world = table.shape[0], table.shape[1], 4
    assert n_rep.max() > 1  # a layer with replicated experts
    raw = RawCtx(0, world, 1, E, 8, 1024, 512, 8192, torch.bfloat16)
    L = _lib.lib()
    try:
        raw.call("mep_set_placement", 0, table.ctypes.data, n_rep.ctypes.data, rmax)
        raw.call("mep_reset_rr", stream())
        rr = torch.zeros(E, dtype=torch.int64, device="cuda")
        rr_cpu = np.zeros(E, dtype=np.int64)
        gen = torch.Generator().manual_seed(123)
        for call, m in enumerate((6000, 65536)):
            p = torch.distributions.Dirichlet(torch.ones(E)).sample()
            ids = torch.multinomial(p, m, replacement=True, generator=gen).to(torch.int64)
            ids_d = ids.cuda()
            want = torch.empty_like(ids_d)
            raw.call("mep_dest_ranks", 0, ids_d.data_ptr(), m, want.data_ptr(), stream())
            got = torch.full_like(ids_d, -7)
            rc = L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                          rr.data_ptr(), ids_d.data_ptr(), m, got.data_ptr(),
                                          stream())
            assert rc == 0, _lib.last_error(None)
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"call {call}"
            ref = O.dest_ranks(table, n_rep, rr_cpu, ids.numpy())
            assert np.array_equal(got.cpu().numpy(), ref), f"call {call}"
            assert np.array_equal(rr.cpu().numpy(), rr_cpu)
        # round-robin state of any sign: the replica is (rr + occurrence) mod n_rep
        # taken non-negative, as Python's % gives it
        rr_cpu = np.arange(E, dtype=np.int64) * -7 - 3
        rr.copy_(torch.from_numpy(rr_cpu))
        ids = torch.randint(0, E, (3000,), generator=gen).to(torch.int64)
        got = torch.full((3000,), -7, dtype=torch.int64, device="cuda")
        assert L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                        rr.data_ptr(), ids.cuda().data_ptr(), 3000,
                                        got.data_ptr(), stream()) == 0, _lib.last_error(None)
        ref = O.dest_ranks(table, n_rep, rr_cpu, ids.numpy())
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy(), ref)
        assert np.array_equal(rr.cpu().numpy(), rr_cpu)
        # an id outside [0, E) gets destination -1 and is left out of the
        # round-robin advance; the valid ids route as if it were absent
        rr.zero_()
        ids = torch.randint(0, E, (500,), generator=gen).to(torch.int64)
        bad = ids.clone()
        bad[[3, 77, 400]] = torch.tensor([E, -1, 10 * E])
        got = torch.full((500,), -7, dtype=torch.int64, device="cuda")
        assert L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                        rr.data_ptr(), bad.cuda().data_ptr(), 500,
                                        got.data_ptr(), stream()) == 0
        keep = torch.ones(500, dtype=torch.bool)
        keep[[3, 77, 400]] = False
        rr_ref = np.zeros(E, dtype=np.int64)
        ref = O.dest_ranks(table, n_rep, rr_ref, bad[keep].numpy())
        torch.cuda.synchronize()
        g = got.cpu()
        assert g[~keep].tolist() == [-1, -1, -1]
        assert np.array_equal(g[keep].numpy(), ref)
        assert np.array_equal(rr.cpu().numpy(), rr_ref)
        # beyond the fixed scratch: rejected with a clear message, nothing launched
        big = torch.zeros(65537, dtype=torch.int64, device="cuda")
        rc = L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                      rr.data_ptr(), big.data_ptr(), big.numel(), big.data_ptr(),
                                      stream())
        assert rc == _lib.MEP_OK + 1 and "65536" in _lib.last_error(None)
        raw.call("mep_check")
    finally:
        raw.close()


def test_noalloc_single_owner_layer_and_empty_call(golden):
    """A layer without replicas takes the reference's fast path (ep.py:84-85):
    destinations straight from the table and the round-robin state untouched;
    a call with no ids launches only the state update, which leaves it alone
    as well."""
    require_gpu()
    g = np.load(golden / "dest_ranks.npz")
    owners = O.owners_from_plan(json.loads(str(g["plan"])))
    single = [l for l in range(len(owners)) if all(len(o) == 1 for o in owners[l])]
    layer = single[0] if single else None
    world = 4
    if layer is None:  # the shipped plan replicates every layer: use the naive placement
        own = O.naive_owners(1, 32, world)[0]
    else:
        own = owners[layer]
    table, n_rep = O.build_table(own)
    E, rmax = table.shape
    assert (n_rep == 1).all()
    L = _lib.lib()
    rr0 = np.arange(E, dtype=np.int64) + 5
    rr = torch.from_numpy(rr0.copy()).cuda()
    ids = torch.randint(0, E, (4097,), generator=torch.Generator().manual_seed(9)).to(torch.int64)
    got = torch.empty(4097, dtype=torch.int64, device="cuda")
    for call in range(2):
        assert L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                        rr.data_ptr(), ids.cuda().data_ptr(), ids.numel(),
                                        got.data_ptr(), stream()) == 0, _lib.last_error(None)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy(), O.dest_ranks(table, n_rep, rr0.copy(), ids.numpy()))
        assert np.array_equal(rr.cpu().numpy(), rr0), call
    assert L.mep_dest_ranks_noalloc(E, world, table.ctypes.data, n_rep.ctypes.data, rmax,
                                    rr.data_ptr(), None, 0, None, stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(rr.cpu().numpy(), rr0)
