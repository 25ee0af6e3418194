"""The single-process drop-in (LocalMoEBackend) and the step timeline, on one GPU.

* ``miniep_b200.LocalMoEBackend`` is the reference's LocalMoEBackend
  (modeling.py:131-145): constructed from the stacked expert weights alone,
  called with the same (x, topk_idx, topk_gate, valid_mask) arguments. Its
  outputs are checked against the reference's own fp32 run (config 1
  fixture) and the checker, and its stats against the routing.
* The step timeline (option "timeline", mep_read_timeline): every stage of a
  block step is stamped, in launch order, and reading clears the stamps.
"""
import numpy as np
import pytest
import torch

from gpu_util import require_gpu
from miniep_b200 import EPStats, LocalMoEBackend, synth
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def test_local_backend_drop_in_matches_reference_config1(golden):
    g = np.load(golden / "router_local_fp32.npz")
    sh = synth.SHAPES["a"]
    n = 512
    lt = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=0)
    stats = EPStats(1, sh["experts"])
    be = LocalMoEBackend(lt.w_in.cuda(), lt.w_out.cuda(), max_tokens=n, topk=sh["topk"],
                         stats=stats)
    idx = torch.from_numpy(g["topk_idx"]).long()
    gate = torch.from_numpy(g["topk_gate"])
    valid = torch.from_numpy(g["valid"]).bool()
    for mask in (None, valid):
        out = be(lt.x.cuda(), idx.cuda(), gate.cuda(),
                 valid_mask=None if mask is None else mask.cuda()).cpu()
        ref = O.local_moe(lt.x, idx, gate, lt.w_in, lt.w_out, mask)
        assert (out - ref).abs().max() <= 1e-5 * ref.abs().max()
        head = g["out_head"] if mask is None else g["outm_head"]
        ref_head = torch.from_numpy(head)
        assert (out[:head.shape[0]] - ref_head).abs().max() <= 1e-5 * ref_head.abs().max()
    be.comm.check()
    snap = stats.snapshot()
    kept = idx.reshape(-1)[valid.repeat_interleave(sh["topk"])]
    want = torch.bincount(idx.reshape(-1), minlength=sh["experts"]) + \
        torch.bincount(kept, minlength=sh["experts"])
    assert snap["route_counts"][0] == want.tolist()
    assert snap["recv_tokens"] == n * sh["topk"] + int(valid.sum()) * sh["topk"]
    be.comm.close()


def test_step_timeline_stamps_every_stage_in_order():
    sh = synth.SHAPES["a"]
    n = 2048
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=2,
                          dtype=torch.bfloat16)
    be = LocalMoEBackend(lb.w_in.cuda(), lb.w_out.cuda(), max_tokens=n, topk=sh["topk"])
    comm = be.comm
    h = synth.make_tokens(n, sh["hidden"], seed=7, dtype=torch.bfloat16).cuda()
    nw = torch.ones(sh["hidden"], dtype=torch.bfloat16, device="cuda")
    args = (h, nw, 1e-6, lb.router.cuda(), synth.GRANITE_RESIDUAL_MULTIPLIER)
    be.moe_block_from_h(*args)  # option off: nothing is stamped
    assert comm.read_timeline() == {}
    comm.set_option("timeline", 1)
    out_on, *_ = be.moe_block_from_h(*args)
    tl = comm.read_timeline()
    comm.set_option("timeline", 0)
    order = ["norm", "router", "route", "dispatch", "gemm1", "gemm2", "combine"]
    assert set(order) <= set(tl), tl
    for name in order:
        s, e = tl[name]
        assert 0 <= s <= e, (name, s, e)
    # one stream: each stage starts after the previous one ended (1 us of slack
    # for stamps taken on different SMs)
    for a, b in zip(order, order[1:]):
        assert tl[a][1] <= tl[b][0] + 1.0, (a, tl[a], b, tl[b])
    assert tl["route"][0] <= tl["counts_sent"] <= tl["layout"] <= tl["route"][1] + 1.0
    assert tl["combine"][0] <= tl["results_in"] <= tl["combine"][1]
    assert comm.read_timeline() == {}  # reading cleared the stamps
    # the stamps do not change the step's results
    out_off, *_ = be.moe_block_from_h(*args)
    assert torch.equal(out_on, out_off)
    comm.check()
    comm.close()


@pytest.mark.parametrize("option", ["dispatch_per_warp=0", "ffn_ast=1", "ffn_prefetch=1"])
@pytest.mark.parametrize("n", [4096, 300])
def test_step_options_change_no_result(option, n):
    """The selectable variants move the same bytes and issue the same MMAs
    in another schedule (streaming dispatch engine, A-stationary GEMM2, L2
    prefetch of the next tile's rows): the block's output, ids and gates are
    bit-identical to the default step's."""
    name, value = option.split("=")
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=6,
                          dtype=torch.bfloat16)
    be = LocalMoEBackend(lb.w_in.cuda(), lb.w_out.cuda(), max_tokens=n, topk=sh["topk"])
    comm = be.comm
    h = synth.make_tokens(n, sh["hidden"], seed=10, dtype=torch.bfloat16).cuda()
    nw = torch.ones(sh["hidden"], dtype=torch.bfloat16, device="cuda")
    bias = synth.zipf_router_bias(1, sh["experts"])[0].cuda()
    args = (h, nw, 1e-6, lb.router.cuda(), synth.GRANITE_RESIDUAL_MULTIPLIER)
    ref = [t.clone() for t in be.moe_block_from_h(*args, bias=bias)[:3]]
    comm.set_option(name, int(value))
    got = [t.clone() for t in be.moe_block_from_h(*args, bias=bias)[:3]]
    comm.check()
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    comm.close()
