"""Pin the CPU checker (oracle/) to the reference's own outputs.

The fixtures in tests/golden/ were produced by running the reference's code
(tests/golden/make_golden.py); here the checker recomputes the same cases from
the same seeds and must agree: integer results (routing indices away from
ties, counts, destinations, plans) exactly, floating-point results within
summation-order noise (1e-5 relative in fp32, 1 bf16 ulp / 2e-2 abs in bf16).
"""
import json

import numpy as np
import pytest
import torch

from miniep_b200 import synth
from oracle import moe_oracle as O


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def _near_tie(logits, k, eps):
    srt = logits.float().sort(dim=-1, descending=True).values[:, : k + 1]
    return ((srt[:, :-1] - srt[:, 1:]).abs() <= eps).any(dim=-1)


def test_router_and_local_fp32(golden):
    g = np.load(golden / "router_local_fp32.npz")
    sh = synth.SHAPES["a"]
    lt = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 512, seed=0)
    idx, gate, logits = O.router_topk(lt.x, lt.router, sh["topk"])
    ref_logits = torch.from_numpy(g["logits"])
    assert torch.allclose(logits, ref_logits, rtol=1e-5, atol=1e-6)
    stable = ~_near_tie(ref_logits, sh["topk"], 1e-5)
    assert stable.float().mean() > 0.95
    assert torch.equal(idx[stable], torch.from_numpy(g["topk_idx"]).long()[stable])
    assert torch.allclose(gate, torch.from_numpy(g["topk_gate"]), rtol=1e-5, atol=1e-6)
    # the rest of the layer on the reference's own routing
    ref_idx = torch.from_numpy(g["topk_idx"]).long()
    ref_gate = torch.from_numpy(g["topk_gate"])
    out = O.local_moe(lt.x, ref_idx, ref_gate, lt.w_in, lt.w_out)
    head = torch.from_numpy(g["out_head"])
    scale = head.abs().max()
    assert (out[:48] - head).abs().max() <= 1e-5 * scale
    rs = torch.from_numpy(g["out_rowsum"])
    assert torch.allclose(out.double().sum(1), rs[:, 0], rtol=1e-4, atol=1e-5)
    valid = torch.from_numpy(g["valid"])
    outm = O.local_moe(lt.x, ref_idx, ref_gate, lt.w_in, lt.w_out, valid_mask=valid)
    assert (outm[:48] - torch.from_numpy(g["outm_head"])).abs().max() <= 1e-5 * scale
    assert torch.all(outm[~valid] == 0)


def test_router_and_block_bf16(golden):
    g = np.load(golden / "router_local_bf16.npz")
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 128, seed=0,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    idx, gate, logits = O.router_topk(lb.x, lb.router, sh["topk"], bias)
    ref_logits = _bf16(g["logits"])
    diff = (logits.float() - ref_logits.float()).abs()
    ulp = ref_logits.float().abs().clamp_min(1e-3) * 2.0 ** -7
    assert torch.all(diff <= ulp)
    assert (logits == ref_logits).float().mean() > 0.99
    ref_idx = torch.from_numpy(g["topk_idx"]).long()
    same = (logits == ref_logits).all(dim=1)
    ok = ~O.boundary_ties(ref_logits, sh["topk"]) & same
    assert ok.float().mean() > 0.5  # bf16 + skew bias: exact ties are common
    assert torch.equal(idx[ok], ref_idx[ok])
    # with ties, the selected values (not their order among equals) must agree
    assert torch.equal(logits.gather(1, idx)[same], ref_logits.gather(1, ref_idx)[same])
    ref_gate = _bf16(g["topk_gate"])
    out = O.local_moe(lb.x, ref_idx, ref_gate, lb.w_in, lb.w_out)
    ref_out = _bf16(g["out"])
    assert (out.float() - ref_out.float()).abs().max() <= 2e-2
    h = synth.make_tokens(128, sh["hidden"], seed=7, dtype=torch.bfloat16)
    blk = O.residual_add(h, out, synth.GRANITE_RESIDUAL_MULTIPLIER)
    assert (blk.float() - _bf16(g["block_out"]).float()).abs().max() <= 2e-2


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("plan", ["naive", "replicated"])
def test_ep_forward_matches_gloo_reference(golden, world, plan):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", golden / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    case = mg.ep_cases(world)[plan]
    g = np.load(golden / "ep_gloo.npz")
    key = f"w{world}_{plan}"
    assert json.loads(str(g[f"{key}_owners"])) == case["owners"]
    rr = [np.zeros(case["E"], dtype=np.int64) for _ in range(world)]
    route = np.zeros((world, case["E"]), dtype=np.int64)
    recv = np.zeros(world, dtype=np.int64)
    for call in range(2):
        res = O.ep_forward(case["x"][call], case["idx"][call], case["gate"][call], case["w_in"],
                           case["w_out"], case["owners"][0], rr=rr, valids=case["valid"][call])
        route += res.route_counts
        recv += res.recv_tokens
        for r in range(world):
            ref = torch.from_numpy(g[f"{key}_r{r}_c{call}_out"])
            assert (res.outputs[r] - ref).abs().max() <= 1e-5 * ref.abs().max()
    for r in range(world):
        assert np.array_equal(route[r], g[f"{key}_r{r}_route_counts"][0])
        assert recv[r] == int(g[f"{key}_r{r}_recv_tokens"])


def test_dest_ranks_round_robin(golden):
    g = np.load(golden / "dest_ranks.npz")
    owners = O.owners_from_plan(json.loads(str(g["plan"])))
    for layer in range(len(owners)):
        table, n_rep = O.build_table(owners[layer])
        rr = np.zeros(len(owners[layer]), dtype=np.int64)
        for call in range(3):
            ids = g[f"l{layer}_c{call}_ids"].astype(np.int64)
            d = O.dest_ranks(table, n_rep, rr, ids)
            assert np.array_equal(d, g[f"l{layer}_c{call}_dest"].astype(np.int64))
        assert np.array_equal(rr, g[f"l{layer}_rr"])


def test_local_equals_world1_ep():
    torch.manual_seed(0)
    lt = synth.make_layer(64, 8, 32, 40, seed=9)
    logits = lt.x @ lt.router.T
    tl, ti = logits.topk(2, dim=-1)
    tg = torch.softmax(tl, -1)
    local = O.local_moe(lt.x, ti, tg, lt.w_in, lt.w_out)
    ep = O.ep_forward([lt.x], [ti], [tg], lt.w_in, lt.w_out, O.naive_owners(1, 8, 1)[0])
    assert torch.allclose(local, ep.outputs[0], rtol=1e-6, atol=1e-7)
    assert ep.recv_tokens[0] == 80


def test_rms_norm_matches_reference(golden):
    """The checker's post-attention RMSNorm is the reference's rms_norm
    (modeling.py:51-52) bit for bit, bf16 and fp32, shapes (a) and (b)."""
    g = np.load(golden / "rms_norm.npz")
    for shape in ("a", "b"):
        for name in ("bf16", "fp32"):
            conv = _bf16 if name == "bf16" else torch.from_numpy
            h, w, y = (conv(g[f"{shape}_{name}_{t}"]) for t in ("h", "w", "y"))
            assert torch.equal(O.rms_norm(h, w, 1e-6), y), (shape, name)
