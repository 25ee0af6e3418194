"""CUDA path vs the CPU checker and the reference's fixtures, through the C ABI.

Bars: routing indices and every count bit-exact (away from exact logit ties,
where the CUDA router's rule is "lower expert index first" and is checked
against its own logits); layer outputs within 1e-5 relative (fp32) and
within 2e-2 max-abs of an fp32 reference (bf16).
"""
import json

import numpy as np
import pytest
import torch

from gpu_util import RawCtx, require_gpu, stream, world1_backend, world1_comm
from miniep_b200 import MEPError, synth
from miniep_b200.ep import router_topk
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

FP32_RTOL = 1e-5       # fp32 outputs: max|gpu - ref| <= 1e-5 * max|ref|
BF16_ATOL = 2e-2       # bf16 outputs vs an fp32 reference, max-abs, for outputs of unit scale
# Tie-free rows whose top-k may differ from the reference's because one bf16
# logit rounded a step the other way (fp32 sums of the router GEMM in another
# order than torch's CPU kernel, which is itself not correctly rounded in about
# 1e-4 of its bf16 logits): at most this fraction of the rows. Measured on a
# B200: 0 of 3342, 803, 889 and 27 tie-free rows.
ROUTER_ROUNDING_ROWS = 0.005


def logit_step(logits, bias=None):
    """One bf16 rounding step of a router logit, from either of its two
    roundings: the dot product (magnitude |logit - bias|) rounds to bf16, then
    the bias is added and the sum rounds again. Two fp32 sums of the same dot
    product that round to neighbouring bf16 values give logits at most one
    step of each apart (with cancellation against the bias the first step can
    exceed the logit's own)."""
    b = 0.0 if bias is None else bias.to(torch.bfloat16).float()
    return ((logits - b).abs() + logits.abs()).clamp_min(2.0 ** -20) * 2.0 ** -7


def bf16_tol(ref32):
    """2e-2 max-abs, scaled by the output magnitude when it exceeds 1: shape
    (b) outputs reach |3.6| and the reference's own bf16 path is already
    2.8e-2 away from fp32 there (one bf16 ulp at 2..4 is 1.6e-2)."""
    return BF16_ATOL * max(1.0, float(ref32.abs().max()))


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    require_gpu()


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def _fp32_ref(x, idx, gate, w_in, w_out, valid=None):
    return O.local_moe(x.float().cpu(), idx.cpu(), gate.float().cpu(), w_in.float().cpu(),
                       w_out.float().cpu(), None if valid is None else valid.cpu())


# ----------------------------------------------------------------- router
def test_router_fp32_config1(golden):
    g = np.load(golden / "router_local_fp32.npz")
    sh = synth.SHAPES["a"]
    lt = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 512, seed=0)
    be = world1_backend(lt.w_in, lt.w_out, sh["topk"], 512)
    idx, gate, logits = router_topk(be.comm, lt.x.cuda(), lt.router.cuda(), return_logits=True)
    ref_logits = torch.from_numpy(g["logits"])
    # 1e-5 relative to the logit scale (fp32 sums of 1024 products in another order)
    assert (logits.cpu() - ref_logits).abs().max() <= FP32_RTOL * ref_logits.abs().max()
    srt = ref_logits.sort(dim=-1, descending=True).values[:, : sh["topk"] + 1]
    stable = ((srt[:, :-1] - srt[:, 1:]) > 1e-4 * srt.abs().max()).all(dim=-1)
    assert stable.float().mean() > 0.9
    ref_idx = torch.from_numpy(g["topk_idx"]).long()
    assert torch.equal(idx.cpu()[stable], ref_idx[stable])
    assert torch.allclose(gate.cpu()[stable], torch.from_numpy(g["topk_gate"])[stable],
                          rtol=1e-5, atol=1e-6)


# 256 and more tokens take the tcgen05 router, fewer the warp-level kernel
@pytest.mark.parametrize("shape,n", [("a", 4096), ("a", 1), ("a", 1000), ("b", 1024), ("b", 33),
                                     ("b", 4100), ("a", 20000)])
def test_router_bf16_skewed(shape, n):
    sh = synth.SHAPES[shape]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=1, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    comm = world1_comm(sh["experts"], sh["topk"], sh["hidden"], sh["inter"], n, torch.bfloat16)
    idx, gate, logits = router_topk(comm, lb.x.cuda(), lb.router.cuda(), bias.cuda(),
                                    return_logits=True)
    idx, gate, logits = idx.cpu(), gate.cpu(), logits.cpu()
    ref_idx, ref_gate, ref_logits = O.router_topk(lb.x, lb.router, sh["topk"], bias)
    # logits: fp32 accumulation in another order, then the same rounding
    assert torch.all((logits - ref_logits.float()).abs() <= logit_step(ref_logits.float(), bias))
    same_row = (logits == ref_logits.float()).all(dim=1)
    if n >= 64:
        assert same_row.float().mean() > 0.9
    # selection rule is exact on the kernel's own logits (lower index first on ties)
    assert torch.equal(idx, O.topk_lowest_index(logits, sh["topk"]))
    # against the reference, every row without an exact tie in its top-(k+1)
    # logits (where torch's CPU topk has no fixed order) is compared
    ties = O.boundary_ties(ref_logits, sh["topk"])
    off = ~(idx == ref_idx).all(dim=1) & ~ties
    # a row whose logits equal the reference's bit for bit selects the same experts
    assert not (off & same_row).any()
    # the rest: a logit one rounding step from the reference's moved the choice
    # (reported apart; bounded by ROUTER_ROUNDING_ROWS of the tie-free rows)
    assert int(off.sum()) <= ROUTER_ROUNDING_ROWS * int((~ties).sum()), \
        (int(off.sum()), int((~ties).sum()))
    ok = ~ties & ~off
    assert torch.equal(idx[ok], ref_idx[ok])
    assert torch.equal(logits.gather(1, idx)[same_row],
                       ref_logits.float().gather(1, ref_idx)[same_row])
    assert (gate.float() - ref_gate.float()).abs()[ok].max() <= 2.0 ** -8
    # per-expert histogram of the kernel's routing == the reference's on tie-free rows
    assert torch.equal(torch.bincount(idx[ok].reshape(-1), minlength=sh["experts"]),
                       torch.bincount(ref_idx[ok].reshape(-1), minlength=sh["experts"]))
    print(f"router {shape} n={n}: exact-tie rows {int(ties.sum())}, "
          f"rounding-moved rows {int(off.sum())} of {int((~ties).sum())} tie-free")


@pytest.mark.parametrize("shape,n", [("a", 8192), ("b", 8192), ("a", 2048), ("b", 300)])
def test_router_tcgen05_and_warp_kernels_agree(shape, n):
    """The tcgen05 router and the warp-level kernel select the same experts
    and gates wherever their fp32 sums round to the same bf16 logits, and
    their logits differ by at most one rounding step (the tcgen05 kernel's
    tiles hold 56 tokens at 8192, 16 at 2048 and 8 at 300 on 148 SMs)."""
    sh = synth.SHAPES[shape]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=5, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0].cuda()
    comm = world1_comm(sh["experts"], sh["topk"], sh["hidden"], sh["inter"], n, torch.bfloat16)
    x, w = lb.x.cuda(), lb.router.cuda()
    got = {}
    for no_tc in (0, 1):
        comm.set_option("router_no_tc", no_tc)
        got[no_tc] = [t.cpu() for t in router_topk(comm, x, w, bias, return_logits=True)]
    comm.check()
    (i_tc, g_tc, l_tc), (i_w, g_w, l_w) = got[0], got[1]
    assert torch.all((l_tc - l_w).abs() <= logit_step(l_w, bias.cpu()))
    same = (l_tc == l_w).all(dim=1)
    assert same.float().mean() > 0.9
    assert torch.equal(i_tc[same], i_w[same])
    assert torch.equal(g_tc[same], g_w[same])
    assert torch.equal(i_tc, O.topk_lowest_index(l_tc, sh["topk"]))


def test_dispatch_rejects_rows_not_16_byte_aligned():
    sh = synth.SHAPES["a"]
    n, H = 64, sh["hidden"]
    lb = synth.make_layer(H, sh["experts"], sh["inter"], n, seed=4, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    buf = torch.empty(n * H + 2, dtype=torch.bfloat16, device="cuda")
    x = buf[2:].view(n, H)
    x.copy_(lb.x)
    idx = torch.stack([torch.randperm(32)[:8] for _ in range(n)]).cuda()
    gate = torch.full((n, 8), 0.125, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(MEPError, match="16-byte"):
        be(x, idx, gate)
    out = be(lb.x.cuda(), idx, gate)  # the context keeps working
    assert torch.isfinite(out.float()).all()
    be.comm.check()


def test_router_bf16_rows_not_16_byte_aligned():
    """x starting 4 bytes past an allocation takes the CUDA-core kernel; its
    logits and selection obey the same contract as the staged kernel's."""
    sh = synth.SHAPES["a"]
    n, H = 200, sh["hidden"]
    lb = synth.make_layer(H, sh["experts"], sh["inter"], n, seed=3, dtype=torch.bfloat16)
    buf = torch.empty(n * H + 2, dtype=torch.bfloat16, device="cuda")
    x = buf[2:].view(n, H)
    x.copy_(lb.x)
    assert x.data_ptr() % 16 == 4
    comm = world1_comm(sh["experts"], sh["topk"], H, sh["inter"], n, torch.bfloat16)
    idx, gate, logits = router_topk(comm, x, lb.router.cuda(), return_logits=True)
    idx, logits = idx.cpu(), logits.cpu()
    _, _, ref_logits = O.router_topk(lb.x, lb.router, sh["topk"])
    assert torch.all((logits - ref_logits.float()).abs() <= logit_step(ref_logits.float()))
    assert torch.equal(idx, O.topk_lowest_index(logits, sh["topk"]))


# ---------------------------------------------------------------- dest ranks
def test_dest_ranks_matches_reference_round_robin(golden):
    g = np.load(golden / "dest_ranks.npz")
    plan = json.loads(str(g["plan"]))
    owners = O.owners_from_plan(plan)
    L, E = len(owners), len(owners[0])
    raw = RawCtx(0, 4, L, E, 8, 1024, 512, 64, torch.bfloat16)
    try:
        for l in range(L):
            table, n_rep = O.build_table(owners[l])
            raw.call("mep_set_placement", l, table.ctypes.data, n_rep.ctypes.data, table.shape[1])
        raw.call("mep_reset_rr", stream())
        for l in range(L):
            for call in range(3):
                ids = torch.from_numpy(g[f"l{l}_c{call}_ids"].astype(np.int64)).cuda()
                out = torch.empty_like(ids)
                raw.call("mep_dest_ranks", l, ids.data_ptr(), ids.numel(), out.data_ptr(), stream())
                want = torch.from_numpy(g[f"l{l}_c{call}_dest"].astype(np.int64))
                assert torch.equal(out.cpu(), want), (l, call)
        # reset_rr restarts the round robin
        raw.call("mep_reset_rr", stream())
        ids = torch.from_numpy(g["l0_c0_ids"].astype(np.int64)).cuda()
        out = torch.empty_like(ids)
        raw.call("mep_dest_ranks", 0, ids.data_ptr(), ids.numel(), out.data_ptr(), stream())
        assert torch.equal(out.cpu(), torch.from_numpy(g["l0_c0_dest"].astype(np.int64)))
        torch.cuda.synchronize()
        raw.call("mep_check")
    finally:
        raw.close()


# ---------------------------------------------------------------- layer
def test_layer_fp32_config1_matches_reference(golden):
    g = np.load(golden / "router_local_fp32.npz")
    sh = synth.SHAPES["a"]
    lt = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 512, seed=0)
    idx = torch.from_numpy(g["topk_idx"]).long()
    gate = torch.from_numpy(g["topk_gate"])
    valid = torch.from_numpy(g["valid"])
    be = world1_backend(lt.w_in, lt.w_out, sh["topk"], 512)
    out = be(lt.x.cuda(), idx.cuda(), gate.cuda()).cpu()
    head = torch.from_numpy(g["out_head"])
    tol = FP32_RTOL * head.abs().max()
    assert (out[:48] - head).abs().max() <= tol
    full = O.local_moe(lt.x, idx, gate, lt.w_in, lt.w_out)
    assert (out - full).abs().max() <= FP32_RTOL * full.abs().max()
    outm = be(lt.x.cuda(), idx.cuda(), gate.cuda(), valid_mask=valid.cuda()).cpu()
    assert (outm[:48] - torch.from_numpy(g["outm_head"])).abs().max() <= tol
    assert torch.all(outm[~valid] == 0)
    snap = be.stats.snapshot()
    kept = int(valid.sum()) * sh["topk"]
    assert snap["recv_tokens"] == 512 * sh["topk"] + kept
    want = torch.bincount(idx.reshape(-1), minlength=sh["experts"]) + \
        torch.bincount(idx[valid].reshape(-1), minlength=sh["experts"])
    assert snap["route_counts"] == [want.tolist()]
    be.comm.check()


@pytest.mark.parametrize("path", ["tcgen05_pair", "tcgen05_single", "cuda_cores"])
@pytest.mark.parametrize("n", [1, 127, 300, 2048])
def test_layer_bf16_shape_a(n, path):
    force_simt, single_cta = path == "cuda_cores", path == "tcgen05_single"
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=2, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    idx, gate, _ = O.router_topk(lb.x, lb.router, sh["topk"], bias)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], max(n, 256), force_simt=force_simt,
                        single_cta=single_cta)
    out = be(lb.x.cuda(), idx.cuda(), gate.cuda()).cpu()
    ref32 = _fp32_ref(lb.x, idx, gate, lb.w_in, lb.w_out)
    assert (out.float() - ref32).abs().max() <= BF16_ATOL
    ref16 = O.local_moe(lb.x, idx, gate, lb.w_in, lb.w_out)
    # against the bf16 reference itself: same roundings, so nearly all equal
    d = (out.float() - ref16.float()).abs()
    assert d.max() <= 2e-2 and (d == 0).float().mean() > 0.8
    be.comm.check()


def test_tcgen05_and_cuda_core_paths_agree():
    sh = synth.SHAPES["a"]
    n = 4096
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=4, dtype=torch.bfloat16)
    idx, gate, _ = O.router_topk(lb.x, lb.router, sh["topk"], synth.zipf_router_bias(1, 32)[0])
    a = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    b = world1_backend(lb.w_in, lb.w_out, sh["topk"], n, force_simt=True)
    c = world1_backend(lb.w_in, lb.w_out, sh["topk"], n, single_cta=True)
    xa, ia, ga = lb.x.cuda(), idx.cuda(), gate.cuda()
    oa, ob, oc = a(xa, ia, ga), b(xa, ia, ga), c(xa, ia, ga)
    d = (oa.float() - ob.float()).abs()
    assert d.max() <= 1e-2 and (d == 0).float().mean() > 0.9
    # CTA pairs and single CTAs run the same MMA chain per row: identical bits
    assert torch.equal(oa, oc)
    for be in (a, b, c):
        be.comm.check()


def test_layer_bf16_shape_b():
    sh = synth.SHAPES["b"]
    n = 384
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=5, dtype=torch.bfloat16)
    idx, gate, _ = O.router_topk(lb.x, lb.router, sh["topk"], synth.zipf_router_bias(1, 64)[0])
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    out = be(lb.x.cuda(), idx.cuda(), gate.cuda()).cpu()
    ref32 = _fp32_ref(lb.x, idx, gate, lb.w_in, lb.w_out)
    assert (out.float() - ref32).abs().max() <= bf16_tol(ref32)
    # and no further from fp32 than the reference's own bf16 path, within one ulp
    ref16 = O.local_moe(lb.x, idx, gate, lb.w_in, lb.w_out)
    assert (out.float() - ref16.float()).abs().max() <= 2.0 ** -6 * max(1.0, float(ref32.abs().max()))
    be.comm.check()


def test_moe_block_matches_reference_block(golden):
    g = np.load(golden / "router_local_bf16.npz")
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 128, seed=0,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    h = synth.make_tokens(128, sh["hidden"], seed=7, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], 128)
    h_out, idx, gate = be.moe_block(h.cuda(), lb.x.cuda(), lb.router.cuda(),
                                    synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias.cuda())
    ref_idx = torch.from_numpy(g["topk_idx"]).long()
    # rows without an exact tie in the reference's top-(k+1) logits select the
    # reference's experts in the reference's order; a row with such a tie may
    # order the tied experts differently (torch's CPU topk has no tie rule)
    ties = O.boundary_ties(_bf16(g["logits"]).float(), sh["topk"])
    same = (idx.cpu() == ref_idx).all(dim=1)
    off = ~same & ~ties
    assert int(off.sum()) <= ROUTER_ROUNDING_ROWS * int((~ties).sum()), int(off.sum())
    same = same & ~ties
    d = (h_out.cpu().float() - _bf16(g["block_out"]).float()).abs()
    assert d[same].max() <= BF16_ATOL
    # rows with a different tie pick still equal h + rm * moe(x) of their own routing
    ref = O.residual_add(h, O.local_moe(lb.x, idx.cpu(), gate.cpu(), lb.w_in, lb.w_out),
                         synth.GRANITE_RESIDUAL_MULTIPLIER)
    assert (h_out.cpu().float() - ref.float()).abs().max() <= BF16_ATOL
    be.comm.check()


# ------------------------------------------------------------- edge cases
def test_empty_masked_and_single_hot_expert():
    sh = synth.SHAPES["a"]
    n = 640
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=6, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    x = lb.x.cuda()
    # n = 0: the step still runs (lockstep) and returns an empty tensor
    out0 = be(x[:0], torch.zeros(0, 8, dtype=torch.long, device="cuda"),
              torch.zeros(0, 8, dtype=torch.bfloat16, device="cuda"))
    assert out0.shape == (0, sh["hidden"])
    # every token masked: zeros, no expert rows received
    idx = torch.stack([torch.randperm(32)[:8] for _ in range(n)])
    gate = torch.full((n, 8), 0.125, dtype=torch.bfloat16)
    outm = be(x, idx.cuda(), gate.cuda(), valid_mask=torch.zeros(n, dtype=torch.bool, device="cuda"))
    assert torch.all(outm == 0)
    assert be.comm.last_recv_rows() == 0
    # one expert in every token's first slot: a 640-row segment (5 tiles)
    idx[:, 0] = 31
    idx[:, 1:] = torch.stack([torch.randperm(31)[:7] for _ in range(n)])
    out = be(x, idx.cuda(), gate.cuda()).cpu()
    ref32 = _fp32_ref(lb.x, idx, gate, lb.w_in, lb.w_out)
    assert (out.float() - ref32).abs().max() <= BF16_ATOL
    assert be.comm.last_recv_rows() == n * 8
    be.comm.check()


@pytest.mark.parametrize("n", [16384, 65536])
def test_full_size_workload_properties(n):
    """BASELINE shape (a) at 16K and 64K tokens (64K: more 256-token routing
    rounds than SMs, so routing CTAs take several rounds each): counts exact,
    sampled rows vs the checker."""
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=0, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    x = lb.x.cuda()
    idx, gate = router_topk(be.comm, x, lb.router.cuda(), bias.cuda())
    out = be(x, idx, gate)
    out2 = be(x, idx, gate)
    assert torch.equal(out, out2)  # deterministic, no atomics
    snap = be.stats.snapshot()
    cnt = torch.bincount(idx.reshape(-1).cpu(), minlength=sh["experts"])
    assert snap["route_counts"][0] == (2 * cnt).tolist()
    assert snap["recv_tokens"] == 2 * n * sh["topk"]
    assert int(cnt.max()) > 2 * int(cnt.float().mean())  # skewed, as configured
    rows = torch.randperm(n, generator=torch.Generator().manual_seed(0))[:192]
    ref32 = _fp32_ref(lb.x[rows], idx.cpu()[rows], gate.cpu()[rows], lb.w_in, lb.w_out)
    assert (out.cpu()[rows].float() - ref32).abs().max() <= BF16_ATOL
    assert torch.isfinite(out.float()).all()
    be.comm.check()


def test_device_errors_are_reported_and_recoverable():
    sh = synth.SHAPES["a"]
    n = 64
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n, seed=8, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    x = lb.x.cuda()
    idx = torch.stack([torch.randperm(32)[:8] for _ in range(n)])
    gate = torch.full((n, 8), 0.125, dtype=torch.bfloat16)
    bad = idx.clone()
    bad[3, 2] = 99
    be(x, bad.cuda(), gate.cuda())
    with pytest.raises(MEPError, match="outside"):
        be.comm.check()
    # a wait that nothing satisfies ends with an error instead of hanging
    from miniep_b200 import _lib
    _lib.check(_lib.lib().mep_debug_wait(be.comm._ctx, 0x7fffffff, 200, stream()), be.comm._ctx)
    with pytest.raises(MEPError, match="debug wait"):
        be.comm.check()
    # the context keeps working
    out = be(x, idx.cuda(), gate.cuda()).cpu()
    ref32 = _fp32_ref(lb.x, idx, gate, lb.w_in, lb.w_out)
    assert (out.float() - ref32).abs().max() <= BF16_ATOL
    be.comm.check()


def test_argument_errors():
    sh = synth.SHAPES["a"]
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 8, seed=8, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], 8)
    idx = torch.zeros(16, 8, dtype=torch.long, device="cuda")
    with pytest.raises(MEPError, match="max_tokens"):
        be(torch.zeros(16, 1024, dtype=torch.bfloat16, device="cuda"), idx,
           torch.zeros(16, 8, dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(MEPError, match="CUDA"):
        be(torch.zeros(8, 1024, dtype=torch.float32, device="cuda"), idx[:8],
           torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda"))
    be.local_experts = [0, 1]
    with pytest.raises(MEPError, match="local_experts"):
        be(lb.x.cuda(), idx[:8], torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda"))


def test_graphed_block_replays_match_eager_calls():
    from miniep_b200 import GraphedMoEBlock
    sh = synth.SHAPES["a"]
    n = 512
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 2 * n, seed=9,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0].cuda()
    hs = synth.make_tokens(2 * n, sh["hidden"], seed=10, dtype=torch.bfloat16).cuda()
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    router = lb.router.cuda()
    blk = GraphedMoEBlock(be, n, router, synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
    for part in (0, 1, 0):
        x, h = lb.x[part * n:(part + 1) * n].cuda(), hs[part * n:(part + 1) * n]
        got = blk(x, h).clone()
        want, _, _ = be.moe_block(h, x, router, synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
        assert torch.equal(got, want)
    be.comm.check()


def test_streamed_block_from_host_matches_unchunked_step():
    """Host batches through StreamedMoEBlock (chunked copies overlapping the
    steps, ragged last chunk) give the unchunked step's rows bit for bit, on
    two consecutive calls that reuse the same pinned buffers."""
    from miniep_b200 import StreamedMoEBlock
    sh = synth.SHAPES["a"]
    n = 1000
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 2 * n, seed=12,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0].cuda()
    hs = synth.make_tokens(2 * n, sh["hidden"], seed=13, dtype=torch.bfloat16)
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    router = lb.router.cuda()
    blk = StreamedMoEBlock(be, n, router, synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias, chunks=3)
    assert blk.sizes == [334, 333, 333]
    x_host = torch.empty(n, sh["hidden"], dtype=torch.bfloat16).pin_memory()
    h_host = torch.empty_like(x_host).pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    for part in (1, 0):
        x_host.copy_(lb.x[part * n:(part + 1) * n])
        h_host.copy_(hs[part * n:(part + 1) * n])
        blk(x_host, h_host, out_host)
        torch.cuda.synchronize()
        want, _, _ = be.moe_block(h_host.cuda(), x_host.cuda(), router,
                                  synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
        assert torch.equal(out_host, want.cpu())
    # the whole pipeline as one graph over these buffers: new contents, same rows
    blk.capture(x_host, h_host, out_host)
    for part in (0, 1):
        x_host.copy_(lb.x[part * n:(part + 1) * n])
        h_host.copy_(hs[part * n:(part + 1) * n])
        out_host.zero_()
        blk(x_host, h_host, out_host)
        torch.cuda.synchronize()
        want, _, _ = be.moe_block(h_host.cuda(), x_host.cuda(), router,
                                  synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
        assert torch.equal(out_host, want.cpu())
    be.comm.check()


# ------------------------------------------------------------ block from h
@pytest.mark.parametrize("shape,dtype", [("a", torch.bfloat16), ("b", torch.bfloat16),
                                         ("a", torch.float32)])
def test_rms_norm_matches_reference_formula(shape, dtype):
    """modeling.py:51-52 in the model dtype: fp32 within 1e-6; bf16 mostly equal
    to the checker. The fp32 sum of squares runs in another order than torch's,
    so a row's bf16 mean can round one step apart; its 1/sqrt then moves one
    step and, through the two rounded products, its outputs up to two."""
    from miniep_b200.ep import rms_norm
    sh = synth.SHAPES[shape]
    n, H = 777, sh["hidden"]
    h = synth.make_tokens(n, H, seed=21, dtype=dtype)
    g = torch.Generator().manual_seed(22)
    w = (1.0 + 0.02 * torch.randn(H, generator=g)).to(dtype)
    comm = world1_comm(sh["experts"], sh["topk"], H, sh["inter"], n, dtype)
    x = rms_norm(comm, h.cuda(), w.cuda(), 1e-6).cpu()
    ref = O.rms_norm(h, w, 1e-6)
    if dtype == torch.float32:
        assert (x - ref).abs().max() <= 1e-6 * ref.abs().max()
    else:
        two_ulp = ref.float().abs().clamp_min(2.0 ** -20) * 2.0 ** -6
        assert torch.all((x.float() - ref.float()).abs() <= two_ulp)
        assert (x == ref).float().mean() > 0.99


def test_moe_block_from_h_is_norm_then_block():
    """The fused entry point equals the norm stage followed by the block, bit
    for bit, and its graphed and host-streamed forms equal it too."""
    from miniep_b200 import GraphedMoEBlock, StreamedMoEBlock
    from miniep_b200.ep import rms_norm
    sh = synth.SHAPES["a"]
    n, H = 1000, sh["hidden"]
    lb = synth.make_layer(H, sh["experts"], sh["inter"], n, seed=23, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0].cuda()
    h = synth.make_tokens(n, H, seed=24, dtype=torch.bfloat16).cuda()
    w = (1.0 + 0.02 * torch.randn(H, generator=torch.Generator().manual_seed(25))).to(
        torch.bfloat16).cuda()
    be = world1_backend(lb.w_in, lb.w_out, sh["topk"], n)
    router, rm = lb.router.cuda(), synth.GRANITE_RESIDUAL_MULTIPLIER
    out, idx, gate, x = be.moe_block_from_h(h, w, 1e-6, router, rm, bias=bias)
    x2 = rms_norm(be.comm, h, w, 1e-6)
    assert torch.equal(x, x2)
    want, idx2, gate2 = be.moe_block(h, x2, router, rm, bias=bias)
    assert torch.equal(out, want) and torch.equal(idx, idx2) and torch.equal(gate, gate2)
    # against the checker: an fp32 block on the same normalised rows and routing
    ref32 = O.residual_add(h.float().cpu(), _fp32_ref(x.cpu(), idx.cpu(), gate.cpu(), lb.w_in,
                                                      lb.w_out), rm)
    assert (out.float().cpu() - ref32).abs().max() <= BF16_ATOL * max(1.0, float(ref32.abs().max()))
    blk = GraphedMoEBlock(be, n, router, rm, bias=bias, norm_w=w, eps=1e-6)
    assert torch.equal(blk(h=h).clone(), out)
    sblk = StreamedMoEBlock(be, n, router, rm, bias=bias, chunks=3, norm_w=w, eps=1e-6)
    h_host = h.cpu().pin_memory()
    out_host = torch.empty_like(h_host).pin_memory()
    sblk(None, h_host, out_host)
    torch.cuda.synchronize()
    assert torch.equal(out_host, out.cpu())
    # two buffer sets, calls that do not wait for their output copies: each
    # call's rows once `done` has passed, over consecutive calls
    h2 = synth.make_tokens(n, H, seed=26, dtype=torch.bfloat16).cuda()
    want2, *_ = be.moe_block_from_h(h2, w, 1e-6, router, rm, bias=bias)
    pblk = StreamedMoEBlock(be, n, router, rm, bias=bias, chunks=1, norm_w=w, eps=1e-6, depth=2)
    ins = [h.cpu().pin_memory(), h2.cpu().pin_memory(), h.cpu().pin_memory()]
    outs = [torch.empty_like(ins[0]).pin_memory() for _ in ins]
    for hi, oi in zip(ins, outs):
        pblk(None, hi, oi, wait_output=False)
    torch.cuda.current_stream().wait_event(pblk.done)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], out.cpu()) and torch.equal(outs[2], out.cpu())
    assert torch.equal(outs[1], want2.cpu())
    be.comm.check()
