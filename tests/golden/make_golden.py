"""Generate the golden fixtures in this folder by running the REFERENCE's own
code (kanwarpal-brar/mini-ep, package ``miniep``) on seeded synthetic inputs.

Run once, where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path to the mini-ep checkout>

The fixtures are small ``.npz``/``.json`` files committed beside this script;
the tests that use them never need the reference at run time. What is pinned:

* ``router_local_fp32.npz``   modeling.py:193-195 router + LocalMoEBackend
                               (modeling.py:131-145), shape (a), fp32, 512 tokens.
* ``router_local_bf16.npz``   same in bf16 with the Zipf router bias of layer 0,
                               plus the Block residual (modeling.py:197).
* ``ep_gloo.npz``             EPMoEBackend (ep.py:186-249) over real gloo ranks,
                               world 2 and 4, naive and replicated plans, masked
                               tokens, two calls without reset_rr.
* ``dest_ranks.npz``          Placement.dest_ranks (ep.py:76-96) on the shipped
                               balanced plan, three calls per layer (rr carry-over).
* ``balancer.json``           plan_balanced (balancer.py:63-89): the shipped
                               known answer plus synthetic skewed count matrices.
* ``stats_schema.json``       EPStats.snapshot keys and the straggler figures
                               recomputed from the shipped bench results.
* ``rms_norm.npz``            rms_norm (modeling.py:51-52) in bf16 and fp32 on
                               shape (a) and (b) rows, the post-attention norm of
                               the MoE block (modeling.py:192).
* ``model_tiny.npz``          GraniteMoeModel (modeling.py:148-262) with
                               LocalMoEBackend, driven like the engine's
                               prefill + greedy decode (worker.py:38-138) over a
                               right-padded shard of three prompts, fp32, on a
                               two-layer model with synthetic weights
                               (miniep_b200.model.random_weights).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "mini-ep_b200"))
from miniep_b200 import synth  # noqa: E402


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def row_checksums(t: torch.Tensor) -> np.ndarray:
    t64 = t.double()
    return np.stack([t64.sum(1).numpy(), (t64 * t64).sum(1).numpy()], axis=1)


def gen_router_local(out: Path):
    from miniep.modeling import LocalMoEBackend
    sh = synth.SHAPES["a"]
    H, E, I, k = sh["hidden"], sh["experts"], sh["inter"], sh["topk"]
    # fp32, config 1: 512 tokens, seed 0
    lt = synth.make_layer(H, E, I, 512, seed=0, dtype=torch.float32)
    logits = lt.x @ lt.router.T
    tl, ti = logits.topk(k, dim=-1)
    tg = torch.softmax(tl.float(), dim=-1).to(lt.x.dtype)
    out32 = LocalMoEBackend(lt.w_in, lt.w_out)(lt.x, ti, tg)
    valid = torch.ones(512, dtype=torch.bool)
    valid[5::7] = False
    out32m = LocalMoEBackend(lt.w_in, lt.w_out)(lt.x, ti, tg, valid_mask=valid)
    np.savez_compressed(
        out / "router_local_fp32.npz",
        topk_idx=ti.numpy().astype(np.int8), topk_gate=tg.numpy(), logits=logits.numpy(),
        out_head=out32[:48].numpy(), out_rowsum=row_checksums(out32),
        valid=valid.numpy(), outm_head=out32m[:48].numpy(), outm_rowsum=row_checksums(out32m))

    # bf16 with the layer-0 Zipf bias and the residual add, 128 tokens, seed 0
    lb = synth.make_layer(H, E, I, 128, seed=0, dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, E)[0]
    logits = lb.x @ lb.router.T
    logits = logits + bias.to(logits.dtype)
    tl, ti = logits.topk(k, dim=-1)
    tg = torch.softmax(tl.float(), dim=-1).to(lb.x.dtype)
    moe = LocalMoEBackend(lb.w_in, lb.w_out)(lb.x, ti, tg)
    h = synth.make_tokens(128, H, seed=7, dtype=torch.bfloat16)
    blk = h + moe * synth.GRANITE_RESIDUAL_MULTIPLIER
    np.savez_compressed(
        out / "router_local_bf16.npz",
        topk_idx=ti.numpy().astype(np.int8), topk_gate=bf16_bits(tg), logits=bf16_bits(logits),
        out=bf16_bits(moe), block_out=bf16_bits(blk))


def _ep_worker(rank, world, ref_path, port, cases, result_dir):
    sys.path.insert(0, ref_path)
    import torch.distributed as dist
    from miniep.ep import Comm, EPMoEBackend, EPStats, Placement
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    comm = Comm()
    res = {}
    for name, case in cases.items():
        placement = Placement(case["owners"])
        stats = EPStats(1, case["E"])
        local = placement.experts_of_rank(rank)[0]
        be = EPMoEBackend(0, comm, placement, local, case["w_in"][local], case["w_out"][local],
                          stats)
        outs = []
        placement.reset_rr()
        for call in range(2):  # two calls without reset_rr: rr carries over
            outs.append(be(case["x"][call][rank], case["idx"][call][rank],
                           case["gate"][call][rank], valid_mask=case["valid"][call][rank]))
        snap = stats.snapshot()
        res[name] = dict(outs=[o.numpy() for o in outs],
                         route_counts=np.array(snap["route_counts"]),
                         recv_tokens=snap["recv_tokens"],
                         recv_tokens_per_layer=np.array(snap["recv_tokens_per_layer"]))
    torch.save(res, Path(result_dir) / f"rank{rank}.pt")
    dist.barrier()
    dist.destroy_process_group()


def ep_cases(world: int):
    """Small fp32 layer: H=128, E=16, I=64, k=4, 32 tokens per rank, two calls.
    Shared with the tests, which rebuild the same inputs from the same seeds."""
    H, E, I, k, n = 128, 16, 64, 4, 32
    lt = synth.make_layer(H, E, I, n * world * 2, seed=3, dtype=torch.float32)
    bias = synth.zipf_router_bias(1, E, seed=5)[0]
    logits = lt.x @ lt.router.T + bias
    tl, ti = logits.topk(k, dim=-1)
    tg = torch.softmax(tl.float(), dim=-1)
    per = E // world
    naive = [[[e // per] for e in range(E)]]
    # replicas: hot experts on extra ranks (each owner list sorted, no duplicates)
    rep = [[sorted({e // per, (e + 1) % world} if e % 3 == 0 else {e // per}) for e in range(E)]]
    rep[0][1] = sorted(set(range(world)))  # one expert on every rank
    xs, idxs, gates, valids = [], [], [], []
    for call in range(2):
        base = call * n * world
        xs.append([lt.x[base + r * n: base + (r + 1) * n] for r in range(world)])
        idxs.append([ti[base + r * n: base + (r + 1) * n] for r in range(world)])
        gates.append([tg[base + r * n: base + (r + 1) * n] for r in range(world)])
        vm = []
        for r in range(world):
            v = torch.ones(n, dtype=torch.bool)
            if call == 1:
                v[(r + 1)::5] = False
            vm.append(v)
        valids.append(vm)
    common = dict(E=E, H=H, I=I, k=k, n=n, w_in=lt.w_in, w_out=lt.w_out, x=xs, idx=idxs,
                  gate=gates, valid=valids)
    return {"naive": dict(common, owners=naive), "replicated": dict(common, owners=rep)}


def gen_ep_gloo(ref_path: str, out: Path):
    import tempfile
    import torch.multiprocessing as mp
    save = {}
    for world, port in ((2, 29611), (4, 29612)):
        cases = ep_cases(world)
        with tempfile.TemporaryDirectory() as td:
            mp.spawn(_ep_worker, args=(world, ref_path, port, cases, td), nprocs=world, join=True)
            ranks = [torch.load(Path(td) / f"rank{r}.pt", weights_only=False) for r in range(world)]
        for name in cases:
            key = f"w{world}_{name}"
            save[f"{key}_owners"] = np.array(json.dumps(cases[name]["owners"]))
            for r in range(world):
                rr = ranks[r][name]
                for call in range(2):
                    save[f"{key}_r{r}_c{call}_out"] = rr["outs"][call]
                save[f"{key}_r{r}_route_counts"] = rr["route_counts"]
                save[f"{key}_r{r}_recv_tokens"] = np.array(rr["recv_tokens"])
                save[f"{key}_r{r}_recv_per_layer"] = rr["recv_tokens_per_layer"]
    np.savez_compressed(out / "ep_gloo.npz", **save)


def gen_dest_ranks(ref_root: Path, out: Path):
    from miniep.ep import Placement
    plan = json.loads((ref_root / "results" / "plan_balanced.json").read_text())
    pl = Placement.from_plan(plan)
    g = torch.Generator().manual_seed(11)
    save = {"plan": np.array(json.dumps(plan))}
    pl.reset_rr()
    for layer in range(pl.num_layers):
        for call in range(3):
            m = 64 + 37 * call
            ids = torch.randint(0, pl.num_experts, (m,), generator=g)
            save[f"l{layer}_c{call}_ids"] = ids.numpy().astype(np.int8)
            save[f"l{layer}_c{call}_dest"] = pl.dest_ranks(layer, ids).numpy().astype(np.int8)
        save[f"l{layer}_rr"] = pl._rr[layer].numpy()
    np.savez_compressed(out / "dest_ranks.npz", **save)


def gen_balancer(ref_root: Path, out: Path):
    from miniep.balancer import plan_balanced
    bench = json.loads((ref_root / "results" / "bench_naive.json").read_text())
    counts = sum(torch.tensor(r["stats"]["route_counts"]) for r in bench["ranks"])
    placement, report = plan_balanced(counts, bench["world"], slots_per_rank=2)
    shipped = json.loads((ref_root / "results" / "plan_balanced.json").read_text())
    assert placement.to_plan() == shipped, "reference planner no longer reproduces its shipped plan"
    cases = [dict(name="shipped_bench_naive", world=bench["world"], slots=2,
                  counts=counts.tolist(), plan=shipped, report=report)]
    # synthetic skewed counts at other worlds / budgets
    sh = synth.SHAPES["a"]
    bias = synth.zipf_router_bias(4, sh["experts"])
    g = torch.Generator().manual_seed(21)
    base = torch.randint(50, 150, (4, sh["experts"]), generator=g).double()
    skew = (base * torch.exp(bias.double())).round().long()
    for world in (2, 4, 8):
        for slots in (1, 2, 3):
            pl, rep = plan_balanced(skew, world, slots_per_rank=slots)
            cases.append(dict(name=f"zipf_w{world}_s{slots}", world=world, slots=slots,
                              counts=skew.tolist(), plan=pl.to_plan(), report=rep))
    (out / "balancer.json").write_text(json.dumps(cases))


MODEL_TINY = dict(
    hidden_size=256, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
    num_key_value_heads=2, num_local_experts=8, num_experts_per_tok=2, vocab_size=512,
    rms_norm_eps=1e-6, rope_theta=10000.0, embedding_multiplier=12.0,
    attention_multiplier=0.015625, residual_multiplier=0.22, logits_scaling=6.0,
    max_position_embeddings=256)
MODEL_TINY_PROMPT_LENS = (7, 12, 4)
MODEL_TINY_NEW = 6


def gen_model(out: Path):
    from miniep.modeling import GraniteMoeModel, LocalMoEBackend, ModelConfig
    from miniep.worker import Shard
    from miniep_b200.model import ModelConfig as Cfg, expert_weight_keys, random_weights
    cfg = ModelConfig(**MODEL_TINY)
    w = random_weights(Cfg.from_dict(MODEL_TINY), seed=5, dtype=torch.float32)
    backends = [LocalMoEBackend(w[a], w[b]) for a, b in map(expert_weight_keys, range(2))]
    model = GraniteMoeModel(cfg, w, backends)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(1, cfg.vocab_size, (n,), generator=g).tolist()
               for n in MODEL_TINY_PROMPT_LENS]
    shard = Shard(prompts, cfg.num_hidden_layers, pad_id=cfg.pad_token_id)
    with torch.no_grad():
        # Engine.prefill (worker.py:100-112)
        mask, moe_valid = shard.prefill_masks()
        logits = model(shard.input, kv_cache=shard.kv, attn_mask=mask, moe_valid=moe_valid,
                       logits_at=shard.lengths - 1)
        prefill = logits[:, 0].clone()
        shard.last_tokens = prefill.argmax(dim=-1)
        steps = []
        # Engine.decode_step (worker.py:126-138), all rows active
        for _ in range(MODEL_TINY_NEW):
            for i in range(shard.B):
                shard.generated[i].append(int(shard.last_tokens[i]))
            mask, _ = shard.decode_masks()
            logits = model(shard.last_tokens.unsqueeze(1), positions=shard.positions_decode(),
                           kv_cache=shard.kv, attn_mask=mask)
            steps.append(logits[:, -1].clone())
            shard.last_tokens = logits[:, -1].argmax(dim=-1)
            shard.decoded_steps += 1
    allv = torch.cat([prefill[None], torch.stack(steps)])  # (1+steps, B, V)
    top2 = allv.topk(2, dim=-1).values
    gap = float((top2[..., 0] - top2[..., 1]).min())
    assert gap > 1e-3, f"greedy choice too close to a tie ({gap})"
    np.savez_compressed(out / "model_tiny.npz", config=json.dumps(MODEL_TINY),
                        prompt_lens=np.array(MODEL_TINY_PROMPT_LENS),
                        prompts=np.array(sum(prompts, [])), generated=np.array(shard.generated),
                        prefill_logits=prefill.numpy(), decode_logits=torch.stack(steps).numpy(),
                        min_top2_gap=gap)


def gen_rms_norm(out: Path):
    from miniep.modeling import rms_norm
    res = {}
    for shape in ("a", "b"):
        H = synth.SHAPES[shape]["hidden"]
        g = torch.Generator().manual_seed(31)
        h = torch.randn(16, H, generator=g)
        w = 1.0 + 0.02 * torch.randn(H, generator=g)
        for name, dt in (("bf16", torch.bfloat16), ("fp32", torch.float32)):
            hd, wd = h.to(dt), w.to(dt)
            y = rms_norm(hd, wd, 1e-6)
            res[f"{shape}_{name}_h"] = bf16_bits(hd) if dt == torch.bfloat16 else hd.numpy()
            res[f"{shape}_{name}_w"] = bf16_bits(wd) if dt == torch.bfloat16 else wd.numpy()
            res[f"{shape}_{name}_y"] = bf16_bits(y) if dt == torch.bfloat16 else y.numpy()
    np.savez_compressed(out / "rms_norm.npz", **res)


def gen_stats(ref_root: Path, out: Path):
    res = {}
    for name in ("naive", "balanced"):
        b = json.loads((ref_root / "results" / f"bench_{name}.json").read_text())
        loads = np.array([r["stats"]["recv_tokens_per_layer"] for r in b["ranks"]])  # (W, L)
        strag = loads.max(0).sum() / loads.mean(0).sum() - 1
        per_layer = loads.max(0) / loads.mean(0)
        res[name] = dict(world=b["world"], recv_tokens_per_layer=loads.tolist(),
                         straggler=float(strag), imbalance_avg=float(per_layer.mean()),
                         imbalance_worst=float(per_layer.max()),
                         snapshot_keys=sorted(b["ranks"][0]["stats"].keys()),
                         bench_keys=list(b.keys()), rank_keys=list(b["ranks"][0].keys()),
                         recv_tokens=[r["stats"]["recv_tokens"] for r in b["ranks"]],
                         positions=[r["positions"] for r in b["ranks"]],
                         wall_time=b["wall_time"], positions_per_s=b["positions_per_s"])
    nb = json.loads((ref_root / "results" / "bench_naive.json").read_text())
    bb = json.loads((ref_root / "results" / "bench_balanced.json").read_text())
    res["route_counts_placement_invariant"] = all(
        a["stats"]["route_counts"] == c["stats"]["route_counts"]
        for a, c in zip(nb["ranks"], bb["ranks"]))
    (out / "stats_schema.json").write_text(json.dumps(res))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the mini-ep checkout")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    ref_root = Path(args.reference).resolve()
    sys.path.insert(0, str(ref_root))
    torch.set_num_threads(8)
    steps = {
        "router_local": lambda: gen_router_local(HERE),
        "ep_gloo": lambda: gen_ep_gloo(str(ref_root), HERE),
        "dest_ranks": lambda: gen_dest_ranks(ref_root, HERE),
        "balancer": lambda: gen_balancer(ref_root, HERE),
        "stats": lambda: gen_stats(ref_root, HERE),
        "model": lambda: gen_model(HERE),
        "rms_norm": lambda: gen_rms_norm(HERE),
    }
    for name, fn in steps.items():
        if args.only and name not in args.only.split(","):
            continue
        fn()
        print("wrote", name)


if __name__ == "__main__":
    main()
