"""End-to-end GraniteMoE serving workloads on B200:
a 24-layer Granite-3.0-1B-A400M-shaped decoder with synthetic weights, every
MoE layer on the expert-parallel CUDA layer, one process per GPU.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 \\
        -m miniep_b200.model_bench --config 2 [--plan naive|balanced|lpt]

  config 2: prefill 8 sequences x 256 random token ids, 32 greedy steps
  config 3: 16 x 512 prefill, 32 greedy steps, Zipf(1.2) router bias per layer;
            run under naive placement, then the balancer's plan and the LPT plan
            from the first run's route counts (2 slots per rank): continuations
            must be identical across the three
  config 4: 64 sequences over a 1024-token random context, 128 decode steps of
            one token per sequence; reports the latency per decode step

Sequences are dealt to ranks round-robin (worker.py:145-146); throughput is
tok-pos/s as the reference counts it (worker.py:214-217: valid prompt
positions plus decode positions, over the wall time of the run). Rank 0
prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch
import torch.distributed as dist

from . import Comm, EPMoEBackend, EPStats, Placement, plan_balanced, plan_lpt, synth
from .model import (GRANITE_1B_A400M, DeviceModel, Engine, ModelConfig, Shard,
                    expert_weight_keys, random_weights)

CONFIGS = {2: dict(seqs=8, prompt=256, new=32, zipf=False),
           3: dict(seqs=16, prompt=512, new=32, zipf=True),
           4: dict(seqs=64, prompt=1024, new=128, zipf=False)}


def _setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _run(cfg, w, placement, prompts, new, biases, rank, local, graphed):
    L, E = cfg.num_hidden_layers, cfg.num_local_experts
    max_tokens = max(1, len(prompts)) * max(len(p) for p in prompts) if prompts else 4
    comm = Comm(num_layers=L, num_experts=E, topk=cfg.num_experts_per_tok, hidden=cfg.hidden_size,
                inter=cfg.intermediate_size, max_tokens=max_tokens, dtype=torch.bfloat16,
                device=local, timeout_ms=60000)
    comm.install(placement)
    stats = EPStats(L, E)
    mine = placement.experts_of_rank(rank)
    backends = []
    for l in range(L):
        a, b = expert_weight_keys(l)
        backends.append(EPMoEBackend(l, comm, placement, mine[l], w[a][mine[l]].cuda(),
                                     w[b][mine[l]].cuda(), stats))

    def moe(l):
        be, bias = backends[l], (None if biases is None else biases[l].cuda())

        def run(h, x, router_w, rm, valid):
            return be.moe_block(h, x, router_w, rm, bias=bias, valid_mask=valid)[0]
        return run

    dense = {k: v.cuda() for k, v in w.items() if ".block_sparse_moe.input_linear" not in k
             and ".block_sparse_moe.output_linear" not in k}
    model = DeviceModel(cfg, dense, [moe(l) for l in range(L)])
    eng = Engine(model, reset_rr=placement.reset_rr)
    dummy = not prompts
    shard = Shard(prompts if prompts else [[1, 2, 3, 4]], cfg, new, "cuda", torch.bfloat16)
    # warm-up, untimed, on a scratch shard of the same shape: a full prefill and
    # two decode steps (kernel selection, library set-up, graph capture)
    warm = Shard(prompts if prompts else [[1, 2, 3, 4]], cfg, 2, "cuda", torch.bfloat16)
    weng = Engine(model, reset_rr=placement.reset_rr)
    weng.prefill(warm, dummy=dummy)
    if graphed:
        weng.decode_graphed(warm, 2, idle=dummy)
    else:
        for _ in range(2):
            weng.decode_step(warm, active=torch.zeros(warm.B, dtype=torch.bool, device="cuda")
                             if dummy else None)
    del warm
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    t0 = time.perf_counter()
    eng.prefill(shard, dummy=dummy)
    torch.cuda.synchronize()
    t_prefill = time.perf_counter() - t0
    if graphed:
        eng.decode_graphed(shard, new, idle=dummy)
    else:
        for _ in range(new):
            eng.decode_step(shard, active=torch.zeros(shard.B, dtype=torch.bool, device="cuda")
                            if dummy else None)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    positions = 0 if dummy else int(shard.lengths.sum()) + shard.B * new
    comm.check()
    out = dict(generated=shard.generated if not dummy else [], positions=positions, wall=wall,
               prefill_s=t_prefill, decode_s=wall - t_prefill,
               route_counts=stats.route_counts.clone())
    comm.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--plan", choices=["naive", "balanced", "lpt"], default="naive",
                    help="placement re-planned from the naive run's counts (config 3 runs both)")
    ap.add_argument("--eager-decode", action="store_true",
                    help="launch each decode step op by op instead of one graph replay")
    a = ap.parse_args()
    world, rank, local = _setup()
    c = CONFIGS[a.config]
    cfg = ModelConfig.from_dict(dict(GRANITE_1B_A400M, num_hidden_layers=a.layers))
    w = random_weights(cfg, seed=0, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    all_prompts = [torch.randint(1, cfg.vocab_size, (c["prompt"],), generator=g).tolist()
                   for _ in range(c["seqs"])]
    prompts = [p for i, p in enumerate(all_prompts) if i % world == rank]
    biases = synth.zipf_router_bias(cfg.num_hidden_layers, cfg.num_local_experts) \
        if c["zipf"] else None
    naive = Placement.naive(cfg.num_hidden_layers, cfg.num_local_experts, world)
    graphed = not a.eager_decode
    res = _run(cfg, w, naive, prompts, c["new"], biases, rank, local, graphed)
    runs = {"naive": res}
    wanted = ["balanced", "lpt"] if a.config == 3 else [a.plan]
    wanted = [p for p in wanted if p != "naive"]
    if wanted:
        counts = res["route_counts"].cuda()
        if world > 1:
            dist.all_reduce(counts)
    for name in wanted:
        planner = plan_balanced if name == "balanced" else plan_lpt
        plan, _ = planner(counts.cpu(), world, slots_per_rank=2)
        runs[name] = _run(cfg, w, plan, prompts, c["new"], biases, rank, local, graphed)
    # whole-job figures: positions summed, wall time max over ranks
    out = {}
    for name, r in runs.items():
        t = torch.tensor([r["positions"], r["wall"], r["prefill_s"], r["decode_s"]],
                         dtype=torch.float64, device="cuda")
        if world > 1:
            pos = t[:1].clone()
            dist.all_reduce(pos)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t[0] = pos[0]
        out[name] = t.tolist()
    same = None
    if len(runs) > 1:
        flag = torch.tensor([int(all(r["generated"] == runs["naive"]["generated"]
                                     for r in runs.values()))], device="cuda")
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        same = bool(flag.item())
    if rank == 0:
        line = {"metric": "e2e tok-pos/s", "config": a.config, "world": world,
                "decode": "eager" if a.eager_decode else "one CUDA graph replay per step",
                "layers": cfg.num_hidden_layers, "dtype": "bf16", "data": "synthetic",
                "sequences": c["seqs"], "prompt_len": c["prompt"], "new_tokens": c["new"]}
        for name, (pos, wall, pre, dec) in out.items():
            line[name] = {"tok_pos_per_s": pos / wall, "positions": int(pos), "wall_s": wall,
                          "prefill_s": pre, "decode_ms_per_step": dec / c["new"] * 1e3}
        if same is not None:
            line["greedy_identical_across_plans"] = same
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
