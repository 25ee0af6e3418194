"""MoE-layer scaling sweep: throughput of the expert-parallel
block step against the layer roofline, over shapes, token counts and plans.

    python -m miniep_b200.sweep [--shapes a,b] [--tokens 1024,4096,16384,65536]
    torchrun --nproc-per-node N -m miniep_b200.sweep --plans naive,balanced,lpt

For every (shape, tokens, plan) it builds the layer (seeded weights drawn on
the GPU: same distribution as the bench's, other values), runs a profiling
pass over the step's tokens for the plan's counts, then times the graphed
block step from h (RMSNorm, router, route, dispatch, experts, combine,
residual) with L2 flushed between steps, max over ranks. Each line reports
tokens/s, the layer roofline max(T_tc, T_nv) with both terms (the north
star's definition: expert FLOPs at the measured burst bf16 peak; dispatch
plus combine rows of the busiest rank, one row per remote entry, at 900 GB/s
per direction), the straggler figure, and (with --timeline) the median
per-stage times of rank 0. Rank 0 prints one JSON line per configuration and
a markdown table at the end.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

from . import (Comm, EPMoEBackend, GraphedMoEBlock, Placement, plan_balanced, plan_lpt,
               straggler_overhead, synth)
from .ep import rms_norm, router_topk

NVLINK_GBS = 900.0


def peak_tflops() -> float:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="a,b")
    ap.add_argument("--tokens", default="1024,4096,16384,65536")
    ap.add_argument("--plans", default="naive,balanced,lpt")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--timeline", action="store_true")
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    peak = peak_tflops()
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    plans = a.plans.split(",") if world > 1 else ["naive"]
    rows = []
    for shape in a.shapes.split(","):
        sh = synth.SHAPES[shape]
        H, E, k, I = sh["hidden"], sh["experts"], sh["topk"], sh["inter"]
        lt = synth.make_layer(H, E, I, 1, seed=0, dtype=torch.bfloat16, device=dev)
        bias = synth.zipf_router_bias(1, E)[0].to(dev)
        nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
        f_tok = 6.0 * k * H * I + 2.0 * H * E
        for tokens in [int(t) for t in a.tokens.split(",")]:
            start, stop = synth.split_tokens(tokens, world, rank)
            n = stop - start
            h = synth.make_tokens(tokens, H, seed=7, dtype=torch.bfloat16,
                                  device=dev)[start:stop].contiguous()
            comm = Comm(num_layers=1, num_experts=E, topk=k, hidden=H, inter=I, max_tokens=n,
                        dtype=torch.bfloat16, device=local, timeout_ms=30000)
            comm.install(Placement.naive(1, E, world))
            idx, _ = router_topk(comm, rms_norm(comm, h, nw, 1e-6), lt.router, bias)
            counts = torch.bincount(idx.reshape(-1), minlength=E)
            if world > 1:
                dist.all_reduce(counts)
            for plan_name in plans:
                if plan_name == "naive":
                    placement, predicted = Placement.naive(1, E, world), None
                else:
                    fn = plan_balanced if plan_name == "balanced" else plan_lpt
                    placement, rep = fn(counts.view(1, E).cpu(), world, slots_per_rank=2)
                    predicted = rep["layers"][0]["imbalance_after"] - 1.0
                comm.install(placement)
                mine = placement.experts_of_rank(rank)[0]
                be = EPMoEBackend(0, comm, placement, mine, lt.w_in[mine].contiguous(),
                                  lt.w_out[mine].contiguous(), None)
                # remote entries each way (one row per entry), round-robin state at zero
                dest = placement.dest_ranks(0, idx.reshape(-1)).cpu()
                placement.reset_rr()
                per_dest = torch.bincount(dest, minlength=world).to(torch.float64)
                mine_t = torch.cat([per_dest, torch.zeros(1, dtype=torch.float64)]).to(dev)
                comm.set_option("timeline", 1 if a.timeline else 0)
                blk = GraphedMoEBlock(be, n, lt.router, 0.22, bias=bias, norm_w=nw)
                comm.set_option("timeline", 0)
                blk.h.copy_(h)
                for _ in range(a.warmup):
                    blk()
                comm.read_timeline()
                times, recs = [], []
                if world > 1:
                    dist.barrier()
                for _ in range(a.steps):
                    flush.zero_()
                    if world > 1:
                        comm.barrier()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    blk()
                    e1.record()
                    if a.timeline:
                        recs.append(comm.read_timeline())
                    times.append((e0, e1))
                torch.cuda.synchronize()
                comm.check()
                ms = sum(s.elapsed_time(e) for s, e in times) / a.steps
                recv = float(comm.last_recv_rows())
                mine_t[world] = recv
                t = torch.tensor([ms], device=dev, dtype=torch.float64)
                if world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    parts = [torch.zeros_like(mine_t) for _ in range(world)]
                    dist.all_gather(parts, mine_t)
                else:
                    parts = [mine_t]
                ms = float(t)
                del blk
                if rank == 0:
                    m = torch.stack(parts).cpu()  # [src][dest counts..., recv]
                    sent = [float(m[r, :world].sum() - m[r, r]) for r in range(world)]
                    got = [float(m[:, r].sum() - m[r, r]) for r in range(world)]
                    nv = max(2.0 * max(s, g) * H * 2.0 for s, g in zip(sent, got))
                    t_tc = tokens * f_tok / world / (peak * 1e12) * 1e6
                    t_nv = nv / (NVLINK_GBS * 1e9) * 1e6
                    roof = max(t_tc, t_nv)
                    recvs = [[float(m[r, world])] for r in range(world)]
                    row = {"shape": shape, "tokens": tokens, "world": world, "plan": plan_name,
                           "ms_per_step": ms, "tokens_per_s": tokens / (ms / 1e3),
                           "t_tc_us": t_tc, "t_nv_us": t_nv,
                           "roofline_tokens_per_s": tokens / (roof / 1e6),
                           "roofline_frac": roof / (ms * 1e3),
                           "straggler_pct": 100.0 * straggler_overhead(recvs),
                           "planner_predicted_pct": None if predicted is None
                           else 100.0 * predicted}
                    if recs:
                        row["stages_us_rank0"] = {
                            key: round(statistics.median(r[key][1] - r[key][0] for r in recs), 1)
                            for key in recs[0] if isinstance(recs[0][key], tuple)}
                    rows.append(row)
                    print(json.dumps(row), flush=True)
            comm.close()
            del h
        del lt
        torch.cuda.empty_cache()
    if rank == 0:
        print("| shape | tokens | GPUs | plan | ms/step | M tokens/s | T_tc us | T_nv us | "
              "of roofline | straggler % |")
        print("|---|---|---|---|---|---|---|---|---|---|")
        for r in rows:
            print(f"| {r['shape']} | {r['tokens']} | {r['world']} | {r['plan']} | "
                  f"{r['ms_per_step']:.3f} | {r['tokens_per_s'] / 1e6:.1f} | {r['t_tc_us']:.0f} | "
                  f"{r['t_nv_us']:.0f} | {r['roofline_frac']:.2f} | {r['straggler_pct']:.1f} |")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
