"""NVLink bandwidth of the layer's all-to-alls, against NCCL on the same bytes.

    torchrun --nproc-per-node N -m miniep_b200.a2a_bench [--tokens 1024,4096,16384,65536]

For each token count (all ranks together, shape (a) or (b), Zipf router,
``plan_lpt`` placement) it runs the expert-parallel MoE block with the step
timeline on and reports, per rank, the bytes that cross NVLink and the stage
times of the two exchanges:

* dispatch: the kernel-issued bulk copies of token rows to the owner ranks'
  landing buffers, one row per (token, remote destination rank);
* return: GEMM2's epilogue stores of expert output rows to their source
  ranks, one row per remote (token, slot) entry, overlapped with the
  tensor-core work of the same kernel (so its rate is a lower bound).

Next to each it times ``torch.distributed.all_to_all_single`` (NCCL over
NVLink) moving the same number of bytes from every rank, split evenly over
the peers: the reference's ``Comm.all_to_all`` (miniep/ep.py:126-136) done by
the library the layer could have called instead. Rank 0 prints one JSON line
per token count and a summary table (GB/s per GPU, max over ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch
import torch.distributed as dist

from . import Comm, EPMoEBackend, GraphedMoEBlock, Placement, plan_lpt, synth
from .ep import rms_norm, router_topk


def nccl_a2a_us(send_bytes: int, world: int, dev, reps: int = 20) -> float:
    """Median device time (us, max over ranks) of one all_to_all_single that
    sends send_bytes from this rank, split evenly over the other ranks."""
    per = max(16, send_bytes // max(world - 1, 1) // 16 * 16)
    splits = [0 if r == dist.get_rank() else per for r in range(world)]
    inp = torch.empty(per * (world - 1), dtype=torch.uint8, device=dev)
    out = torch.empty_like(inp)
    for _ in range(3):
        dist.all_to_all_single(out, inp, splits, splits)
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dist.all_to_all_single(out, inp, splits, splits)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    t = torch.tensor([statistics.median(times)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1024,4096,16384,65536")
    ap.add_argument("--shape", choices=["a", "b"], default="a")
    ap.add_argument("--steps", type=int, default=10)
    a = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        raise SystemExit("run under torchrun with 2 or more GPUs")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sh = synth.SHAPES[a.shape]
    H, E, k, I = sh["hidden"], sh["experts"], sh["topk"], sh["inter"]
    lt = synth.make_layer(H, E, I, 1, seed=0, dtype=torch.bfloat16)
    router = lt.router.to(dev)
    bias = synth.zipf_router_bias(1, E)[0].to(dev)
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    rows = []
    for tokens in [int(t) for t in a.tokens.split(",")]:
        start, stop = synth.split_tokens(tokens, world, rank)
        n = stop - start
        h = synth.make_tokens(tokens, H, seed=7, dtype=torch.bfloat16)[start:stop].to(dev)
        comm = Comm(num_layers=1, num_experts=E, topk=k, hidden=H, inter=I, max_tokens=n,
                    dtype=torch.bfloat16, device=local, timeout_ms=20000)
        comm.install(Placement.naive(1, E, world))
        idx, _ = router_topk(comm, rms_norm(comm, h, nw, 1e-6), router, bias)
        counts = torch.bincount(idx.reshape(-1), minlength=E)
        dist.all_reduce(counts)
        placement, _ = plan_lpt(counts.view(1, E).cpu(), world)
        comm.install(placement)
        mine = placement.experts_of_rank(rank)[0]
        be = EPMoEBackend(0, comm, placement, mine, lt.w_in[mine].to(dev),
                          lt.w_out[mine].to(dev), None)
        # bytes over NVLink from this rank: dispatch rows (one per token and
        # remote destination rank), return rows (one per remote entry it owns)
        table, n_rep = placement.table(0)
        dest = placement.dest_ranks(0, idx.reshape(-1)).view(n, k).cpu()
        placement.reset_rr()
        remote_rows = sum(len(set(d) - {rank}) for d in dest.tolist())
        comm.set_option("timeline", 1)
        blk = GraphedMoEBlock(be, n, router, 0.22, bias=bias, norm_w=nw)
        blk.h.copy_(h)
        comm.read_timeline()
        recs = []
        for _ in range(a.steps):
            comm.barrier()
            blk()
            recs.append(comm.read_timeline())
        recv_total = comm.last_recv_rows()
        del blk
        comm.set_option("timeline", 0)
        med = lambda key: statistics.median(r[key][1] - r[key][0] for r in recs)  # noqa: E731
        local_entries = int((dest == rank).sum())
        mine_stats = torch.tensor([remote_rows * 2.0 * H, med("dispatch"),
                                   (recv_total - local_entries) * 2.0 * H, med("gemm2")],
                                  device=dev, dtype=torch.float64)
        parts = [torch.zeros_like(mine_stats) for _ in range(world)]
        dist.all_gather(parts, mine_stats)
        per = torch.stack(parts).cpu()
        disp_bytes = int(per[:, 0].max())
        ret_bytes = int(per[:, 2].max())
        row = {
            "tokens": tokens, "world": world, "shape": a.shape,
            "dispatch_bytes_max_rank": disp_bytes,
            "dispatch_us_max_rank": float(per[:, 1].max()),
            "dispatch_gbs_per_gpu": disp_bytes / (float(per[:, 1].max()) * 1e-6) / 1e9,
            "return_bytes_max_rank": ret_bytes,
            "gemm2_us_max_rank": float(per[:, 3].max()),
            "return_gbs_per_gpu_lower_bound": ret_bytes / (float(per[:, 3].max()) * 1e-6) / 1e9,
        }
        for name, b in (("dispatch", disp_bytes), ("return", ret_bytes)):
            us = nccl_a2a_us(b, world, dev)
            row[f"nccl_{name}_us"] = us
            row[f"nccl_{name}_gbs_per_gpu"] = b / (us * 1e-6) / 1e9
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
        comm.close()
    if rank == 0:
        print("| tokens | dispatch MB | P2P dispatch GB/s | NCCL a2a GB/s | return MB | "
              "P2P return GB/s (lower bound) | NCCL a2a GB/s |")
        print("|---|---|---|---|---|---|---|")
        for r in rows:
            print(f"| {r['tokens']} | {r['dispatch_bytes_max_rank'] / 1e6:.1f} | "
                  f"{r['dispatch_gbs_per_gpu']:.0f} | {r['nccl_dispatch_gbs_per_gpu']:.0f} | "
                  f"{r['return_bytes_max_rank'] / 1e6:.1f} | "
                  f"{r['return_gbs_per_gpu_lower_bound']:.0f} | "
                  f"{r['nccl_return_gbs_per_gpu']:.0f} |")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
