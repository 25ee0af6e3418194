"""MoE-layer throughput on B200: one expert-parallel GraniteMoE-shaped MoE block
step from the residual stream h (post-attention RMSNorm + router + route +
dispatch + grouped SwiGLU experts + combine + residual, modeling.py:192-197).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (shape (a)): hidden 1024, 32 experts, top-8,
intermediate 512, bf16, Zipf(1.2)-skewed router (layer-0 bias), 16384 tokens
per step in total, split evenly over the ranks (strong scaling), balanced
replica plan (2 slots per rank) from a naive profiling pass when N > 1.
Seeded synthetic tensors stand in for the checkpoint and prompts.

Prints one JSON line (rank 0). `value` is whole-job tokens/s of the device
step (inputs resident in HBM, L2 flushed between steps, per-step CUDA events,
max over ranks); `e2e` is the same metric through the public API with the
step's inputs copied from pinned host memory and its output copied back
inside the timed region (h is the block's only input). `--impl reference`
times the CPU checker's restatement of the reference's block (RMSNorm,
router, LocalMoEBackend, residual) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / "mini-ep_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import torch  # noqa: E402

METRIC = "MoE layer tokens/s"
UNIT = "tokens/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes (read + write) of the expert FFN stage (both tcgen05 launches) per
# layer step, from one ncu capture of this bench at N=1 (profiles/
# ffn_tc_shape_a_16k_dram.txt): keyed by (shape, tokens per step)
FFN_DRAM_BYTES = {("a", 16384): 325.20e6 + 110.93e6 + 163.11e6 + 215.29e6}
# norm, router, routing (+ layout), dispatch, gemm1, gemm2, combine (+ data wait and fan-out when N > 1)
KERNELS_PER_STEP = 7


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--shape", choices=["a", "b"], default="a")
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per step, all ranks")
    ap.add_argument("--plan", choices=["naive", "balanced"], default="balanced")
    ap.add_argument("--cpu-sample", type=int, default=2048, help="tokens per CPU sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=0,
                    help="pieces per host batch in the e2e leg (0: 4 from 4096 tokens per rank, else 2)")
    ap.add_argument("--force-simt", action="store_true")
    ap.add_argument("--e2e-graph", choices=["on", "off"], default="off",
                    help="capture the e2e host pipeline as one CUDA graph per step "
                         "(measured slower at N=1 and 2: consecutive steps stop overlapping)")
    ap.add_argument("--report", default=None,
                    help="also write a bench report in the reference's results/bench_*.json layout")
    return ap.parse_args()


def workload_name(a) -> str:
    return f"moe_layer_shape_{a.shape}_{a.tokens}tok_zipf1.2_{a.plan}"


def config(a, sh) -> dict:
    return {"workload": workload_name(a), "tokens_per_step": a.tokens, "hidden": sh["hidden"],
            "experts": sh["experts"], "topk": sh["topk"], "inter": sh["inter"],
            "block": "post-attention RMSNorm + router + experts + residual from h "
                     "(modeling.py:192-197)",
            "router": "zipf(1.2) bias x2.0, layer 0", "placement": a.plan,
            "l2": "flushed between timed steps (512 MiB write + 256 MiB read, outside the step events)"}


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None
            return
        # the timed region starts once sampling runs
        t0 = time.perf_counter()
        while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 5.0:
            time.sleep(0.02)
        self.lines.clear()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        time.sleep(0.05)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# --------------------------------------------------------------- CPU legs
def cpu_sample_inputs(sh, n_tokens, seed=0):
    from miniep_b200 import synth
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], n_tokens, seed=seed,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    h = synth.make_tokens(n_tokens, sh["hidden"], seed=seed + 7, dtype=torch.bfloat16)
    return lb, bias, h


NORM_EPS = 1e-6


def norm_weight(hidden: int, device=None):
    """Synthetic post-attention RMSNorm weight: 1 + N(0, 1) * 0.02 (seed 8)."""
    g = torch.Generator().manual_seed(8)
    return (1.0 + 0.02 * torch.randn(hidden, generator=g)).to(torch.bfloat16).to(device)


def cpu_step(oracle, lb, bias, h, k):
    from miniep_b200 import synth
    out, _, _, _ = oracle.moe_block_from_h(h, norm_weight(h.shape[1]), NORM_EPS, lb.router,
                                           lb.w_in, lb.w_out, k,
                                           synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
    return out


def cpu_baseline(sh, sample_tokens, min_seconds=10.0, max_reps=2000) -> dict:
    """The CPU checker's restatement of the reference path (router +
    LocalMoEBackend + residual) on this host's cores, on a bounded sample."""
    from oracle import moe_oracle
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    lb, bias, h = cpu_sample_inputs(sh, sample_tokens)
    cpu_step(moe_oracle, lb, bias, h, sh["topk"])  # warm-up
    reps, t0 = 0, time.perf_counter()
    while reps < max_reps:
        cpu_step(moe_oracle, lb, bias, h, sh["topk"])
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": reps * sample_tokens / dt, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{reps} x {sample_tokens} tokens of the same workload (bf16, shape, "
                      f"Zipf router) through oracle.moe_block_from_h, {dt:.1f} s"}


def run_reference(a):
    """--impl reference: the CPU path of the reference, timed on host cores."""
    from miniep_b200 import synth
    from oracle import moe_oracle
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sh = synth.SHAPES[a.shape]
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    sample = min(a.cpu_sample, a.tokens)
    lb, bias, h = cpu_sample_inputs(sh, sample)
    for _ in range(a.warmup):
        cpu_step(moe_oracle, lb, bias, h, sh["topk"])
    t0 = time.perf_counter()
    for _ in range(a.steps):
        cpu_step(moe_oracle, lb, bias, h, sh["topk"])
    dt = time.perf_counter() - t0
    value = a.steps * sample / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": dt / a.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config(a, sh),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{sample} tokens per step through oracle.moe_block_from_h "
                                   f"(router + LocalMoEBackend + residual restated in torch CPU)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU leg
def main_b200(a):
    import torch.distributed as dist
    from miniep_b200 import (Comm, EPMoEBackend, EPStats, GraphedMoEBlock, Placement,
                             StreamedMoEBlock, _lib, plan_balanced, report, straggler_overhead,
                             synth)
    from miniep_b200.ep import rms_norm, router_topk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)
    sh = synth.SHAPES[a.shape]
    H, E, k, I = sh["hidden"], sh["experts"], sh["topk"], sh["inter"]
    start, stop = synth.split_tokens(a.tokens, world, rank)
    n = stop - start
    # same weights on every rank (same seed), each rank its own token shard
    lt = synth.make_layer(H, E, I, a.tokens, seed=0, dtype=torch.bfloat16, device=dev)
    bias = synth.zipf_router_bias(1, E)[0].to(dev)
    h = synth.make_tokens(a.tokens, H, seed=7, dtype=torch.bfloat16, device=dev)[start:stop].contiguous()
    nw = norm_weight(H, dev)
    rm = synth.GRANITE_RESIDUAL_MULTIPLIER

    comm = Comm(num_layers=1, num_experts=E, topk=k, hidden=H, inter=I, max_tokens=n,
                dtype=torch.bfloat16, device=local, timeout_ms=20000)
    if a.force_simt:
        comm.set_option("force_simt", 1)
    placement = Placement.naive(1, E, world)
    counts = None
    if world > 1 and a.plan == "balanced":
        comm.install(placement)
        idx, _ = router_topk(comm, rms_norm(comm, h, nw, NORM_EPS), lt.router, bias)
        counts = torch.bincount(idx.reshape(-1), minlength=E).to(torch.int64)
        dist.all_reduce(counts)
        placement, _ = plan_balanced(counts.view(1, E).cpu(), world, slots_per_rank=2)
    comm.install(placement)
    mine = placement.experts_of_rank(rank)[0]
    w_in, w_out = lt.w_in[mine].contiguous(), lt.w_out[mine].contiguous()
    lt_router = lt.router.contiguous()
    del lt
    stats = EPStats(1, E)  # device counters; the report covers the timed graph steps only
    be = EPMoEBackend(0, comm, placement, mine, w_in, w_out, stats)

    L, ctx = _lib.lib(), comm._ctx
    idx = torch.empty(n, k, dtype=torch.int64, device=dev)
    gate = torch.empty(n, k, dtype=torch.bfloat16, device=dev)
    h_out = torch.empty_like(h)
    P = _lib.ptr
    # L2 flush between steps: write 512 MiB, then read 256 MiB so that the
    # written lines are evicted (written back) before the step, not during it
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    flush_rd = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def flush_l2():
        flush.zero_()
        flush_rd.sum()

    x = torch.empty_like(h)

    def eager_step(st, ev_ffn=None):
        # mep_moe_block_from_h's sequence, with events around the expert FFN stage
        _lib.check(L.mep_rmsnorm(ctx, P(h), P(nw), NORM_EPS, n, P(x), st), ctx)
        _lib.check(L.mep_router_topk(ctx, P(x), P(lt_router), P(bias), n, P(idx), P(gate),
                                     None, st), ctx)
        _lib.check(L.mep_route(ctx, 0, P(idx), None, n, len(mine), st), ctx)
        _lib.check(L.mep_dispatch(ctx, P(x), P(idx), n, st), ctx)
        if ev_ffn:
            ev_ffn[0].record()
        _lib.check(L.mep_expert_ffn(ctx, P(w_in), P(w_out), len(mine), st), ctx)
        if ev_ffn:
            ev_ffn[1].record()
        _lib.check(L.mep_combine(ctx, P(gate), None, n, P(h), rm, None, P(h_out), st), ctx)

    def timed(run, steps):
        """Per-step device time (L2 flushed before each step, outside the events).
        The region is bracketed by a host barrier and a synchronize; inside it
        the ranks meet before every step in a device-side barrier (mep_barrier),
        so no host wake-up latency lands inside a step and the host keeps the
        queue ahead of the GPU."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(steps):
            flush_l2()
            if world > 1:
                comm.barrier()
            starts[i].record()
            run(i)
            ends[i].record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        return [s.elapsed_time(e) for s, e in zip(starts, ends)]

    st = torch.cuda.current_stream().cuda_stream
    for _ in range(a.warmup):
        eager_step(st)
    torch.cuda.synchronize()
    comm.check()

    # 1) eager stages: FFN-stage time for the roofline, and the eager step time
    n_eager = max(10, a.steps // 4)
    ffn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_eager)]
    eager_ms = timed(lambda i: eager_step(st, ffn[i]), n_eager)
    ffn_ms = [s.elapsed_time(e) for s, e in ffn]
    recv_rows = comm.last_recv_rows()
    comm.check()

    # 2) the step as one CUDA graph (GraphedMoEBlock): the reported value
    blk = GraphedMoEBlock(be, n, lt_router, rm, bias=bias, norm_w=nw, eps=NORM_EPS)
    blk.h.copy_(h)
    for _ in range(a.warmup):
        blk()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    _lib.check(L.mep_reset_stats(ctx, st), ctx)
    clocks.start()
    wall0 = time.perf_counter()
    step_ms = timed(lambda i: blk(), a.steps)
    wall = time.perf_counter() - wall0
    comm.check()
    t_step = torch.tensor([sum(step_ms) / a.steps, sum(ffn_ms) / n_eager,
                           sum(eager_ms) / n_eager], device=dev, dtype=torch.float64)
    rows_t = torch.tensor([recv_rows], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_step, op=dist.ReduceOp.MAX)
    ms_step, ms_ffn, ms_eager = t_step.tolist()
    snap = stats.snapshot()  # route counts and received entries of the timed steps

    # 3) e2e: the public graphed API with host buffers, copies inside the timed region
    e2e = None
    if not a.no_e2e:
        h_host = h.cpu().pin_memory()
        out_host = torch.empty_like(h_host).pin_memory()

        chunks = a.e2e_chunks or (4 if n >= 4096 else 2)
        sblk = StreamedMoEBlock(be, n, lt_router, rm, bias=bias, chunks=chunks, norm_w=nw,
                                eps=NORM_EPS)
        graphed = a.e2e_graph == "on"
        if graphed:
            sblk.capture(None, h_host, out_host)  # one graph launch per step

        def e2e_step():
            sblk(None, h_host, out_host)

        for _ in range(max(1, a.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": a.tokens / (te.item() / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h_host.numel() * 2,
               "d2h_bytes_per_step": out_host.numel() * 2,
               "ms_per_step": te.item(),
               "path": f"StreamedMoEBlock: h from pinned host memory in {chunks} pieces, "
                       "copies overlapping the pieces' steps"
                       + (", one CUDA graph per step" if graphed else
                          ", eager (consecutive steps overlap)")}
        comm.check()
    clk = clocks.stop()

    # per-rank received rows and expert-stage time: the straggler figures
    per_rank = torch.tensor([[float(recv_rows), sum(ffn_ms) / n_eager]], device=dev,
                            dtype=torch.float64)
    if world > 1:
        parts = [torch.zeros_like(per_rank) for _ in range(world)]
        dist.all_gather(parts, per_rank)
        per_rank = torch.cat(parts)
        dist.all_reduce(rows_t)
    total_rows = rows_t.item()
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(sh, a.cpu_sample)

    if rank == 0:
        peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
        # burst figure: the clock samples show the step running at full SM clock,
        # not at the power-capped clock of the sustained figure
        peak = peaks.get("bf16_tflops")
        peak_src = "measured burst bf16 (MEASURED_PEAKS.json)"
        if peak is None:
            peak, peak_src = FALLBACK_BF16_TFLOPS, "fallback"
        flops_rank0 = recv_rows * 6.0 * H * I  # algorithmic FLOPs of this rank's FFN launch
        # GEMM1 reads rows (H) and writes act (I); GEMM2 reads act (I), writes rows (H);
        # plus this rank's expert weights once per launch
        n_local_w_bytes = len(mine) * 3.0 * H * I * 2
        achieved = flops_rank0 / (sum(ffn_ms) / n_eager / 1e3) / 1e12
        line = {
            "metric": METRIC, "value": a.tokens / (ms_step / 1e3), "unit": UNIT,
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights/tokens, Zipf-skewed router)",
            "config": dict(config(a, sh), parallelism=f"ep{world}"),
            "roofline": {"bound": "tensor", "kernel": "expert FFN stage (tcgen05 GEMM1+SwiGLU, "
                                                      "GEMM2+return stores), rank 0",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": peak_src,
                         "flops_per_launch": flops_rank0, "ms_per_launch": sum(ffn_ms) / n_eager,
                         "traffic": (FFN_DRAM_BYTES.get((a.shape, a.tokens)) if world == 1
                                     else None),
                         "traffic_unit": "bytes per launch (dram read + write, ncu)",
                         "algorithmic_bytes": recv_rows * (2 * H + 2 * I) * 2.0
                         + n_local_w_bytes},
            "ffn_ms_per_step_max_rank": ms_ffn,
            "eager": {"value": a.tokens / (ms_eager / 1e3), "ms_per_step": ms_eager,
                      "note": "same kernels launched one by one from Python"},
            "layer_roofline_frac": (a.tokens * (6.0 * k * H * I + 2.0 * H * E) / world
                                    / (ms_step / 1e3) / 1e12) / peak,
            "recv_rows_total": total_rows,
            "wall_s_timed_region": wall,
            "gpu_launches": (KERNELS_PER_STEP + 2 * (world > 1)) * a.steps,
            "clocks": clk,
        }
        if world > 1:
            loads = per_rank[:, 0].cpu().view(world, 1)
            t_ffn = per_rank[:, 1].cpu()
            strag = {"formula": "sum_l max_r recv / sum_l mean_r recv - 1 (1 layer)",
                     "plan": a.plan,
                     "load_pct": 100.0 * straggler_overhead(loads),
                     "ffn_time_pct": 100.0 * float(t_ffn.max() / t_ffn.mean() - 1.0),
                     "recv_rows_per_rank": loads.view(-1).tolist()}
            if counts is not None:  # what the naive placement would have given
                per = E // world
                naive = counts.cpu().view(world, per).sum(dim=1).view(world, 1)
                strag["naive_load_pct"] = 100.0 * straggler_overhead(naive)
            line["straggler"] = strag
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if a.report:
        # every rank: its tokens, its counters, and (from the stage events) the
        # time of its expert stage vs the rest of the step, over the timed steps
        my_ffn, my_step = sum(ffn_ms) / n_eager, sum(step_ms) / a.steps
        snap.update(compute_time=my_ffn * a.steps / 1e3,
                    a2a_time=max(my_step - my_ffn, 0.0) * a.steps / 1e3, steps=a.steps)
        got = report.gather_payloads(report.rank_payload(rank, n * a.steps, snap))
        if rank == 0:
            rep = report.bench_report(got, plan=a.plan, iters=a.steps, wall_time=wall,
                                      iter_times=[t / 1e3 for t in step_ms])
            report.write_bench_report(a.report, rep)
            for line_ in report.summary_lines(rep):
                print(line_, file=sys.stderr)
    del blk
    comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return
    main_b200(a)


if __name__ == "__main__":
    main()
