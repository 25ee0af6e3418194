"""MoE-layer throughput on B200: one expert-parallel GraniteMoE-shaped MoE block
step from the residual stream h (post-attention RMSNorm + router + route +
dispatch + grouped SwiGLU experts + combine + residual, modeling.py:192-197).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (shape (a) by default): hidden 1024, 32 experts,
top-8, intermediate 512, bf16, Zipf(1.2)-skewed router (layer-0 bias), 16384
tokens per step in total, split evenly over the ranks (strong scaling). The
placement comes from a profiling pass over the same tokens: ``lpt`` (default,
``plan_lpt``: experts re-placed by load, at most E/N + 2 experts per rank),
``balanced`` (the reference's replica planner, 2 slots per rank) or
``naive``. Seeded synthetic tensors stand in for the checkpoint and prompts.

Prints one JSON line (rank 0). `value` is whole-job tokens/s of the device
step (inputs resident in HBM, L2 flushed between steps, per-step CUDA events,
max over ranks); `e2e` is the same metric through the public API with the
step's input copied from pinned host memory and its output copied back inside
the timed region. After the timed steps every rank runs one checked step:
route counts, received rows and sampled output rows against the CPU checker
(`parity`). A timeline pass records per-stage device stamps on every rank
(`stages_us`). `--impl reference` times the CPU checker's restatement of the
reference's block (RMSNorm, router, LocalMoEBackend, residual) on this host's
cores, on the same tokens.
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
NVLINK_NOMINAL_GBS = 900.0   # per direction per GPU (NVLink 5 through NVSwitch)
NVLINK_MEASURED_GBS = 770.0  # peer copy per direction, measured on this pool's B200s
# DRAM bytes (read + write) of the expert FFN stage (both tcgen05 launches) per
# layer step, from one ncu capture of this bench at N=1 (profiles/
# ffn_tc_shape_a_16k_dram.txt): keyed by (shape, tokens per step)
FFN_DRAM_BYTES = {("a", 16384): 325.20e6 + 110.93e6 + 163.11e6 + 215.29e6}
# the algorithmic bytes of that capture's launches (receive rows, act, output
# rows, all 32 experts' weights): other workloads scale the traffic by it
FFN_ALG_BYTES = {("a", 16384): 131072 * (2 * 1024 + 2 * 512) * 2.0 + 32 * 3.0 * 1024 * 512 * 2}
NORM_EPS = 1e-6


def ffn_traffic(shape: str, tokens: int, world: int, alg_bytes: float):
    """DRAM traffic of the FFN stage per step on rank 0: the ncu capture of
    this workload at one GPU when there is one, else that capture scaled by
    the ratio of algorithmic bytes (traffic tracked the algorithmic bytes,
    0.90 of them, in the capture). With several GPUs part of GEMM2's writes
    go to peers over NVLink, so the scaled figure is an upper bound on the
    local DRAM traffic."""
    key = (shape, tokens)
    if world == 1 and key in FFN_DRAM_BYTES:
        return FFN_DRAM_BYTES[key], "ncu capture of this workload (profiles/ffn_tc_shape_a_16k_dram.txt)"
    base = ("a", 16384)
    if shape != base[0]:
        return None, "no capture of this shape"
    return (FFN_DRAM_BYTES[base] * alg_bytes / FFN_ALG_BYTES[base],
            "1-GPU 16384-token capture scaled by this rank's algorithmic bytes (upper bound "
            "on local DRAM traffic when N > 1: part of GEMM2's writes go to peers)")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--shape", choices=["a", "b"], default="a")
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per step, all ranks")
    ap.add_argument("--plan", choices=["naive", "balanced", "lpt"], default="lpt")
    ap.add_argument("--slots", type=int, default=2, help="extra expert slots per rank for the plan")
    ap.add_argument("--cpu-sample", type=int, default=0,
                    help="tokens per CPU step (0: the whole step, shrunk only if the "
                         "reference arm would run for more than a few minutes)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="length of the cpu_baseline measurement in the GPU arm")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--timeline-steps", type=int, default=10,
                    help="steps of the per-stage timeline pass (0: skip)")
    ap.add_argument("--parity-rows", type=int, default=256, help="output rows checked per rank")
    ap.add_argument("--e2e-chunks", type=int, default=1, help="pieces per host batch in the e2e leg")
    ap.add_argument("--e2e-warmup", type=int, default=20,
                    help="untimed e2e steps before the timed ones (host copies, pipeline fill)")
    ap.add_argument("--e2e-depth", type=int, default=2,
                    help="device buffer sets the e2e leg's consecutive steps rotate through")
    ap.add_argument("--force-simt", action="store_true")
    ap.add_argument("--ffn-ast", action="store_true",
                    help="A-stationary GEMM2 (keeps a row tile's activations resident)")
    ap.add_argument("--ffn-prefetch", action="store_true",
                    help="GEMMs prefetch their next tile's rows into L2")
    ap.add_argument("--dispatch-stream", action="store_true",
                    help="dispatch with the streaming engine instead of one warp per token")
    ap.add_argument("--e2e-graph", choices=["on", "off"], default="off",
                    help="capture the e2e host pipeline as one CUDA graph per step "
                         "(measured slower at N=1 and 2: consecutive steps stop overlapping)")
    ap.add_argument("--report", default=None,
                    help="also write a bench report in the reference's results/bench_*.json layout")
    return ap.parse_args()


def workload_name(a) -> str:
    return f"moe_layer_shape_{a.shape}_{a.tokens}tok_zipf1.2_{a.plan}"


PLAN_NOTES = {
    "naive": "naive contiguous placement (Placement.naive)",
    "balanced": "the reference's replica planner (plan_balanced, 2 extra slots per rank)",
    "lpt": "plan_lpt: experts re-placed by profiled load, longest first, at most E/N + 2 "
           "experts per rank (same plan JSON)",
}


def config(a, sh) -> dict:
    return {"workload": workload_name(a), "tokens_per_step": a.tokens, "hidden": sh["hidden"],
            "experts": sh["experts"], "topk": sh["topk"], "inter": sh["inter"],
            "block": "post-attention RMSNorm + router + experts + residual from h "
                     "(modeling.py:192-197)",
            "router": "zipf(1.2) bias x2.0, layer 0", "placement": a.plan,
            "placement_note": PLAN_NOTES[a.plan].replace("2 extra", f"{a.slots} extra")
                                                .replace("E/N + 2", f"E/N + {a.slots}"),
            "l2": "flushed between timed steps (512 MiB write + 256 MiB read, outside the step events)"}


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU over the bench's GPU phase (warm-up,
    timed graph steps, timeline, e2e)."""

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
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, ValueError):
            self.proc = None
            return
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
                "samples": len(sm), "reasons": sorted(reasons),
                "window": "every 100 ms over the GPU phase (warm-up, timed steps, timeline, e2e)"}


# --------------------------------------------------------------- CPU legs
def norm_weight(hidden: int, device=None):
    """Synthetic post-attention RMSNorm weight: 1 + N(0, 1) * 0.02 (seed 8)."""
    g = torch.Generator().manual_seed(8)
    return (1.0 + 0.02 * torch.randn(hidden, generator=g)).to(torch.bfloat16).to(device)


def cpu_inputs(sh, n_tokens):
    """The bench's own tokens and weights on the host (drawn on the CPU with the
    same seeds as the GPU arm's CPU copies)."""
    from miniep_b200 import synth
    lb = synth.make_layer(sh["hidden"], sh["experts"], sh["inter"], 1, seed=0,
                          dtype=torch.bfloat16)
    bias = synth.zipf_router_bias(1, sh["experts"])[0]
    h = synth.make_tokens(n_tokens, sh["hidden"], seed=7, dtype=torch.bfloat16)
    return lb, bias, h


def cpu_step(oracle, lb, bias, h, k):
    from miniep_b200 import synth
    out, _, _, _ = oracle.moe_block_from_h(h, norm_weight(h.shape[1]), NORM_EPS, lb.router,
                                           lb.w_in, lb.w_out, k,
                                           synth.GRANITE_RESIDUAL_MULTIPLIER, bias=bias)
    return out


def cpu_baseline(sh, tokens, seconds) -> dict:
    """The CPU checker's restatement of the reference path (RMSNorm, router,
    LocalMoEBackend, residual) on this host's cores, on the bench's own
    token batch, repeated for about `seconds`."""
    from oracle import moe_oracle
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    lb, bias, h = cpu_inputs(sh, tokens)
    cpu_step(moe_oracle, lb, bias, h, sh["topk"])  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        cpu_step(moe_oracle, lb, bias, h, sh["topk"])
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": reps * tokens / dt, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{reps} x the full {tokens}-token step (bf16, same shape, Zipf router) "
                      f"through oracle.moe_block_from_h in one process, {dt:.1f} s"}


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
    sample = min(a.cpu_sample or a.tokens, a.tokens)
    lb, bias, h = cpu_inputs(sh, sample)
    t0 = time.perf_counter()
    cpu_step(moe_oracle, lb, bias, h, sh["topk"])
    t_one = time.perf_counter() - t0
    if not a.cpu_sample and (a.steps + a.warmup) * t_one > 150.0:
        # keep the whole run within a few minutes: a bounded sample per step
        sample = max(256, int(sample * 150.0 / ((a.steps + a.warmup) * t_one)) // 256 * 256)
        h = h[:sample].contiguous()
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
        "same_config": sample == a.tokens,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{sample} of the step's {a.tokens} tokens per step through "
                                   f"oracle.moe_block_from_h (router + LocalMoEBackend + residual "
                                   f"restated in torch CPU ops, one process on all host threads)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU leg
_T0 = time.perf_counter()


def progress(rank: int, what: str):
    """One stderr line per phase (rank, seconds since start): where a run
    that stalls stopped."""
    print(f"[bench r{rank} {time.perf_counter() - _T0:7.1f}s] {what}", file=sys.stderr, flush=True)


def make_plan(kind, counts, world, slots):
    from miniep_b200 import Placement, plan_balanced, plan_lpt
    E = counts.numel()
    if world == 1 or kind == "naive":
        return Placement.naive(1, E, world), None
    if kind == "balanced":
        return plan_balanced(counts.view(1, E).cpu(), world, slots_per_rank=slots)
    return plan_lpt(counts.view(1, E).cpu(), world, slots_per_rank=slots)


def layer_roofline(sh, tokens, world, ms_step, remote_entries, peak_tflops):
    """The north-star layer roofline: the slower of the expert FLOPs at the
    tensor peak and the dispatch + combine bytes at NVLink bandwidth.
    remote_entries: per rank (entries it sends to other ranks, entries it
    receives from other ranks), one row each way per phase (no dedup)."""
    H, E, k, I = sh["hidden"], sh["experts"], sh["topk"], sh["inter"]
    f_tok = 6.0 * k * H * I + 2.0 * H * E
    t_tc = tokens * f_tok / world / (peak_tflops * 1e12) * 1e6
    row = H * 2.0
    # per direction per phase: the busiest rank's remote rows; dispatch sends
    # what combine later receives, so each phase moves max(sent, received)
    nv_bytes = max((2.0 * max(s, r) * row for s, r in remote_entries), default=0.0)
    t_nv = {bw: nv_bytes / (bw * 1e9) * 1e6 for bw in (NVLINK_NOMINAL_GBS, NVLINK_MEASURED_GBS)}
    roof_us = max(t_tc, t_nv[NVLINK_NOMINAL_GBS])
    return {"t_tc_us": t_tc, "t_nv_us": t_nv[NVLINK_NOMINAL_GBS],
            "t_nv_us_at_measured_770": t_nv[NVLINK_MEASURED_GBS],
            "nvlink_bytes_max_rank": nv_bytes, "roofline_us": roof_us,
            "roofline_tokens_per_s": tokens / (roof_us / 1e6),
            "frac": roof_us / (ms_step * 1e3),
            "assumptions": f"T_tc: {f_tok:.0f} FLOP/token at the measured burst bf16 peak "
                           f"{peak_tflops} TFLOP/s; T_nv: per-entry rows (no dedup), both "
                           f"phases, at {NVLINK_NOMINAL_GBS:.0f} GB/s per direction (nominal "
                           "NVLink 5)"}


def main_b200(a):
    import torch.distributed as dist
    from miniep_b200 import (Comm, EPMoEBackend, EPStats, GraphedMoEBlock, StreamedMoEBlock,
                             _lib, report, straggler_overhead, synth)
    from miniep_b200.ep import rms_norm, router_topk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    progress(rank, "process group up")
    clocks = ClockSampler(local)
    clocks.start()
    sh = synth.SHAPES[a.shape]
    H, E, k, I = sh["hidden"], sh["experts"], sh["topk"], sh["inter"]
    start, stop = synth.split_tokens(a.tokens, world, rank)
    n = stop - start
    # same weights on every rank (same seed), each rank its own token shard;
    # drawn on the host, so they are the reference arm's tensors too
    lt_cpu = synth.make_layer(H, E, I, 1, seed=0, dtype=torch.bfloat16)
    lt = synth.LayerTensors(lt_cpu.router.to(dev), lt_cpu.w_in.to(dev), lt_cpu.w_out.to(dev), None)
    bias = synth.zipf_router_bias(1, E)[0].to(dev)
    h = synth.make_tokens(a.tokens, H, seed=7, dtype=torch.bfloat16)[start:stop].to(dev)
    nw = norm_weight(H, dev)
    rm = synth.GRANITE_RESIDUAL_MULTIPLIER

    comm = Comm(num_layers=1, num_experts=E, topk=k, hidden=H, inter=I, max_tokens=n,
                dtype=torch.bfloat16, device=local, timeout_ms=20000)
    if a.force_simt:
        comm.set_option("force_simt", 1)
    if a.dispatch_stream:
        comm.set_option("dispatch_per_warp", 0)
    if a.ffn_ast:
        comm.set_option("ffn_ast", 1)
    if a.ffn_prefetch:
        comm.set_option("ffn_prefetch", 1)
    from miniep_b200 import Placement
    comm.install(Placement.naive(1, E, world))
    # profiling pass: the global per-expert load of these tokens
    idx0, _ = router_topk(comm, rms_norm(comm, h, nw, NORM_EPS), lt.router, bias)
    counts = torch.bincount(idx0.reshape(-1), minlength=E).to(torch.int64)
    if world > 1:
        dist.all_reduce(counts)
    placement, plan_report = make_plan(a.plan, counts, world, a.slots)
    progress(rank, f"plan {a.plan}: experts {placement.experts_of_rank(rank)[0]}")
    comm.install(placement)
    mine = placement.experts_of_rank(rank)[0]
    w_in, w_out = lt.w_in[mine].contiguous(), lt.w_out[mine].contiguous()
    router_w = lt.router.contiguous()
    w_in_all, w_out_all = ((lt_cpu.w_in, lt_cpu.w_out) if rank == 0 and not a.no_parity
                           else (None, None))
    del lt, lt_cpu
    stats = EPStats(1, E)
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
        _lib.check(L.mep_router_topk(ctx, P(x), P(router_w), P(bias), n, P(idx), P(gate),
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

    progress(rank, "warm-up done")
    # 1) eager stages: FFN-stage time for the roofline, and the eager step time
    n_eager = max(10, min(a.steps // 4, 50))
    ffn = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_eager)]
    eager_ms = timed(lambda i: eager_step(st, ffn[i]), n_eager)
    ffn_ms = [s.elapsed_time(e) for s, e in ffn]
    recv_rows = comm.last_recv_rows()
    comm.check()

    progress(rank, "eager stages timed")
    # 2) the step as one CUDA graph (GraphedMoEBlock): the reported value
    blk = GraphedMoEBlock(be, n, router_w, rm, bias=bias, norm_w=nw, eps=NORM_EPS)
    blk.h.copy_(h)
    for _ in range(a.warmup):
        blk()
    torch.cuda.synchronize()
    _lib.check(L.mep_reset_stats(ctx, st), ctx)
    wall0 = time.perf_counter()
    step_ms = timed(lambda i: blk(), a.steps)
    wall = time.perf_counter() - wall0
    comm.check()
    t_step = torch.tensor([sum(step_ms) / a.steps, sum(ffn_ms) / n_eager,
                           sum(eager_ms) / n_eager], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_step, op=dist.ReduceOp.MAX)
    ms_step, ms_ffn, ms_eager = t_step.tolist()
    snap = stats.snapshot()  # route counts and received entries of the timed steps
    timed_recv = snap["recv_tokens"] / a.steps

    progress(rank, f"graphed steps timed: {ms_step:.3f} ms")
    # 3) timeline: per-stage device stamps of the graphed step on every rank
    stages = None
    if a.timeline_steps > 0:
        comm.set_option("timeline", 1)
        tblk = GraphedMoEBlock(be, n, router_w, rm, bias=bias, norm_w=nw, eps=NORM_EPS)
        comm.set_option("timeline", 0)
        tblk.h.copy_(h)
        comm.read_timeline()  # clears the construction step's stamps
        recs = []
        if world > 1:
            dist.barrier()
        for _ in range(a.timeline_steps):
            flush_l2()
            if world > 1:
                comm.barrier()
            tblk()
            recs.append(comm.read_timeline())
        comm.check()
        del tblk
        stages = {}
        for key in recs[0]:
            vals = [r[key] for r in recs if key in r]
            if isinstance(vals[0], tuple):
                stages[key] = [round(statistics.median(v[0] for v in vals), 1),
                               round(statistics.median(v[1] for v in vals), 1)]
            else:
                stages[key] = round(statistics.median(vals), 1)

    progress(rank, "timeline done")
    # 4) e2e: the public graphed API with host buffers, copies inside the timed region
    e2e = None
    if not a.no_e2e:
        h_host = h.cpu().pin_memory()
        out_host = torch.empty_like(h_host).pin_memory()
        chunks = a.e2e_chunks
        sblk = StreamedMoEBlock(be, n, router_w, rm, bias=bias, chunks=chunks, norm_w=nw,
                                eps=NORM_EPS, depth=a.e2e_depth)
        graphed = a.e2e_graph == "on"
        if graphed:
            sblk.capture(None, h_host, out_host)  # one graph launch per step

        def e2e_step():
            # the next step's copy in and this step's copy out overlap the steps
            # around them; the timed region ends once the last copy out is done
            sblk(None, h_host, out_host, wait_output=False)

        for _ in range(max(1, a.e2e_warmup)):
            e2e_step()
        torch.cuda.current_stream().wait_event(sblk.done)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        h0 = time.perf_counter()
        for _ in range(a.steps):
            e2e_step()
        host_ms = (time.perf_counter() - h0) * 1e3 / a.steps  # enqueue time per step on the host
        torch.cuda.current_stream().wait_event(sblk.done)
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1) / a.steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": a.tokens / (te.item() / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h_host.numel() * 2,
               "d2h_bytes_per_step": out_host.numel() * 2,
               "ms_per_step": te.item(),
               "path": f"StreamedMoEBlock: h from pinned host memory ({chunks} piece(s), "
                       f"{a.e2e_depth} device buffer sets), each step's copy in and copy out "
                       "overlapping the neighbouring steps"
                       + (", one CUDA graph per step" if graphed else "")}
        # the host link alone: the same copies in and out, overlapped the same
        # way, with no layer step between them (every rank at once)
        dbuf = torch.empty_like(h)
        ci, co = torch.cuda.Stream(), torch.cuda.Stream()
        if world > 1:
            dist.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        ci.wait_stream(torch.cuda.current_stream())
        co.wait_stream(torch.cuda.current_stream())
        for _ in range(a.steps):
            with torch.cuda.stream(ci):
                dbuf.copy_(h_host, non_blocking=True)
            with torch.cuda.stream(co):
                out_host.copy_(h, non_blocking=True)
        torch.cuda.current_stream().wait_stream(ci)
        torch.cuda.current_stream().wait_stream(co)
        c1.record()
        torch.cuda.synchronize()
        tc = torch.tensor([c0.elapsed_time(c1) / a.steps], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tc, op=dist.ReduceOp.MAX)
        e2e["copies_only_ms_per_step"] = tc.item()
        th = torch.tensor([host_ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(th, op=dist.ReduceOp.MAX)
        e2e["host_enqueue_ms_per_step"] = th.item()
        del dbuf
        comm.check()
        del sblk
    clk = clocks.stop()

    progress(rank, "e2e done")
    # 5) one checked step: round-robin state reset, so the checker can follow it
    parity_in = None
    if not a.no_parity:
        be.placement.reset_rr()
        _lib.check(L.mep_reset_stats(ctx, st), ctx)
        p_out, p_idx, p_gate, p_x = be.moe_block_from_h(h, nw, NORM_EPS, router_w, rm, bias=bias)
        comm.check()
        psnap = stats.snapshot()
        g = torch.Generator().manual_seed(1000 + rank)
        rows = torch.randperm(n, generator=g)[:min(a.parity_rows, n)].sort().values
        parity_in = {"rank": rank, "idx": p_idx.cpu(), "recv": psnap["recv_tokens"],
                     "route_counts": psnap["route_counts"][0], "rows": rows,
                     "h": h[rows.to(dev)].cpu(), "x": p_x[rows.to(dev)].cpu(),
                     "gate": p_gate[rows.to(dev)].cpu(), "out": p_out[rows.to(dev)].cpu()}
        del p_out, p_idx, p_gate, p_x

    progress(rank, "checked step done")
    # gather the per-rank figures on rank 0
    per_rank = {"rank": rank, "recv_rows": recv_rows, "timed_recv_per_step": timed_recv,
                "ffn_ms": sum(ffn_ms) / n_eager, "step_ms": sum(step_ms) / a.steps,
                "stages_us": stages, "parity_in": parity_in}
    if world > 1:
        got = [None] * world if rank == 0 else None
        dist.gather_object(per_rank, got, dst=0)
    else:
        got = [per_rank]

    progress(rank, "gathered")
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(sh, a.tokens, a.cpu_seconds)

    if rank == 0:
        got.sort(key=lambda r: r["rank"])
        peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
        # burst figure: the clock samples show the step running at full SM clock,
        # not at the power-capped clock of the sustained figure
        peak = peaks.get("bf16_tflops")
        peak_src = "measured burst bf16 (MEASURED_PEAKS.json)"
        if peak is None:
            peak, peak_src = FALLBACK_BF16_TFLOPS, "fallback"
        flops_rank0 = recv_rows * 6.0 * H * I  # algorithmic FLOPs of this rank's FFN launch
        n_local_w_bytes = len(mine) * 3.0 * H * I * 2
        achieved = flops_rank0 / (sum(ffn_ms) / n_eager / 1e3) / 1e12
        alg_bytes = recv_rows * (2 * H + 2 * I) * 2.0 + n_local_w_bytes
        parity, remote = None, None
        if parity_in is not None:
            parity, remote = check_parity(got, placement, w_in_all, w_out_all, router_w.cpu(),
                                          bias.cpu(), sh, rm, world)
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
                         "traffic": ffn_traffic(a.shape, a.tokens, world, alg_bytes)[0],
                         "traffic_unit": "bytes per launch (dram read + write, ncu)",
                         "traffic_source": ffn_traffic(a.shape, a.tokens, world, alg_bytes)[1],
                         "algorithmic_bytes": alg_bytes},
            "ffn_ms_per_step_max_rank": ms_ffn,
            "eager": {"value": a.tokens / (ms_eager / 1e3), "ms_per_step": ms_eager,
                      "note": "same kernels launched one by one from Python"},
            "recv_rows_per_rank": [r["recv_rows"] for r in got],
            "wall_s_timed_region": wall,
            # per step: norm, router, routing, dispatch, gemm1, gemm2, combine
            # (+ the fan-out, which waits for the peers' rows, and the step-start
            # rank barrier, when N > 1)
            "gpu_launches": (7 + 2 * (world > 1)) * a.steps,
            "clocks": clk,
        }
        if remote is not None:
            line["layer_roofline"] = layer_roofline(sh, a.tokens, world, ms_step, remote, peak)
        if stages is not None:
            line["stages_us"] = {str(r["rank"]): r["stages_us"] for r in got}
            line["stages_note"] = ("median device stamps (us) of the graphed step, after the "
                                   "step-start rank barrier (N = 1: after the first stamp); "
                                   "[start, end] per stage, single values are wait ends")
            if remote is not None:
                line["nvlink"] = nvlink_rates(got, remote, H)
        if parity is not None:
            line["parity"] = parity
        if world > 1:
            loads = [[r["timed_recv_per_step"]] for r in got]
            t_ffn = torch.tensor([r["ffn_ms"] for r in got])
            strag = {"formula": "sum_l max_r recv / sum_l mean_r recv - 1 (1 layer)",
                     "plan": a.plan, "slots_per_rank": a.slots,
                     "load_pct": 100.0 * straggler_overhead(loads),
                     "ffn_time_pct": 100.0 * float(t_ffn.max() / t_ffn.mean() - 1.0),
                     "recv_rows_per_rank_per_step": [l[0] for l in loads]}
            if plan_report is not None:
                strag["planner_predicted_pct"] = 100.0 * (
                    plan_report["layers"][0]["imbalance_after"] - 1.0)
                strag["replicas"] = plan_report["replicas_total"]
            strag.update(planner_alternatives(counts, world))
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
        rep_in = report.gather_payloads(report.rank_payload(rank, n * a.steps, snap))
        if rank == 0:
            rep = report.bench_report(rep_in, plan=a.plan, iters=a.steps, wall_time=wall,
                                      iter_times=[t / 1e3 for t in step_ms])
            report.write_bench_report(a.report, rep)
            for line_ in report.summary_lines(rep):
                print(line_, file=sys.stderr)
    del blk
    comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def planner_alternatives(counts, world) -> dict:
    """What the other planners predict for the same counts (max/mean - 1, %),
    with the extra expert slots per rank each needs (the memory cost)."""
    from miniep_b200 import plan_balanced, plan_lpt
    from miniep_b200.balancer import rank_loads
    E = counts.numel()
    c = counts.view(1, E).cpu()
    loads = [float(v) for v in c[0]]
    mean = sum(loads) / world
    naive = rank_loads(loads, [[e // (E // world)] for e in range(E)], world)
    out = {"naive_predicted_pct": 100.0 * (max(naive) / mean - 1.0)}
    for slots in (2, 4, 8):
        for name, fn in (("balanced", plan_balanced), ("lpt", plan_lpt)):
            _, rep = fn(c, world, slots_per_rank=slots)
            out[f"{name}_slots{slots}_predicted_pct"] = round(
                100.0 * (rep["layers"][0]["imbalance_after"] - 1.0), 2)
    return out


def check_parity(got, placement, w_in_all, w_out_all, router_w, bias, sh, rm, world):
    """Rank 0: the checked step of every rank against the CPU checker.

    * counts_exact: each rank's device route counts equal the histogram of
      its own top-k ids (route_counts, ep.py:216-217);
    * recv_rows_exact: each rank's received rows equal what the checker's
      replica round-robin (dest_ranks, ep.py:76-96, state reset to zero)
      sends it from all ranks' ids;
    * output rows: sampled rows of h_out against the checker's expert math on
      the device's own routing (run_experts + slot-order sum + residual,
      modeling.py:83-128, :197) in fp32 (tolerance 2e-2 max-abs, scaled by
      max(1, |ref|)) and in bf16 with the reference's rounding points;
    * router: the checker's top-k on the same normalised rows, rows with an
      exact tie in the top-(k+1) logits excluded, and the rows whose choice
      differs only because a logit rounded one step apart counted apart."""
    import numpy as np
    from oracle import moe_oracle as O
    k, E = sh["topk"], sh["experts"]
    table, n_rep = O.build_table(placement.owners[0])
    counts_ok, recv_expect = True, np.zeros(world, dtype=np.int64)
    remote_in = np.zeros(world, dtype=np.int64)
    sent = []
    for r in got:
        pin = r["parity_in"]
        ids = pin["idx"].reshape(-1).numpy()
        hist = np.bincount(ids, minlength=E)
        counts_ok &= hist.tolist() == list(pin["route_counts"])
        dest = O.dest_ranks(table, n_rep, np.zeros(E, dtype=np.int64), ids)
        per_dest = np.bincount(dest, minlength=world)
        recv_expect += per_dest
        sent.append(int(per_dest.sum() - per_dest[r["rank"]]))
        remote_in += per_dest
        remote_in[r["rank"]] -= per_dest[r["rank"]]
    recv_got = [int(r["parity_in"]["recv"]) for r in got]
    # per rank: (entries sent to other ranks, entries received from other ranks)
    remote = [(sent[i], int(remote_in[i])) for i in range(world)]
    x = torch.cat([r["parity_in"]["x"] for r in got])
    hh = torch.cat([r["parity_in"]["h"] for r in got])
    out = torch.cat([r["parity_in"]["out"] for r in got])
    gate = torch.cat([r["parity_in"]["gate"] for r in got])
    idx = torch.cat([r["parity_in"]["idx"][r["parity_in"]["rows"]] for r in got])
    moe32 = O.local_moe(x.float(), idx, gate.float(), w_in_all.float().cpu(),
                        w_out_all.float().cpu())
    ref32 = O.residual_add(hh.float(), moe32, rm)
    err32 = (out.float() - ref32).abs()
    tol = 2e-2 * max(1.0, float(ref32.abs().max()))
    moe16 = O.local_moe(x, idx, gate, w_in_all.cpu(), w_out_all.cpu())
    ref16 = O.residual_add(hh, moe16, rm)
    d16 = (out.float() - ref16.float()).abs()
    logits = O.router_logits(x, router_w, bias)
    ties = O.boundary_ties(logits, k)
    ref_idx = O.topk_lowest_index(logits, k)
    same = (ref_idx.sort(dim=1).values == idx.sort(dim=1).values).all(dim=1)
    return {"counts_exact": bool(counts_ok),
            "recv_rows_exact": [int(v) for v in recv_expect] == recv_got,
            "recv_rows": recv_got,
            "rows": int(out.shape[0]),
            "max_abs": float(err32.max()), "tol": tol, "ok": bool(float(err32.max()) <= tol),
            "max_abs_vs_bf16_ref": float(d16.max()),
            "bitexact_frac_vs_bf16_ref": float((d16 == 0).float().mean()),
            "router_rows_checked": int((~ties).sum()),
            "router_mismatch_rows": int((~same & ~ties).sum()),
            "router_exact_tie_rows": int(ties.sum()),
            "checker": "oracle/moe_oracle.py (dest_ranks, local_moe, residual_add, router_logits)",
            }, remote


def nvlink_rates(got, remote, H) -> dict:
    """Per rank: bytes its kernels push over NVLink and the stage time they
    took (from the timeline): dispatch sends each token row once per remote
    destination rank it needs (deduplicated rows are fewer than the remote
    entries; the entry count is the upper bound used here), GEMM2 returns one
    row per remote entry it computed, overlapped with its tensor-core work."""
    out = {}
    for r in got:
        st = r["stages_us"] or {}
        sent, recv_remote = remote[r["rank"]]
        row = 2.0 * H
        d = st.get("dispatch")
        g2 = st.get("gemm2")
        out[str(r["rank"])] = {
            "dispatch_remote_entries": sent,
            "dispatch_us": None if not d else round(d[1] - d[0], 1),
            "gemm2_return_rows": recv_remote,
            "gemm2_us": None if not g2 else round(g2[1] - g2[0], 1),
            "return_gbs_lower_bound": None if not g2 else round(
                recv_remote * row / ((g2[1] - g2[0]) * 1e-6) / 1e9, 1),
        }
    return out


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
        return
    main_b200(a)


if __name__ == "__main__":
    main()
