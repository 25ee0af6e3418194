"""bench.py's reference arm runs on the host alone and prints one JSON line
with the contract's keys, on the same workload and metric as the GPU arm."""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def _run(*args):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], capture_output=True,
                         text=True, timeout=600, env=env, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line():
    line = _run("--impl", "reference", "--steps", "2", "--warmup", "1", "--cpu-sample", "128")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == "MoE layer tokens/s" and line["unit"] == "tokens/s"
    assert line["steps"] == 2 and line["warmup"] == 1 and line["value"] > 0
    assert line["config"]["workload"].startswith("moe_layer_shape_a_16384tok")
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", RANK="1", WORLD_SIZE="2")
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--cpu-sample", "64"],
                         capture_output=True, text=True, timeout=300, env=env, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [l for l in out.stdout.splitlines() if l.startswith("{")]


def test_ffn_traffic_is_the_capture_or_scaled_from_it():
    """roofline.traffic: the ncu capture for the captured workload, else the
    capture scaled by the algorithmic bytes, with the source stated."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    base = b.FFN_ALG_BYTES[("a", 16384)]
    t, src = b.ffn_traffic("a", 16384, 1, base)
    assert t == b.FFN_DRAM_BYTES[("a", 16384)] and "capture of this workload" in src
    t8, src8 = b.ffn_traffic("a", 16384, 8, base / 8)
    assert abs(t8 - t / 8) < 1e-3 * t and "scaled" in src8
    assert b.ffn_traffic("b", 16384, 1, 1e9)[0] is None
