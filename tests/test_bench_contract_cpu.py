"""bench.py's driver contract, exercised through its CPU reference arm (no GPU):
one JSON line with the required keys, and torchrun-style non-zero ranks print
nothing."""

import json
import os
import pathlib
import subprocess
import sys

ROOT = pathlib.Path(__file__).resolve().parent.parent

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e", "gpu_launches"}


def run_bench(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, env=env,
                         cwd=str(ROOT), timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return [json.loads(ln) for ln in out.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    lines = run_bench("--impl", "reference", "--m", "512", "--k", "1024", "--steps", "2", "--warmup", "3")
    assert len(lines) == 1
    r = lines[0]
    assert REQUIRED <= set(r), REQUIRED - set(r)
    assert r["impl"] == "reference" and r["unit"] == "TB/s" and r["value"] > 0
    assert r["cpu_baseline"]["kind"] == "port" and r["cpu_baseline"]["cores"] >= 1
    assert r["e2e"]["h2d_bytes_per_step"] == 0 and r["e2e"]["d2h_bytes_per_step"] == 0
    assert r["config"]["workload"].startswith("512x1024")


def test_reference_arm_is_silent_on_nonzero_ranks():
    lines = run_bench("--impl", "reference", "--m", "256", "--k", "256", "--steps", "1", "--warmup", "3",
                      env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert lines == []


def test_launches_per_call_follows_the_split_rule():
    """bench.py's gpu_launches count: one launch up to 148*128 tiles (148*64
    for X rows that are not 16-byte aligned), then whole 128-row tiles per
    launch.  The GPU suite checks the same numbers against profiler counts."""
    import bench

    assert bench.launches_per_call(8192, 8192, 8192) == 1
    assert bench.launches_per_call(8192, 8191, 8191) == 1
    assert bench.launches_per_call(32768, 16384, 16384) == 2
    assert bench.launches_per_call(131072, 16384, 16384) == 7
    assert bench.launches_per_call(16384, 16383, 16383) == 2
    assert bench.launches_per_call(38000, 8192, 8192) == 2
    assert bench.launches_per_call(38000, 8191, 8191) == 3
    assert bench.launches_per_call(1, 65535 * 256, 65535 * 256) == 1
    # Q at any offset: the two-CTA split too
    assert bench.launches_per_call(8192, 8192, 8192, q_any_offset=True) == 1
    assert bench.launches_per_call(16384, 16384, 16384, q_any_offset=True) == 2
    assert bench.launches_per_call(38000, 8192, 8192, q_any_offset=True) == 3
