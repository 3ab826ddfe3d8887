"""Quantizer benchmark CLI, flag-compatible with the reference's benchmark.py.

    python benchmark.py [--m 16384] [--k 16384] [--input-dtype bf16|fp16]
                        [--warmup-iterations 10] [--iterations 50]
                        [--benchmark-repeats 5] [--cold-l2] [--seed 0]

Verifies the output first (a failed check raises before any timing), then
times the B200 kernel and prints the same JSON summary keys as the
reference's CLI (benchmark.py:39-126 there).
"""

from __future__ import annotations

import argparse
import json

from MXFP8_quantizer import DEFAULT_K_TILE, DEFAULT_ROWS_PER_CTA, run_quantizer

SUMMARY_KEYS = (
    "launch_success", "verification_ran", "verification_passed", "q_max_byte_diff", "q_exact_fraction",
    "scale_bytes_exact", "dispatch_mode", "runtime_min_s", "runtime_min_us", "runtime_mean_s",
    "runtime_mean_us", "runtime_std_us", "effective_gb_s", "effective_gb_s_mean", "effective_tb_s",
    "logical_bytes_moved", "physical_bytes_moved", "input_dtype", "rows_per_cta", "k_tile", "grid_m",
    "grid_k", "total_ctas", "benchmark_repeats", "workspace_count", "cold_l2", "is_full_tile",
)


def main() -> None:
    ap = argparse.ArgumentParser(description="Benchmark the MXFP8 quantizer kernel on a local B200.")
    ap.add_argument("--m", type=int, default=16384, help="rows of X")
    ap.add_argument("--k", type=int, default=16384, help="columns of X (the scale blocks run along them)")
    ap.add_argument("--input-dtype", type=str, default="bf16", choices=["bf16", "fp16"])
    ap.add_argument("--warmup-iterations", type=int, default=10)
    ap.add_argument("--iterations", type=int, default=50)
    ap.add_argument("--benchmark-repeats", type=int, default=5)
    ap.add_argument("--cold-l2", action="store_true",
                    help="cycle through distinct workspaces so every launch starts with a cold L2")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    r = run_quantizer(m=a.m, k=a.k, rows_per_cta=DEFAULT_ROWS_PER_CTA, k_tile=DEFAULT_K_TILE,
                      input_dtype=a.input_dtype, warmup_iterations=a.warmup_iterations, iterations=a.iterations,
                      benchmark_repeats=a.benchmark_repeats, cold_l2=a.cold_l2, skip_verification=False,
                      seed=a.seed)
    print(json.dumps({k: r[k] for k in SUMMARY_KEYS}, indent=2, sort_keys=True))


if __name__ == "__main__":
    main()
