"""End-to-end layout check CLI, flag-compatible with the reference's e2e.py.

    python e2e.py [--m 1024] [--n 1024] [--k 2048] [--input-dtype bf16|fp16] [--seed 0]
                  [--gemm-tolerance 1e-2] [--mma-tiler-mn 128,128] [--cluster-shape-mn 1,1] [--suite]

Quantizes A (M, K) and B (N, K), feeds the payloads and the packed scales
unmodified into a block-scaled GEMM and compares C with an fp32 GEMM of the
dequantized operands (the reference's e2e.py:39-94 flow).
"""

from __future__ import annotations

import argparse
import json

from MXFP8_quantizer import run_e2e_suite, run_e2e_verification


def main() -> None:
    ap = argparse.ArgumentParser(description="End-to-end MXFP8 quantizer + block-scaled GEMM check on a B200.")
    ap.add_argument("--m", type=int, default=1024)
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--input-dtype", type=str, default="bf16", choices=["bf16", "fp16"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--gemm-tolerance", type=float, default=1.0e-2)
    ap.add_argument("--mma-tiler-mn", type=str, default="128,128")
    ap.add_argument("--cluster-shape-mn", type=str, default="1,1")
    ap.add_argument("--suite", action="store_true", help="run DEFAULT_E2E_SUITE instead of one configuration")
    a = ap.parse_args()
    if a.suite:
        result = run_e2e_suite(gemm_tolerance=a.gemm_tolerance)
    else:
        result = run_e2e_verification(
            m=a.m, n=a.n, k=a.k, input_dtype=a.input_dtype, seed=a.seed, gemm_tolerance=a.gemm_tolerance,
            mma_tiler_mn=tuple(int(v) for v in a.mma_tiler_mn.split(",")),
            cluster_shape_mn=tuple(int(v) for v in a.cluster_shape_mn.split(",")))
    print(json.dumps(result, indent=2, sort_keys=True))


if __name__ == "__main__":
    main()
