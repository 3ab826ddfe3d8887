"""The reference's own SM100 block-scaled GEMM on this library's Q and S ->
reference_gemm_e2e.json.

    python tests/golden/make_reference_gemm_golden.py --reference <dir holding the
        reference's MXFP8_quantizer.py and blockscaled_gemm.py>

Runs the reference's end-to-end check, ``run_e2e_verification``
(MXFP8_quantizer.py:1037-1223), unmodified, except that the quantizer it
calls is this library's: the ``prepare_and_quantize`` its closure holds is
swapped for this package's drop-in of the same name (same seeded CUDA
``torch.randn`` inputs, same result keys), so A and B are quantized by
libmxfp8.so and go unmodified into the reference's vendored CUTLASS GEMM
(blockscaled_gemm.py, ``Sm100BlockScaledPersistentDenseGemmKernel`` +
``scaled_mm``), whose fp32 C the reference compares with an fp32 GEMM of the
dequantized operands (rtol = atol = 1e-2).  Only the suite rows with a 1x1
cluster run (one CTA per cluster); one B200.  The published errors
for these rows are README.md:164 and README.md:169 of the reference.
Needs a B200, CuTeDSL and the reference's two files; nothing else reads the
reference at run time.
"""

from __future__ import annotations

import argparse
import datetime
import json
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

CLUSTER_1X1_ROWS = [
    # (m, n, k, dtype, seed, mma_tiler_mn, cluster_shape_mn): DEFAULT_E2E_SUITE rows 1 and 6
    (1024, 1024, 2048, "bf16", 0, (128, 128), (1, 1)),
    (1024, 1024, 2048, "bf16", 3, (128, 64), (1, 1)),
]


def swap_closure(fn, name, value):
    for var, cell in zip(fn.__code__.co_freevars, fn.__closure__ or ()):
        if var == name:
            cell.cell_contents = value
            return
    raise KeyError(name)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=str(HERE / "reference_gemm_e2e.json"))
    args = ap.parse_args()
    import importlib.util

    import torch

    import MXFP8_quantizer as ours_module

    ours = ours_module.load_package()
    sys.path.insert(0, args.reference)  # blockscaled_gemm is imported by name inside the check
    spec = importlib.util.spec_from_file_location("reference_mxfp8_quantizer",
                                                  pathlib.Path(args.reference) / "MXFP8_quantizer.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    rt = ref.build_runtime()
    check = rt["run_e2e_verification"]
    calls = []

    def prepare_and_quantize(m, k, dtype_name, seed, stream):
        calls.append((m, k, dtype_name, seed))
        return ours.prepare_and_quantize(m, k, dtype_name, seed, stream)

    swap_closure(check, "prepare_and_quantize", prepare_and_quantize)
    out = {"generator": "tests/golden/make_reference_gemm_golden.py",
           "made": datetime.datetime.now(datetime.timezone.utc).isoformat(timespec="seconds"),
           "device": torch.cuda.get_device_name(0), "rows": []}
    for m, n, k, dt, seed, tiler, cluster in CLUSTER_1X1_ROWS:
        before = len(calls)
        r = check(m, n, k, dt, seed, 1.0e-2, tiler, cluster)
        assert len(calls) == before + 2, "the reference check did not quantize through this library"
        out["rows"].append({"m": m, "n": n, "k": k, "input_dtype": dt, "seed": seed, "mma_tiler_mn": list(tiler),
                            "cluster_shape_mn": list(cluster), "consumer": "reference blockscaled_gemm.py",
                            "e2e_verification_passed": r["e2e_verification_passed"],
                            "max_abs_err": r["max_abs_err"], "pass_margin": r["pass_margin"],
                            "max_err_ratio": r["max_err_ratio"], "sfa_layout": r["sfa_layout"],
                            "quantizer_verify_a": r["quantizer_verify_a"],
                            "quantizer_verify_b": r["quantizer_verify_b"]})
        print(json.dumps(out["rows"][-1]), flush=True)
    pathlib.Path(args.out).write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
