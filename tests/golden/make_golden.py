"""Generate tests/golden/golden.json from the reference's own torch recipe.

Run once in a container that has the reference checkout (it is not needed,
and not read, anywhere else):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

For each case it builds the seeded input (tests/inputs.py), zero-pads it to
the reference's launch shape exactly as ``materialize_quantizer_buffers``
does (MXFP8_quantizer.py:554-562), runs the reference's
``reference_quantize`` (MXFP8_quantizer.py:610-641) on the CPU and scatters
its dense scale matrix into packed storage through the reference's own
layout map ``decode_scale_bytes`` (MXFP8_quantizer.py:643-662).  Rows between
the launch shape and the next multiple of 128 stay 0, as in the reference's
``torch.zeros`` scale buffer (MXFP8_quantizer.py:567).  It records SHA-256
digests of the E4M3 payload and of the packed scales, plus the scale byte of
every finite amax bit pattern for both input dtypes.

Only finite inputs are recorded: for blocks holding inf/NaN the reference's
torch restatement disagrees with its own kernel (it yields scale 256 for a
NaN block), so those cases are pinned elsewhere.
"""

from __future__ import annotations

import argparse
import base64
import hashlib
import json
import pathlib
import sys
import zlib

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import inputs  # noqa: E402


def closure_of(fn, name):
    for var, cell in zip(fn.__code__.co_freevars, fn.__closure__ or ()):
        if var == name:
            return cell.cell_contents
    raise KeyError(name)


def load_reference(path: str):
    sys.path.insert(0, path)
    import MXFP8_quantizer as ref  # the reference module, read-only

    rt = ref.build_runtime()
    verify = closure_of(rt["run_quantizer"], "verify_quantizer_outputs")
    shape_problem = closure_of(rt["run_quantizer"], "shape_problem")
    reference_quantize = closure_of(verify, "reference_quantize")
    decode_scale_bytes = closure_of(verify, "decode_scale_bytes")
    return reference_quantize, decode_scale_bytes, shape_problem


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ceil_div(a, b):
    return (a + b - 1) // b


def run_case(ref_q, decode, shape_problem, bits: np.ndarray, dtype: str):
    m, k = bits.shape
    kernel_m, kernel_k, _, _ = shape_problem(m, k, 8, 256)
    x = inputs.bits_to_torch(bits, dtype)
    xp = torch.zeros((kernel_m, kernel_k), dtype=x.dtype)
    xp[:m, :k] = x
    scale_bytes, q = ref_q(xp)
    assert int(scale_bytes.min()) >= 0 and int(scale_bytes.max()) <= 255
    scale_cols = kernel_k // 32
    nbytes = ceil_div(kernel_m, 128) * 128 * ceil_div(scale_cols, 4) * 4
    offs = decode(torch.arange(nbytes, dtype=torch.int64), kernel_m, kernel_k)
    packed = torch.zeros(nbytes, dtype=torch.uint8)
    packed[offs.reshape(-1)] = scale_bytes.reshape(-1).to(torch.uint8)
    qb = q.view(torch.uint8).numpy()
    return {
        "m": m, "k": k, "dtype": dtype, "kernel_m": kernel_m, "kernel_k": kernel_k,
        "q_sha256": sha(qb), "s_sha256": sha(packed.numpy()), "s_bytes": nbytes,
        "s_dense_sha256": sha(scale_bytes.to(torch.uint8).numpy()),
    }, scale_bytes


def finite_only(bits: np.ndarray, dtype: str) -> np.ndarray:
    b = bits.copy()
    if dtype == "bf16":
        bad = (b & 0x7F80) == 0x7F80
        b[bad] = 0x3F80
    else:
        bad = (b & 0x7C00) == 0x7C00
        b[bad] = 0x3C00
    return b


CASES = {
    "c1": ("normal(256, 1024, seed=0) bf16", lambda: inputs.normal(256, 1024, 0), "bf16"),
    "c2": ("normal(8192, 8192, seed=1) bf16", lambda: inputs.normal(8192, 8192, 1), "bf16"),
    "c3": ("llm_activation_fp16(16384, 4096, seed=3)", lambda: inputs.llm_activation_fp16(), "fp16"),
    "c4_finite": ("special_values_bf16(1000, 4064, seed=2) with inf/NaN replaced by 1.0",
                  lambda: finite_only(inputs.special_values_bf16(), "bf16"), "bf16"),
    "ragged_1x1": ("normal(1, 1, seed=11) bf16", lambda: inputs.normal(1, 1, 11), "bf16"),
    "ragged_7x33": ("normal(7, 33, seed=12) fp16", lambda: inputs.normal(7, 33, 12, "fp16"), "fp16"),
    "ragged_129x4064": ("normal(129, 4064, seed=13) bf16", lambda: inputs.normal(129, 4064, 13), "bf16"),
    "ragged_2051x2080": ("normal(2051, 2080, seed=14) fp16", lambda: inputs.normal(2051, 2080, 14, "fp16"), "fp16"),
    "sweep_bf16": ("amax_sweep('bf16', seed=7)", lambda: inputs.amax_sweep("bf16"), "bf16"),
    "sweep_fp16": ("amax_sweep('fp16', seed=7)", lambda: inputs.amax_sweep("fp16"), "fp16"),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE / "golden.json"))
    args = ap.parse_args()
    torch.set_num_threads(8)
    ref_q, decode, shape_problem = load_reference(args.reference)
    out = {"generator": "tests/golden/make_golden.py", "cases": {}, "scale_tables": {}}
    for name, (desc, gen, dtype) in CASES.items():
        bits = gen()
        rec, scale_bytes = run_case(ref_q, decode, shape_problem, bits, dtype)
        rec["input"] = desc
        out["cases"][name] = rec
        print(name, rec["q_sha256"][:16], rec["s_sha256"][:16], flush=True)
        if name.startswith("sweep_"):
            # block b of the sweep holds amax pattern b: keep the scale byte per pattern
            top = 0x7F7F if dtype == "bf16" else inputs.FP16_MAX
            per_pattern = scale_bytes[: bits.shape[0]].reshape(-1)[: top + 1].to(torch.uint8).numpy()
            out["scale_tables"][dtype] = base64.b64encode(zlib.compress(per_pattern.tobytes(), 9)).decode()
    pathlib.Path(args.out).write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
