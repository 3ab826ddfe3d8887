"""Digests of the reference *kernel's* outputs (run on a B200) -> golden_kernel.json.

    python tests/golden/make_kernel_golden.py --reference <dir holding MXFP8_quantizer.py>

The reference's torch restatement (used by make_golden.py) is only right for
finite blocks.  This script runs the reference's own CuTeDSL kernel
(MXFP8_quantizer.py:262-525) through its own buffer and launch helpers
(``materialize_quantizer_buffers`` MXFP8_quantizer.py:554-608,
``make_compiled_quantizer`` MXFP8_quantizer.py:699-728, launched as at
MXFP8_quantizer.py:836-844) on the seeded inputs of tests/inputs.py,
including every inf/NaN bit pattern, and records SHA-256 digests of the
padded payload buffer and of the packed scale storage.  Those digests pin
the special-value semantics that the oracle and the CUDA kernels follow.
Needs a B200, CuTeDSL and the reference module; nothing else reads the
reference at run time.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))
import inputs  # noqa: E402
from make_golden import CASES, closure_of  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


KERNEL_CASES = dict(CASES)
KERNEL_CASES.update({
    "c4": ("special_values_bf16(1000, 4064, seed=2)", lambda: inputs.special_values_bf16(), "bf16"),
    "c4_ragged": ("special_values_bf16(129, 4064, seed=5)[:, :4000]",
                  lambda: inputs.special_values_bf16(129, 4064, seed=5)[:, :4000].copy(), "bf16"),
    "nonfinite_bf16": ("nonfinite_patterns('bf16')", lambda: inputs.nonfinite_patterns("bf16"), "bf16"),
    "nonfinite_fp16": ("nonfinite_patterns('fp16')", lambda: inputs.nonfinite_patterns("fp16"), "fp16"),
})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=str(HERE / "golden_kernel.json"))
    args = ap.parse_args()
    import importlib.util

    spec = importlib.util.spec_from_file_location("reference_mxfp8_quantizer",
                                                  pathlib.Path(args.reference) / "MXFP8_quantizer.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    rt = ref.build_runtime()
    pq = rt["prepare_and_quantize"]
    materialize = closure_of(pq, "materialize_quantizer_buffers")
    make_compiled = closure_of(pq, "make_compiled_quantizer")
    Config = closure_of(pq, "MXFP8QuantizerConfig")
    shape_problem = closure_of(pq, "shape_problem")
    resolve = closure_of(pq, "_resolve_input_dtype")
    Int32 = closure_of(pq, "Int32")
    cuda = closure_of(pq, "cuda")
    stream = cuda.CUstream(torch.cuda.current_stream().cuda_stream)

    out = {"generator": "tests/golden/make_kernel_golden.py",
           "device": torch.cuda.get_device_name(0), "torch": torch.__version__, "cases": {}}
    try:
        import cutlass

        out["cutlass_dsl"] = getattr(cutlass, "__version__", "unknown")
    except Exception:
        pass
    for name, (desc, gen, dtype) in KERNEL_CASES.items():
        bits = gen()
        m, k = bits.shape
        kernel_m, kernel_k, _, _ = shape_problem(m, k, 8, 256)
        tdt, cdt = resolve(dtype)
        x = inputs.bits_to_torch(bits, dtype).cuda()
        buf = materialize(kernel_m, kernel_k, tdt, cdt, x)
        compiled = make_compiled(Config(input_dtype=cdt), buf["x_ptr"], buf["q_dwords_ptr"], buf["s_words_ptr"],
                                 kernel_m, kernel_k, buf["s_storage_word_count"], stream)
        compiled(buf["x_ptr"], buf["q_dwords_ptr"], buf["s_words_ptr"], Int32(kernel_m), Int32(kernel_k),
                 Int32(buf["s_storage_word_count"]), stream)
        torch.cuda.synchronize()
        q = buf["q_bytes"].view(torch.uint8).cpu().numpy()
        s = buf["s_storage_bytes"].cpu().numpy()
        out["cases"][name] = {"input": desc, "m": m, "k": k, "dtype": dtype, "kernel_m": kernel_m,
                              "kernel_k": kernel_k, "q_sha256": sha(q), "s_sha256": sha(s), "s_bytes": int(s.size)}
        print(name, out["cases"][name]["q_sha256"][:16], out["cases"][name]["s_sha256"][:16], flush=True)
    pathlib.Path(args.out).write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
