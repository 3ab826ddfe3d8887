"""Drop-in for the reference's ``MXFP8_quantizer`` module.

``from MXFP8_quantizer import run_quantizer, run_e2e_verification,
run_e2e_suite, prepare_and_quantize`` keeps working, with the same
signatures, return keys and exceptions, backed by the B200 CUDA library in
``mxfp8-quantizer_b200/`` (whose directory name is not an importable
identifier, so it is loaded here under the name ``mxfp8_quantizer_b200``).
"""

from __future__ import annotations

import importlib.util
import pathlib
import sys

PACKAGE_NAME = "mxfp8_quantizer_b200"
PACKAGE_DIR = pathlib.Path(__file__).resolve().parent / "mxfp8-quantizer_b200"


def load_package():
    mod = sys.modules.get(PACKAGE_NAME)
    if mod is not None:
        return mod
    spec = importlib.util.spec_from_file_location(
        PACKAGE_NAME, PACKAGE_DIR / "__init__.py", submodule_search_locations=[str(PACKAGE_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PACKAGE_NAME] = mod
    try:
        spec.loader.exec_module(mod)
    except BaseException:
        sys.modules.pop(PACKAGE_NAME, None)
        raise
    return mod


_pkg = load_package()

DEFAULT_ROWS_PER_CTA = _pkg.DEFAULT_ROWS_PER_CTA
DEFAULT_K_TILE = _pkg.DEFAULT_K_TILE
DEFAULT_E2E_SUITE = _pkg.DEFAULT_E2E_SUITE
build_runtime = _pkg.build_runtime
run_quantizer = _pkg.run_quantizer
run_e2e_verification = _pkg.run_e2e_verification
run_e2e_suite = _pkg.run_e2e_suite
prepare_and_quantize = _pkg.prepare_and_quantize
quantize = _pkg.quantize
dequantize = _pkg.dequantize
