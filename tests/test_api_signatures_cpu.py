"""The drop-in module MXFP8_quantizer.py offers the reference module's public
functions with the same parameter names and defaults, and its constants
(tests/golden/api_signatures.json, made by tests/golden/make_api_signatures.py
from the reference's MXFP8_quantizer.py)."""

import ast
import inspect
import json
import pathlib

import pytest

import MXFP8_quantizer

ROOT = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = json.loads((ROOT / "tests" / "golden" / "api_signatures.json").read_text())


def test_constants_match():
    for name, value in GOLDEN["constants"].items():
        assert getattr(MXFP8_quantizer, name) == value, name


@pytest.mark.parametrize("name", sorted(GOLDEN["functions"]))
def test_function_signature_matches(name):
    ref = GOLDEN["functions"][name]
    sig = inspect.signature(getattr(MXFP8_quantizer, name))
    assert list(sig.parameters) == ref["params"]
    for param, text in ref["defaults"].items():
        ours = sig.parameters[param].default
        try:
            expect = ast.literal_eval(text)
        except ValueError:                       # a module-level name, e.g. DEFAULT_ROWS_PER_CTA
            expect = getattr(MXFP8_quantizer, text)
        assert ours == expect, (name, param, ours, expect)


@pytest.mark.parametrize("name", sorted(GOLDEN["return_keys"]))
def test_returned_dict_keys_match(name):
    """The dict each entry point returns has the reference's keys (read from
    this repository's source the same way the fixture was read)."""
    from make_api_signatures import return_keys

    ours = return_keys(ROOT / "mxfp8-quantizer_b200" / "quantizer.py")
    assert ours.get(name) == GOLDEN["return_keys"][name]
