"""The C ABI library without a GPU: it loads, exports every symbol that
include/mxfp8.h declares, and rejects bad arguments before touching a device
(the reference raises ValueError for the same cases, MXFP8_quantizer.py:544-552,
766-791, 801-807)."""

import ctypes
import pathlib
import re

import pytest

import MXFP8_quantizer

ROOT = pathlib.Path(__file__).resolve().parent.parent
pkg = MXFP8_quantizer.load_package()
capi = pkg._capi


def declared_symbols(header="mxfp8.h"):
    text = (ROOT / "include" / header).read_text()
    return sorted(set(re.findall(r"MXFP8_API\s+[\w\s\*]+?\b(mxfp8_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(capi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_checked_library_exports_both_headers():
    """libmxfp8_checked.so: the whole C ABI plus the checked-build hook, which
    the product library does not carry."""
    checked = capi.checked_lib()
    for name in declared_symbols() + declared_symbols("mxfp8_checked.h"):
        assert hasattr(checked, name), name
    assert declared_symbols("mxfp8_checked.h") == ["mxfp8_checked_window_slack"]
    assert not hasattr(capi.lib(), "mxfp8_checked_window_slack")
    assert checked.mxfp8_checked_window_slack(-1) == capi.ERR_SHAPE
    assert checked.mxfp8_checked_window_slack(0) == capi.OK


def test_library_is_sm100a_only():
    data = capi.LIB_PATH.read_bytes()
    assert b"sm_100a" in data


@pytest.mark.parametrize("rows,cols,expect", [
    (256, 1024, 256 * 32), (1000, 4096, 1024 * 128), (1000, 4064, 1024 * 128), (1, 1, 128 * 4),
    (129, 33, 256 * 4), (0, 0, 0), (8192, 8192, 8192 * 256),
])
def test_scale_storage_bytes(rows, cols, expect):
    assert capi.scale_storage_bytes(rows, cols) == expect
    assert pkg.packed_scale_storage_bytes(rows, cols) == expect


def test_launch_shape_matches_reference_rules():
    assert capi.launch_shape(1000, 4064) == (1000, 4096)
    assert capi.launch_shape(16385, 16384) == (16392, 16384)
    assert capi.launch_shape(2051, 2080) == (2056, 2304)
    for m, k in [(0, 5), (5, 0), (2 ** 31, 8), (8, 65535 * 256 + 1)]:
        with pytest.raises(ValueError):
            capi.launch_shape(m, k)
        with pytest.raises(ValueError):
            pkg.shape_problem(m, k)
    assert pkg.shape_problem(1000, 4064) == (1000, 4096, 125, 16)


@pytest.mark.parametrize("args,match", [
    (dict(dtype=7), "dtype"),
    (dict(q_cols=1000), "sizes"),            # not a multiple of 32
    (dict(q_rows=10), "sizes"),              # fewer rows than m
    (dict(ld_x=100), "sizes"),               # row stride shorter than k
    (dict(ld_q=200), "sizes"),
    (dict(q=0), "NULL"),
    (dict(s=0), "NULL"),
    (dict(x=0), "NULL"),
    (dict(x=0x1001), "alignment"),
    (dict(s=0x1002), "alignment"),
    (dict(s_bytes=100), "scale buffer"),
])
def test_quantize_rejects_bad_arguments_without_a_device(args, match):
    a = dict(x=0x1000, dtype=0, m=16, k=256, ld_x=256, q=0x2000, q_rows=16, q_cols=256, ld_q=256, s=0x3000,
             s_bytes=capi.scale_storage_bytes(16, 256), stream=0)
    a.update(args)
    with pytest.raises(ValueError, match=match):
        capi.quantize(a["x"], a["dtype"], a["m"], a["k"], a["ld_x"], a["q"], a["q_rows"], a["q_cols"], a["ld_q"],
                      a["s"], a["s_bytes"], a["stream"])


def test_empty_geometry_is_a_no_op():
    capi.quantize(0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0)


def test_padded_entry_rejects_unpadded_shapes():
    for m, k in [(7, 256), (8, 100), (0, 256)]:
        with pytest.raises(ValueError):
            capi.quantize_padded(0x1000, 0x2000, 0x3000, m, k, 1 << 20, 0, 0)


def test_dequantize_rejects_bad_arguments():
    ok_s = capi.scale_storage_bytes(4, 32)
    with pytest.raises(ValueError):
        capi.dequantize(0x1000, 4, 33, 33, 0x2000, ok_s, 0x3000, 2, 33, 0)    # cols % 32
    with pytest.raises(ValueError):
        capi.dequantize(0x1000, 4, 32, 32, 0x2000, ok_s, 0x3000, 9, 32, 0)    # dtype
    with pytest.raises(ValueError, match="scale buffer"):
        capi.dequantize(0x1000, 4, 32, 32, 0x2000, ok_s - 1, 0x3000, 2, 32, 0)  # S too small


def test_strerror_names_every_code():
    for code in range(-8, 1):
        assert capi.strerror(code) != "unknown status"
    assert capi.strerror(-99) == "unknown status"


def test_product_path_does_not_touch_the_oracle():
    src = "\n".join(p.read_text() for p in (ROOT / "mxfp8-quantizer_b200").rglob("*.py"))
    src += (ROOT / "MXFP8_quantizer.py").read_text()
    assert "oracle" not in src

