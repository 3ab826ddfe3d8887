"""The reference's own SM100 block-scaled GEMM (blockscaled_gemm.py, run by its
own end-to-end check, MXFP8_quantizer.py:1037-1223) on this library's Q and S:
the fixture tests/golden/make_reference_gemm_golden.py recorded on a B200 for
the suite rows with a 1x1 cluster.  Its errors and margins equal the reference
README's published ones (README.md:164 and README.md:169 of the reference) to
the digits printed there, and the quantizer outputs fed to the GEMM were
bit-exact by the reference's own verifier."""

import json
import pathlib

import pytest

FIXTURE = pathlib.Path(__file__).resolve().parent / "golden" / "reference_gemm_e2e.json"

# (mma_tiler_mn, seed) -> published (max abs error, pass margin), 3 significant digits
PUBLISHED = {((128, 128), 0): (1.07e-4, 650), ((128, 64), 3): (9.16e-5, 379)}


def test_reference_gemm_on_this_librarys_outputs_matches_the_published_errors():
    rows = json.loads(FIXTURE.read_text())["rows"]
    assert len(rows) == len(PUBLISHED)
    for r in rows:
        assert r["consumer"] == "reference blockscaled_gemm.py"
        assert r["cluster_shape_mn"] == [1, 1]
        assert r["e2e_verification_passed"] and r["max_err_ratio"] < 1.0
        for side in ("quantizer_verify_a", "quantizer_verify_b"):
            assert r[side]["scale_bytes_exact"] and r[side]["q_max_byte_diff"] == 0
        err, margin = PUBLISHED[(tuple(r["mma_tiler_mn"]), r["seed"])]
        assert float(f"{r['max_abs_err']:.2e}") == pytest.approx(err, rel=1e-9)
        assert round(r["pass_margin"]) == margin
