"""benchmark.py and e2e.py accept exactly the reference CLIs' flags, with the
same defaults (tests/golden/cli_flags.json, made by
tests/golden/make_cli_flags.py from the reference's benchmark.py and e2e.py),
so scripts that drive the reference's tools drive these unchanged."""

import json
import pathlib

import pytest

from make_cli_flags import cli_flags

ROOT = pathlib.Path(__file__).resolve().parent.parent
GOLDEN = json.loads((ROOT / "tests" / "golden" / "cli_flags.json").read_text())


@pytest.mark.parametrize("tool", sorted(GOLDEN))
def test_cli_flags_match_the_reference(tool):
    assert cli_flags(ROOT / tool) == GOLDEN[tool]
