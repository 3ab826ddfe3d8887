"""Write tests/golden/cli_flags.json: the flags and defaults of the reference's
two command-line tools (benchmark.py, e2e.py), read from their source with
the ast module.  Run in a container that holds the reference checkout:

    python tests/golden/make_cli_flags.py /path/to/reference

tests/test_cli_flags_cpu.py compares this repository's benchmark.py and e2e.py
against the file, so the CLIs stay drop-in.
"""

import ast
import json
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent


def cli_flags(path: pathlib.Path) -> dict:
    """{flag: default} of every add_argument call in a Python source file
    (defaults that are not literals are recorded as their source text)."""
    tree = ast.parse(path.read_text())
    flags = {}
    for node in ast.walk(tree):
        if not (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and node.func.attr == "add_argument" and node.args):
            continue
        first = node.args[0]
        if not (isinstance(first, ast.Constant) and isinstance(first.value, str)):
            continue
        default = None
        for kw in node.keywords:
            if kw.arg == "default":
                try:
                    default = ast.literal_eval(kw.value)
                except ValueError:
                    default = ast.unparse(kw.value)
            if kw.arg == "action" and isinstance(kw.value, ast.Constant) and kw.value.value == "store_true":
                default = False if default is None else default
        flags[first.value] = default
    return flags


def main() -> None:
    ref = pathlib.Path(sys.argv[1])
    out = {name: cli_flags(ref / name) for name in ("benchmark.py", "e2e.py")}
    (HERE / "cli_flags.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(json.dumps(out, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
