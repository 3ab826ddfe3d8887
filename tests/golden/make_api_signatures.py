"""Write tests/golden/api_signatures.json: the module-level functions of the
reference's MXFP8_quantizer.py with their parameter names and defaults, and
its module-level constants, read from the source with the ast module.  Run in
a container that holds the reference checkout:

    python tests/golden/make_api_signatures.py /path/to/reference

tests/test_api_signatures_cpu.py checks that the root MXFP8_quantizer.py of this
repository offers the same functions with the same parameters and defaults.
"""

import ast
import json
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent


def api_signatures(path: pathlib.Path) -> dict:
    tree = ast.parse(path.read_text())
    funcs, consts = {}, {}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and not node.name.startswith("_"):
            params = [a.arg for a in node.args.args]
            defaults = dict(zip(params[len(params) - len(node.args.defaults):],
                                (ast.unparse(d) for d in node.args.defaults)))
            funcs[node.name] = {"params": params, "defaults": defaults}
        elif isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            try:
                consts[node.targets[0].id] = ast.literal_eval(node.value)
            except ValueError:
                pass
    return {"functions": funcs, "constants": consts}


def main() -> None:
    out = api_signatures(pathlib.Path(sys.argv[1]) / "MXFP8_quantizer.py")
    (HERE / "api_signatures.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(json.dumps(out, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
