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


RETURNING = ("run_quantizer", "prepare_and_quantize", "run_e2e_verification", "run_e2e_suite",
             "verify_quantizer_outputs", "materialize_quantizer_buffers", "benchmark_compiled_quantizer",
             "build_runtime")


def own_nodes(fn: ast.FunctionDef):
    """The nodes of a function's body, not descending into nested functions."""
    stack = list(fn.body)
    while stack:
        node = stack.pop()
        yield node
        if not isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda)):
            stack.extend(ast.iter_child_nodes(node))


def return_keys(path: pathlib.Path) -> dict:
    """Keys of the dict each function in RETURNING returns, wherever it is
    defined (the reference defines them inside build_runtime): a dict literal
    in the return statement, or the literal assigned to the returned name."""
    tree = ast.parse(path.read_text())
    out = {}
    for fn in ast.walk(tree):
        if not (isinstance(fn, ast.FunctionDef) and fn.name in RETURNING):
            continue
        literals = {}
        for node in own_nodes(fn):
            if isinstance(node, ast.Assign) and isinstance(node.value, ast.Dict):
                for t in node.targets:
                    if isinstance(t, ast.Name):
                        literals[t.id] = node.value
        for node in own_nodes(fn):
            if isinstance(node, ast.Return) and node.value is not None:
                d = node.value if isinstance(node.value, ast.Dict) else (
                    literals.get(node.value.id) if isinstance(node.value, ast.Name) else None)
                if d is not None:
                    out[fn.name] = sorted(k.value for k in d.keys if isinstance(k, ast.Constant))
    return out


def main() -> None:
    out = api_signatures(pathlib.Path(sys.argv[1]) / "MXFP8_quantizer.py")
    out["return_keys"] = return_keys(pathlib.Path(sys.argv[1]) / "MXFP8_quantizer.py")
    (HERE / "api_signatures.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(json.dumps(out, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
