"""Every name the Python sources load is bound somewhere in their module.

A coarse static check (no GPU, no import side effects): for each module of
the package, the oracle, the tests and bench.py, the set of names read
anywhere must lie within the names the module binds anywhere (imports,
definitions, assignments, parameters, loop and comprehension targets,
exception aliases, globals) or the builtins.  It catches a name that exists
only in another module, which the CPU tests cannot reach when the code path
runs only on GPUs (a multi-rank data-parallel call, for instance).
"""
import ast
import builtins
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = sorted(
    [os.path.join(d, f) for d in ("glt_b200", "oracle", "tests", os.path.join("tests", "golden"))
     for f in os.listdir(os.path.join(ROOT, d)) if f.endswith(".py")]
    + ["bench.py", "__graft_entry__.py"]
)


def bound_and_loaded(tree: ast.AST) -> tuple[set, set]:
    bound, loaded = set(), set()
    for node in ast.walk(tree):
        if isinstance(node, ast.Name):
            (loaded if isinstance(node.ctx, ast.Load) else bound).add(node.id)
        elif isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
            bound.add(node.name)
        elif isinstance(node, ast.arg):
            bound.add(node.arg)
        elif isinstance(node, (ast.Import, ast.ImportFrom)):
            for a in node.names:
                bound.add((a.asname or a.name).split(".")[0])
        elif isinstance(node, ast.ExceptHandler) and node.name:
            bound.add(node.name)
        elif isinstance(node, (ast.Global, ast.Nonlocal)):
            bound.update(node.names)
        elif isinstance(node, ast.alias):
            pass
    return bound, loaded


@pytest.mark.parametrize("rel", FILES)
def test_every_loaded_name_is_bound(rel):
    with open(os.path.join(ROOT, rel)) as f:
        tree = ast.parse(f.read(), filename=rel)
    bound, loaded = bound_and_loaded(tree)
    missing = sorted(n for n in loaded - bound if not hasattr(builtins, n) and n != "__file__")
    assert not missing, f"{rel}: names read but never bound: {missing}"
