"""CPU check of bench.py: every name a function reads is bound somewhere it can see (its own
scope, an enclosing function, the module, or builtins). bench.py's configurations run only on
a GPU box, so a NameError in a rarely taken branch (a JSON field of one configuration) would
otherwise surface only there."""
import ast
import builtins
import os

BENCH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")


def _targets(node):
    for n in ast.walk(node):
        if isinstance(n, ast.Name) and isinstance(n.ctx, (ast.Store, ast.Del)):
            yield n.id


def _bound(fn):
    names = {a.arg for a in fn.args.args + fn.args.kwonlyargs + fn.args.posonlyargs}
    if fn.args.vararg:
        names.add(fn.args.vararg.arg)
    if fn.args.kwarg:
        names.add(fn.args.kwarg.arg)
    for n in ast.walk(fn):
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef)) and n is not fn:
            names.add(n.name)  # a nested function: its name and its parameters
            names.update(a.arg for a in n.args.args + n.args.kwonlyargs)
            names.update(a.arg for a in (n.args.vararg, n.args.kwarg) if a)
        elif isinstance(n, ast.ClassDef):
            names.add(n.name)
        elif isinstance(n, (ast.Import, ast.ImportFrom)):
            names.update((a.asname or a.name).split(".")[0] for a in n.names)
        elif isinstance(n, ast.ExceptHandler) and n.name:
            names.add(n.name)
        elif isinstance(n, ast.Lambda):
            names.update(a.arg for a in n.args.args)
    names.update(_targets(fn))
    return names


def test_bench_functions_read_only_bound_names():
    tree = ast.parse(open(BENCH).read())
    module = set()
    for n in tree.body:
        if isinstance(n, (ast.FunctionDef, ast.ClassDef)):
            module.add(n.name)
        elif isinstance(n, (ast.Import, ast.ImportFrom)):
            module.update((a.asname or a.name).split(".")[0] for a in n.names)
        elif isinstance(n, (ast.Assign, ast.AnnAssign, ast.AugAssign)):
            module.update(_targets(n))
    missing = []

    def visit(fn, outer):
        scope = outer | _bound(fn)
        for n in ast.walk(fn):
            if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Load):
                if n.id not in scope and n.id not in module and not hasattr(builtins, n.id):
                    missing.append(f"{fn.name}:{n.lineno}: {n.id}")

    for n in tree.body:
        if isinstance(n, ast.FunctionDef):
            visit(n, set())
    assert not missing, missing
