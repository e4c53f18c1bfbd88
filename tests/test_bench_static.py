"""CPU check of bench.py (the driver runs it on GPUs only): every name a
function of bench.py reads is defined -- as a parameter, a local, a global
of the module or a builtin -- so a refactor cannot leave a NameError for the
GPU run to find."""

import ast
import builtins
import os
import symtable

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _undefined_names(path):
    src = open(path).read()
    top = symtable.symtable(src, path, "exec")
    module_names = set(top.get_identifiers())
    bad = []

    def visit(table, enclosing):
        names = set(enclosing)
        names.update(s.get_name() for s in table.get_symbols()
                     if s.is_assigned() or s.is_parameter() or s.is_imported() or s.is_namespace())
        for sym in table.get_symbols():
            n = sym.get_name()
            if sym.is_referenced() and not (n in names or n in module_names or hasattr(builtins, n)):
                bad.append(f"{table.get_name()}:{n}")
        for child in table.get_children():
            visit(child, names if table.get_type() == "function" else enclosing)

    for child in top.get_children():
        visit(child, set())
    return bad


def _deleted_but_never_bound(path):
    """`del x` inside a function that never binds x (symtable counts the
    `del` itself as a binding, so the check above cannot see it)."""
    bad = []
    for fn in ast.walk(ast.parse(open(path).read())):
        if not isinstance(fn, (ast.FunctionDef, ast.AsyncFunctionDef)):
            continue
        bound = {a.arg for a in fn.args.args + fn.args.kwonlyargs + fn.args.posonlyargs}
        deleted = []
        for node in ast.walk(fn):
            if isinstance(node, ast.Name) and isinstance(node.ctx, ast.Store):
                bound.add(node.id)
            elif isinstance(node, ast.Name) and isinstance(node.ctx, ast.Del):
                deleted.append(node.id)
            elif isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)) and node is not fn:
                bound.add(node.name)
            elif isinstance(node, (ast.Import, ast.ImportFrom)):
                bound.update((a.asname or a.name).split(".")[0] for a in node.names)
        bad += [f"{fn.name}:{n}" for n in deleted if n not in bound]
    return bad


def test_bench_has_no_undefined_names():
    ast.parse(open(os.path.join(REPO, "bench.py")).read())
    assert _undefined_names(os.path.join(REPO, "bench.py")) == []
    assert _deleted_but_never_bound(os.path.join(REPO, "bench.py")) == []
