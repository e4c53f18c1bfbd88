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


def test_bench_has_no_undefined_names():
    ast.parse(open(os.path.join(REPO, "bench.py")).read())
    assert _undefined_names(os.path.join(REPO, "bench.py")) == []
