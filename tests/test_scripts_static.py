"""Static checks of the top-level scripts that only run in full on a GPU box:
every global name a function uses must be defined at module level or be a
builtin (catches a helper lost in an edit before a GPU run does)."""
import builtins
import os
import symtable

import pytest

from conftest import ROOT

SCRIPTS = ["bench.py", "__graft_entry__.py", os.path.join("tests", "mp_tp_worker.py"),
           os.path.join("tests", "mp_stress_worker.py")]


def _undefined_globals(path):
    src = open(path).read()
    top = symtable.symtable(src, path, "exec")
    defined = set(dir(builtins)) | {"__file__", "__name__", "__doc__"}
    for sym in top.get_symbols():
        if sym.is_assigned() or sym.is_imported() or sym.is_namespace():
            defined.add(sym.get_name())
    missing = set()

    def walk(table):
        for sym in table.get_symbols():
            if (sym.is_global() or (sym.is_free() is False and sym.is_referenced()
                                    and not sym.is_local() and not sym.is_parameter()
                                    and not sym.is_free() and table.get_type() != "module")):
                if sym.get_name() not in defined and not sym.is_local():
                    missing.add((table.get_name(), sym.get_name()))
        for child in table.get_children():
            walk(child)

    for child in top.get_children():
        walk(child)
    return sorted(missing)


@pytest.mark.parametrize("script", SCRIPTS)
def test_no_undefined_globals(script):
    assert _undefined_globals(os.path.join(ROOT, script)) == []


def test_checker_catches_a_missing_helper(tmp_path):
    p = tmp_path / "s.py"
    p.write_text("def f(x):\n    return helper(x) + len(x)\n")
    assert ("f", "helper") in _undefined_globals(str(p))
