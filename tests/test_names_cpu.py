"""Every name a function of the host package reads resolves.

A name that is neither local, an argument, a closure variable, a module
global nor a builtin only fails when its line runs; several such lines run
only on a multi-GPU box (the sharded chain's constructor, for one).  This
check walks the symbol tables of every module instead, on the CPU."""

from __future__ import annotations

import builtins
import symtable
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SOURCES = sorted((ROOT / "videolingo-user_b200" / "vlasr").glob("*.py")) + [
    ROOT / "bench.py", ROOT / "__graft_entry__.py", ROOT / "bench" / "asr_rtfx.py"] + sorted(
    (ROOT / "tests").glob("*.py"))


MODULE_ATTRS = {"__file__", "__name__", "__doc__", "__spec__", "__loader__", "__package__",
                "__path__", "__builtins__"}


def _module_names(table: symtable.SymbolTable) -> set[str]:
    return MODULE_ATTRS | {s.get_name() for s in table.get_symbols()
                           if s.is_assigned() or s.is_imported() or s.is_namespace()}


def _unresolved(table: symtable.SymbolTable, module: set[str], path: str) -> list[str]:
    bad = []
    for child in table.get_children():
        if child.get_type() in ("function", "class"):
            for s in child.get_symbols():
                if (s.is_global() and s.is_referenced() and s.get_name() not in module
                        and not hasattr(builtins, s.get_name())):
                    bad.append(f"{path}: {child.get_name()}: {s.get_name()}")
        bad += _unresolved(child, module, path)
    return bad


@pytest.mark.parametrize("path", SOURCES, ids=lambda p: p.name)
def test_every_global_name_resolves(path):
    top = symtable.symtable(path.read_text(), str(path), "exec")
    module = _module_names(top)
    assert _unresolved(top, module, path.name) == []
