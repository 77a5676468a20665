"""Every name a module's functions use resolves to something: much of the
GPU path (bench.py's GPU arms, the multi-GPU exchanges) cannot run on a CPU,
so a NameError there would otherwise surface first on a B200.  Checked with
symtable: a name that is neither local, enclosing, module-level, imported
nor builtin is reported.  CPU only."""

import builtins
import os
import symtable

import pytest

from conftest import REPO

FILES = ["bench.py", "__graft_entry__.py", "mtp-engine_b200/_mtp_native.py", "mtp-engine_b200/mtp_kernels.py",
         "mtp-engine_b200/mtp_fused_verify.py", "mtp-engine_b200/mtp_parallel.py",
         "mtp-engine_b200/mtp_draft_tree.py", "mtp-engine_b200/_build.py", "oracle/mtp_oracle.py"]
# the GPU tests too: on a CPU they are collected but never run
FILES += sorted(os.path.join("tests", f) for f in os.listdir(os.path.join(REPO, "tests"))
                if f.startswith("test_") and f.endswith(".py"))
MODULE_DUNDERS = {"__file__", "__name__", "__doc__", "__spec__", "__loader__", "__package__", "__path__"}


def unresolved(path):
    src = open(os.path.join(REPO, path)).read()
    top = symtable.symtable(src, path, "exec")
    defined = {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported()}
    out = []

    def walk(t, where):
        for s in t.get_symbols():
            n = s.get_name()
            if s.is_global() and n not in defined and not hasattr(builtins, n) and n not in MODULE_DUNDERS:
                out.append(f"{where}: {n}")
        for c in t.get_children():
            walk(c, f"{where}.{c.get_name()}")

    walk(top, path)
    return out


@pytest.mark.parametrize("path", FILES)
def test_every_name_resolves(path):
    assert unresolved(path) == []
