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


PROJECT_MODULES = {"_mtp_native", "mtp_kernels", "mtp_fused_verify", "mtp_parallel", "mtp_draft_tree",
                   "oracle.mtp_oracle", "protocol_models"}


def bad_attributes(path):
    """`alias.name` uses, where alias is an imported project module (at any
    scope), naming something the module does not define."""
    import ast
    import importlib
    tree = ast.parse(open(os.path.join(REPO, path)).read())
    aliases = {}
    for node in ast.walk(tree):
        if isinstance(node, ast.Import):
            for a in node.names:
                if a.name in PROJECT_MODULES:
                    aliases[a.asname or a.name] = a.name
        elif isinstance(node, ast.ImportFrom) and node.module == "oracle":
            for a in node.names:
                if a.name == "mtp_oracle":
                    aliases[a.asname or a.name] = "oracle.mtp_oracle"
    # uses inside `with pytest.raises(...)` are meant to fail (out-of-scope names)
    expected = set()
    for node in ast.walk(tree):
        if isinstance(node, ast.With) and any(
                isinstance(i.context_expr, ast.Call) and isinstance(i.context_expr.func, ast.Attribute)
                and i.context_expr.func.attr == "raises" for i in node.items):
            expected.update(id(n) for stmt in node.body for n in ast.walk(stmt))
    out = []
    for node in ast.walk(tree):
        if id(node) in expected:
            continue
        if isinstance(node, ast.Attribute) and isinstance(node.value, ast.Name) and node.value.id in aliases:
            mod = importlib.import_module(aliases[node.value.id])
            if not hasattr(mod, node.attr):
                out.append(f"{path}:{node.lineno}: {node.value.id}.{node.attr}")
    return out


@pytest.mark.parametrize("path", FILES)
def test_project_attributes_exist(path):
    assert bad_attributes(path) == []


@pytest.mark.parametrize("path", FILES)
def test_library_calls_have_signatures(path):
    """Every C entry point the Python side calls (`....mtp_name`) has its
    argument and result types in _mtp_native.SIGNATURES: without them ctypes
    would pass 64-bit sizes and pointers as C ints."""
    import re
    import _mtp_native as N
    src = open(os.path.join(REPO, path)).read()
    used = set(re.findall(r"\.(mtp_[a-z0-9_]+)\s*\(", src))  # calls only
    assert sorted(used - set(N.SIGNATURES)) == []


@pytest.mark.parametrize("path", FILES)
def test_library_call_arity(path):
    """Each call of a C entry point passes as many arguments as the header
    declares (ctypes would raise only when the call runs -- on a GPU for
    most of them)."""
    import ast
    import _mtp_native as N
    tree = ast.parse(open(os.path.join(REPO, path)).read())
    bad = []
    for node in ast.walk(tree):
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and node.func.attr in N.SIGNATURES
                and not any(isinstance(a, ast.Starred) for a in node.args) and not node.keywords):
            want = len(N.SIGNATURES[node.func.attr][1])
            if len(node.args) != want:
                bad.append(f"{path}:{node.lineno}: {node.func.attr} with {len(node.args)} arguments, declared {want}")
    assert bad == []


def header_declarations():
    import re
    src = open(os.path.join(REPO, "include", "mtp_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = {}
    for ret, name, params in re.findall(r"\b(int|size_t|const char\*|uint64_t)\s+(mtp_[a-z0-9_]+)\s*\(([^)]*)\)\s*;",
                                        src):
        ps = [p.strip() for p in params.split(",") if p.strip() and p.strip() != "void"]
        decls[name] = (ret, ps)
    return decls


def test_binding_types_match_header():
    """_mtp_native.SIGNATURES against include/mtp_b200.h, parameter by
    parameter: pointers as pointers, int64_t as c_int64, size_t as c_size_t,
    int as c_int, float as c_float, and the result type."""
    import ctypes
    import _mtp_native as N

    def kind_c(p):
        if "*" in p:
            return "ptr"
        t = p.split()[0] if not p.startswith("const") else p.split()[1]
        return {"int64_t": "i64", "size_t": "u64", "int": "int", "float": "float", "uint64_t": "u64"}[t]

    def kind_py(t):
        if t in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
            return "ptr"
        # c_size_t is c_uint64 on this ABI (LP64)
        return {ctypes.c_int64: "i64", ctypes.c_size_t: "u64", ctypes.c_int: "int", ctypes.c_float: "float",
                ctypes.c_uint64: "u64"}[t]

    decls = header_declarations()
    assert sorted(decls) == sorted(N.SIGNATURES)
    bad = []
    for name, (ret, params) in decls.items():
        rt, argtypes = N.SIGNATURES[name]
        want_ret = {"int": ctypes.c_int, "size_t": ctypes.c_size_t, "const char*": ctypes.c_char_p,
                    "uint64_t": ctypes.c_uint64}[ret]
        if rt is not want_ret:
            bad.append(f"{name}: result {rt} vs {ret}")
        if [kind_c(p) for p in params] != [kind_py(t) for t in argtypes]:
            bad.append(f"{name}: {[kind_c(p) for p in params]} vs {[kind_py(t) for t in argtypes]}")
    assert bad == []


def test_product_never_uses_the_oracle():
    """The oracle is test infrastructure: nothing in the product package
    imports, loads or names it (the product has no CPU fallback)."""
    pkg = os.path.join(REPO, "mtp-engine_b200")
    hits = []
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                src = open(os.path.join(root, f)).read()
                if "oracle" in src or "mtp_oracle" in src:
                    hits.append(os.path.relpath(os.path.join(root, f), REPO))
    assert hits == []


def reads_before_assignment(path):
    """Names a function reads on an earlier line than its first assignment
    of them in its own body (an UnboundLocalError waiting for the call),
    for every top-level and nested function; lambdas and comprehensions are
    left to their own scopes."""
    import ast
    tree = ast.parse(open(os.path.join(REPO, path)).read())
    out = []
    scopes = (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda, ast.ListComp, ast.GeneratorExp, ast.DictComp,
              ast.SetComp, ast.ClassDef)

    def check(fn):
        assigned, reads = {}, []

        def visit(node):
            for ch in ast.iter_child_nodes(node):
                if isinstance(ch, scopes):
                    continue
                if isinstance(ch, ast.Name):
                    if isinstance(ch.ctx, ast.Store):
                        assigned[ch.id] = min(assigned.get(ch.id, 10 ** 9), ch.lineno)
                    elif isinstance(ch.ctx, ast.Load):
                        reads.append((ch.id, ch.lineno))
                visit(ch)

        for arg in fn.args.args + fn.args.kwonlyargs:
            assigned[arg.arg] = 0
        visit(fn)
        declared = {n for st in ast.walk(fn) if isinstance(st, (ast.Global, ast.Nonlocal)) for n in st.names}
        out.extend(f"{path}:{l} {fn.name}: {n}" for n, l in sorted(set(reads))
                   if n in assigned and l < assigned[n] and n not in declared)

    for node in ast.walk(tree):
        if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef)):
            check(node)
    return out


@pytest.mark.parametrize("path", [f for f in FILES if not f.startswith("tests/")])
def test_no_read_before_assignment(path):
    assert reads_before_assignment(path) == []
