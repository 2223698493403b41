"""Static check of the Julia binding (qwendecisioncore.jl_b200/julia/
QwenDecisionCoreB200Ext.jl) against the C header: Julia is not installed
here, so every `ccall` is parsed and its return type, argument types and
argument count are compared with the declaration in include/qdc_b200.h."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
JL = os.path.join(ROOT, "qwendecisioncore.jl_b200", "julia", "QwenDecisionCoreB200Ext.jl")
HEADER = os.path.join(ROOT, "include", "qdc_b200.h")


def _split_top(text):
    """Split on commas that are not inside (), {} or []."""
    parts, depth, cur = [], 0, []
    for ch in text:
        if ch in "({[":
            depth += 1
        elif ch in ")}]":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        parts.append("".join(cur).strip())
    return parts


def _ccalls(src):
    out = []
    for m in re.finditer(r"ccall\(", src):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        items = _split_top(src[m.end():i - 1])
        name = re.match(r"\(:(\w+),", items[0]).group(1)
        types = _split_top(items[2].strip()[1:-1])
        out.append((name, items[1], types, items[3:]))
    return out


def _jl_kind(t):
    if t.startswith("Ptr{") or t == "Cstring":
        return "ptr"
    return {"Int64": "i64", "Cint": "i32", "Cfloat": "f32", "Csize_t": "usize"}[t]


def _c_kind(param):
    if "*" in param:
        return "ptr"
    words = param.replace("const", "").split()
    return {"int64_t": "i64", "int": "i32", "float": "f32", "size_t": "usize"}[words[0]]


def _header():
    src = open(HEADER).read()
    decls = {}
    for m in re.finditer(r"QDC_API\s+(int|const char \*)\s*(qdc_\w+)\s*\(([^;]*?)\)\s*;", src, re.S):
        params = [p.strip() for p in m.group(3).split(",") if p.strip() and p.strip() != "void"]
        decls[m.group(2)] = ("Cstring" if "char" in m.group(1) else "Cint", [_c_kind(p) for p in params])
    return decls


CALLS = _ccalls(open(JL).read())


def test_binding_calls_something():
    assert len(CALLS) >= 12


@pytest.mark.parametrize("name,ret,types,args", CALLS, ids=[c[0] + f"#{i}" for i, c in enumerate(CALLS)])
def test_ccall_matches_header(name, ret, types, args):
    decls = _header()
    assert name in decls, f"{name} is not declared in include/qdc_b200.h"
    c_ret, c_kinds = decls[name]
    assert ret == c_ret
    assert [_jl_kind(t) for t in types] == c_kinds
    assert len(args) == len(types), f"{name}: {len(args)} arguments for {len(types)} types"


def test_every_declared_entry_point_is_bound():
    """Every QDC_API function of the header has a ccall in the binding."""
    bound = {c[0] for c in CALLS}
    missing = sorted(set(_header()) - bound)
    assert not missing, f"declared in include/qdc_b200.h but not bound in the Julia extension: {missing}"
