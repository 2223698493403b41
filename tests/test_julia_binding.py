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


# ---- the CUDA extension's side: qwendecisioncore.jl_b200/julia/patch_cuda_ext.py

def _jl_functions(src):
    """name -> (required positional count, total positional count, keyword names)
    for every `function name(...)` and one-line `name(...) = ...` of the binding."""
    out = {}
    for m in re.finditer(r"^(?:function\s+)?([A-Za-z_]\w*!?)\(", src, re.M):
        name, i, depth = m.group(1), m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        rest = src[i:i + 40]
        if not (m.group(0).startswith("function") or re.match(r"\s*=", rest)):
            continue
        inner = src[m.end():i - 1]
        pos, _, kw = inner.partition(";")
        params = _split_top(pos)
        required = sum(1 for p in params if "=" not in p)
        out[name] = (required, len(params), {k.split("::")[0].split("=")[0].strip() for k in _split_top(kw)})
    return out


def _hook_calls(text):
    """(name, positional count, keyword names) of every B200Kernels[].name(...) call."""
    calls = []
    for m in re.finditer(r"B200Kernels\[\]\.(\w+!?)\(", text):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(text[i], 0)
            i += 1
        pos, _, kw = text[m.end():i - 1].partition(";")
        calls.append((m.group(1), len(_split_top(pos)), {k.split("=")[0].strip() for k in _split_top(kw)}))
    return calls


def _patch_module():
    import importlib.util
    path = os.path.join(ROOT, "qwendecisioncore.jl_b200", "julia", "patch_cuda_ext.py")
    spec = importlib.util.spec_from_file_location("patch_cuda_ext", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_every_hook_call_names_a_binding_function_with_its_arguments():
    """Each call the CUDA-extension edits make through the hook table names a
    function of the binding, with a positional argument count it accepts
    and keywords it declares; and every such function is in the table the
    binding's __init__ fills."""
    src = open(JL).read()
    defs = _jl_functions(src)
    table = re.search(r"B200Kernels\[\] = \(;(.*?)\)\)", src, re.S).group(1)
    exported = {n.strip() for n in table.replace("\n", " ").split(",") if n.strip()}
    calls = [c for e in _patch_module().EDITS for c in _hook_calls(e.text)]
    assert len(calls) >= 12
    for name, npos, kws in calls:
        assert name in defs, f"{name} is not defined in the binding"
        required, total, declared = defs[name]
        assert required <= npos <= total, f"{name}: {npos} positional arguments, takes {required}..{total}"
        assert kws <= declared, f"{name}: keywords {kws - declared} not declared"
        assert name in exported, f"{name} is not in the hook table"


@pytest.mark.skipif(not os.path.isdir("/root/reference/ext"), reason="the reference tree is not present")
def test_cuda_extension_edits_apply_to_the_reference():
    """Every edit's anchor line is where it was recorded (checked by hash) in
    the reference's ext/ files, and the patched files bracket each routed
    kernel launch with an if/else on the hook table."""
    files = _patch_module().patched("/root/reference")
    assert set(files) == {"ext/cuda_workspace.jl", "ext/cuda_mlp.jl", "ext/cuda_delta.jl",
                          "ext/cuda_attention.jl"}
    for name, (old, new) in files.items():
        added = len(new.split("\n")) - len(old.split("\n"))
        assert added > 0
        # every `if B200Kernels[] === nothing` opened before a launch is closed
        opens = new.count("    if B200Kernels[] === nothing\n")
        assert new.count("\n    else\n") >= opens
