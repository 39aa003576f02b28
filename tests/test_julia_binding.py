"""The committed Julia extension (ext/B200Ext/B200Ext.jl) against the C ABI:
every ccall names an entry point the header declares and the library
exports, with as many arguments as the declaration and the same kind at
each position (pointer, int, int64_t, size_t, double).  No Julia toolchain
exists here, so the binding is checked by its signatures."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
JL = os.path.join(ROOT, "ext", "B200Ext", "B200Ext.jl")
HDR = os.path.join(ROOT, "include", "jlust_b200.h")


def _balanced(s, i):
    """Index just past the parenthesis group opening at s[i] == '('."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] == "(":
            depth += 1
        elif s[j] == ")":
            depth -= 1
            if depth == 0:
                return j + 1
    raise ValueError("unbalanced")


def _split_top(s):
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch in "({[":
            depth += 1
        elif ch in ")}]":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur.strip())
    return out


def _jl_kind(t):
    t = t.strip()
    if t.startswith(("Ptr{", "CuPtr{", "Ref{")):
        return "ptr"
    return {"Cint": "int", "Int64": "int64", "Csize_t": "size_t", "Cdouble": "double"}[t]


def julia_ccalls():
    src = open(JL).read()
    calls = []
    for m in re.finditer(r"ccall\(\(:(\w+), lib\),\s*(\w+),\s*", src):
        name, ret = m.group(1), m.group(2)
        i = m.end()
        assert src[i] == "(", f"{name}: argument types must be a tuple"
        j = _balanced(src, i)
        types = _split_top(src[i + 1:j - 1])
        calls.append((name, ret, [_jl_kind(t) for t in types if t]))
    return calls


def _c_kind(a):
    a = a.strip()
    if "*" in a or re.match(r"(const\s+)?jlb_\w+_plan\b", a):
        return "ptr"
    t = re.sub(r"\bconst\b", "", a).split()[0]
    return {"int": "int", "int64_t": "int64", "size_t": "size_t", "double": "double",
            "float": "float", "uint64_t": "uint64"}[t]


def header_decls():
    src = re.sub(r"/\*.*?\*/", "", open(HDR).read(), flags=re.S)
    decls = {}
    for m in re.finditer(r"JLB_API\s+([\w\s\*]+?)\s*\b(jlb_\w+)\s*\(([^;]*?)\)\s*;", src, re.S):
        ret, name, args = m.group(1).strip(), m.group(2), m.group(3).strip()
        kinds = [] if args in ("", "void") else [_c_kind(a) for a in args.split(",")]
        decls[name] = (ret, kinds)
    return decls


def test_every_ccall_matches_the_header():
    calls = julia_ccalls()
    decls = header_decls()
    assert len(calls) >= 15
    ret_kind = {"Cint": "int", "Csize_t": "size_t"}
    for name, ret, kinds in calls:
        assert name in decls, f"{name} is not declared in include/jlust_b200.h"
        c_ret, c_kinds = decls[name]
        assert kinds == c_kinds, f"{name}: Julia passes {kinds}, the header declares {c_kinds}"
        assert ret_kind[ret] == c_ret.replace("const char *", "ptr"), f"{name}: return type"


def test_every_ccall_is_exported():
    from jlust_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\b(jlb_\w+)$", out, re.M))
    for name, _, _ in julia_ccalls():
        assert name in exported, name


def test_status_codes_mapped():
    """Statuses 1-7 rethrow JLUST's own exceptions (src/errors.jl:1-9), 10 a
    timeout exception; the rest fall through to a generic error."""
    src = open(JL).read()
    for code, exc in ((1, "UnsupportedFormat"), (2, "UnsupportedIndexType"),
                      (3, "UnsupportedValueType"), (4, "IndexOriginMismatch"),
                      (5, "DeviceMismatch"), (6, "IncompatibleExtents"),
                      (7, "NonCanonicalStorage"), (10, "B200DeviceTimeout")):
        assert re.search(rf"st == {code} && throw\((JLUST\.)?{exc}\(", src), code
