"""Every binding of the C ABI agrees with include/hsb.h, parameter by
parameter.

ctypes does not read the header: an argtypes list with one entry too few, a
size_t bound as int, or a float bound as double passes garbage to the
library without any error.  So the header's prototypes are parsed here and
compared with hillserve_b200/_capi.py's table -- count, and the C type class
of every parameter and of the return value.  The C snippets of the
integration guide are checked the same way for their argument counts, so
the guide cannot drift from the header either.  CPU only."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _strip_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    return re.sub(r"//[^\n]*", " ", text)


def header_prototypes(header: str = "hsb.h") -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, [parameter declarations]) of every hsb_ function."""
    text = _strip_comments((ROOT / "include" / header).read_text())
    text = re.sub(r"^\s*#[^\n]*", " ", text, flags=re.M)
    out: dict[str, tuple[str, list[str]]] = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(hsb_\w+)\s*\(([^;{}]*?)\)\s*;", text):
        ret, name, params = m.group(1), m.group(2), m.group(3)
        ret = ret.split(";")[-1].split("}")[-1].strip()
        ret = re.sub(r"\bextern\b|\"C\"|\bstatic\b|\binline\b", " ", ret).strip()
        plist = [p.strip() for p in params.split(",")] if params.strip() not in ("", "void") else []
        out[name] = (ret, plist)
    return out


def c_class(decl: str) -> str:
    """The ctypes class a C declaration (parameter or return type) needs."""
    d = re.sub(r"\bconst\b", " ", decl)
    if "*" in d or "[" in d:
        return "char_p" if re.fullmatch(r"\s*char\s*\*\s*\w*\s*", d) else "pointer"
    words = d.split()
    # drop the parameter name, if any
    if len(words) > 1 and words[-1] not in ("int", "long", "char", "short"):
        words = words[:-1]
    t = " ".join(words)
    table = {
        "void": "void",
        "int": "int", "int32_t": "int",
        "unsigned": "uint", "unsigned int": "uint", "uint32_t": "uint",
        "size_t": "size",
        "uint64_t": "u64", "unsigned long long": "u64",
        "int64_t": "i64",
        "float": "float",
        "double": "double",
    }
    if t not in table:
        raise AssertionError(f"unknown C type {t!r} in {decl!r}")
    return table[t]


def ctypes_class(t) -> str:
    if t is None:
        return "void"
    if t is C.c_char_p:
        return "char_p"
    if t is C.c_void_p or (isinstance(t, type) and issubclass(t, C._Pointer)):
        return "pointer"
    for cls, name in ((C.c_size_t, "size"), (C.c_uint64, "u64"), (C.c_int64, "i64"), (C.c_float, "float"),
                      (C.c_double, "double"), (C.c_uint32, "uint"), (C.c_int32, "int")):
        if t is cls:
            return name
    # ctypes aliases (c_int is c_int32, c_uint is c_uint32, c_ulonglong is c_uint64 on LP64)
    if C.sizeof(t) == 8 and t in (C.c_ulong, C.c_ulonglong):
        return "u64" if t is not C.c_size_t else "size"
    raise AssertionError(f"unexpected ctypes type {t}")


def _same(header: str, binding: str) -> bool:
    # size_t and uint64_t are both 64-bit unsigned on the LP64 targets this
    # library builds for, and ctypes gives them one type.
    wide = {"size", "u64"}
    return header == binding or (header in wide and binding in wide)


def test_header_parser_sees_every_export():
    from hillserve_b200 import _capi

    protos = header_prototypes()
    assert set(protos) == set(_capi.declared_symbols())


@pytest.mark.parametrize("name", sorted(header_prototypes()))
def test_ctypes_signature_matches_header(name):
    from hillserve_b200 import _capi

    ret, params = header_prototypes()[name]
    restype, argtypes = _capi._SIGNATURES[name]
    assert len(argtypes) == len(params), (name, params)
    for i, (decl, t) in enumerate(zip(params, argtypes)):
        assert _same(c_class(decl), ctypes_class(t)), (name, i, decl, t)
    assert _same(c_class(ret), ctypes_class(restype)), (name, ret, restype)


def _calls(code: str):
    """(name, argument count) of every hsb_ call in a C snippet."""
    for m in re.finditer(r"\b(hsb_\w+)\s*\(", code):
        depth, i, args, cur = 1, m.end(), 0, ""
        while i < len(code) and depth:
            ch = code[i]
            if ch in "([{":
                depth += 1
            elif ch in ")]}":
                depth -= 1
            elif ch == "," and depth == 1:
                args += 1
            if depth:
                cur += ch
            i += 1
        yield m.group(1), (args + 1 if cur.strip() else 0)


def test_integration_snippets_match_header():
    protos = header_prototypes()
    text = (ROOT / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```c\n(.*?)```", text, flags=re.S)
    assert blocks
    seen = 0
    for block in blocks:
        for name, nargs in _calls(_strip_comments(block)):
            assert name in protos, name
            assert nargs == len(protos[name][1]), (name, nargs, protos[name][1])
            seen += 1
    assert seen >= 10


def test_names_in_docs_exist():
    """Every hsb_ function the integration guide and the README name is declared."""
    protos = header_prototypes()
    headers = "".join((ROOT / "include" / h).read_text() for h in ("hsb.h", "hsb_compat.h"))
    libraries = {"hsb_compat"}  # the C++ drop-in's link target (libhsb_compat.so)
    for doc in ("INTEGRATION.md", "README.md"):
        for name in set(re.findall(r"`(hsb_\w+)", (ROOT / doc).read_text())):
            if name.endswith("_"):  # a family, written `hsb_history_*`
                assert any(p.startswith(name) for p in protos), (doc, name)
                continue
            assert name in protos or name in libraries or re.search(rf"\b{name}\b", headers), (doc, name)


def test_integration_ctypes_snippets_match_headers():
    """The guide's ctypes examples declare argtypes / restype that agree with
    include/hsb.h and include/hsb_compat.h (char* may be bound as c_char_p)."""
    protos = {**header_prototypes("hsb.h"), **header_prototypes("hsb_compat.h")}
    text = (ROOT / "INTEGRATION.md").read_text()
    blocks = re.findall(r"```python\n(.*?)```", text, flags=re.S)
    seen = 0
    for block in blocks:
        for name, expr in re.findall(r"\w+\.(hsb_\w+)\.argtypes\s*=\s*(.+)", block):
            argtypes = eval(expr, {"C": C})  # noqa: S307 - the guide's own list expression
            params = protos[name][1]
            assert len(argtypes) == len(params), (name, len(argtypes), params)
            for decl, t in zip(params, argtypes):
                want, got = c_class(decl), ctypes_class(t)
                assert _same(want, got) or (want == "char_p" and got == "pointer") or \
                    (want == "pointer" and got == "char_p" and "char" in decl), (name, decl, t)
            seen += 1
        for name, expr in re.findall(r"\w+\.(hsb_\w+)\.restype\s*=\s*(.+)", block):
            restype = eval(expr, {"C": C})  # noqa: S307
            want = c_class(protos[name][0])
            assert _same(want, ctypes_class(restype)), (name, protos[name][0], restype)
    assert seen >= 3
