"""The bindings of the C ABI against the compiled library (no GPU needed).

The library reports sizeof / offsetof of every struct of include/orda.h as it
was compiled (orda_abi_layout). Checked against it:
  * the Python ctypes mirrors (orda_b200/_abi.py);
  * the Rust #[repr(C)] mirrors of orda-cutile-rs_b200/rust/src/cuda/ffi.rs,
    the binding that replaces the reference crate's src/cuda/launch.rs: this
    file parses the Rust source and lays each struct out by the repr(C) rules
    (no Rust compiler is needed for that);
and that ffi.rs declares exactly the entry points the header declares.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
FFI_RS = REPO / "orda-cutile-rs_b200" / "rust" / "src" / "cuda" / "ffi.rs"
HEADER = REPO / "include" / "orda.h"


@pytest.fixture(scope="module")
def layout(ob):
    from orda_b200 import _abi

    lib = ob.load_library()
    p = C.POINTER(_abi.OrdaFieldLayout)()
    n = lib.orda_abi_layout(C.byref(p))
    table = {}
    for i in range(n):
        e = p[i]
        s, f = e.struct_name.decode(), e.field.decode()
        table.setdefault(s, {"size": None, "fields": []})
        if f == "":
            table[s]["size"] = int(e.size)
        else:
            table[s]["fields"].append((f, int(e.offset), int(e.size)))
    return table


def _header_structs():
    text = HEADER.read_text()
    return set(re.findall(r"typedef struct (\w+) \{", text))


def test_every_header_struct_is_in_the_layout_table(layout):
    assert _header_structs() == set(layout)


def test_ctypes_mirrors_match_the_library(layout):
    from orda_b200 import _abi

    for name, rec in layout.items():
        cls = getattr(_abi, name, None)
        assert cls is not None, f"no ctypes mirror of {name}"
        assert C.sizeof(cls) == rec["size"], name
        names = [f[0] for f in cls._fields_]
        assert names == [f for f, _, _ in rec["fields"]], name
        for f, off, size in rec["fields"]:
            desc = getattr(cls, f)
            assert (desc.offset, desc.size) == (off, size), f"{name}.{f}"


# ------------------------------------------------------------------ Rust

_PRIM = {"f32": (4, 4), "f64": (8, 8), "i8": (1, 1), "u8": (1, 1), "i16": (2, 2), "u16": (2, 2), "i32": (4, 4),
         "u32": (4, 4), "i64": (8, 8), "u64": (8, 8), "usize": (8, 8), "isize": (8, 8), "c_int": (4, 4),
         "c_char": (1, 1)}


def _rust_structs():
    """name -> [(field, type)] of every #[repr(C)] struct in ffi.rs."""
    src = FFI_RS.read_text()
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*(?:#\[derive\([^)]*\)\]\s*)*pub struct (\w+) \{(.*?)\n\}", src, re.S):
        fields = []
        for line in m.group(2).splitlines():
            line = line.split("//")[0].strip().rstrip(",")
            if not line:
                continue
            fm = re.match(r"(?:pub )?(\w+): (.+)$", line)
            assert fm, f"cannot parse field line {line!r} of {m.group(1)}"
            fields.append((fm.group(1), fm.group(2).strip()))
        out[m.group(1)] = fields
    return out


def _rust_size_align(ty, structs, memo):
    ty = ty.strip()
    if ty in _PRIM:
        return _PRIM[ty]
    if ty.startswith(("*const ", "*mut ")):
        return 8, 8
    am = re.match(r"\[(.+); (\d+)\]$", ty)
    if am:
        s, a = _rust_size_align(am.group(1), structs, memo)
        return s * int(am.group(2)), a
    if ty in structs:
        return _rust_layout(ty, structs, memo)[:2]
    raise AssertionError(f"unknown Rust type {ty}")


def _rust_layout(name, structs, memo):
    """(size, align, [(field, offset, size)]) of a #[repr(C)] struct."""
    if name in memo:
        return memo[name]
    off, align, fields = 0, 1, []
    for f, ty in structs[name]:
        s, a = _rust_size_align(ty, structs, memo)
        off = -(-off // a) * a
        fields.append((f, off, s))
        off += s
        align = max(align, a)
    size = -(-off // align) * align if off else 0
    memo[name] = (size, align, fields)
    return memo[name]


def test_rust_repr_c_mirrors_match_the_library(layout):
    structs = _rust_structs()
    memo = {}
    for name, rec in layout.items():
        assert name in structs, f"ffi.rs has no #[repr(C)] mirror of {name}"
        size, _align, fields = _rust_layout(name, structs, memo)
        assert size == rec["size"], f"{name}: Rust size {size}, library {rec['size']}"
        assert fields == rec["fields"], f"{name}: Rust {fields} vs library {rec['fields']}"


def test_rust_extern_block_declares_every_entry_point():
    hdr = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    declared = set(re.findall(r"ORDA_API\s+[\w\s\*]+?\b(orda_\w+)\s*\(", hdr))
    rust = set(re.findall(r"pub fn (orda_\w+)\(", FFI_RS.read_text()))
    assert declared and declared == rust, (sorted(declared - rust), sorted(rust - declared))


def test_rust_constants_match_the_header():
    hdr = HEADER.read_text()
    rust = FFI_RS.read_text()
    consts = dict(re.findall(r"pub const (ORDA_\w+): \w+ = (\d+);", rust))
    for name, val in re.findall(r"\b(ORDA_[A-Z0-9_]+) = (\d+)", hdr):
        assert consts.get(name) == val, name
    for name, val in re.findall(r"#define (ORDA_[A-Z0-9_]+) (\d+)", hdr):
        assert consts.get(name) == val, name
