"""The Rust binding (glypr_b200/rust/glypr-cuda) against the C header it binds: every function
include/glypr_cuda.h declares is declared in src/ffi.rs with the same name, the same number of
parameters and the Rust type of each C parameter and return type, and the #[repr(C)] structs
carry the header's fields in order.  (No Rust toolchain exists in this image, so the crate is
checked by reading both files; a maintainer builds it with cargo next to glypr-core.)"""
from __future__ import annotations

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "glypr_cuda.h")
CRATE = os.path.join(ROOT, "glypr_b200", "rust", "glypr-cuda")

BASE = {"char": "c_char", "int": "c_int", "int32_t": "i32", "int64_t": "i64", "size_t": "usize",
        "float": "c_float", "double": "c_double", "void": "c_void"}


def c_to_rust(ctype: str) -> str:
    """C declaration type -> the Rust FFI type (pointer constness read from the qualifiers)."""
    t = ctype.replace("*", " * ").split()
    base_const = False
    while t and t[0] == "const":
        base_const = True
        t.pop(0)
    base = t.pop(0)
    if t and t[0] == "const":  # "char const *"
        base_const = True
        t.pop(0)
    rust = BASE.get(base, base)
    pointee_const = base_const
    while t:
        assert t.pop(0) == "*", ctype
        rust = ("*const " if pointee_const else "*mut ") + rust
        pointee_const = bool(t) and t[0] == "const"
        if pointee_const:
            t.pop(0)
    return rust


def header_functions():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"([\w\s\*]+?)\b(glp_\w+)\s*\(([^)]*)\)\s*;", text):
        ret = " ".join(m.group(1).strip().split("\n")[-1].split())
        args = " ".join(m.group(3).split())
        params = [] if args in ("", "void") else [a.strip() for a in args.split(",")]
        ptypes = []
        for p in params:
            name = re.findall(r"(\w+)\s*$", p)[0]
            ptypes.append(c_to_rust(p[: p.rindex(name)].strip()))
        out[m.group(2)] = (None if ret == "void" else c_to_rust(ret), ptypes)
    return out


def rust_functions():
    text = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    block = text[text.index('extern "C" {'):]
    out = {}
    for m in re.finditer(r"pub fn (glp_\w+)\((.*?)\)\s*(->\s*([^;]+))?;", block, flags=re.S):
        params = [p.strip() for p in m.group(2).split(",") if p.strip()]
        ptypes = [" ".join(p.split(":", 1)[1].split()) for p in params]
        out[m.group(1)] = (" ".join(m.group(4).split()) if m.group(4) else None, ptypes)
    return out


def test_every_header_function_is_bound_with_matching_types():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 35
    assert set(h) == set(r), (set(h) ^ set(r))
    for name, (ret, params) in h.items():
        rret, rparams = r[name]
        assert rret == ret, (name, ret, rret)
        assert rparams == params, (name, params, rparams)


def _c_struct_fields(name):
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        ty, names = decl.split(" ", 1) if not decl.startswith("const ") else (" ".join(decl.split(" ")[:2]), decl.split(" ", 2)[2])
        for n in names.split(","):
            fields.append(re.sub(r"[\*\[\]\w]*\[.*\]", lambda m: m.group(0).split("[")[0], n.strip()).lstrip("*"))
    return fields


def _rust_struct_fields(name):
    text = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    body = re.search(r"pub struct %s \{(.*?)\}" % name, text, flags=re.S).group(1)
    return re.findall(r"pub (\w+):", body)


def test_structs_have_the_header_fields_in_order():
    for s in ("glp_options", "glp_model_info_t", "glp_timing", "glp_profile"):
        assert _c_struct_fields(s) == _rust_struct_fields(s), s


def test_crate_files_present():
    for f in ("Cargo.toml", "build.rs", os.path.join("src", "lib.rs"), os.path.join("src", "ffi.rs")):
        assert os.path.exists(os.path.join(CRATE, f)), f
    lib = open(os.path.join(CRATE, "src", "lib.rs")).read()
    for item in ("pub struct CudaEmbedder", "pub struct CudaQ8Linear", "pub unsafe fn flash_attention",
                 "pub struct Engine", "pub struct Tokenizer"):
        assert item in lib, item
