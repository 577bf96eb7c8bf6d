"""The C structs of ``include/s1c.h`` and their ctypes mirrors in ``sys1rust_b200.backend`` have the
same size, field offsets and field sizes: a probe compiled with the system C compiler against the
header prints ``sizeof`` / ``offsetof`` for every field, and the test compares them with ctypes. The
Rust cuda-ffi crate (``rust/cuda-ffi/src/lib.rs``) is checked the same way, and its functions'
arity and status constants against the header; the laya-cuda crate calls only functions it
declares."""
import os
import shutil
import subprocess

import pytest

from sys1rust_b200 import backend as bk

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STRUCTS = {
    "s1c_model_desc": bk.ModelDesc, "s1c_tensor": bk.Tensor, "s1c_batch": bk.CBatch, "s1c_varlen": bk.CVarlen,
    "s1c_server_opts": bk.ServerOpts, "s1c_request": bk.CRequest, "s1c_server_stats": bk.ServerStats,
    "s1c_act_head": bk.CActHead, "s1c_answer": bk.CAnswer,
}


def _probe(tmp_path, structs=None):
    """{(struct, field): offset, (struct, field.size): size, (struct, "size"): size} of the header's
    structs, from gcc."""
    structs = structs or {c: [f for f, _ in py._fields_] for c, py in STRUCTS.items()}
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "s1c.h"', "int main(void) {"]
    for cname, fields in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname in fields:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
            lines.append(f'  printf("{cname} {fname}.size %zu\\n", sizeof((({cname}*)0)->{fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "probe"
    subprocess.run([cc, "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {tuple(l.split()[:2]): int(l.split()[2]) for l in out.splitlines()}


def test_struct_layouts_match_the_header(tmp_path):
    got = _probe(tmp_path)
    for cname, py in STRUCTS.items():
        assert got[(cname, "size")] == bk.C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
            assert got[(cname, fname + ".size")] == getattr(py, fname).size, (cname, fname)


# The Rust cuda-ffi crate is not compiled here (no cargo in this image): its #[repr(C)] structs are
# checked field by field against the header through ctypes structures built from the Rust field
# types (repr(C) lays them out as C does), and its extern functions' arity against the header's
# declarations.
RUST_FFI = os.path.join(ROOT, "rust", "cuda-ffi", "src", "lib.rs")
RUST_BACKEND = os.path.join(ROOT, "rust", "laya-cuda", "src", "lib.rs")
_RUST_CTYPES = {"i32": bk.C.c_int32, "u32": bk.C.c_uint32, "i64": bk.C.c_int64, "u64": bk.C.c_uint64,
                "f32": bk.C.c_float, "f64": bk.C.c_double, "usize": bk.C.c_size_t, "u8": bk.C.c_uint8}


def _rust_source():
    with open(RUST_FFI) as f:
        return f.read()


def _rust_type(t):
    import re
    t = t.strip()
    if t.startswith("*"):
        return bk.C.c_void_p
    m = re.fullmatch(r"\[(\w+);\s*(\d+)\]", t)
    if m:
        return _RUST_CTYPES[m.group(1)] * int(m.group(2))
    return _RUST_CTYPES[t]


def _rust_structs():
    import re
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\](?:\s*#\[derive\([^)]*\)\])?\s*pub struct (\w+)\s*\{(.*?)\}", _rust_source(),
                         re.S):
        fields = re.findall(r"pub (\w+):\s*([^,]+?)\s*(?=,|$)", m.group(2).strip())
        if fields:  # opaque handles ({ _p: [u8; 0] }) have no public fields
            out[m.group(1)] = [(f, _rust_type(t)) for f, t in fields]
    return out


def test_rust_binding_structs_match_the_header(tmp_path):
    rs = _rust_structs()
    assert set(STRUCTS) <= set(rs), set(STRUCTS) - set(rs)
    got = _probe(tmp_path, {c: [f for f, _ in fs] for c, fs in rs.items()})
    for cname, fields in rs.items():
        py = type(cname, (bk.C.Structure,), {"_fields_": fields})
        assert got[(cname, "size")] == bk.C.sizeof(py), cname
        for fname, _ in fields:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
            assert got[(cname, fname + ".size")] == getattr(py, fname).size, (cname, fname)


def test_rust_binding_functions_match_the_header():
    import re
    src = _rust_source()
    with open(os.path.join(ROOT, "include", "s1c.h")) as f:
        hdr = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    hdr = re.sub(r"typedef\s+\w+\s*\(\s*\*\s*\w+\s*\)\s*\([^;]*\);", "", hdr)
    decl = {}
    for m in re.finditer(r"\b(s1c_[a-z_]+)\s*\(([^;]*?)\)\s*;", hdr):
        p = m.group(2).strip()
        decl[m.group(1)] = 0 if p in ("", "void") else p.count(",") + 1
    fns = re.findall(r"pub fn (s1c_\w+)\s*\(([^)]*)\)", src)
    assert {name for name, _ in fns} == set(decl)  # every header function, nothing else
    for name, params in fns:
        assert name in decl, name
        n = 0 if not params.strip() else params.count(",") + 1 - (1 if params.strip().endswith(",") else 0)
        assert n == decl[name], (name, n, decl[name])
    consts = dict(re.findall(r"pub const (S1C_\w+): i32 = (-?\d+);", src))
    with open(os.path.join(ROOT, "include", "s1c.h")) as f:
        hdr_consts = dict(re.findall(r"#define (S1C_(?:OK|ERR_\w+|DT_\w+))\s+\(?(-?\d+)\)?", f.read()))
    assert set(consts) == set(hdr_consts)  # every status code and dtype
    for name, v in consts.items():
        assert hdr_consts[name] == v, name


def test_rust_backend_calls_only_declared_functions():
    """laya-cuda (the Backend implementation) calls libs1c only through functions cuda-ffi declares,
    and implements the trait methods the reference's backends implement."""
    import re
    decl = set(re.findall(r"pub fn (s1c_\w+)", _rust_source()))
    with open(RUST_BACKEND) as f:
        src = f.read()
    used = set(re.findall(r"ffi::(s1c_[a-z_]+)\s*\(", src))
    assert used and used <= decl, used - decl
    for m in ("fn name", "fn forward", "fn active_kernels", "fn padded_len", "fn warmup", "fn encoder_hidden",
              "pub fn make_backend", "pub fn factory"):
        assert m in src, m
