"""The C structs of ``include/s1c.h`` and their ctypes mirrors in ``sys1rust_b200.backend`` have the
same size and field offsets: a probe compiled with the system C compiler against the header prints
``sizeof`` / ``offsetof`` for every field, and the test compares them with ctypes. A Rust FFI
binding of the header relies on the same layout."""
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


def _probe(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "s1c.h"', "int main(void) {"]
    for cname, py in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
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
