"""The C-ABI library builds, loads without a GPU, and exports every function ``include/s1c.h``
declares. No compute calls are made here."""
import ctypes
import os
import subprocess

import pytest

from sys1rust_b200 import build as b
from sys1rust_b200.backend import header_functions, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    return b.build()


def test_header_declares_the_backend_surface():
    fns = header_functions()
    for want in ["s1c_create", "s1c_destroy", "s1c_forward_padded", "s1c_forward_varlen", "s1c_forward_device",
                 "s1c_encoder_hidden", "s1c_name", "s1c_active_kernels", "s1c_padded_len", "s1c_warmup",
                 "s1c_last_error"]:
        assert want in fns


def test_library_exports_every_declared_symbol(built):
    L = ctypes.CDLL(built)
    missing = [f for f in header_functions() if not hasattr(L, f)]
    assert not missing, missing


def test_only_declared_symbols_are_exported(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    s1c = {s for s in exported if s.startswith("s1c_")}
    assert s1c == set(header_functions())


def test_library_is_built_for_sm100a(built):
    """The embedded device code targets sm_100a only (checked from the build flags)."""
    assert "arch=compute_100a,code=sm_100a" in " ".join(b.NVCC_FLAGS)
    assert os.path.getsize(built) > 100_000


def test_create_without_gpu_fails_cleanly(built):
    """With no usable device the library returns an error code, not a crash."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from sys1rust_b200.backend import ModelDesc, Tensor
    L = lib()
    desc = ModelDesc()
    h = ctypes.c_void_p()
    rc = L.s1c_create(ctypes.byref(desc), (Tensor * 1)(), 0, 0, ctypes.byref(h))
    assert rc < 0
    assert L.s1c_create_error()


def test_python_constants_match_the_header():
    """Every status code and tensor type of ``include/s1c.h`` has the same value in the Python
    mirror, so errors map to the same exception classes on both sides of the ABI."""
    import re
    from sys1rust_b200 import backend
    with open(os.path.join(ROOT, "include", "s1c.h")) as f:
        text = f.read()
    defs = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (S1C_(?:OK|ERR_\w+|DT_\w+))\s+\(?(-?\d+)\)?", text)}
    assert {"S1C_OK", "S1C_ERR_ARG", "S1C_ERR_SELFCHECK", "S1C_DT_BF16"} <= set(defs)
    for name, value in defs.items():
        py = name if hasattr(backend, name) else name.replace("S1C_", "", 1)
        assert getattr(backend, py, None) == value, (name, value, getattr(backend, py, None))


def test_ctypes_signatures_match_the_header():
    """The Python binding declares each function with as many arguments as ``include/s1c.h``
    gives it (a mismatch would pass garbage through the ABI without an error)."""
    import re
    with open(os.path.join(ROOT, "include", "s1c.h")) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    text = re.sub(r"typedef\s+\w+\s*\(\s*\*\s*\w+\s*\)\s*\([^;]*\);", "", text)
    decl = {}
    for m in re.finditer(r"\b(s1c_[a-z_]+)\s*\(([^;]*?)\)\s*;", text):
        params = m.group(2).strip()
        decl[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    assert set(decl) == set(header_functions())
    L = lib()
    for name, n in decl.items():
        fn = getattr(L, name)
        assert fn.argtypes is not None, name
        assert len(fn.argtypes) == n, (name, len(fn.argtypes), n)
