"""Load-time kernel self-check (setting ``check=1``) on the GPU, through the C ABI.

The reference checks its fused kernels at load against the op chains they replace and turns a
failing kernel off for that load with one stderr line (``laya-mlx/src/lib.rs:319-362``); its tests
drive that rule by handing the check a failing build. Here ``check=1`` runs every kernel family the
forward can pick on small seeded problems against a host double-precision computation, and
``check_fail=<kernel>`` plants a wrong value in the host-side expected result of that kernel's
check, so the fallback rule runs without a faulty kernel:
  * a failing two-CTA / cluster split-K GEMM or tcgen05 attention is turned off for the handle
    (the one-CTA GEMM / mma.sync attention take over) and the forward still matches the oracle;
  * a failing one-CTA GEMM or mma.sync attention, or a failing kernel the settings force, makes
    ``s1c_create`` fail with ``S1C_ERR_SELFCHECK``.
"""
import os

import numpy as np
import pytest

from test_gpu_forward import check_against_oracle, make_rows

pytestmark = pytest.mark.gpu


def _backend(model, settings):
    from sys1rust_b200.backend import CudaBackend
    from conftest import get_backend
    cfg, w, _ = get_backend(model)
    old = os.environ.get("S1C_SETTINGS")
    os.environ["S1C_SETTINGS"] = settings
    try:
        return cfg, w, CudaBackend.from_synthetic(cfg, w.tensors)
    finally:
        if old is None:
            del os.environ["S1C_SETTINGS"]
        else:
            os.environ["S1C_SETTINGS"] = old


def _batch(cfg):
    from sys1rust_b200.batch import collate_to
    items = make_rows(cfg, 31, [1, 9, 64, 130, 300, 700], [0, 2, 3, 4, 6, 9])
    return collate_to(items, cfg.encoder.pad_token_id)


def test_check_passes_and_forward_unchanged(cuda_lib):
    """Every kernel passes its load check; the checked handle's forward is bit-identical to an
    unchecked one (the check changes no kernel choice when everything passes)."""
    cfg, w, be = _backend("small:3", "check=1")
    _, _, plain = _backend("small:3", "check=0")
    try:
        ks = be.active_kernels()
        assert "load_check(passed)" in ks, ks
        assert "attention_varlen_tcgen05" in ks and "gemm_tcgen05_2cta" in ks
        b = _batch(cfg)
        got, ref = be.forward(b), plain.forward(b)
        assert np.array_equal(got.logits, ref.logits) and np.array_equal(got.pooled, ref.pooled)
        check_against_oracle(cfg, w, be, b)
    finally:
        be.close()
        plain.close()


@pytest.mark.parametrize("fail,off,kept", [
    ("2cta", "gemm_tcgen05_2cta", "gemm_tcgen05_cluster_splitk"),
    ("csk", "gemm_tcgen05_cluster_splitk", "gemm_tcgen05_2cta"),
    ("tc", "attention_varlen_tcgen05", "attention_varlen_mma"),
    ("2cta+csk+tc", "gemm_tcgen05_2cta", "gemm_tcgen05_1cta"),
])
def test_failing_fast_kernel_falls_back(cuda_lib, capfd, fail, off, kept):
    cfg, w, be = _backend("small:3", f"check=1,check_fail={fail}")
    try:
        ks = be.active_kernels()
        assert off not in ks and kept in ks, ks
        assert any(k.startswith("load_check(off:") for k in ks), ks
        err = capfd.readouterr().err
        assert "is off for this load" in err and "runs instead" in err
        check_against_oracle(cfg, w, be, _batch(cfg))
    finally:
        be.close()


@pytest.mark.parametrize("settings", [
    "check=1,check_fail=1cta",
    "check=1,check_fail=mma",
    "check=1,gemm=2cta,check_fail=2cta",
    "check=1,attn=tc,check_fail=tc",
    "check=1,gemm=splitk,check_fail=splitk",
])
def test_failing_base_or_forced_kernel_refuses_to_load(cuda_lib, settings):
    from sys1rust_b200.backend import BackendError, S1C_ERR_SELFCHECK
    with pytest.raises(BackendError) as ei:
        _backend("small:3", settings)
    assert ei.value.code == S1C_ERR_SELFCHECK
    assert "load check" in str(ei.value) and "differs from the plain computation" in str(ei.value)


def test_large_model_check_passes(cuda_lib):
    cfg, w, be = _backend("large:0", "check=1")
    try:
        assert "load_check(passed)" in be.active_kernels()
    finally:
        be.close()
