"""Packed-token buckets on the GPU (settings ``buckets=`` / ``warm=``; the reference's length buckets
and load-time warm-up, ``laya-mlx/src/lib.rs:89-94, :1152-1173``).

A batch whose tokens fit a bucket runs as the bucket's shape (dummy rows hold the remaining tokens,
marker slots padded to a multiple of 4), so requests of different lengths replay one captured graph.
The padding must not change what a batch's own rows get: checked against a handle without buckets
(within rounding: the GEMMs' split-K plan depends on the token count), against the CPU oracle, and
bit for bit against a handle with the same buckets but no graphs.
"""
import contextlib
import os

import numpy as np
import pytest

from sys1rust_b200.batch import Varlen, collate_to

from test_gpu_forward import check_against_oracle, make_rows

pytestmark = pytest.mark.gpu


@contextlib.contextmanager
def settings(extra: str):
    old = os.environ.get("S1C_SETTINGS")
    os.environ["S1C_SETTINGS"] = (old + "," if old else "") + extra
    try:
        yield
    finally:
        if old is None:
            del os.environ["S1C_SETTINGS"]
        else:
            os.environ["S1C_SETTINGS"] = old


def backend_with(cfg, w, extra: str):
    from sys1rust_b200.backend import CudaBackend
    with settings(extra):
        return CudaBackend.from_synthetic(cfg, w.tensors)


def test_bucketed_replay_equals_direct_launches(cuda_lib):
    """After warmup(), single requests of new lengths (one bucket, marker counts 0..9) replay the
    bucket's graph; every output equals, bit for bit, a handle that launches kernel by kernel with
    the same buckets."""
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    be.warmup()
    direct = backend_with(cfg, w, "graphs=0")
    try:
        lens = [70, 71, 90, 100, 111, 126, 97, 83]
        ks = [0, 1, 2, 3, 4, 5, 9, 7]
        for i, it in enumerate(make_rows(cfg, 40, lens, ks)):
            v = Varlen.from_rows([it])
            a, b = be.forward_varlen(v), direct.forward_varlen(v)
            assert a.logits.shape == (len(it.markers),)
            assert np.array_equal(a.logits, b.logits) and np.array_equal(a.pooled, b.pooled), i
            assert np.all(np.isfinite(a.pooled))
    finally:
        direct.close()


def test_buckets_leave_rows_unchanged(cuda_lib):
    """The same batches with and without buckets agree to rounding, and the bucketed ones match the
    CPU oracle (single rows, a multi-row batch, a row with no markers, kmax past a bucket step)."""
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    plain = backend_with(cfg, w, "buckets=0")
    try:
        cases = [([5], [2]), ([64], [5]), ([127], [0]), ([128], [3]), ([33, 12, 90], [3, 9, 1]),
                 ([200, 1, 17, 40, 3], [4, 0, 2, 13, 1]), ([100, 28], [2, 2])]
        for seed, (lens, ks) in enumerate(cases):
            items = make_rows(cfg, 50 + seed, lens, ks)
            batch = collate_to(items, cfg.encoder.pad_token_id)
            a, b = be.forward(batch), plain.forward(batch)
            assert a.logits.shape == b.logits.shape
            if a.logits.size:
                assert np.abs(a.logits - b.logits).max() < 2e-3
            assert np.linalg.norm(a.pooled - b.pooled) / np.linalg.norm(b.pooled) < 1e-2
            masked = np.ones(batch.n * batch.kmax, bool)
            for r in range(batch.n):
                masked[r * batch.kmax: r * batch.kmax + int(batch.marker_count[r])] = False
            assert np.all(a.logits[masked] == -1e4)
            check_against_oracle(cfg, w, be, batch)
    finally:
        plain.close()


def test_bucketed_device_and_hidden_entry_points(cuda_lib):
    """The device-resident entry point (logits copied out of the bucket's wider rows) and the
    hidden-state output (the batch's own tokens only) give the host entry point's outputs."""
    import torch
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    items = make_rows(cfg, 60, [45, 9, 77], [5, 2, 6])
    v = Varlen.from_rows(items)
    ref = be.forward_varlen(v)
    hid = be.forward_varlen(v, hidden=True)
    assert np.array_equal(hid.logits, ref.logits) and np.array_equal(hid.pooled, ref.pooled)
    assert hid.hidden.shape == (v.total * cfg.encoder.hidden_size,)
    assert np.all(np.isfinite(hid.hidden))
    ids = torch.from_numpy(v.ids.astype(np.int32)).cuda()
    lg = torch.full((v.n * v.kmax + 8,), 7.0, device="cuda")
    pl = torch.empty(v.n * cfg.encoder.hidden_size, device="cuda")
    be.forward_device(v, ids.data_ptr(), lg.data_ptr(), pl.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(lg[: v.n * v.kmax].cpu().numpy(), ref.logits)
    assert np.all(lg[v.n * v.kmax:].cpu().numpy() == 7.0)  # nothing written past the batch's logits
    assert np.array_equal(pl.cpu().numpy(), ref.pooled)


def test_bucket_settings_are_checked(cuda_lib):
    from conftest import get_backend
    from sys1rust_b200.config import ConfigError
    cfg, w, _ = get_backend("small:3")
    for bad in ("buckets=12x", "buckets=128:-4", "warm=a"):
        with pytest.raises(ConfigError, match="is not a whole number"):
            backend_with(cfg, w, bad)
    be = backend_with(cfg, w, "buckets=256:64,warm=1:3")
    try:
        be.warmup()
        out = be.forward_varlen(Varlen.from_rows(make_rows(cfg, 61, [300], [2])))  # past the largest bucket
        assert np.all(np.isfinite(out.pooled))
    finally:
        be.close()


def test_trace_layers_and_ops_lines(cuda_lib, capfd):
    """`trace`, `layers` and `ops` (the reference's tracing knobs) print one line per forward, the
    device time of every encoder layer and the per-kernel sums to stderr; outputs are unchanged."""
    from conftest import get_backend
    cfg, w, be = get_backend("small:3")
    v = Varlen.from_rows(make_rows(cfg, 80, [50, 70], [2, 3]))
    ref = be.forward_varlen(v)
    capfd.readouterr()
    tr = backend_with(cfg, w, "trace=1,layers=1,ops")
    try:
        out = tr.forward_varlen(v)
        err = capfd.readouterr().err
        assert "s1c trace: rows 2 tokens 120 kmax 3 bucket 128x4x4, direct" in err, err
        layer_line = [l for l in err.splitlines() if l.startswith("s1c layers (ms):")]
        assert len(layer_line) == 1 and len(layer_line[0].split()) == 3 + cfg.encoder.num_hidden_layers
        assert "s1c ops: gemm_qkv_rope" in err and "attn_global" in err
        assert np.array_equal(out.logits, ref.logits) and np.array_equal(out.pooled, ref.pooled)
    finally:
        tr.close()
