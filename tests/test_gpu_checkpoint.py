"""A checkpoint directory loaded through the library's reader (``CudaBackend.from_dir``:
``s1c_weights_open`` + ``s1c_create_from_weights``) gives the same forward as the same tensors
handed over in memory, for BF16 files and for F16 files (the reference's checkpoint dtype,
converted to bf16 at load, laya-core/src/weights.rs:82-115); and a truncated file is refused before
anything reaches the GPU.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _batch(vocab):
    from sys1rust_b200.batch import Varlen
    from sys1rust_b200.workloads import _row
    rng = np.random.default_rng(7)
    return Varlen.from_rows([_row(rng, vocab, L, q) for L, q in [(40, [0, 1]), (97, [2]), (5, [1])]])


@pytest.mark.parametrize("dtype", ["BF16", "F16"])
def test_checkpoint_dir_matches_in_memory_tensors(cuda_lib, tmp_path, dtype):
    from sys1rust_b200.backend import CudaBackend
    from sys1rust_b200.config import small_model
    from sys1rust_b200.weights import SyntheticWeights, bf16_bits_to_f16_bits
    cfg = small_model()
    w = SyntheticWeights(cfg, seed=11)
    w.save(str(tmp_path), dtype=dtype)
    v = _batch(cfg.encoder.vocab_size)
    a = CudaBackend.from_dir(str(tmp_path))
    if dtype == "BF16":
        b = CudaBackend.from_synthetic(cfg, w.tensors)
    else:
        b = CudaBackend(cfg, {k: ("F16", t.shape, bf16_bits_to_f16_bits(t)) for k, t in w.tensors.items()})
    try:
        oa, ob = a.forward_varlen(v), b.forward_varlen(v)
        assert np.array_equal(oa.logits, ob.logits)
        assert np.array_equal(oa.pooled, ob.pooled)
        assert np.isfinite(oa.logits).all()
    finally:
        a.close()
        b.close()


def test_truncated_checkpoint_is_refused_before_the_gpu(cuda_lib, tmp_path):
    from sys1rust_b200.backend import CudaBackend, WeightsError
    from sys1rust_b200.config import small_model
    from sys1rust_b200.weights import SyntheticWeights
    w = SyntheticWeights(small_model(), seed=12)
    w.save(str(tmp_path), dtype="F16")
    p = tmp_path / "model.safetensors"
    full = p.read_bytes()
    p.write_bytes(full[: len(full) // 2])
    with pytest.raises(WeightsError, match=rf"model.safetensors \({len(full) // 2} bytes\) is truncated"):
        CudaBackend.from_dir(str(tmp_path))
