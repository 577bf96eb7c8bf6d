"""The CPU oracle pinned against golden outputs of the model the reference reproduces
(transformers' ModernBertModel + torch TransformerEncoderLayer head + scorer, fp32), written by
``tests/golden/make_golden.py``. Also bounds the bf16-storage emulation of the oracle, which is
the precision budget the device path works within."""
import os

import numpy as np
import pytest

from sys1rust_b200.batch import Batch
from sys1rust_b200.config import large_model, small_model
from sys1rust_b200.weights import SyntheticWeights

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(name):
    z = np.load(os.path.join(HERE, "golden", f"hf_{name}.npz"))
    b = Batch(int(z["n"]), int(z["len"]), int(z["kmax"]), z["input_ids"], z["attention_mask"], z["seq_lens"],
              z["marker_pos"], z["marker_count"], z["qtype"])
    return z, b


@pytest.mark.parametrize("name,cfgf", [("small", small_model), ("large", large_model)])
def test_oracle_matches_hf_golden(name, cfgf):
    from oracle.forward_ref import OracleModel
    z, b = _load(name)
    cfg = cfgf()
    w = SyntheticWeights(cfg, seed=int(z["weight_seed"]))
    logits, pooled, hidden = OracleModel(cfg, w.tensors).forward(b)
    am = b.attention_mask.reshape(b.n, b.len).astype(bool)
    ref = z["hidden_real"]
    assert np.linalg.norm(hidden[am] - ref) / np.linalg.norm(ref) < 1e-5
    assert np.abs(logits - z["logits"]).max() < 1e-5
    assert np.abs(pooled - z["pooled"].reshape(-1)).max() < 1e-4
    # masked marker slots
    for r in range(b.n):
        for k in range(int(b.marker_count[r]), b.kmax):
            assert logits[r * b.kmax + k] == np.float32(-1e4)


def test_bf16_storage_emulation_within_tolerance():
    """bf16 storage of GEMM inputs, q/k/v and activations with an fp32 residual stream stays well
    inside the 2e-2 relative hidden-state bound on the large config."""
    from oracle.forward_ref import OracleModel
    z, b = _load("large")
    cfg = large_model()
    w = SyntheticWeights(cfg, seed=int(z["weight_seed"]))
    _, _, hidden = OracleModel(cfg, w.tensors, emulate_bf16=True).forward(b)
    am = b.attention_mask.reshape(b.n, b.len).astype(bool)
    ref = z["hidden_real"]
    assert np.linalg.norm(hidden[am] - ref) / np.linalg.norm(ref) < 1e-2


def test_weights_are_seeded_and_order_independent():
    cfg = small_model()
    a = SyntheticWeights(cfg, seed=5)
    b = SyntheticWeights(cfg, seed=5)
    c = SyntheticWeights(cfg, seed=6)
    for k in a.tensors:
        assert np.array_equal(a.tensors[k], b.tensors[k])
    assert not np.array_equal(a.tensors["type_emb.weight"], c.tensors["type_emb.weight"])
    from sys1rust_b200.weights import gen_tensor
    assert np.array_equal(gen_tensor(5, "type_emb.weight", (3, 256), "w"), a.tensors["type_emb.weight"])
    ln = a.f32("encoder.final_norm.weight")
    assert abs(float(ln.mean()) - 1.0) < 0.01


def test_checkpoint_roundtrip(tmp_path):
    from sys1rust_b200.config import ModelConfig
    from sys1rust_b200.weights import load_safetensors_bits
    cfg = small_model()
    w = SyntheticWeights(cfg, seed=1)
    w.save(str(tmp_path))
    t = load_safetensors_bits(str(tmp_path / "model.safetensors"))
    assert set(t) == set(w.tensors)
    for k, (dt, shape, arr) in t.items():
        assert dt == "BF16" and tuple(shape) == w.tensors[k].shape
        assert np.array_equal(arr, w.tensors[k])
    cfg2 = ModelConfig.load(str(tmp_path))
    assert cfg2.encoder.layer_is_local == cfg.encoder.layer_is_local
    assert cfg2.encoder.hidden_size == cfg.encoder.hidden_size
