"""The C restatement of the forward (``oracle/forward_ref.c``, the timed CPU baseline's second
form) against the PyTorch oracle (``oracle/forward_ref.py``) on the small config: two independent
fp32 restatements of ``MlxBackend::forward`` (runtime/crates/laya-mlx/src/lib.rs:1833-1863) that
must agree to fp32 rounding, including the pruned last head layer (lib.rs:1726-1760) and the
masked marker slots (lib.rs:1851-1857)."""
import numpy as np
import pytest

from oracle.forward_c import CForwardModel
from oracle.forward_ref import OracleModel
from sys1rust_b200.batch import collate_to
from sys1rust_b200.config import small_model
from sys1rust_b200.weights import SyntheticWeights
from sys1rust_b200.workloads import _row


@pytest.fixture(scope="module")
def models():
    cfg = small_model()
    w = SyntheticWeights(cfg, seed=3)
    return cfg, OracleModel(cfg, w.tensors), CForwardModel(cfg, w.tensors)


@pytest.mark.parametrize("L,qtypes", [(1, []), (2, [2]), (40, [0, 1]), (130, [1, 1, 0]), (300, [2])])
def test_c_restatement_matches_the_torch_oracle(models, L, qtypes):
    cfg, om, cm = models
    rng = np.random.default_rng(L)
    it = _row(rng, cfg.encoder.vocab_size, L, qtypes) if L > 2 else None
    if it is None:  # rows too short for [CLS] ... [SEP] with markers: ids and markers by hand
        from sys1rust_b200.batch import EncodedItem
        it = EncodedItem([1] * (L - 1) + [2], [0] * (2 if qtypes else 0), qtypes[0] if qtypes else 0)
    b = collate_to([it], cfg.encoder.pad_token_id)
    lo, po, _ = om.forward(b)
    kmax = max(len(it.markers), 1) + 2  # two padded slots past marker_count
    lc, pc = cm.forward_row(np.array(it.ids), it.markers, it.qtype, kmax=kmax)
    assert np.all(lc[len(it.markers):] == np.float32(-1e4))
    assert np.abs(lc[:len(it.markers)] - lo[:len(it.markers)]).max(initial=0) < 1e-5
    assert np.abs(pc - po).max() < 1e-5 * max(1.0, np.abs(po).max())
