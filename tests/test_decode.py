"""Answer decoding (``s1c_decode`` through ``sys1rust_b200.decode``) on CPU: the known answers of the
reference's decode tests (runtime/crates/laya-core/src/decode.rs:425-640), and random rows against
the CPU restatement in ``oracle/decode_ref.py``.
"""
import math

import numpy as np
import pytest

from oracle import decode_ref
from sys1rust_b200.backend import WeightsError
from sys1rust_b200.decode import ActHead, Temperatures, clamp_temperature, decode, temp_bucket


def _zero_head(d):
    """decode.rs:527-537: one hidden unit, two classes, all zero (probabilities 0.5 / 0.5)."""
    return ActHead(np.zeros((1, d + 4)), np.zeros(1), np.zeros((2, 1)), np.zeros(2))


def test_temperature_clamping_and_buckets():
    # decode.rs:425-435
    assert clamp_temperature(0.1006) == 0.5
    assert clamp_temperature(7.0) == 5.0
    assert clamp_temperature("1.5") == 1.5
    assert clamp_temperature("abc") == 1.0
    assert clamp_temperature(None) == 1.0
    assert clamp_temperature(float("nan")) == 1.0
    assert temp_bucket(0, 20) == "choice:11+"
    assert temp_bucket(2, 2) == "noul:2"
    assert temp_bucket(1, 5) == "score:3-5"
    assert temp_bucket(0, 6) == "choice:6-10"
    t = Temperatures.from_config([0.1, "2", 1.0], {"choice:2": 9})
    assert t.by_type == [0.5, 2.0, 1.0] and t.scale(0, 2) == 5.0 and t.scale(0, 3) == 0.5
    assert len(t.rejected) == 3


def test_answer_confidence_per_type():
    # decode.rs:560-625: choice over 3, score over 3, noul over 2 (kmax 3), temperatures 1
    logits = np.array([2.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, -1.0, -1e4], np.float32)
    ans, probs = decode(logits, np.zeros(6, np.float32), [3, 3, 2], [0, 1, 2], 3, 2, Temperatures(), _zero_head(2))
    pick, rate, yes = ans
    assert pick["argmax"] == 0
    assert round(pick["answer_confidence"], 4) == 0.787 and abs(pick["answer_confidence"] - probs[0, 0]) == 0
    assert abs(pick["answer_confidence"] - math.exp(2) / (math.exp(2) + 2)) < 1e-12
    assert round(rate["answer_confidence"], 4) == 0.5761
    assert abs(rate["score"] - (1 * math.e + 2 * 1) / (math.e + 2)) < 1e-12
    assert round(yes["noul"], 4) == 0.2689 and round(yes["confidence"], 4) == 0.7311
    assert yes["answer_confidence"] == yes["confidence"]
    assert all(a["act_probability"] == 0.5 for a in ans)  # zero head: 0.5 / 0.5
    assert probs[2, 2] == 0.0  # past marker_count


def test_confidence_known_answers():
    # decode.rs:521-525
    assert decode_ref.confidence_from_probs([1.0], 1) == 1.0
    lg = np.array([0.0, 0.0, 50.0, -50.0], np.float32)
    ans, _ = decode(lg, np.zeros(4, np.float32), [2, 2], [0, 0], 2, 2, Temperatures(), _zero_head(2))
    assert abs(ans[0]["confidence"]) < 1e-12
    assert abs(ans[1]["confidence"] - 1.0) < 1e-9


def test_act_head_shape_checks():
    # decode.rs:459-517
    with pytest.raises(WeightsError, match="needs at least 5"):
        ActHead(np.zeros((8, 4)), np.zeros(8), np.zeros((2, 8)), np.zeros(2))
    with pytest.raises(WeightsError, match="biases have 7 and 2 values"):
        ActHead(np.zeros((8, 6)), np.zeros(7), np.zeros((2, 8)), np.zeros(2))
    head = ActHead(np.zeros((8, 6)), np.zeros(8), np.zeros((2, 8)), np.zeros(2))
    assert (head.d_in, head.hidden, head.n_act) == (6, 8, 2)
    with pytest.raises(WeightsError, match="not the encoder hidden size 1024 plus 4 scalar features"):
        decode(np.zeros(2, np.float32), np.zeros(1024, np.float32), [2], [2], 2, 1024, Temperatures(), head)


def test_random_rows_match_the_restatement():
    rng = np.random.default_rng(0)
    d, H, n_act, kmax, n = 32, 16, 3, 6, 40
    w0 = rng.standard_normal((H, d + 4)).astype(np.float32) * 0.3
    b0 = rng.standard_normal(H).astype(np.float32) * 0.1
    w2 = rng.standard_normal((n_act, H)).astype(np.float32) * 0.3
    b2 = rng.standard_normal(n_act).astype(np.float32) * 0.1
    head = ActHead(w0, b0, w2, b2)
    mc = rng.integers(0, kmax + 1, n)
    qt = rng.integers(0, 3, n)
    logits = (rng.standard_normal((n, kmax)) * 3).astype(np.float32)
    for r in range(n):
        logits[r, mc[r]:] = -1e4
    pooled = rng.standard_normal((n, d)).astype(np.float32)
    temps = Temperatures.from_config([0.7, 1.3, 2.0], {"score:3-5": 0.9})
    ans, probs = decode(logits, pooled, mc, qt, kmax, d, temps, head)
    for r in range(n):
        ref, p = decode_ref.decode_row(logits[r], pooled[r], int(mc[r]), int(qt[r]), temps.scale(int(qt[r]), int(mc[r])),
                                       (w0, b0, w2, b2))
        a = ans[r]
        assert a["type"] == ref["type"] and a["k"] == ref["k"]
        for key in ("confidence", "answer_confidence", "score", "noul"):
            if key in ref:
                assert abs(a[key] - ref[key]) < 1e-12, (r, key)
        if "argmax" in ref:
            assert a["argmax"] == ref["argmax"]
        assert np.allclose(probs[r, :mc[r]], p, atol=1e-12, rtol=0)
        assert abs(a["act_probability"] - ref["act_probability"]) < 2e-6, (r, a["act_probability"], ref["act_probability"])
