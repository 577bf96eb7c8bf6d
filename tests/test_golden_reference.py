"""Host logic against the reference's own known answers (``tests/golden/reference_vectors.json``,
transcribed from the reference's unit tests; each entry names its source test)."""
import json
import os

import numpy as np
import pytest

from sys1rust_b200.batch import Batch, Packing, Varlen, collate_to, EncodedItem
from sys1rust_b200.config import ConfigError, EncoderConfig

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "reference_vectors.json")) as f:
    GOLD = json.load(f)


def _gold_batch():
    b = GOLD["packing"]["batch"]
    return Batch(b["n"], b["len"], b["kmax"], np.array(b["input_ids"], np.uint32),
                 np.array(b["attention_mask"], np.uint32), np.array(b["seq_lens"], np.int64),
                 np.array(b["marker_pos"], np.uint32), np.array(b["marker_count"], np.int64),
                 np.array(b["qtype"], np.uint32))


def test_packing_matches_reference_vectors():
    g = GOLD["packing"]
    p = Packing.new(_gold_batch())
    assert p.offsets.tolist() == g["offsets"]
    assert p.pack.tolist() == g["pack"]
    assert p.unpack.tolist() == g["unpack"]
    assert p.row.tolist() == g["row"]


def test_scorer_rows_match_reference_vectors():
    g = GOLD["packing"]
    b = _gold_batch()
    v = Varlen.from_batch(b)
    assert v.scorer_rows().tolist() == g["scorer_rows_packed"]
    # padded layout: row starts r * len
    padded = []
    for r in range(b.n):
        base = r * b.len
        padded += [base] + [base + int(m) for m in b.marker_pos[r * b.kmax:(r + 1) * b.kmax]]
    assert padded == g["scorer_rows_padded"]


def test_varlen_positions_and_cu_seqlens():
    b = _gold_batch()
    v = Varlen.from_batch(b)
    assert v.cu_seqlens.tolist() == [0, 2, 6, 7]
    assert v.positions.tolist() == [0, 1, 0, 1, 2, 3, 0]
    assert v.ids.tolist() == [1, 2, 3, 4, 5, 6, 7]


def test_window_rule_matches_reference_mask():
    g = GOLD["window_mask"]
    L, w = g["len"], g["w"]
    want = np.array(g["values"], np.float32)
    i, j = np.meshgrid(np.arange(L), np.arange(L), indexing="ij")
    got = np.where(np.abs(i - j) <= w, 0.0, -1e4).astype(np.float32)
    assert np.array_equal(got, want)


def test_window_key_idx_formula():
    """The chunked-path gather index rule of the reference (its windows cover exactly the keys
    the varlen kernel's per-tile key range [q0 - w, q1 + w] covers)."""
    for s, rows, L in GOLD["window_key_idx"]["cases"]:
        nc = -(-L // s)
        idx = [r * L + min(max((c - 1) * s + j, 0), L - 1) for r in range(rows) for c in range(nc) for j in range(3 * s)]
        # every query position of chunk c, window s, finds all its keys inside chunk c's gather
        for c in range(nc):
            for q in range(c * s, min(c * s + s, L)):
                needed = {k for k in range(max(0, q - s), min(L, q + s + 1))}
                have = {min(max((c - 1) * s + j, 0), L - 1) for j in range(3 * s)}
                assert needed <= have
        assert len(idx) == rows * nc * 3 * s


def test_chunked_mask_tables_equal_the_varlen_window_rule():
    """The reference's chunked local-attention masks on its own padded fixture (``chunked_mask``):
    key slot j of chunk c is position (c - 1) S + j, valid when inside the row's real tokens; the
    band allows i + 2S >= j >= i; a padded query row is all true. For every real query the allowed
    positions are exactly the key range the varlen kernels compute from the row bounds,
    [max(0, q - w), min(len_b, q + w + 1)) with w = S (attention_tc.cuh / attention.cuh), and no
    query row is empty."""
    g = GOLD["chunked_mask"]
    mask, n, L, S, nc = np.array(g["mask"]), g["n"], g["len"], g["s"], g["nc"]
    for b in range(n):
        real = int(mask[b * L:(b + 1) * L].sum())  # right-padded rows: real tokens [0, real)
        for c in range(nc):
            slots = [(c - 1) * S + j for j in range(3 * S)]
            key_ok = [0 <= p < L and mask[b * L + p] == 1 for p in slots]
            for i in range(S):
                q = c * S + i
                padded = q >= L or mask[b * L + q] != 1
                band = [i + 2 * S >= j >= i for j in range(3 * S)]
                row = [(k and bd) or padded for k, bd in zip(key_ok, band)]
                assert any(row), (b, q)
                if not padded:
                    got = {p for p, v in zip(slots, row) if v}
                    k_lo, k_hi = max(0, q - S), min(real, q + S + 1)
                    assert got == set(range(k_lo, k_hi)), (b, q, got)
    # row 1's last chunk holds padding only
    b, c = 1, 3
    assert not any(0 <= (c - 1) * S + j < L and mask[b * L + (c - 1) * S + j] == 1 for j in range(3 * S))


def test_head_scale_matches_reference():
    for hidden, heads, want in GOLD["head_scale"]["cases"]:
        got = float(np.float32(1.0) / np.sqrt(np.float32(hidden // heads)))
        assert got == pytest.approx(want, rel=0, abs=0) or abs(got - want) < 1e-7


def _minimal(extra):
    v = {"model_type": "modernbert", "vocab_size": 100, "hidden_size": 64, "num_hidden_layers": 6,
         "num_attention_heads": 2, "intermediate_size": 96}
    v.update(extra)
    return v


def test_layer_pattern_matches_reference():
    g = GOLD["layer_pattern"]
    assert EncoderConfig.from_value(_minimal({})).layer_is_local == g["every3_6"]
    assert EncoderConfig.from_value(_minimal({"global_attn_every_n_layers": 2})).layer_is_local == g["every2_6"]
    types = ["sliding_attention", "full_attention", "sliding_attention", "sliding_attention", "full_attention",
             "sliding_attention"]
    assert EncoderConfig.from_value(_minimal({"layer_types": types})).layer_is_local == g["override"]
    big = EncoderConfig.from_value({"model_type": "modernbert", "vocab_size": 50368, "hidden_size": 1024,
                                    "num_hidden_layers": 28, "num_attention_heads": 16, "intermediate_size": 2560,
                                    "global_attn_every_n_layers": 3, "local_attention": 128})
    assert big.layer_is_local == g["large_28"]


def test_config_shape_errors_match_reference_messages():
    with pytest.raises(ConfigError, match="num_attention_heads must be at least 1"):
        EncoderConfig.from_value(_minimal({"num_attention_heads": 0}))
    with pytest.raises(ConfigError, match="hidden_size 65 is not a multiple of num_attention_heads 2"):
        EncoderConfig.from_value(_minimal({"hidden_size": 65}))
    with pytest.raises(ConfigError, match="not a multiple of the 3 decision-head attention heads"):
        EncoderConfig.from_value(_minimal({"hidden_size": 200, "num_attention_heads": 2}))
    for w in (0, 1):
        with pytest.raises(ConfigError, match="local_attention must be at least 2"):
            EncoderConfig.from_value(_minimal({"local_attention": w}))
    with pytest.raises(ConfigError, match="global_attn_every_n_layers must be at least 1"):
        EncoderConfig.from_value(_minimal({"global_attn_every_n_layers": 0}))
    with pytest.raises(ConfigError, match="only 'modernbert'"):
        EncoderConfig.from_value({**_minimal({}), "model_type": "bert"})


def test_rope_theta_layouts():
    v4 = EncoderConfig.from_value(_minimal({"global_rope_theta": 1234.0, "local_rope_theta": 55.0}))
    assert (v4.global_rope_theta, v4.local_rope_theta) == (1234.0, 55.0)
    v5 = EncoderConfig.from_value(_minimal({"rope_parameters": {"full_attention": {"rope_theta": 99.0},
                                                                "sliding_attention": {"rope_theta": 7.0}}}))
    assert (v5.global_rope_theta, v5.local_rope_theta) == (99.0, 7.0)


def test_collate_right_pads_and_validates():
    items = [EncodedItem([1, 5, 6, 2], [1, 2], 0), EncodedItem([1, 2], [], 2)]
    b = collate_to(items, pad_id=9)
    assert (b.n, b.len, b.kmax) == (2, 4, 2)
    assert b.input_ids.tolist() == [1, 5, 6, 2, 1, 2, 9, 9]
    assert b.attention_mask.tolist() == [1, 1, 1, 1, 1, 1, 0, 0]
    assert b.marker_pos.tolist() == [1, 2, 0, 0]
    b.validate()
    b.attention_mask[3] = 0
    with pytest.raises(ValueError, match="attention mask"):
        b.validate()


def test_noul_decode_known_answer():
    g = GOLD["noul_decode"]
    z = np.array(g["logits"], np.float64)
    p = np.exp(z - z.max())
    p /= p.sum()
    assert round(float(p[1]), 4) == g["noul"]
