"""Generate the golden fixtures under ``tests/golden/``.

Two kinds of fixture are written:

1. ``reference_vectors.json`` -- known answers taken from the reference's own unit tests
   (read as text; each entry cites the test it comes from). They pin the integer parts of the
   path: packing indices, scorer rows, the window rule, the head scale, the layer pattern.

2. ``hf_<name>.npz`` -- outputs of the model the reference reproduces, built from
   transformers' ``ModernBertModel`` (encoder) plus ``torch.nn.TransformerEncoderLayer``
   (pre-norm decision-head layers) plus the scorer ``LayerNorm -> Linear -> GELU -> Linear``,
   loaded with the seeded synthetic weights of ``sys1rust_b200.weights`` and run in fp32 on
   the CPU. The reference checks its MLX forward against exactly this model's fp32 answers
   (``runtime/crates/laya-mlx/tests/reference.rs:22-29``), so these outputs pin the CPU oracle
   without depending on it. The weights are regenerated from the seed by the tests, so only
   the inputs and outputs are stored.

Run from the repository root: ``python tests/golden/make_golden.py``. Needs transformers
(present in the build container, not needed on the GPU box).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from sys1rust_b200.batch import EncodedItem, collate_to  # noqa: E402
from sys1rust_b200.config import ModelConfig, large_model, small_model  # noqa: E402
from sys1rust_b200.weights import SyntheticWeights, bf16_to_f32  # noqa: E402


def reference_vectors() -> dict:
    """Known answers transcribed from the reference's tests (file:line cited per entry)."""
    return {
        "packing": {
            "source": "runtime/crates/laya-mlx/src/lib.rs:2008-2032 packing_indexes_real_tokens_and_scorer_rows",
            "batch": {"n": 3, "len": 4, "kmax": 2,
                      "input_ids": [1, 2, 0, 0, 3, 4, 5, 6, 7, 0, 0, 0],
                      "attention_mask": [1, 1, 0, 0, 1, 1, 1, 1, 1, 0, 0, 0],
                      "seq_lens": [2, 4, 1], "marker_pos": [1, 0, 1, 3, 0, 0],
                      "marker_count": [1, 2, 0], "qtype": [0, 1, 2]},
            "offsets": [0, 2, 6],
            "pack": [0, 1, 4, 5, 6, 7, 8],
            "unpack": [0, 1, 0, 0, 2, 3, 4, 5, 6, 6, 6, 6],
            "row": [0, 0, 1, 1, 1, 1, 2],
            "scorer_rows_padded": [0, 1, 0, 4, 5, 7, 8, 8, 8],
            "scorer_rows_packed": [0, 1, 0, 2, 3, 5, 6, 6, 6],
        },
        "head_scale": {
            "source": "runtime/crates/laya-mlx/src/lib.rs:2125-2132 head_scale_follows_the_head_dim",
            "cases": [[768, 12, 0.125], [1024, 16, 0.125], [512, 8, 0.125],
                      [96, 1, float(1.0 / np.sqrt(np.float32(96)))],
                      [160, 2, float(1.0 / np.sqrt(np.float32(80)))]],
        },
        "layer_pattern": {
            "source": "runtime/crates/laya-core/src/config.rs:249-308",
            "every3_6": [False, True, True, False, True, True],
            "every2_6": [False, True, False, True, False, True],
            "large_28": [i % 3 != 0 for i in range(28)],
            "base_22": [i % 3 != 0 for i in range(22)],
            "override": [True, False, True, True, False, True],
        },
        "window_mask": {
            "source": "runtime/crates/laya-mlx/src/lib.rs:2135-2156 window_view_is_the_corner_of_the_longer_mask",
            "rule": "|i - j| > w is MASK_NEG (-1e4), else 0",
            "len": 8, "w": 2,
            "values": [[0.0 if abs(i - j) <= 2 else -1e4 for j in range(8)] for i in range(8)],
        },
        "window_key_idx": {
            "source": "runtime/crates/laya-mlx/src/lib.rs:2160-2173 window_key_idx_matches_the_host_formula",
            "rule": "r * len + clamp((c - 1) * S + j, 0, len - 1), row-major over (r, c, j)",
            "cases": [[2, 3, 7], [4, 1, 4], [64, 2, 130]],
        },
        "noul_decode": {
            "source": "runtime/crates/laya-core/src/testing.rs:744-748",
            "logits": [0.0, 1.0], "noul": 0.7311,
        },
        "mask_neg": {"source": "runtime/crates/laya-mlx/src/lib.rs:43-45", "mask_neg": -1e4, "logit_masked": -1e4},
    }


def build_hf_model(cfg: ModelConfig, w: SyntheticWeights):
    from transformers import ModernBertConfig, ModernBertModel
    e = cfg.encoder
    hcfg = ModernBertConfig(
        vocab_size=e.vocab_size, hidden_size=e.hidden_size, num_hidden_layers=e.num_hidden_layers,
        num_attention_heads=e.num_attention_heads, intermediate_size=e.intermediate_size,
        norm_eps=e.norm_eps, global_attn_every_n_layers=e.global_attn_every_n_layers,
        local_attention=e.local_attention, pad_token_id=e.pad_token_id,
        global_rope_theta=e.global_rope_theta, local_rope_theta=e.local_rope_theta,
        max_position_embeddings=e.max_position_embeddings,
        hidden_activation="gelu", norm_bias=False, attention_bias=False, mlp_bias=False,
        attention_dropout=0.0, embedding_dropout=0.0, mlp_dropout=0.0,
    )
    hcfg._attn_implementation = "eager"
    enc = ModernBertModel(hcfg).eval()
    sd = {}
    for k in enc.state_dict().keys():
        name = "encoder." + k
        sd[k] = torch.from_numpy(bf16_to_f32(w.bits(name)).copy())
    enc.load_state_dict(sd, strict=True)

    d, nh = e.hidden_size, e.head_nheads()
    head = torch.nn.ModuleList([
        torch.nn.TransformerEncoderLayer(d, nh, dim_feedforward=cfg.head_ffn, dropout=0.0,
                                         activation="relu", batch_first=True, norm_first=True,
                                         layer_norm_eps=1e-5)
        for _ in range(cfg.head_layers)]).eval()
    hsd = {k: torch.from_numpy(bf16_to_f32(w.bits("head.layers." + k)).copy()) for k in head.state_dict()}
    head.load_state_dict(hsd, strict=True)
    type_emb = torch.from_numpy(bf16_to_f32(w.bits("type_emb.weight")).copy())
    scorer = torch.nn.Sequential(torch.nn.LayerNorm(d, eps=1e-5), torch.nn.Linear(d, cfg.scorer_hidden),
                                 torch.nn.GELU(), torch.nn.Linear(cfg.scorer_hidden, 1)).eval()
    ssd = {k: torch.from_numpy(bf16_to_f32(w.bits("scorer." + k)).copy()) for k in scorer.state_dict()}
    scorer.load_state_dict(ssd, strict=True)
    return enc, head, type_emb, scorer


@torch.no_grad()
def hf_forward(cfg, w, batch):
    enc, head, type_emb, scorer = build_hf_model(cfg, w)
    n, L, kmax = batch.n, batch.len, batch.kmax
    ids = torch.from_numpy(batch.input_ids.astype(np.int64)).view(n, L)
    am = torch.from_numpy(batch.attention_mask.astype(np.int64)).view(n, L)
    hidden = enc(input_ids=ids, attention_mask=am).last_hidden_state
    qt = torch.from_numpy(batch.qtype.astype(np.int64))
    h = hidden + type_emb[qt].view(n, 1, -1)
    kpm = am == 0
    for layer in head:
        # The slow path (training-mode semantics, dropout 0) keeps every position computed.
        layer.train()
        h = layer(h, src_key_padding_mask=kpm)
        layer.eval()
    mp = torch.from_numpy(batch.marker_pos.astype(np.int64)).view(n, kmax)
    rows = torch.arange(n).view(n, 1).expand(n, kmax)
    m = h[rows.reshape(-1), mp.reshape(-1)]
    logits = scorer(m).reshape(-1).numpy().astype(np.float32)
    for r in range(n):
        logits[r * kmax + int(batch.marker_count[r]):(r + 1) * kmax] = -1e4
    return logits, h[:, 0, :].numpy().astype(np.float32), hidden.numpy().astype(np.float32)


def golden_batch(cfg: ModelConfig, seed: int, lens, markers_per_row, qtypes) -> "Batch":
    rng = np.random.Generator(np.random.PCG64(seed))
    e = cfg.encoder
    items = []
    for L, k, qt in zip(lens, markers_per_row, qtypes):
        ids = rng.integers(4, e.vocab_size, size=L).astype(np.uint32)
        ids[0], ids[-1] = 1, 2  # CLS / SEP stand-ins
        markers = sorted(rng.choice(np.arange(1, L - 1), size=k, replace=False).tolist())
        items.append(EncodedItem(ids.tolist(), markers, qt))
    return collate_to(items, e.pad_token_id)


def main() -> None:
    with open(os.path.join(HERE, "reference_vectors.json"), "w") as f:
        json.dump(reference_vectors(), f, indent=1)
    torch.manual_seed(0)
    cases = [
        ("small", small_model(), 7, [37, 12, 50, 1 + 1], [3, 2, 4, 0], [0, 2, 1, 2]),
        ("large", large_model(), 11, [80, 23, 150], [2, 3, 4], [2, 0, 1]),
    ]
    for name, cfg, seed, lens, ks, qts in cases:
        w = SyntheticWeights(cfg, seed=seed)
        batch = golden_batch(cfg, seed + 100, lens, ks, qts)
        logits, pooled, hidden = hf_forward(cfg, w, batch)
        am = batch.attention_mask.reshape(batch.n, batch.len).astype(bool)
        np.savez_compressed(
            os.path.join(HERE, f"hf_{name}.npz"),
            weight_seed=np.int64(seed), n=np.int64(batch.n), len=np.int64(batch.len), kmax=np.int64(batch.kmax),
            input_ids=batch.input_ids, attention_mask=batch.attention_mask, seq_lens=batch.seq_lens,
            marker_pos=batch.marker_pos, marker_count=batch.marker_count, qtype=batch.qtype,
            logits=logits, pooled=pooled, hidden_real=hidden[am])
        print(name, "logits", logits[:6], "pooled[0,:4]", pooled[0, :4])


if __name__ == "__main__":
    main()
