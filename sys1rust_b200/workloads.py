"""Seeded synthetic workloads with the shapes of the benchmark configs.

Rows follow the reference's ``Batch`` contract (``laya-core/src/backend.rs:74-98``): one qtype
per row (the type embedding is row-wide, ``laya-mlx/src/lib.rs:1702-1708``), one marker per
answer option. A request with several questions is one row holding the state and every
question segment; its markers are the options of all its questions (choice 3, score 4, noul 2)
and its row qtype is that of its first question. Token ids are uniform in [4, vocab), with
id 1 standing in for [CLS] at position 0 and id 2 for [SEP] at the end (the tokenizer is absent).

* cfg1 -- 1 row x 128 tokens, one noul question (2 markers).
* cfg2 -- 1 row x 512 tokens, 10 questions (4 choice, 3 score, 3 noul = 30 markers).
* cfg3 -- 64 rows, lengths U[64, 512], 3 questions each (3 + 4 + 2 markers).
* latency stream -- single requests of U[64, 200] tokens with 1-3 questions, no shape repeated.
* cfg5 -- 8192 requests, lengths clip(round(exp(ln 200 + 0.6 z)), 32, 1024), 1..10 questions
          of uniform type; packed into varlen batches of at most 16384 tokens per GPU.
"""
from __future__ import annotations

from typing import List

import numpy as np

from .batch import EncodedItem, Varlen

LABELS = {0: 3, 1: 4, 2: 2}  # markers per question: choice, score, noul


def _row(rng, vocab: int, L: int, qtypes: List[int]) -> EncodedItem:
    ids = rng.integers(4, vocab, size=L).astype(np.uint32)
    ids[0] = 1
    if L > 1:
        ids[-1] = 2
    n_markers = min(sum(LABELS[q] for q in qtypes), max(L - 2, 0))
    markers = sorted(rng.choice(np.arange(1, L - 1), size=n_markers, replace=False).tolist()) if n_markers else []
    return EncodedItem(ids.tolist(), markers, int(qtypes[0]) if qtypes else 2)


def cfg1(vocab: int = 50368, seed: int = 101) -> List[EncodedItem]:
    rng = np.random.Generator(np.random.PCG64(seed))
    return [_row(rng, vocab, 128, [2])]


def cfg2(vocab: int = 50368, seed: int = 102) -> List[EncodedItem]:
    rng = np.random.Generator(np.random.PCG64(seed))
    return [_row(rng, vocab, 512, [0] * 4 + [1] * 3 + [2] * 3)]


def cfg3(vocab: int = 50368, seed: int = 103) -> List[EncodedItem]:
    rng = np.random.Generator(np.random.PCG64(seed))
    return [_row(rng, vocab, int(rng.integers(64, 513)), [0, 1, 2]) for _ in range(64)]


def latency_stream(n: int = 200, vocab: int = 50368, seed: int = 104, lo: int = 64, hi: int = 200,
                   max_questions: int = 3) -> List[EncodedItem]:
    """``n`` single requests whose shapes never repeat: lengths U[lo, hi], 1..max_questions questions
    of uniform type, and no two requests with the same (length, marker count)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out, shapes = [], set()
    while len(out) < n:
        L = int(rng.integers(lo, hi + 1))
        qs = [int(t) for t in rng.integers(0, 3, size=int(rng.integers(1, max_questions + 1)))]
        k = min(sum(LABELS[q] for q in qs), L - 2)
        if (L, k) in shapes:
            continue
        shapes.add((L, k))
        out.append(_row(rng, vocab, L, qs))
    return out


def cfg5_requests(n: int = 8192, vocab: int = 50368, seed: int = 1) -> List[EncodedItem]:
    rng = np.random.Generator(np.random.PCG64(seed))
    lens = np.clip(np.round(np.exp(np.log(200.0) + 0.6 * rng.standard_normal(n))), 32, 1024).astype(int)
    nq = rng.integers(1, 11, size=n)
    out = []
    for L, q in zip(lens, nq):
        out.append(_row(rng, vocab, int(L), [int(t) for t in rng.integers(0, 3, size=int(q))]))
    return out


def request_cost(L: int, d: int = 1024, I: int = 2624, n_layers: int = 28, window: int = 64) -> float:
    """Encoder FLOPs of one request of ``L`` tokens (``encoder_flops`` of one row): the GEMMs grow
    with L, global attention with L^2."""
    i = np.arange(L)
    pl = float(np.sum(np.minimum(i, window) + np.minimum(L - 1 - i, window) + 1))
    n_global = (n_layers + 2) // 3
    return 2.0 * (d * 3 * d + d * d + d * 2 * I + I * d) * n_layers * L + 4.0 * d * (
        n_global * float(L) * L + (n_layers - n_global) * pl)


def shard_lpt(items: List[EncodedItem], n_shards: int) -> List[List[EncodedItem]]:
    """Longest-processing-time assignment by cost (``request_cost``: GEMM work plus the quadratic
    global attention): each request goes to the shard with the least cost so far (costliest
    requests first), then each shard keeps arrival order."""
    costs = {L: request_cost(L) for L in {len(it.ids) for it in items}}
    order = sorted(range(len(items)), key=lambda i: -len(items[i].ids))
    load = [0.0] * n_shards
    owner = [0] * len(items)
    for i in order:
        s = min(range(n_shards), key=lambda k: load[k])
        owner[i] = s
        load[s] += costs[len(items[i].ids)]
    return [[items[i] for i in range(len(items)) if owner[i] == s] for s in range(n_shards)]


def pack_batches(items: List[EncodedItem], max_tokens: int = 16384) -> List[Varlen]:
    """Requests into varlen batches of at most ``max_tokens`` tokens, first-fit decreasing by
    length: the fewest batches (ceil(tokens / max_tokens) for workloads of many short requests)
    where packing in arrival order can leave a batch short. Rows keep arrival order inside a
    batch; a request longer than ``max_tokens`` runs alone."""
    bins: List[List[int]] = []
    room: List[int] = []
    for i in sorted(range(len(items)), key=lambda i: -len(items[i].ids)):
        L = len(items[i].ids)
        for b in range(len(bins)):
            if room[b] >= L:
                bins[b].append(i)
                room[b] -= L
                break
        else:
            bins.append([i])
            room.append(max_tokens - L)
    return [Varlen.from_rows([items[i] for i in sorted(b)]) for b in bins]


def encoder_flops(lens, d: int = 1024, I: int = 2624, n_layers: int = 28, window: int = 64,
                  local=None) -> float:
    """Algorithmic encoder FLOPs: GEMMs 2 * (d*3d + d*d + d*2I + I*d) per token per layer, plus
    attention 4 * d per attended (query, key) pair (L^2 global; min(i, w) + min(L-1-i, w) + 1 local)."""
    local = local if local is not None else [i % 3 != 0 for i in range(n_layers)]
    gemm = 2.0 * (d * 3 * d + d * d + d * 2 * I + I * d) * n_layers
    tot = 0.0
    for L in lens:
        i = np.arange(L)
        pl = float(np.sum(np.minimum(i, window) + np.minimum(L - 1 - i, window) + 1))
        pg = float(L) * L
        tot += gemm * L + sum(4.0 * d * (pl if lo else pg) for lo in local)
    return tot
