"""Host-side batch formats: the reference's padded ``Batch`` and its unpadded packing.

``Batch`` mirrors ``laya_core::Batch`` (``runtime/crates/laya-core/src/backend.rs:74-98``):
row-major padded token ids, a 1/0 attention mask (right padding), per-row lengths, marker
positions (``n * kmax``, zero past ``marker_count``), and one question type per row.

``Packing`` restates ``Packing::new`` (``runtime/crates/laya-mlx/src/lib.rs:894-943``) bit for
bit: ``pack`` (padded index of every real token, row-major), ``unpack`` (packed index of every
padded position; padding points at its row's token 0), ``row`` and ``offsets``.

``Varlen`` is the layout the CUDA path runs on: real tokens only, ``cu_seqlens`` row offsets
(equal to ``Packing.offsets`` plus the total) and the position of every token inside its row
(0 .. seq_len - 1, the RoPE position of ``split_rope.metal:26-76``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import numpy as np


@dataclass
class Batch:
    n: int
    len: int
    kmax: int
    input_ids: np.ndarray       # u32 [n * len]
    attention_mask: np.ndarray  # u32 [n * len], 1 real / 0 padding
    seq_lens: np.ndarray        # i64 [n]
    marker_pos: np.ndarray      # u32 [n * kmax]
    marker_count: np.ndarray    # i64 [n]
    qtype: np.ndarray           # u32 [n]  (0 choice, 1 score, 2 noul)

    def total_tokens(self) -> int:
        return int(np.sum(self.seq_lens))

    def marker_mask(self, row: int, k: int) -> bool:
        return k < int(self.marker_count[row])

    def validate(self) -> None:
        """The invariants ``Batch`` producers (``collate_to``) guarantee; checked before the
        batch crosses into the device library so that a malformed batch is an error, never an
        out-of-bounds access."""
        n, L, k = self.n, self.len, self.kmax
        if self.input_ids.shape != (n * L,) or self.attention_mask.shape != (n * L,):
            raise ValueError("batch: input_ids/attention_mask must hold n*len entries")
        if self.seq_lens.shape != (n,) or self.marker_count.shape != (n,) or self.qtype.shape != (n,):
            raise ValueError("batch: seq_lens/marker_count/qtype must hold n entries")
        if self.marker_pos.shape != (n * k,):
            raise ValueError("batch: marker_pos must hold n*kmax entries")
        m = self.attention_mask.reshape(n, L) if n * L else np.zeros((n, L), np.uint32)
        for r in range(n):
            s = int(self.seq_lens[r])
            if s < 1 or s > L:
                raise ValueError(f"row {r}: seq_len {s} outside 1..{L}")
            if np.any(m[r, :s] != 1) or np.any(m[r, s:] != 0):
                raise ValueError(f"row {r}: attention mask does not match seq_len {s}")
            c = int(self.marker_count[r])
            if c < 0 or c > k:
                raise ValueError(f"row {r}: marker_count {c} outside 0..{k}")
            if np.any(self.marker_pos[r * k:r * k + c] >= s):
                raise ValueError(f"row {r}: marker position past seq_len {s}")
        if n and np.any(self.qtype > 2):
            raise ValueError("batch: qtype must be 0, 1 or 2")


@dataclass
class EncodedItem:
    """One question row before collation (``sequence.rs:11-17``)."""
    ids: Sequence[int]
    markers: Sequence[int]
    qtype: int


def collate_to(items: List[EncodedItem], pad_id: int, min_len: int = 0) -> Batch:
    """Right-pad rows with ``pad_id`` to the longest row (``sequence.rs:132-166``)."""
    n = len(items)
    L = max([len(it.ids) for it in items] + [0])
    L = max(L, min_len)
    kmax = max([len(it.markers) for it in items] + [0])
    input_ids = np.full(n * L, pad_id, dtype=np.uint32)
    attention_mask = np.zeros(n * L, dtype=np.uint32)
    marker_pos = np.zeros(n * kmax, dtype=np.uint32)
    seq_lens = np.zeros(n, dtype=np.int64)
    marker_count = np.zeros(n, dtype=np.int64)
    qtype = np.zeros(n, dtype=np.uint32)
    for i, it in enumerate(items):
        s = len(it.ids)
        input_ids[i * L:i * L + s] = np.asarray(it.ids, dtype=np.uint32)
        attention_mask[i * L:i * L + s] = 1
        marker_pos[i * kmax:i * kmax + len(it.markers)] = np.asarray(it.markers, dtype=np.uint32)
        seq_lens[i] = s
        marker_count[i] = len(it.markers)
        qtype[i] = it.qtype
    return Batch(n, L, kmax, input_ids, attention_mask, seq_lens, marker_pos, marker_count, qtype)


@dataclass
class Packing:
    pack: np.ndarray     # u32 [T]
    unpack: np.ndarray   # u32 [n * len]
    row: np.ndarray      # u32 [T]
    offsets: np.ndarray  # u32 [n]

    @staticmethod
    def new(batch: Batch) -> "Packing":
        """``Packing::new`` (``lib.rs:906-930``), vectorised; same values bit for bit."""
        n, L = batch.n, batch.len
        m = batch.attention_mask.reshape(n, L).astype(bool)
        flat = np.arange(n * L, dtype=np.uint32).reshape(n, L)
        pack = flat[m].astype(np.uint32)
        row = np.repeat(np.arange(n, dtype=np.uint32), m.sum(axis=1))
        counts = m.sum(axis=1)
        offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint32) if n else np.zeros(0, np.uint32)
        unpack = np.empty((n, L), dtype=np.uint32)
        rank = np.cumsum(m, axis=1) - 1 + offsets[:, None]
        unpack[:] = np.where(m, rank, offsets[:, None])
        return Packing(pack, unpack.reshape(-1).astype(np.uint32), row, offsets)


@dataclass
class Varlen:
    """Real tokens only: what the device library consumes."""
    ids: np.ndarray         # u32 [T]
    cu_seqlens: np.ndarray  # i32 [n + 1]
    positions: np.ndarray   # i32 [T], index within the row
    marker_pos: np.ndarray  # u32 [n * kmax] (position within the row)
    marker_count: np.ndarray  # i32 [n]
    qtype: np.ndarray       # u32 [n]
    kmax: int

    @property
    def n(self) -> int:
        return len(self.cu_seqlens) - 1

    @property
    def total(self) -> int:
        return int(self.cu_seqlens[-1])

    @staticmethod
    def from_batch(batch: Batch) -> "Varlen":
        p = Packing.new(batch)
        ids = batch.input_ids[p.pack.astype(np.int64)].astype(np.uint32)
        cu = np.concatenate([p.offsets.astype(np.int64), [batch.total_tokens()]]).astype(np.int32)
        positions = (p.pack % max(batch.len, 1)).astype(np.int32)
        return Varlen(ids, cu, positions, batch.marker_pos.astype(np.uint32),
                      batch.marker_count.astype(np.int32), batch.qtype.astype(np.uint32), batch.kmax)

    @staticmethod
    def from_rows(rows: List[EncodedItem], kmax: int | None = None) -> "Varlen":
        """Pack rows directly, without the padded intermediate."""
        n = len(rows)
        k = max([len(r.markers) for r in rows] + [0]) if kmax is None else kmax
        lens = np.array([len(r.ids) for r in rows], dtype=np.int64)
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        ids = np.concatenate([np.asarray(r.ids, dtype=np.uint32) for r in rows]) if n else np.zeros(0, np.uint32)
        positions = np.concatenate([np.arange(l, dtype=np.int32) for l in lens]) if n else np.zeros(0, np.int32)
        mp = np.zeros(n * k, dtype=np.uint32)
        mc = np.zeros(n, dtype=np.int32)
        for i, r in enumerate(rows):
            mp[i * k:i * k + len(r.markers)] = r.markers
            mc[i] = len(r.markers)
        qt = np.array([r.qtype for r in rows], dtype=np.uint32)
        return Varlen(ids, cu, positions, mp, mc, qt, k)

    def scorer_rows(self) -> np.ndarray:
        """Packed token index of position 0 of every row followed by its ``kmax`` marker slots
        (padded slots point at position 0), ``MlxBackend::scorer_rows`` (``lib.rs:1512-1523``)."""
        n, k = self.n, self.kmax
        base = self.cu_seqlens[:-1].astype(np.int64)
        out = np.empty((n, 1 + k), dtype=np.uint32)
        out[:, 0] = base
        if k:
            out[:, 1:] = base[:, None] + self.marker_pos.reshape(n, k)
        return out.reshape(-1)
