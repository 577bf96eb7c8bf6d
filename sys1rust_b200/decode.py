"""Answers from the forward's outputs: the host side of the reference's ``decode_answers``
(``runtime/crates/laya-core/src/decode.rs``), with the arithmetic in the library (``s1c_decode``).

* ``clamp_temperature`` / ``Temperatures``: the calibration temperatures as the runtime applies them
  (decode.rs:16-86): confined to [0.5, 5.0], ``1.0`` when not a number, per question type or per
  ``"<type>:<size bucket>"`` entry of ``temperature_by_options``.
* ``ActHead``: the action head's tensors (``act_head.0`` / ``act_head.2``, decode.rs:117-207) with the
  reference's shape checks, as fp32 arrays.
* ``decode``: per row the option probabilities, confidence, the per-type answer value and the
  action probability (unrounded; the JSON result object and its 4-decimal rounding are the
  caller's).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from .backend import CActHead, CAnswer, S1C_OK, WeightsError, _raise, lib

TEMP_MIN, TEMP_MAX = 0.5, 5.0
QTYPES = ("choice", "score", "noul")


def clamp_temperature(v) -> float:
    """``clamp_temperature`` (decode.rs:19-31): a number, a numeric string or a bool; anything else
    (or a non-finite value) is 1.0; the result is confined to [0.5, 5.0]."""
    t = None
    if isinstance(v, bool):
        t = 1.0 if v else 0.0
    elif isinstance(v, (int, float)):
        t = float(v)
    elif isinstance(v, str):
        try:
            t = float(v.strip())
        except ValueError:
            t = None
    if t is None or not math.isfinite(t):
        return 1.0
    return min(max(t, TEMP_MIN), TEMP_MAX)


def temp_bucket(qtype: int, k: int) -> str:
    """``Temperatures::temp_bucket`` (decode.rs:68-79)."""
    size = "2" if k <= 2 else "3-5" if k <= 5 else "6-10" if k <= 10 else "11+"
    return f"{QTYPES[qtype]}:{size}"


@dataclass
class Temperatures:
    by_type: List[float] = field(default_factory=lambda: [1.0, 1.0, 1.0])
    by_options: Dict[str, float] = field(default_factory=dict)
    rejected: List[str] = field(default_factory=list)

    @staticmethod
    def from_config(temperature: Sequence = (), temperature_by_options: Optional[dict] = None) -> "Temperatures":
        """``Temperatures::from_config`` (decode.rs:43-65)."""
        t = Temperatures()
        for i, raw in enumerate(list(temperature)[:3]):
            t.by_type[i] = clamp_temperature(raw)
            if not (isinstance(raw, (int, float)) and not isinstance(raw, bool) and float(raw) == t.by_type[i]):
                t.rejected.append(f"temperature[{i}]={raw} -> {t.by_type[i]}")
        for k, raw in (temperature_by_options or {}).items():
            v = clamp_temperature(raw)
            if not (isinstance(raw, (int, float)) and not isinstance(raw, bool) and float(raw) == v):
                t.rejected.append(f"{k}={raw} -> {v}")
            t.by_options[k] = v
        return t

    def scale(self, qtype: int, k: int) -> float:
        """``Temperatures::scale`` (decode.rs:80-86)."""
        return float(self.by_options.get(temp_bucket(qtype, k), self.by_type[qtype]))


class ActHead:
    """``act_head = Linear(d + 4, H) -> GELU -> Linear(H, n_act)`` (decode.rs:117-207)."""

    def __init__(self, w0, b0, w2, b2):
        w0, b0, w2, b2 = (np.ascontiguousarray(x, dtype=np.float32) for x in (w0, b0, w2, b2))
        if w0.ndim != 2 or w2.ndim != 2 or w2.shape[1] != w0.shape[0]:
            raise WeightsError(-3, f"act_head shapes {list(w0.shape)} / {list(w2.shape)} are not a 2-layer MLP")
        self.hidden, self.d_in = w0.shape
        self.n_act = w2.shape[0]
        if self.d_in <= 4:
            raise WeightsError(-3, f"act_head.0.weight has input width {self.d_in}, but the action head reads the "
                                   "pooled hidden state plus 4 scalar features, so it needs at least 5")
        if self.hidden == 0 or self.n_act == 0:
            raise WeightsError(-3, f"act_head shapes {list(w0.shape)} / {list(w2.shape)} have an empty layer")
        if b0.size != self.hidden or b2.size != self.n_act:
            raise WeightsError(-3, f"act_head biases have {b0.size} and {b2.size} values; the layers have "
                                   f"{self.hidden} and {self.n_act} outputs")
        self.w0, self.b0, self.w2, self.b2 = w0, b0, w2, b2

    @staticmethod
    def from_weights(wf) -> "ActHead":
        """From an open ``WeightsFile`` (``ActHead::load``, decode.rs:130-136)."""
        def f32(name):
            dt, shape, a = wf.tensor(name)
            if dt == "F32":
                return a
            if dt == "F64":
                return a.astype(np.float32)
            if dt == "F16":
                return a.view(np.float16).astype(np.float32)
            return (a.astype(np.uint32) << 16).view(np.float32)  # BF16
        return ActHead(f32("act_head.0.weight"), f32("act_head.0.bias"), f32("act_head.2.weight"),
                       f32("act_head.2.bias"))

    def c(self) -> CActHead:
        return CActHead(self.d_in, self.hidden, self.n_act, self.w0.ctypes.data, self.b0.ctypes.data,
                        self.w2.ctypes.data, self.b2.ctypes.data)


def decode(logits: np.ndarray, pooled: np.ndarray, marker_count: Sequence[int], qtype: Sequence[int], kmax: int,
           hidden: int, temps: Temperatures, head: ActHead):
    """Decode n rows; returns (answers, probs [n, kmax]). Each answer is a dict with ``type``,
    ``k``, ``confidence``, ``answer_confidence``, ``act_probability`` and ``argmax`` (choice),
    ``score`` (score) or ``noul`` (noul)."""
    n = len(marker_count)
    lg = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1)
    pl = np.ascontiguousarray(pooled, dtype=np.float32).reshape(-1)
    mc = np.ascontiguousarray(marker_count, dtype=np.int32)
    qt = np.ascontiguousarray(qtype, dtype=np.uint32)
    tt = np.array([temps.scale(int(q), int(k)) for q, k in zip(qt, mc)], dtype=np.float64)
    probs = np.zeros((max(n, 1), max(kmax, 1)), dtype=np.float64)
    out = (CAnswer * max(n, 1))()
    h = head.c()
    rc = lib().s1c_decode(lg.ctypes.data, pl.ctypes.data, n, kmax, hidden, mc.ctypes.data, qt.ctypes.data,
                          tt.ctypes.data, C.byref(h), probs.ctypes.data, out)
    if rc != S1C_OK:
        _raise(rc, lib().s1c_create_error().decode())
    answers = []
    for r in range(n):
        a = out[r]
        d = {"type": QTYPES[a.qtype], "k": a.k, "confidence": a.confidence,
             "answer_confidence": a.answer_confidence, "act_probability": float(a.act_probability)}
        if a.qtype == 0:
            d["argmax"] = a.argmax
        elif a.qtype == 1:
            d["score"] = a.score
        else:
            d["noul"] = a.noul
        answers.append(d)
    return answers, probs[:n, :kmax]
