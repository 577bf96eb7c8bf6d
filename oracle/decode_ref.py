"""CPU restatement of the reference's answer decoding, for tests only (test infrastructure: the
product path is ``s1c_decode`` in the library; nothing here is called by it).

Follows runtime/crates/laya-core/src/decode.rs:
  confidence_from_probs   decode.rs:88-94
  softmax (f64 / f32)     decode.rs:96-108
  gelu (erf, in f64)      decode.rs:110-114
  ActHead::probs          decode.rs:232-253
  act_features            decode.rs:257-267
  decode_answers values   decode.rs:318-413 (without the JSON formatting and rounding)
"""
from __future__ import annotations

import math

import numpy as np


def softmax_f64(z):
    m = max(z) if len(z) else -math.inf
    e = [math.exp(x - m) for x in z]
    s = sum(e)
    return [x / s for x in e]


def softmax_f32(z):
    z = np.asarray(z, dtype=np.float32)
    m = np.float32(z.max())
    e = np.exp(z - m).astype(np.float32)
    s = np.float32(0)
    for x in e:
        s = np.float32(s + x)
    return (e / s).astype(np.float32)


def confidence_from_probs(p, k):
    if k < 2:
        return 1.0
    ent = sum(-x * math.log(min(max(x, 1e-12), 1.0)) for x in p[:k])
    return min(max(1.0 - ent / math.log(k), 0.0), 1.0)


def gelu(x):
    return np.float32(0.5 * float(x) * (1.0 + math.erf(float(x) / math.sqrt(2.0))))


def act_features(row, marker_count):
    p = softmax_f32(row)
    k = np.float32(max(marker_count, 2))
    ent = np.float32(0)
    for x in p:
        ent = np.float32(ent + np.float32(x * np.float32(math.log(max(float(x), 1e-9)))))
    ent = np.float32(-ent / np.float32(math.log(k)))
    s = sorted(p.tolist(), reverse=True)
    top1 = np.float32(s[0]) if s else np.float32(0)
    top2 = np.float32(s[1]) if len(s) > 1 else np.float32(0)
    return [top1, np.float32(top1 - top2), ent, np.float32(k / np.float32(255.0))]


def act_probs(w0, b0, w2, b2, pooled, feats):
    d = w0.shape[1] - 4
    h = []
    for j in range(w0.shape[0]):
        acc = np.float32(b0[j])
        for a, b in zip(w0[j, :d], pooled):
            acc = np.float32(acc + np.float32(a * b))
        for a, b in zip(w0[j, d:], feats):
            acc = np.float32(acc + np.float32(a * b))
        h.append(gelu(acc))
    out = []
    for j in range(w2.shape[0]):
        acc = np.float32(0)
        for a, b in zip(w2[j], h):
            acc = np.float32(acc + np.float32(a * b))
        out.append(np.float32(b2[j] + acc))
    return softmax_f32(out)


def decode_row(row, pooled, k, qtype, t, head):
    """(answer dict, probabilities) of one row; head = (w0, b0, w2, b2) fp32 arrays."""
    p = softmax_f64([float(x) / t for x in row[:k]])
    conf = confidence_from_probs(p, k)
    am = 0
    for i, x in enumerate(p):
        if x > p[am]:
            am = i
    a = {"k": k}
    if qtype == 0:
        a.update(type="choice", argmax=am, confidence=conf, answer_confidence=p[am] if k else 0.0)
    elif qtype == 1:
        a.update(type="score", score=sum(i * x for i, x in enumerate(p)), confidence=conf,
                 answer_confidence=max(p) if p else 0.0)
    else:
        p1 = p[1] if k > 1 else 0.0
        top = max(p1, 1.0 - p1)
        a.update(type="noul", noul=p1, confidence=top, answer_confidence=top)
    a["act_probability"] = float(act_probs(*head, pooled, act_features(row, k))[0])
    return a, p
