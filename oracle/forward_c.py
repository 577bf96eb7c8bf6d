"""ctypes wrapper of the C restatement of the forward (``oracle/forward_ref.c``) -- TEST
INFRASTRUCTURE ONLY: loaded by the tests (as a second checker beside ``forward_ref.OracleModel``)
and by ``bench.py``'s CPU-baseline leg, never by the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Dict, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libforward_ref.so")

_FP = C.POINTER(C.c_float)
_FPP = C.POINTER(_FP)


class _Model(C.Structure):
    _fields_ = [("d", C.c_int), ("heads", C.c_int), ("inter", C.c_int), ("n_layers", C.c_int), ("window", C.c_int),
                ("head_layers", C.c_int), ("head_heads", C.c_int), ("head_ffn", C.c_int),
                ("scorer_hidden", C.c_int),
                ("eps", C.c_float), ("theta_global", C.c_float), ("theta_local", C.c_float),
                ("layer_is_local", C.POINTER(C.c_int32)),
                ("tok_emb", _FP), ("emb_norm", _FP),
                ("attn_norm", _FPP), ("wqkv", _FPP), ("wo", _FPP), ("mlp_norm", _FPP), ("wi", _FPP), ("wo2", _FPP),
                ("final_norm", _FP), ("type_emb", _FP), ("head", _FPP),
                ("sc0_w", _FP), ("sc0_b", _FP), ("sc1_w", _FP), ("sc1_b", _FP), ("sc3_w", _FP), ("sc3_b", _FP)]


def build() -> str:
    """Compile the library with ``oracle/Makefile`` (no-op when it is up to date)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def _load():
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "forward_ref.c")):
        build()
    lib = C.CDLL(LIB)
    lib.ofr_forward_row.restype = C.c_int
    lib.ofr_forward_row.argtypes = [C.POINTER(_Model), C.POINTER(C.c_uint32), C.c_int, C.POINTER(C.c_uint32), C.c_int,
                                    C.c_int, C.c_int, _FP, _FP]
    return lib


class CForwardModel:
    """fp32 copies of one checkpoint's tensors (bf16 bit arrays by reference name) and the C forward."""

    def __init__(self, cfg, weights: Dict[str, np.ndarray]):
        self.lib = _load()
        e = cfg.encoder
        self.cfg = cfg
        self._keep = []

        def f32(name):
            bits = np.ascontiguousarray(weights[name]).astype(np.uint32) << 16
            a = bits.view(np.float32)
            self._keep.append(a)
            return a

        def ptr(a):
            return a.ctypes.data_as(_FP)

        def ptrs(arrs):
            arr = (_FP * len(arrs))(*[ptr(a) if a is not None else _FP() for a in arrs])
            self._keep.append(arr)
            return C.cast(arr, _FPP)

        L = e.num_hidden_layers
        p = "encoder.layers.{}."
        lay = lambda s: [f32(p.format(i) + s) for i in range(L)]
        attn_norm = [None] + [f32(p.format(i) + "attn_norm.weight") for i in range(1, L)]
        head = []
        for j in range(cfg.head_layers):
            q = f"head.layers.{j}."
            for s in ("norm1.weight", "norm1.bias", "self_attn.in_proj_weight", "self_attn.in_proj_bias",
                      "self_attn.out_proj.weight", "self_attn.out_proj.bias", "norm2.weight", "norm2.bias",
                      "linear1.weight", "linear1.bias", "linear2.weight", "linear2.bias"):
                head.append(f32(q + s))
        local = np.array([1 if x else 0 for x in e.layer_is_local], np.int32)
        self._keep.append(local)
        ffn = weights["head.layers.0.linear1.weight"].shape[0] if cfg.head_layers else 0
        self.m = _Model(
            d=e.hidden_size, heads=e.num_attention_heads, inter=e.intermediate_size, n_layers=L, window=e.window(),
            head_layers=cfg.head_layers, head_heads=e.head_nheads(), head_ffn=ffn,
            scorer_hidden=weights["scorer.1.weight"].shape[0],
            eps=e.norm_eps, theta_global=e.global_rope_theta, theta_local=e.local_rope_theta,
            layer_is_local=local.ctypes.data_as(C.POINTER(C.c_int32)),
            tok_emb=ptr(f32("encoder.embeddings.tok_embeddings.weight")),
            emb_norm=ptr(f32("encoder.embeddings.norm.weight")),
            attn_norm=ptrs(attn_norm), wqkv=ptrs(lay("attn.Wqkv.weight")), wo=ptrs(lay("attn.Wo.weight")),
            mlp_norm=ptrs(lay("mlp_norm.weight")), wi=ptrs(lay("mlp.Wi.weight")), wo2=ptrs(lay("mlp.Wo.weight")),
            final_norm=ptr(f32("encoder.final_norm.weight")), type_emb=ptr(f32("type_emb.weight")),
            head=ptrs(head),
            sc0_w=ptr(f32("scorer.0.weight")), sc0_b=ptr(f32("scorer.0.bias")),
            sc1_w=ptr(f32("scorer.1.weight")), sc1_b=ptr(f32("scorer.1.bias")),
            sc3_w=ptr(f32("scorer.3.weight")), sc3_b=ptr(f32("scorer.3.bias")))

    def forward_row(self, ids, markers, qtype: int, kmax: int = None) -> Tuple[np.ndarray, np.ndarray]:
        """(logits [kmax], pooled [d]) of one row: ids, marker positions, qtype."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        kmax = len(markers) if kmax is None else kmax
        mp = np.zeros(max(kmax, 1), np.uint32)
        mp[:len(markers)] = markers
        logits = np.empty(max(kmax, 1), np.float32)
        pooled = np.empty(self.cfg.encoder.hidden_size, np.float32)
        rc = self.lib.ofr_forward_row(C.byref(self.m), ids.ctypes.data_as(C.POINTER(C.c_uint32)), len(ids),
                                      mp.ctypes.data_as(C.POINTER(C.c_uint32)), kmax, len(markers), int(qtype),
                                      logits.ctypes.data_as(_FP), pooled.ctypes.data_as(_FP))
        if rc != 0:
            raise MemoryError("ofr_forward_row: out of host memory")
        return logits[:kmax], pooled
