"""Seeded synthetic checkpoints with the reference's tensor names.

The names are the ones ``MlxBackend::new`` reads (``runtime/crates/laya-mlx/src/lib.rs:990-1131``)
plus the ``act_head.*`` pair of ``ActHead::load`` (``runtime/crates/laya-core/src/decode.rs:130-135``),
so that a file written here carries every family ``Weights::verify`` requires
(``runtime/crates/laya-core/src/weights.rs:68-79``).

Values: every matrix, embedding and bias is N(0, 0.02); LayerNorm weights are 1 + N(0, 0.02).
Each tensor draws from its own ``numpy`` PCG64 stream keyed by ``(seed, crc32(name))``, so a
tensor's values do not depend on which other tensors are generated or in what order. Values are
rounded to bf16 (round to nearest even): the checkpoint is a bf16 model, and the CPU oracle and
the device path see the same weights exactly.
"""
from __future__ import annotations

import json
import os
import zlib
from typing import Dict, Iterator, List, Tuple

import numpy as np

from .config import ModelConfig

STD = 0.02


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


def tensor_specs(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape, kind) for every tensor; kind is ``w`` (N(0, s)) or ``ln`` (1 + N(0, s))."""
    e = cfg.encoder
    d, I, F, S = e.hidden_size, e.intermediate_size, cfg.head_ffn, cfg.scorer_hidden
    out: List[Tuple[str, Tuple[int, ...], str]] = [
        ("encoder.embeddings.tok_embeddings.weight", (e.vocab_size, d), "w"),
        ("encoder.embeddings.norm.weight", (d,), "ln"),
    ]
    for i in range(e.num_hidden_layers):
        p = f"encoder.layers.{i}"
        if i > 0:  # layer 0's attn_norm is the identity (lib.rs:993-997)
            out.append((f"{p}.attn_norm.weight", (d,), "ln"))
        out += [(f"{p}.attn.Wqkv.weight", (3 * d, d), "w"),
                (f"{p}.attn.Wo.weight", (d, d), "w"),
                (f"{p}.mlp_norm.weight", (d,), "ln"),
                (f"{p}.mlp.Wi.weight", (2 * I, d), "w"),
                (f"{p}.mlp.Wo.weight", (d, I), "w")]
    out.append(("encoder.final_norm.weight", (d,), "ln"))
    out.append(("type_emb.weight", (cfg.n_qtypes, d), "w"))
    for j in range(cfg.head_layers):
        p = f"head.layers.{j}"
        out += [(f"{p}.norm1.weight", (d,), "ln"), (f"{p}.norm1.bias", (d,), "w"),
                (f"{p}.self_attn.in_proj_weight", (3 * d, d), "w"),
                (f"{p}.self_attn.in_proj_bias", (3 * d,), "w"),
                (f"{p}.self_attn.out_proj.weight", (d, d), "w"),
                (f"{p}.self_attn.out_proj.bias", (d,), "w"),
                (f"{p}.norm2.weight", (d,), "ln"), (f"{p}.norm2.bias", (d,), "w"),
                (f"{p}.linear1.weight", (F, d), "w"), (f"{p}.linear1.bias", (F,), "w"),
                (f"{p}.linear2.weight", (d, F), "w"), (f"{p}.linear2.bias", (d,), "w")]
    out += [("scorer.0.weight", (d,), "ln"), ("scorer.0.bias", (d,), "w"),
            ("scorer.1.weight", (S, d), "w"), ("scorer.1.bias", (S,), "w"),
            ("scorer.3.weight", (1, S), "w"), ("scorer.3.bias", (1,), "w"),
            ("act_head.0.weight", (256, d + 4), "w"), ("act_head.0.bias", (256,), "w"),
            ("act_head.2.weight", (2, 256), "w"), ("act_head.2.bias", (2,), "w")]
    return out


def gen_tensor(seed: int, name: str, shape: Tuple[int, ...], kind: str) -> np.ndarray:
    """bf16 bit patterns of one seeded tensor."""
    rng = np.random.Generator(np.random.PCG64([seed, zlib.crc32(name.encode())]))
    x = rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(STD)
    if kind == "ln":
        x += np.float32(1.0)
    return bf16_bits(x).reshape(shape)


class SyntheticWeights:
    """Seeded weights held as bf16 bit patterns, looked up by reference tensor name."""

    def __init__(self, cfg: ModelConfig, seed: int = 0):
        self.cfg = cfg
        self.seed = seed
        self.tensors: Dict[str, np.ndarray] = {}
        for name, shape, kind in tensor_specs(cfg):
            self.tensors[name] = gen_tensor(seed, name, shape, kind)

    def bits(self, name: str) -> np.ndarray:
        return self.tensors[name]

    def f32(self, name: str) -> np.ndarray:
        return bf16_to_f32(self.tensors[name])

    def items(self) -> Iterator[Tuple[str, np.ndarray]]:
        return iter(self.tensors.items())

    def save(self, model_dir: str, dtype: str = "BF16") -> None:
        """Write ``model.safetensors`` (``BF16``, or ``F16`` as the reference's checkpoints are
        stored: each bf16 value converted to the nearest half), ``encoder/config.json`` and
        ``rl_agent_config.json`` in the checkpoint layout ``Agent::load`` reads."""
        os.makedirs(os.path.join(model_dir, "encoder"), exist_ok=True)
        path = os.path.join(model_dir, "model.safetensors")
        if dtype == "BF16":
            write_safetensors_bf16(path, self.tensors)
        elif dtype == "F16":
            write_safetensors(path, {k: ("F16", bf16_bits_to_f16_bits(v)) for k, v in self.tensors.items()})
        else:
            raise ValueError(f"unsupported checkpoint dtype {dtype}")
        with open(os.path.join(model_dir, "encoder", "config.json"), "w") as f:
            json.dump(self.cfg.encoder.to_value(), f, indent=1)
        with open(os.path.join(model_dir, "rl_agent_config.json"), "w") as f:
            json.dump({"encoder": "encoder", "head_layers": self.cfg.head_layers,
                       "max_len": self.cfg.max_len, "head_max_len": self.cfg.head_max_len,
                       "act_costs": {"ask": 1.0}, "temperature": [1.0, 1.0, 1.0]}, f, indent=1)


def bf16_bits_to_f16_bits(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> IEEE half bit patterns (round to nearest even)."""
    f = (bits.astype(np.uint32) << 16).view(np.float32)
    return f.astype(np.float16).view(np.uint16)


_ST_SIZE = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "U8": 1}


def write_safetensors(path: str, tensors: Dict[str, Tuple[str, np.ndarray]]) -> None:
    """Write ``name -> (dtype, array)`` (arrays holding the raw element bits or values of that
    dtype) as a safetensors file: 8-byte little-endian header length, JSON header padded with
    spaces to a multiple of 8 bytes, then the tensors' bytes back to back in header order."""
    header, off, blobs = {}, 0, []
    for name, (dt, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        if len(b) != int(np.prod(a.shape)) * _ST_SIZE[dt]:
            raise ValueError(f"{name}: {len(b)} bytes do not match {dt} x {a.shape}")
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_safetensors_bf16(path: str, tensors: Dict[str, np.ndarray]) -> None:
    """Write bf16 bit patterns (uint16 arrays) as a safetensors file with dtype ``BF16``:
    an 8-byte little-endian header length, the JSON header (padded with spaces to a multiple of
    8 bytes), then the tensors' bytes back to back."""
    header, off = {}, 0
    for name, a in tensors.items():
        nbytes = int(a.size) * 2
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for a in tensors.values():
            f.write(np.ascontiguousarray(a, dtype=np.uint16).tobytes())


def load_safetensors_bits(path: str) -> Dict[str, Tuple[str, Tuple[int, ...], np.ndarray]]:
    """Read a safetensors file into ``name -> (dtype, shape, raw array)`` without torch.
    dtype is ``BF16``, ``F16`` or ``F32`` (the formats ``weights.rs:82-115`` converts)."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        hdr = json.loads(f.read(n))
        base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in hdr.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        a, b = meta["data_offsets"]
        raw = mm[base + a: base + b]
        shape = tuple(meta["shape"])
        if dt in ("BF16", "F16"):
            arr = np.frombuffer(raw, dtype=np.uint16)
        elif dt == "F32":
            arr = np.frombuffer(raw, dtype=np.float32)
        else:
            raise ValueError(f"{name}: unsupported dtype {dt}")
        if arr.size != int(np.prod(shape)):
            raise ValueError(f"{name}: data holds {arr.size} elements, shape {shape} needs {int(np.prod(shape))}")
        out[name] = (dt, shape, arr.reshape(shape))
    return out
