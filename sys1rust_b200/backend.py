"""``CudaBackend``: the host-side mirror of ``laya_core::Backend`` over ``libs1c.so``.

Same methods and meanings as the reference trait (``runtime/crates/laya-core/src/backend.rs:109-133``):
``name``, ``forward(batch) -> BackendOutput``, ``active_kernels``, ``padded_len``, ``warmup``,
``encoder_hidden``. Errors surface as ``BackendError`` (``Error::Backend``), weight problems as
``WeightsError`` and config problems as ``ConfigError``, like the reference's ``Error`` enum.

There is no CPU fallback: constructing a backend needs the CUDA library and an sm_100 GPU, and
fails loudly otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from .batch import Batch, Varlen
from .config import ConfigError, ModelConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libs1c.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "s1c.h")

S1C_OK, S1C_ERR_ARG, S1C_ERR_CUDA, S1C_ERR_WEIGHTS, S1C_ERR_CONFIG, S1C_ERR_DEVICE_TIMEOUT, S1C_ERR_UNSUPPORTED = \
    0, -1, -2, -3, -4, -5, -6
S1C_ERR_BUSY, S1C_ERR_DEAD, S1C_ERR_TIMEOUT = -7, -8, -9
S1C_ERR_SELFCHECK = -10
DT_F32, DT_F16, DT_BF16, DT_F64 = 0, 1, 2, 3


class BackendError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"backend error {code}: {msg}")
        self.code = code


class WeightsError(BackendError):
    pass


class DeviceTimeout(BackendError):
    pass


class ModelDesc(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("num_layers", C.c_int32),
                ("num_heads", C.c_int32), ("intermediate_size", C.c_int32), ("norm_eps", C.c_float),
                ("local_attention", C.c_int32), ("global_rope_theta", C.c_float),
                ("local_rope_theta", C.c_float), ("layer_is_local", C.POINTER(C.c_uint8)),
                ("head_layers", C.c_int32), ("max_position", C.c_int32), ("max_tokens", C.c_int32)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("ndim", C.c_int32),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p)]


class CBatch(C.Structure):
    _fields_ = [("n", C.c_size_t), ("len", C.c_size_t), ("kmax", C.c_size_t),
                ("input_ids", C.c_void_p), ("attention_mask", C.c_void_p), ("seq_lens", C.c_void_p),
                ("marker_pos", C.c_void_p), ("marker_count", C.c_void_p), ("qtype", C.c_void_p)]


class CVarlen(C.Structure):
    _fields_ = [("n", C.c_int32), ("kmax", C.c_int32), ("ids", C.c_void_p), ("cu_seqlens", C.c_void_p),
                ("marker_pos", C.c_void_p), ("marker_count", C.c_void_p), ("qtype", C.c_void_p)]


class ServerOpts(C.Structure):
    _fields_ = [("max_concurrent", C.c_int32), ("max_batch_tokens", C.c_int32), ("max_batch_rows", C.c_int32),
                ("linger_us", C.c_int32)]


class CRequest(C.Structure):
    _fields_ = [("ids", C.c_void_p), ("len", C.c_int32), ("marker_pos", C.c_void_p), ("n_markers", C.c_int32),
                ("qtype", C.c_uint32)]


class ServerStats(C.Structure):
    _fields_ = [("batches", C.c_uint64), ("rows", C.c_uint64), ("tokens", C.c_uint64),
                ("failed_batches", C.c_uint64), ("busy_rejections", C.c_uint64),
                ("cancelled_skipped", C.c_uint64), ("in_flight", C.c_int32), ("queued", C.c_int32),
                ("workers_alive", C.c_int32)]


class CActHead(C.Structure):
    _fields_ = [("d_in", C.c_int32), ("hidden", C.c_int32), ("n_act", C.c_int32), ("w0", C.c_void_p),
                ("b0", C.c_void_p), ("w2", C.c_void_p), ("b2", C.c_void_p)]


class CAnswer(C.Structure):
    _fields_ = [("qtype", C.c_int32), ("k", C.c_int32), ("argmax", C.c_int32), ("score", C.c_double),
                ("noul", C.c_double), ("confidence", C.c_double), ("answer_confidence", C.c_double),
                ("act_probability", C.c_float)]


# s1c_server_forward_fn
SERVER_FORWARD_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.POINTER(CVarlen), C.POINTER(C.c_float),
                                C.POINTER(C.c_float), C.POINTER(C.c_char_p))


_lib = None


def lib() -> C.CDLL:
    """Load ``libs1c.so`` (built in-tree by ``sys1rust_b200.build``); raises when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m sys1rust_b200.build`")
    L = C.CDLL(LIB_PATH)
    P, I32, I64, F32, SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t
    sig = {
        "s1c_create": (I32, [C.POINTER(ModelDesc), C.POINTER(Tensor), I32, I32, C.POINTER(P)]),
        "s1c_create_with_settings": (I32, [C.POINTER(ModelDesc), C.POINTER(Tensor), I32, I32, C.c_char_p,
                                           C.POINTER(P)]),
        "s1c_destroy": (None, [P]),
        "s1c_last_error": (C.c_char_p, [P]),
        "s1c_create_error": (C.c_char_p, []),
        "s1c_name": (C.c_char_p, [P]),
        "s1c_active_kernels": (C.c_char_p, [P]),
        "s1c_padded_len": (SZ, [P, SZ, SZ]),
        "s1c_warmup": (I32, [P]),
        "s1c_forward_padded": (I32, [P, C.POINTER(CBatch), P, P]),
        "s1c_forward_varlen": (I32, [P, C.POINTER(CVarlen), P, P, P]),
        "s1c_forward_device": (I32, [P, C.POINTER(CVarlen), P, P, P, P]),
        "s1c_forward_device_async": (I32, [P, C.POINTER(CVarlen), P, P, P, P]),
        "s1c_synchronize": (I32, [P]),
        "s1c_encoder_hidden": (I32, [P, C.POINTER(CBatch), P]),
        "s1c_gemm": (I32, [I32, P, P, P, I32, I32, I32, P, I32, I32, P, F32, I32, I32, I32, P]),
        "s1c_attention": (I32, [P, P, P, P, I32, I32, I32, I32, I32, P, I32, I32, F32, I32, P]),
        "s1c_last_launch_count": (I64, [P]),
        "s1c_set_stream": (I32, [P, P]),
        "s1c_profile": (I32, [P, I32]),
        "s1c_profile_report": (SZ, [P, C.c_char_p, SZ]),
        "s1c_gemm_splitk_noalloc": (I32, [I32, P, P, P, I32, I32, I32, P, I32, I32, P, F32, I32, I32, P]),
        "s1c_weights_open": (I32, [C.c_char_p, C.POINTER(P)]),
        "s1c_weights_close": (None, [P]),
        "s1c_weights_count": (I32, [P]),
        "s1c_weights_find": (I32, [P, C.c_char_p]),
        "s1c_weights_tensor": (I32, [P, I32, C.POINTER(Tensor)]),
        "s1c_weights_verify": (I32, [P]),
        "s1c_create_from_weights": (I32, [C.POINTER(ModelDesc), P, I32, C.POINTER(P)]),
        "s1c_server_create": (I32, [C.POINTER(P), I32, C.POINTER(ServerOpts), C.POINTER(P)]),
        "s1c_server_create_with": (I32, [SERVER_FORWARD_FN, C.POINTER(P), I32, I32, C.POINTER(ServerOpts),
                                         C.POINTER(P)]),
        "s1c_server_submit": (I32, [P, C.POINTER(CRequest), C.POINTER(C.c_uint64)]),
        "s1c_server_wait": (I32, [P, C.c_uint64, I32, P, P, C.POINTER(F32)]),
        "s1c_server_cancel": (I32, [P, C.c_uint64]),
        "s1c_server_get_stats": (I32, [P, C.POINTER(ServerStats)]),
        "s1c_server_stop": (None, [P]),
        "s1c_server_destroy": (None, [P]),
        "s1c_decode": (I32, [P, P, I32, I32, I32, P, P, P, C.POINTER(CActHead), P, C.POINTER(CAnswer)]),
        "s1c_selftest_wait_timeout": (I32, [I32, I64, C.POINTER(C.c_int32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def header_functions() -> List[str]:
    """Every function ``include/s1c.h`` declares."""
    with open(HEADER) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    text = re.sub(r"typedef\s+\w+\s*\(\s*\*\s*\w+\s*\)\s*\([^;]*\);", "", text)  # function-pointer types
    return sorted(set(re.findall(r"\b(s1c_[a-z_]+)\s*\(", text)))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _raise(code: int, msg: str) -> None:
    if code == S1C_OK:
        return
    if code == S1C_ERR_WEIGHTS:
        raise WeightsError(code, msg)
    if code == S1C_ERR_CONFIG:
        raise ConfigError(msg)
    if code == S1C_ERR_DEVICE_TIMEOUT:
        raise DeviceTimeout(code, msg)
    raise BackendError(code, msg)


@dataclass
class BackendOutput:
    """``BackendOutput`` (``backend.rs:100-108``): masked logits ``[n * kmax]``, pooled ``[n * d]``."""
    logits: np.ndarray
    pooled: np.ndarray
    hidden: Optional[np.ndarray] = None


_DT_NAME = {DT_F32: "F32", DT_F16: "F16", DT_BF16: "BF16", DT_F64: "F64"}
_DT_NP = {"F32": np.float32, "F16": np.uint16, "BF16": np.uint16, "F64": np.float64}


class WeightsFile:
    """A memory-mapped ``model.safetensors`` read by the library (``laya_core::Weights``,
    ``weights.rs:10-77``): validated at open, so a missing or truncated file raises ``WeightsError``
    with the reference's wording; tensors are views into the mapping until ``close``."""

    def __init__(self, model_dir: str):
        L = lib()
        h = C.c_void_p()
        rc = L.s1c_weights_open(os.fsencode(model_dir), C.byref(h))
        if rc != S1C_OK:
            _raise(rc, L.s1c_create_error().decode())
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().s1c_weights_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _tensor(self, i: int) -> Tensor:
        t = Tensor()
        rc = lib().s1c_weights_tensor(self._h, i, C.byref(t))
        if rc != S1C_OK:
            _raise(rc, lib().s1c_create_error().decode())
        return t

    def names(self) -> List[str]:
        """Names of the tensors (every dtype), in header order."""
        out = []
        for i in range(lib().s1c_weights_count(self._h)):
            t = Tensor()
            if lib().s1c_weights_tensor(self._h, i, C.byref(t)) == S1C_OK:
                out.append(t.name.decode())
            else:
                out.append(None)
        return out

    def shape(self, name: str) -> Tuple[int, ...]:
        i = lib().s1c_weights_find(self._h, name.encode())
        if i < 0:
            raise WeightsError(S1C_ERR_WEIGHTS, f"{name}: tensor not found")
        t = self._tensor(i)
        return tuple(int(t.shape[d]) for d in range(t.ndim))

    def tensor(self, name: str) -> Tuple[str, Tuple[int, ...], np.ndarray]:
        """``(dtype, shape, raw array)`` of a float tensor (a copy of the mapped bytes)."""
        i = lib().s1c_weights_find(self._h, name.encode())
        if i < 0:
            raise WeightsError(S1C_ERR_WEIGHTS, f"{name}: tensor not found")
        t = self._tensor(i)
        dt = _DT_NAME[t.dtype]
        shape = tuple(int(t.shape[d]) for d in range(t.ndim))
        n = int(np.prod(shape)) if shape else 1
        buf = (C.c_char * (n * np.dtype(_DT_NP[dt]).itemsize)).from_address(t.data)
        return dt, shape, np.frombuffer(bytes(buf), dtype=_DT_NP[dt]).reshape(shape)

    def verify(self) -> None:
        rc = lib().s1c_weights_verify(self._h)
        if rc != S1C_OK:
            _raise(rc, lib().s1c_create_error().decode())


class CudaBackend:
    """One model on one GPU. Calls on one instance must be serialised."""

    def _desc(self, cfg: ModelConfig, max_tokens: int) -> ModelDesc:
        e = cfg.encoder
        self.cfg = cfg
        self.hidden = e.hidden_size
        self._local = np.array([1 if x else 0 for x in e.layer_is_local], dtype=np.uint8)
        return ModelDesc(e.vocab_size, e.hidden_size, e.num_hidden_layers, e.num_attention_heads,
                         e.intermediate_size, e.norm_eps, e.local_attention, e.global_rope_theta,
                         e.local_rope_theta, self._local.ctypes.data_as(C.POINTER(C.c_uint8)),
                         cfg.head_layers, e.max_position_embeddings, max_tokens)

    def __init__(self, cfg: ModelConfig, tensors: Optional[Dict[str, Tuple[str, Tuple[int, ...], np.ndarray]]],
                 device: int = 0, max_tokens: int = 16384, weights_file: Optional[WeightsFile] = None,
                 settings: Optional[str] = None):
        """``settings``: the library's comma list of kernel / bucket settings (``s1c_create_with_settings``);
        None reads the ``S1C_SETTINGS`` environment variable."""
        L = lib()
        desc = self._desc(cfg, max_tokens)
        if weights_file is not None:
            h = C.c_void_p()
            rc = L.s1c_create_from_weights(C.byref(desc), weights_file._h, device, C.byref(h))
            if rc != S1C_OK:
                _raise(rc, L.s1c_create_error().decode())
            self._h = h
            self.device = device
            return
        keep = []
        arr = (Tensor * len(tensors))()
        for i, (name, (dt, shape, data)) in enumerate(tensors.items()):
            data = np.ascontiguousarray(data)
            keep.append(data)
            nb = name.encode()
            keep.append(nb)
            code = {"F32": DT_F32, "F16": DT_F16, "BF16": DT_BF16, "F64": DT_F64}[dt]
            sh = (C.c_int64 * 4)(*(list(shape) + [0] * (4 - len(shape))))
            arr[i] = Tensor(nb, code, len(shape), sh, data.ctypes.data)
        h = C.c_void_p()
        rc = L.s1c_create_with_settings(C.byref(desc), arr, len(tensors), device,
                                        settings.encode() if settings is not None else None, C.byref(h))
        if rc != S1C_OK:
            _raise(rc, L.s1c_create_error().decode())
        self._h = h
        self.device = device

    @staticmethod
    def from_synthetic(cfg: ModelConfig, weights, device: int = 0, max_tokens: int = 16384,
                       settings: Optional[str] = None) -> "CudaBackend":
        t = {name: ("BF16", bits.shape, bits) for name, bits in weights.items()}
        return CudaBackend(cfg, t, device=device, max_tokens=max_tokens, settings=settings)

    @staticmethod
    def from_dir(model_dir: str, device: int = 0, max_tokens: int = 16384) -> "CudaBackend":
        """Load a checkpoint directory (``Agent::load``): ``encoder/config.json`` and
        ``rl_agent_config.json`` here, ``model.safetensors`` mapped and converted by the library."""
        cfg = ModelConfig.load(model_dir)
        with WeightsFile(model_dir) as wf:
            wf.verify()
            cfg.head_ffn = wf.shape("head.layers.0.linear1.weight")[0]
            cfg.scorer_hidden = wf.shape("scorer.1.weight")[0]
            return CudaBackend(cfg, None, device=device, max_tokens=max_tokens, weights_file=wf)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().s1c_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self) -> str:
        return lib().s1c_last_error(self._h).decode()

    def _check(self, rc: int) -> None:
        if rc != S1C_OK:
            _raise(rc, self._err())

    # -- the Backend trait ------------------------------------------------------------------
    def name(self) -> str:
        return lib().s1c_name(self._h).decode()

    def active_kernels(self) -> List[str]:
        s = lib().s1c_active_kernels(self._h).decode()
        return re.findall(r"[a-z0-9_]+(?:\([^)]*\))?", s)

    def padded_len(self, length: int, rows: int) -> int:
        return int(lib().s1c_padded_len(self._h, length, rows))

    def warmup(self) -> None:
        self._check(lib().s1c_warmup(self._h))

    def forward(self, batch: Batch) -> BackendOutput:
        cb, keep = self._cbatch(batch)
        logits = np.empty(batch.n * batch.kmax, dtype=np.float32)
        pooled = np.empty(batch.n * self.hidden, dtype=np.float32)
        self._check(lib().s1c_forward_padded(self._h, C.byref(cb), _ptr(logits), _ptr(pooled)))
        return BackendOutput(logits, pooled)

    def encoder_hidden(self, batch: Batch) -> np.ndarray:
        cb, keep = self._cbatch(batch)
        out = np.empty(batch.n * batch.len * self.hidden, dtype=np.float32)
        self._check(lib().s1c_encoder_hidden(self._h, C.byref(cb), _ptr(out)))
        return out

    # -- unpadded entry points --------------------------------------------------------------
    def forward_varlen(self, v: Varlen, hidden: bool = False) -> BackendOutput:
        cv, keep = self._cvarlen(v)
        logits = np.empty(v.n * v.kmax, dtype=np.float32)
        pooled = np.empty(v.n * self.hidden, dtype=np.float32)
        hid = np.empty(v.total * self.hidden, dtype=np.float32) if hidden else None
        self._check(lib().s1c_forward_varlen(self._h, C.byref(cv), _ptr(logits), _ptr(pooled),
                                             _ptr(hid) if hidden else None))
        return BackendOutput(logits, pooled, hid)

    def forward_device(self, v: Varlen, d_ids: int, d_logits: int, d_pooled: int, d_hidden: int = 0) -> None:
        """Device-resident inputs/outputs (raw device pointers, e.g. ``tensor.data_ptr()``)."""
        cv, keep = self._cvarlen(v)
        self._check(lib().s1c_forward_device(self._h, C.byref(cv), d_ids, d_logits, d_pooled, d_hidden or None))

    def forward_device_async(self, v: Varlen, d_ids: int, d_logits: int, d_pooled: int, d_hidden: int = 0) -> None:
        """Enqueue a forward without waiting; ``synchronize()`` waits and reports device errors."""
        cv, keep = self._cvarlen(v)
        self._check(lib().s1c_forward_device_async(self._h, C.byref(cv), d_ids, d_logits, d_pooled,
                                                   d_hidden or None))

    def synchronize(self) -> None:
        self._check(lib().s1c_synchronize(self._h))

    def last_launch_count(self) -> int:
        return int(lib().s1c_last_launch_count(self._h))

    def set_stream(self, stream: int) -> None:
        """Run forwards on ``stream`` (a raw ``cudaStream_t``, e.g. ``torch.cuda.current_stream().cuda_stream``)."""
        self._check(lib().s1c_set_stream(self._h, stream or None))

    def profile(self, on: bool) -> None:
        self._check(lib().s1c_profile(self._h, 1 if on else 0))

    def profile_report(self) -> Dict[str, Dict[str, float]]:
        """Per-kernel totals since ``profile(True)``: launches, ms, algorithmic flops and bytes."""
        n = int(lib().s1c_profile_report(self._h, None, 0))
        buf = C.create_string_buffer(n)
        lib().s1c_profile_report(self._h, buf, n)
        out = {}
        for line in buf.value.decode().splitlines():
            name, launches, ms, flops, nbytes = line.split()
            out[name] = {"launches": int(launches), "ms": float(ms), "flops": float(flops), "bytes": float(nbytes)}
        return out

    # -- marshalling ------------------------------------------------------------------------
    @staticmethod
    def _cbatch(b: Batch):
        arrs = [np.ascontiguousarray(b.input_ids, dtype=np.uint32),
                np.ascontiguousarray(b.attention_mask, dtype=np.uint32),
                np.ascontiguousarray(b.seq_lens, dtype=np.uint64),
                np.ascontiguousarray(b.marker_pos, dtype=np.uint32),
                np.ascontiguousarray(b.marker_count, dtype=np.uint64),
                np.ascontiguousarray(b.qtype, dtype=np.uint32)]
        cb = CBatch(b.n, b.len, b.kmax, *[_ptr(a) for a in arrs])
        return cb, arrs

    @staticmethod
    def _cvarlen(v: Varlen):
        arrs = [np.ascontiguousarray(v.ids, dtype=np.uint32), np.ascontiguousarray(v.cu_seqlens, dtype=np.int32),
                np.ascontiguousarray(v.marker_pos, dtype=np.uint32),
                np.ascontiguousarray(v.marker_count, dtype=np.int32), np.ascontiguousarray(v.qtype, dtype=np.uint32)]
        cv = CVarlen(v.n, v.kmax, *[_ptr(a) for a in arrs])
        return cv, arrs


# -- isolated kernels (tests, GEMM sweep) ---------------------------------------------------
EPI_STORE, EPI_ROPE, EPI_GEGLU, EPI_RESID, EPI_RESID16 = 0, 1, 2, 3, 4


def gemm(epi: int, a_ptr: int, b_ptr: int, out_ptr: int, M: int, N: int, K: int, bias_ptr: int = 0, act: int = 0,
         out_f32: int = 0, pos_ptr: int = 0, rope_theta: float = 10000.0, rope_cols: int = 0, out_cols: int = 0,
         variant: int = 0, stream: int = 0) -> None:
    """variant 0: by shape; 1: one-CTA 128x256 tiles; 2: two-CTA 256x256 tiles; 3: one-CTA split-K through
    a workspace; 4: cluster split-K (partials reduced in distributed shared memory)."""
    L = lib()
    rc = L.s1c_gemm(epi, a_ptr, b_ptr, out_ptr, M, N, K, bias_ptr or None, act, out_f32, pos_ptr or None,
                    rope_theta, rope_cols, out_cols, variant, stream or None)
    if rc != S1C_OK:
        _raise(rc, L.s1c_create_error().decode())


def gemm_splitk_noalloc(epi: int, a_ptr: int, b_ptr: int, out_ptr: int, M: int, N: int, K: int, bias_ptr: int = 0,
                        act: int = 0, out_f32: int = 0, pos_ptr: int = 0, rope_theta: float = 10000.0,
                        rope_cols: int = 0, out_cols: int = 0, stream: int = 0) -> None:
    """Split-K GEMM whose partial sums live in the library's fixed 4 MiB device array: no device
    allocation on any call (``s1c_gemm_splitk_noalloc``)."""
    L = lib()
    rc = L.s1c_gemm_splitk_noalloc(epi, a_ptr, b_ptr, out_ptr, M, N, K, bias_ptr or None, act, out_f32,
                                   pos_ptr or None, rope_theta, rope_cols, out_cols, stream or None)
    if rc != S1C_OK:
        _raise(rc, L.s1c_create_error().decode())


def attention(q_ptr: int, k_ptr: int, v_ptr: int, o_ptr: int, q_stride: int, k_stride: int, v_stride: int,
              o_stride: int, heads: int, cu_seqlens: np.ndarray, window: int, scale: float, impl: int = 0,
              stream: int = 0) -> None:
    """impl 0: tcgen05 kernel; 1: mma.sync kernel."""
    L = lib()
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    rc = L.s1c_attention(q_ptr, k_ptr, v_ptr, o_ptr, q_stride, k_stride, v_stride, o_stride, heads, _ptr(cu),
                         len(cu) - 1, window, scale, impl, stream or None)
    if rc != S1C_OK:
        _raise(rc, L.s1c_create_error().decode())


def selftest_wait_timeout(device: int = 0, budget_ns: int = 50_000_000) -> list:
    """Run the bounded-wait self-test kernel (``s1c_selftest_wait_timeout``): returns the four result
    words [single-thread wait code, warp wait code, single-thread success, warp success]."""
    L = lib()
    codes = (C.c_int32 * 4)()
    rc = L.s1c_selftest_wait_timeout(device, budget_ns, codes)
    if rc != S1C_OK:
        _raise(rc, L.s1c_create_error().decode())
    return list(codes)


def interleave_wi(wi: np.ndarray, I: int) -> np.ndarray:
    """The row order the GeGLU epilogue expects (what ``s1c_create`` does to ``mlp.Wi``): per
    256-row tile, 128 input rows then the matching 128 gate rows, zero rows past ``I``."""
    tiles = (I + 127) // 128
    out = np.zeros((tiles * 256, wi.shape[1]), dtype=wi.dtype)
    for t in range(tiles):
        c0, c1 = 128 * t, min(128 * t + 128, I)
        out[256 * t: 256 * t + (c1 - c0)] = wi[c0:c1]
        out[256 * t + 128: 256 * t + 128 + (c1 - c0)] = wi[I + c0: I + c1]
    return out
