"""Python face of the library's serving queue (``s1c_server_*``): cross-request varlen batching
over one worker per GPU, with the reference server's admission contract.

The reference serves one request at a time on one inference thread
(``runtime/crates/sys1rust/src/worker.rs:1-4``) behind a non-blocking admission semaphore
(``runtime/crates/sys1rust/src/http.rs:168-181``: over the cap the answer is 503 "server busy, try
again later" with ``Retry-After: 1``). Here the queue and the workers are native (``server.h``); this
module maps its statuses onto exceptions an HTTP layer turns into the reference's responses:

* ``ServerBusy`` -> 503 with ``Retry-After: ServerBusy.retry_after`` (1 s);
* ``WorkerNotRunning`` -> 503 "inference worker is not running";
* ``BackendError`` (a failed forward) -> 500 with an opaque body;
* ``BackendError`` with code ``S1C_ERR_ARG`` for a malformed row (422-class input).

    srv = Server([backend_gpu0, backend_gpu1], max_concurrent=64)
    ticket = srv.submit(item)            # EncodedItem: ids, marker positions, qtype
    logits, pooled, infer_ms = srv.wait(ticket)
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

from .backend import (S1C_ERR_ARG, S1C_ERR_BUSY, S1C_ERR_DEAD, S1C_ERR_TIMEOUT, S1C_OK, SERVER_FORWARD_FN,
                      BackendError, CRequest, CVarlen, ServerOpts, ServerStats, _raise, lib)
from .batch import EncodedItem


class ServerBusy(BackendError):
    """Over the admission cap: refused without queueing (HTTP 503, ``Retry-After: 1``)."""
    retry_after = 1


class WorkerNotRunning(BackendError):
    """No inference worker is running (HTTP 503)."""


class WaitTimeout(BackendError):
    """The result was not ready within the wait's timeout; the ticket stays valid."""


def _check(rc: int) -> None:
    if rc == S1C_OK:
        return
    msg = lib().s1c_create_error().decode()
    if rc == S1C_ERR_BUSY:
        raise ServerBusy(rc, msg)
    if rc == S1C_ERR_DEAD:
        raise WorkerNotRunning(rc, msg)
    if rc == S1C_ERR_TIMEOUT:
        raise WaitTimeout(rc, msg)
    _raise(rc, msg)


# A Python forward for ``Server(forward=...)``: (worker index, n, kmax, ids, cu_seqlens, marker_pos
# [n, kmax], marker_count, qtype) -> (logits [n, kmax], pooled [n, hidden]); raising fails the batch.
PyForward = Callable[[int, int, int, np.ndarray, np.ndarray, np.ndarray, np.ndarray, np.ndarray],
                     Tuple[np.ndarray, np.ndarray]]


class Server:
    def __init__(self, backends: Optional[Sequence] = None, *, forward: Optional[PyForward] = None,
                 n_workers: int = 1, hidden: Optional[int] = None, max_concurrent: int = 16,
                 max_batch_tokens: int = 16384, max_batch_rows: int = 1024, linger_us: int = 0):
        """Workers over ``backends`` (``CudaBackend`` instances, one worker each), or over a Python
        ``forward`` callable (``n_workers`` workers, pooled rows of ``hidden`` floats)."""
        L = lib()
        opts = ServerOpts(max_concurrent, max_batch_tokens, max_batch_rows, linger_us)
        h = C.c_void_p()
        self._cb = None
        self._err = []
        if backends is not None:
            self.hidden = backends[0].hidden
            self._backends = list(backends)  # kept alive while the server runs
            arr = (C.c_void_p * len(backends))(*[b._h.value for b in backends])
            rc = L.s1c_server_create(arr, len(backends), C.byref(opts), C.byref(h))
        else:
            if forward is None or hidden is None:
                raise ValueError("give backends, or a forward callable and hidden")
            self.hidden = hidden
            self._backends = []
            self._cb = SERVER_FORWARD_FN(self._trampoline(forward, hidden))
            ctx = (C.c_void_p * n_workers)(*range(n_workers))
            rc = L.s1c_server_create_with(self._cb, ctx, n_workers, hidden, C.byref(opts), C.byref(h))
        _check(rc)
        self._h = h

    def _trampoline(self, forward: PyForward, hidden: int):
        keep = self._err

        def cb(ctx, vp, lp, pp, errp):
            try:
                v = vp.contents
                n, kmax = v.n, v.kmax
                cu = np.ctypeslib.as_array(C.cast(v.cu_seqlens, C.POINTER(C.c_int32)), (n + 1,)).copy()
                ids = np.ctypeslib.as_array(C.cast(v.ids, C.POINTER(C.c_uint32)), (int(cu[-1]),)).copy()
                km = max(kmax, 1)
                mp = np.ctypeslib.as_array(C.cast(v.marker_pos, C.POINTER(C.c_uint32)), (n * km,)).reshape(n, km).copy()
                mc = np.ctypeslib.as_array(C.cast(v.marker_count, C.POINTER(C.c_int32)), (n,)).copy()
                qt = np.ctypeslib.as_array(C.cast(v.qtype, C.POINTER(C.c_uint32)), (n,)).copy()
                logits, pooled = forward(int(ctx or 0), n, kmax, ids, cu, mp, mc, qt)
                np.ctypeslib.as_array(lp, (n * km,))[:] = np.asarray(logits, np.float32).reshape(-1)[: n * km]
                np.ctypeslib.as_array(pp, (n * hidden,))[:] = np.asarray(pooled, np.float32).reshape(-1)
                return S1C_OK
            except Exception as e:  # the batch fails; the worker keeps serving
                msg = C.create_string_buffer(f"forward failed: {e}".encode())
                keep.append(msg)
                del keep[:-4]
                errp[0] = C.cast(msg, C.c_char_p)
                return -2
        return cb

    def submit(self, item: EncodedItem) -> int:
        ids = np.ascontiguousarray(item.ids, dtype=np.uint32)
        mk = np.ascontiguousarray(item.markers, dtype=np.uint32)
        req = CRequest(ids.ctypes.data if ids.size else None, int(ids.size), mk.ctypes.data if mk.size else None,
                       int(mk.size), int(item.qtype))
        t = C.c_uint64()
        _check(lib().s1c_server_submit(self._h, C.byref(req), C.byref(t)))
        return int(t.value)

    def wait(self, ticket: int, n_markers: int, timeout_ms: int = -1) -> Tuple[np.ndarray, np.ndarray, float]:
        """(logits [n_markers], pooled [hidden], forward ms of the request's batch)."""
        logits = np.empty(max(n_markers, 1), dtype=np.float32)
        pooled = np.empty(self.hidden, dtype=np.float32)
        ms = C.c_float()
        _check(lib().s1c_server_wait(self._h, ticket, timeout_ms, logits.ctypes.data, pooled.ctypes.data,
                                     C.byref(ms)))
        return logits[:n_markers], pooled, float(ms.value)

    def predict(self, item: EncodedItem, timeout_ms: int = -1):
        return self.wait(self.submit(item), len(item.markers), timeout_ms)

    def cancel(self, ticket: int) -> None:
        _check(lib().s1c_server_cancel(self._h, ticket))

    def stats(self) -> dict:
        s = ServerStats()
        _check(lib().s1c_server_get_stats(self._h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in ServerStats._fields_}

    def stop(self) -> None:
        if getattr(self, "_h", None):
            lib().s1c_server_stop(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().s1c_server_destroy(self._h)
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
