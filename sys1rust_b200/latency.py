"""Single-request latency through the host API (``s1c_forward_varlen``: host buffers in, logits and
pooled rows back on the host).

    python -m sys1rust_b200.latency [--reps 50] [--warm 5] [--stream 200]

Builds the ModernBERT-large model from seeded weights and runs ``warmup()`` (the reference warms
its length buckets at load, ``laya-mlx/src/lib.rs:1152-1173``; here that captures one CUDA graph
per packed-token bucket). Then prints one JSON line with:

* ``cfg1``: p50 / p90 wall milliseconds over ``--reps`` calls of benchmark config 1 (one row of
  128 tokens, one noul question), and the device milliseconds of that forward run back to back
  from device-resident inputs (CUDA events);
* ``stream``: p50 / p90 over ``--stream`` single requests whose shapes never repeat (lengths
  U[64, 200], 1-3 questions; ``workloads.latency_stream``), each run once.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def stream_latency(be, reqs) -> dict:
    """Wall milliseconds of each request of ``reqs`` run once through ``forward_varlen``."""
    from .batch import Varlen
    ts = []
    for it in reqs:
        v = Varlen.from_rows([it])
        t = time.perf_counter()
        be.forward_varlen(v)
        ts.append((time.perf_counter() - t) * 1e3)
    return {"p50_ms": float(np.median(ts)), "p90_ms": float(np.percentile(ts, 90)),
            "max_ms": float(np.max(ts)), "n": len(ts),
            "distinct_shapes": len({(len(r.ids), len(r.markers)) for r in reqs})}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--warm", type=int, default=5)
    ap.add_argument("--stream", type=int, default=200)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args()

    import torch
    from .backend import CudaBackend
    from .batch import Varlen
    from .config import large_model
    from .weights import SyntheticWeights
    from .workloads import cfg1, latency_stream

    cfg = large_model()
    w = SyntheticWeights(cfg, seed=0)
    be = CudaBackend.from_synthetic(cfg, w.tensors, device=args.device, max_tokens=4096)
    t0 = time.perf_counter()
    be.warmup()
    warm_s = time.perf_counter() - t0
    stream = stream_latency(be, latency_stream(args.stream)) if args.stream else None

    one = Varlen.from_rows(cfg1())
    for _ in range(args.warm):
        be.forward_varlen(one)
    ts = []
    for _ in range(args.reps):
        t = time.perf_counter()
        be.forward_varlen(one)
        ts.append((time.perf_counter() - t) * 1e3)

    st = torch.cuda.Stream(args.device)
    be.set_stream(st.cuda_stream)
    ids = torch.from_numpy(one.ids.astype(np.int32)).cuda(args.device)
    lg = torch.empty(max(one.n * one.kmax, 1), device=f"cuda:{args.device}")
    pl = torch.empty(one.n * cfg.encoder.hidden_size, device=f"cuda:{args.device}")
    for _ in range(args.warm):
        be.forward_device(one, ids.data_ptr(), lg.data_ptr(), pl.data_ptr())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.reps):
        be.forward_device_async(one, ids.data_ptr(), lg.data_ptr(), pl.data_ptr())
    e1.record(st)
    be.synchronize()
    torch.cuda.synchronize()
    print(json.dumps({"cfg1": {"workload": "1 row x 128 tokens, 1 noul question", "p50_ms": float(np.median(ts)),
                               "p90_ms": float(np.percentile(ts, 90)), "reps": args.reps,
                               "device_ms_per_forward": e0.elapsed_time(e1) / args.reps,
                               "launches_per_forward": be.last_launch_count()},
                      "stream": stream, "warmup_s": warm_s}))
    be.close()


if __name__ == "__main__":
    main()
