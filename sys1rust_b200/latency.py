"""Single-request latency (benchmark config 1): one row of 128 tokens with one noul question through
the host API (``s1c_forward_varlen``: host buffers in, logits and pooled rows back on the host).

    python -m sys1rust_b200.latency [--reps 50] [--warm 5]

Builds the ModernBERT-large model from seeded weights, runs ``--warm`` forwards (the second one
records the shape's CUDA graph), then prints one JSON line: p50 / p90 wall milliseconds per call
over ``--reps`` calls and the device milliseconds of a forward run back to back from device-
resident inputs (CUDA events).
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--warm", type=int, default=5)
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args()

    import torch
    from .backend import CudaBackend
    from .batch import Varlen
    from .config import large_model
    from .weights import SyntheticWeights
    from .workloads import cfg1

    cfg = large_model()
    w = SyntheticWeights(cfg, seed=0)
    be = CudaBackend.from_synthetic(cfg, w.tensors, device=args.device, max_tokens=4096)
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
    print(json.dumps({"workload": "cfg1: 1 row x 128 tokens, 1 noul question", "p50_ms": float(np.median(ts)),
                      "p90_ms": float(np.percentile(ts, 90)), "reps": args.reps,
                      "device_ms_per_forward": e0.elapsed_time(e1) / args.reps,
                      "launches_per_forward": be.last_launch_count()}))
    be.close()


if __name__ == "__main__":
    main()
