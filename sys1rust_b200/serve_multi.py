"""Serving throughput of one queue over several GPUs in one process.

    python -m sys1rust_b200.serve_multi [--gpus 2] [--handles-per-gpu 2] [--steps 3]

The reference serves every request on one inference thread (``runtime/crates/sys1rust/src/
worker.rs:1-4``); here one ``s1c_server`` queue feeds ``handles-per-gpu`` workers on each of
``--gpus`` GPUs (ModernBERT-large, seeded weights, ``warmup()`` at load). The cfg5 stream's first
1024 x gpus requests are submitted one by one from host arrays, packed across requests into
varlen batches of at most 16384 tokens, and every result is collected (logits and pooled rows back
on the host). One untimed pass, then ``--steps`` passes submitted as one stream and timed by the
wall clock around submission and collection. Prints one JSON line: tokens/s for the whole job and
per GPU, batches, the number of handles that served batches.
"""
from __future__ import annotations

import argparse
import json
import time


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--handles-per-gpu", type=int, default=2)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--requests-per-gpu", type=int, default=1024)
    args = ap.parse_args()

    import torch
    from .backend import CudaBackend
    from .config import large_model
    from .server import Server
    from .weights import SyntheticWeights
    from .workloads import cfg5_requests

    n_dev = torch.cuda.device_count()
    if n_dev < args.gpus:
        raise SystemExit(f"{args.gpus} GPUs asked for, {n_dev} visible")
    cfg = large_model()
    w = SyntheticWeights(cfg, seed=0)
    t0 = time.time()
    bes = []
    for dev in range(args.gpus):
        for _ in range(args.handles_per_gpu):
            be = CudaBackend.from_synthetic(cfg, w.tensors, device=dev, max_tokens=16384)
            be.warmup()
            bes.append(be)
    load_s = time.time() - t0
    reqs = cfg5_requests(n=args.requests_per_gpu * args.gpus, seed=1)
    tokens = sum(len(r.ids) for r in reqs)
    with Server(bes, max_concurrent=(args.steps + 1) * len(reqs) + 1, max_batch_tokens=16384,
                linger_us=1000) as srv:
        def serve(steps):
            tk = [srv.submit(it) for _ in range(steps) for it in reqs]
            for i, t in enumerate(tk):
                srv.wait(t, len(reqs[i % len(reqs)].markers))
        serve(1)
        t = time.perf_counter()
        serve(args.steps)
        dt = time.perf_counter() - t
        st = srv.stats()
    served = sum(1 for b in bes if b.last_launch_count() > 0)
    v = tokens * args.steps / dt
    print(json.dumps({"metric": "serving tokens/s, one queue over several GPUs (host buffers, copies and "
                                "result collection included)", "value": v, "unit": "tokens/s",
                      "per_gpu": v / args.gpus, "gpus": args.gpus, "handles": len(bes),
                      "handles_that_served": served, "steps": args.steps, "requests_per_step": len(reqs),
                      "tokens_per_step": tokens, "batches": int(st["batches"]), "load_s": load_s,
                      "workload": "cfg5's first 1024 x gpus requests, one queue, varlen batches <= 16384 tokens"}))
    for b in bes:
        b.close()


if __name__ == "__main__":
    main()
