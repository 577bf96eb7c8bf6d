"""Single-kernel timing through the C ABI, for profiling one kernel on one shape.

    python -m sys1rust_b200.kernel_bench gemm --shape wi_geglu --m 16384 [--variant 1] [--reps 20]
    (variants as s1c_gemm: 0 by shape, 1 one-CTA 128x256, 2 two-CTA, 3 workspace split-K,
    4 cluster split-K, 5 one-CTA 128x128)
    python -m sys1rust_b200.kernel_bench attention --window 64 --tokens 16384 [--impl 1] [--reps 20]
    python -m sys1rust_b200.kernel_bench forward --workload cfg5 [--warm 3]

``gemm`` runs one encoder GEMM with its fused epilogue (shapes as in ``gemm_sweep``); ``attention``
runs the varlen attention over a packed batch of cfg5-distributed sequence lengths (lognormal,
median 200, clipped to [32, 1024]) filling ``--tokens`` tokens, 16 heads of 64, ``--window`` -1 for
global layers. Prints one JSON line: mean time per launch from CUDA events over ``--reps`` launches
after 3 warm-up launches, and the algorithmic TFLOP/s (attention: 4 * 64 per valid (query, key)
pair and head, the key set of the reference's masks). ``s1c_attention`` uploads its work list and
waits for the kernel on every call, so the attention figures are per call and include that upload
(a lower bound on the kernel's rate; the forward's per-launch profile times the kernel alone).
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .backend import EPI_RESID16, attention, gemm, interleave_wi
from .gemm_sweep import SHAPES as SWEEP_SHAPES

# The sweep's three shapes plus the attention output projection Wo (K 1024, N 1024, the f16
# residual add).
SHAPES = SWEEP_SHAPES + [("wo_resid", 1024, 1024, EPI_RESID16)]


def _time(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def bench_gemm(shape: str, M: int, variant: int, reps: int, seed: int = 0) -> dict:
    from .backend import EPI_GEGLU
    name, K, N, epi = next(s for s in SHAPES if s[0] == shape)
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    if epi == EPI_GEGLU:
        w = torch.randn(N, K, generator=g).to(torch.bfloat16)
        b = torch.from_numpy(interleave_wi(w.view(torch.int16).numpy(), N // 2)).view(torch.bfloat16).cuda()
        o = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda")
    else:
        b = torch.randn(N, K, generator=g).to(torch.bfloat16).cuda()
        o = torch.zeros(M, N, dtype=torch.float16 if epi == EPI_RESID16 else torch.bfloat16, device="cuda")
    pos = torch.from_numpy((np.arange(M) % 512).astype(np.int32)).cuda()

    def launch():
        gemm(epi, a.data_ptr(), b.data_ptr(), o.data_ptr(), M, b.shape[0], K, pos_ptr=pos.data_ptr(),
             rope_theta=10000.0, rope_cols=2048, out_cols=N // 2, variant=variant,
             stream=torch.cuda.current_stream().cuda_stream)

    ms = _time(launch, reps)
    return {"kernel": "gemm", "shape": name, "M": M, "N": N, "K": K, "variant": variant, "ms": ms,
            "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12}


def cfg5_lengths(tokens: int, seed: int = 1) -> list:
    rng = np.random.default_rng(seed)
    out, tot = [], 0
    while True:
        L = int(np.clip(np.round(np.exp(np.log(200.0) + 0.6 * rng.standard_normal())), 32, 1024))
        if tot + L > tokens:
            break
        out.append(L)
        tot += L
    return out


def valid_pairs(lens, window: int) -> int:
    tot = 0
    for L in lens:
        if window < 0:
            tot += L * L
        else:
            i = np.arange(L)
            tot += int((np.minimum(i, window) + np.minimum(L - 1 - i, window) + 1).sum())
    return tot


def bench_attention(tokens: int, window: int, impl: int, reps: int, heads: int = 16, seed: int = 0) -> dict:
    lens = cfg5_lengths(tokens)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, d = int(cu[-1]), heads * 64
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(T, 3 * d, generator=g).to(torch.bfloat16).cuda()
    o = torch.empty(T, d, dtype=torch.bfloat16, device="cuda")
    q, k, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]

    def launch():
        attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 3 * d, 3 * d, 3 * d, d, heads, cu, window,
                  0.125, impl=impl, stream=torch.cuda.current_stream().cuda_stream)

    ms = _time(launch, reps)
    flops = 4.0 * 64 * heads * valid_pairs(lens, window)
    return {"kernel": "attention", "impl": impl, "window": window, "tokens": T, "sequences": len(lens),
            "ms_per_call": ms, "tflops_per_call": flops / (ms / 1e3) / 1e12, "flops": flops}


def bench_forward(workload: str, warm: int) -> dict:
    """``warm`` untimed passes, then one pass, of a whole workload through the forward on one
    handle and stream (load check off, no warm-up captures): ``cfg5`` the bench's 15 varlen batches of
    one GPU's cfg5 share, ``cfg1`` one 128-token request. Every pass launches the same kernels, so
    an ncu launch list can skip ``warm`` passes (``launches_per_pass`` each) and capture the last."""
    from .backend import CudaBackend
    from .batch import Varlen
    from .config import large_model
    from .dist import shard_for_rank
    from .weights import SyntheticWeights
    from .workloads import cfg1, cfg5_requests, pack_batches
    cfg = large_model()
    w = SyntheticWeights(cfg, seed=0)
    be = CudaBackend.from_synthetic(cfg, w.tensors, max_tokens=16384, settings="check=0")
    st = torch.cuda.Stream()
    be.set_stream(st.cuda_stream)
    if workload == "cfg1":
        batches = [Varlen.from_rows(cfg1())]
    else:
        batches = pack_batches(shard_for_rank(cfg5_requests(n=1024, seed=1), 1, 0), 16384)
    ids = [torch.from_numpy(b.ids.astype(np.int32)).cuda() for b in batches]
    lg = torch.empty(max(max(b.n * b.kmax for b in batches), 1), device="cuda")
    pl = torch.empty(max(b.n for b in batches) * cfg.encoder.hidden_size, device="cuda")
    per_pass = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for p in range(warm + 1):
        if p == warm:
            torch.cuda.synchronize()
            e0.record(st)
        n = 0
        for b, i in zip(batches, ids):
            be.forward_device_async(b, i.data_ptr(), lg.data_ptr(), pl.data_ptr())
            n += be.last_launch_count()
        be.synchronize()
        per_pass = n
    e1.record(st)
    torch.cuda.synchronize()
    be.close()
    return {"kernel": "forward", "workload": workload, "batches": len(batches),
            "tokens": int(sum(b.total for b in batches)), "launches_per_pass": per_pass, "warm": warm,
            "ms_last_pass": e0.elapsed_time(e1)}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="kernel", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--shape", default="wi_geglu", choices=[s[0] for s in SHAPES])
    g.add_argument("--m", type=int, default=16384)
    g.add_argument("--variant", type=int, default=0)
    g.add_argument("--reps", type=int, default=20)
    a = sub.add_parser("attention")
    a.add_argument("--tokens", type=int, default=16384)
    a.add_argument("--window", type=int, default=64)
    a.add_argument("--impl", type=int, default=1)
    a.add_argument("--reps", type=int, default=20)
    f = sub.add_parser("forward")
    f.add_argument("--workload", default="cfg5", choices=["cfg5", "cfg1"])
    f.add_argument("--warm", type=int, default=3)
    args = ap.parse_args()
    if args.kernel == "gemm":
        r = bench_gemm(args.shape, args.m, args.variant, args.reps)
    elif args.kernel == "forward":
        r = bench_forward(args.workload, args.warm)
    else:
        r = bench_attention(args.tokens, args.window, args.impl, args.reps)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
