"""Encoder GEMM sweep (benchmark config 4): M in {128, 512, 2048, 8192, 32768} against the three
encoder shapes with their fused epilogues -- Wqkv (K 1024, N 3072, RoPE), Wi (K 1024, N 5248,
GeGLU) and Wo2 (K 2624, N 1024, the f16 residual add of the forward) -- with A and B drawn N(0, 1) from a seed.

``python -m sys1rust_b200.gemm_sweep [--variants 1,2] [--cublas]`` prints one JSON line per
(shape, M, variant): achieved TFLOP/s from CUDA events over repeated launches (inputs larger than
L2 are not needed here: the operands of one launch stay L2-resident across repeats, as they do
inside the forward). ``--cublas`` adds torch.matmul on the same shapes (no epilogue) for scale.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .backend import EPI_GEGLU, EPI_RESID16, EPI_ROPE, gemm, interleave_wi

SHAPES = [("wqkv_rope", 1024, 3072, EPI_ROPE), ("wi_geglu", 1024, 5248, EPI_GEGLU), ("wo2_resid", 2624, 1024, EPI_RESID16)]
MS = [128, 512, 2048, 8192, 32768]


def run(variants=(1, 2), cublas=False, reps=20, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for name, K, N, epi in SHAPES:
        Mmax = max(MS)
        a = torch.randn(Mmax, K, generator=g).to(torch.bfloat16).cuda()
        if epi == EPI_GEGLU:
            I = N // 2
            w = torch.randn(N, K, generator=g).to(torch.bfloat16)
            b = torch.from_numpy(interleave_wi(w.view(torch.int16).numpy(), I)).view(torch.bfloat16).cuda()
            Nk, o = b.shape[0], torch.empty(Mmax, I, dtype=torch.bfloat16, device="cuda")
        else:
            b = torch.randn(N, K, generator=g).to(torch.bfloat16).cuda()
            Nk = N
            o = torch.zeros(Mmax, N, dtype=torch.float16 if epi == EPI_RESID16 else torch.bfloat16, device="cuda")
        pos = torch.from_numpy((np.arange(Mmax) % 512).astype(np.int32)).cuda()
        flops_per_row = 2.0 * K * N
        for M in MS:
            for v in variants:
                def launch():
                    gemm(epi, a.data_ptr(), b.data_ptr(), o.data_ptr(), M, Nk, K, pos_ptr=pos.data_ptr(),
                         rope_theta=10000.0, rope_cols=2048, out_cols=N // 2, variant=v,
                         stream=torch.cuda.current_stream().cuda_stream)
                for _ in range(3):
                    launch()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    launch()
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / reps
                out.append({"shape": name, "M": M, "K": K, "N": N, "variant": v, "ms": ms,
                            "tflops": flops_per_row * M / (ms / 1e3) / 1e12})
            if cublas:
                bt = b[:N].t() if epi != EPI_GEGLU else b.t()
                for _ in range(3):
                    torch.matmul(a[:M], bt)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    torch.matmul(a[:M], bt)
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / reps
                out.append({"shape": name, "M": M, "K": K, "N": N, "variant": "cublas_matmul", "ms": ms,
                            "tflops": flops_per_row * M / (ms / 1e3) / 1e12})
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--variants", default="1,2")
    ap.add_argument("--cublas", action="store_true")
    args = ap.parse_args()
    for r in run(tuple(int(x) for x in args.variants.split(",")), args.cublas):
        print(json.dumps(r))
