"""Benchmark of the sys1rust model forward on B200: encoder tokens/s on packed varlen batches.

    python bench.py --gpus N --steps K --warmup W            # this implementation
    python bench.py --impl reference --steps K --warmup W    # the reference's CPU path (oracle port)

A step is one pass over this GPU's share of the cfg5 serving workload: 1024 requests per GPU
(lognormal lengths, median 200, sigma 0.6, clipped to [32, 1024]; 1-10 questions each), packed
into varlen batches of at most 16384 tokens, each batch one full forward (encoder + decision head +
scorer). At N GPUs the job is the first N x 1024 requests of the cfg5 stream, shard-balanced by
estimated cost (LPT over GEMM work plus the quadratic global attention): weak scaling, and at N = 8 exactly cfg5's 8192 requests. Ranks share nothing on the
data path (replicas, no collective); the barrier and the max-over-ranks reduction are the only
collectives. ``value`` is the whole job's tokens / max-over-ranks device time.

Each GPU runs two handles of the model on two streams and alternates its batches between them.
Rank 0 prints one JSON line. Extra keys: ``e2e`` (the same requests submitted one by one from host
arrays to the serving queue, one native worker per handle, copies and result collection included;
the timed steps' requests form one stream, so the queue does not drain between steps;
``e2e_batched``: the pre-packed batches through ``s1c_forward_varlen``), ``roofline`` (dominant
kernel, from per-launch CUDA events over a second, single-stream pass of the timed steps),
``cpu_baseline`` (the PyTorch oracle on a bounded sample, with the C restatement beside it; N = 1
only), ``latency_cfg1`` (p50 ms of one 128-token request through the host API), ``cfg3_tokens_per_s``,
``clocks`` (nvidia-smi during the timed region), ``gpu_launches`` (this library's launches in the
timed region).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encoder tokens/sec/GPU (packed varlen) at 1/2/4/8 B200; p50 ms per 128-tok request"
# DRAM bytes (read + write) per algorithmic FLOP of a kernel, from one ncu capture of the Wi + GeGLU
# GEMM at M = 16384 (84.8 MB for 176.09 GFLOP); a launch's traffic is this times its FLOPs.
DRAM_BYTES_PER_FLOP = {"gemm_wi_geglu": 84.80e6 / 176.09e9}
REQ_PER_GPU = 1024
BATCH_TOKENS = 16384


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    from sys1rust_b200.dist import env_rank
    r = env_rank()
    return r.rank, r.world, r.local


def workload(world: int, rank: int):
    from sys1rust_b200.dist import shard_for_rank
    from sys1rust_b200.workloads import cfg5_requests
    reqs = cfg5_requests(n=REQ_PER_GPU * world, seed=1)
    return reqs, shard_for_rank(reqs, world, rank)


CPU_SAMPLE_REQUESTS = 32


def cpu_sample_requests():
    """The fixed request sample both CPU legs time: the first 1024 requests of the cfg5 stream
    sorted by length, every 32nd one (32 requests stratified by length, ~7 k tokens). The same
    requests at every N and in every step, so the reference rate does not depend on which requests
    a step happened to draw."""
    from sys1rust_b200.workloads import cfg5_requests
    reqs = sorted(cfg5_requests(n=REQ_PER_GPU, seed=1), key=lambda r: len(r.ids))
    step = len(reqs) // CPU_SAMPLE_REQUESTS
    return [reqs[i * step + step // 2] for i in range(CPU_SAMPLE_REQUESTS)]


def cpu_oracle_sample(cfg, weights, items, budget_s: float, kind: str = "torch"):
    """tokens/s (total tokens / total seconds) of a CPU restatement (fp32, all host threads) over
    requests of the workload, one row per forward, until every request has run or ``budget_s``
    seconds have passed (at least one request). ``kind`` "torch" is the PyTorch oracle
    (oracle/forward_ref.py), "c" the C / OpenMP one (oracle/forward_ref.c)."""
    import torch
    from sys1rust_b200.batch import collate_to
    torch.set_num_threads(os.cpu_count() or 1)
    if kind == "c":
        from oracle.forward_c import CForwardModel
        cm = CForwardModel(cfg, weights.tensors)
        run = lambda it: cm.forward_row(np.asarray(it.ids), it.markers, it.qtype)
        cores = int(os.environ.get("OMP_NUM_THREADS", len(os.sched_getaffinity(0))))
    else:
        from oracle.forward_ref import OracleModel
        om = OracleModel(cfg, weights.tensors)
        run = lambda it: om.forward(collate_to([it], cfg.encoder.pad_token_id))
        cores = torch.get_num_threads()
    run(items[0])  # warm
    t0 = time.perf_counter()
    tok = nreq = 0
    for it in items:
        run(it)
        tok += len(it.ids)
        nreq += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return tok / dt, {"cores": cores, "tokens": tok, "requests": nreq, "seconds": dt}


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            p = [x.strip() for x in l.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def arm_config(world: int, tokens_total: int, n_batches: int) -> dict:
    """The workload both arms report (the reference arm runs a bounded sample of it)."""
    return {"workload": f"cfg5 shard: {REQ_PER_GPU} lognormal requests per GPU (first "
                        f"{REQ_PER_GPU * world} of cfg5's stream, LPT by estimated cost), varlen batches "
                        f"<= {BATCH_TOKENS} tokens, full forward (encoder + head + scorer)",
            "model": "ModernBERT-large encoder (28 layers, d 1024, 16x64 heads, GeGLU 2x2624) + "
                     "2 decision-head layers + scorer, seeded N(0,0.02) bf16 weights",
            "tokens_per_step": tokens_total, "batches_per_gpu_step": n_batches,
            "l2": "inputs larger than L2: 686 MB of encoder weights stream every forward",
            "parallelism": f"dp{world} replicas, no data-path collective",
            "streams_per_gpu": 2}


def run_reference(args):
    """The reference arm: the CPU restatement of the forward (the reference's MLX-CPU path does
    not build here), all host threads, on this arm's workload, each step a bounded sample."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from sys1rust_b200.config import large_model
    from sys1rust_b200.weights import SyntheticWeights
    cfg = large_model()
    w = SyntheticWeights(cfg, seed=0)
    all_reqs, mine = workload(world, 0)
    from sys1rust_b200.workloads import pack_batches
    config = arm_config(world, sum(len(r.ids) for r in all_reqs), len(pack_batches(mine, BATCH_TOKENS)))
    config["reference_arm"] = ("rank 0 times the CPU restatement of the forward on a bounded sample of "
                               "this shard's requests, one row per forward, all host threads")
    config["reference_arm"] += (f"; at N > 1 only rank 0 runs it, so the value is one host's rate, not "
                                f"N hosts'")
    sample = cpu_sample_requests()
    sample_tokens = sum(len(r.ids) for r in sample)
    vals = []
    steps = args.steps
    for s in range(args.warmup + steps):
        v, info = cpu_oracle_sample(cfg, w, sample, 60.0)
        if s >= args.warmup:
            vals.append(v)
    v = float(np.median(vals))
    vc, infoc = cpu_oracle_sample(cfg, w, sample, 60.0, kind="c")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
                         "sample": f"each step the same {len(sample)} requests ({sample_tokens} tokens, cfg5 "
                                   f"stratified by length), one row per forward, torch fp32 oracle; median "
                                   f"of the timed steps; the reference's MLX-CPU path needs cargo + MLX, "
                                   f"absent here",
                         "steps_tokens_per_s": vals,
                         "c_restatement": {"value": vc, "cores": infoc["cores"],
                                           "sample": "the same requests once, oracle/forward_ref.c (fp32, "
                                                     "AVX2, OpenMP)"}},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    args.warmup = max(args.warmup, 3)
    # the in-tree library, compiled here if it is missing or older than its sources (nvcc ships
    # with the image; concurrent ranks serialise on a file lock)
    from sys1rust_b200 import build as lib_build
    lib_build.build()

    import torch
    from sys1rust_b200 import dist
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist.init(world, backend="nccl", timeout_s=120, device=torch.device("cuda", local))

    from sys1rust_b200.backend import CudaBackend
    from sys1rust_b200.config import large_model
    from sys1rust_b200.weights import SyntheticWeights
    from sys1rust_b200.workloads import cfg1, cfg3, pack_batches
    from sys1rust_b200.batch import Varlen

    cfg = large_model()
    t0 = time.time()
    w = SyntheticWeights(cfg, seed=0)
    # Two handles of the same model on this GPU, each on its own stream: consecutive batches go to
    # alternate handles, so one batch's kernels fill the SMs another batch's kernels leave idle
    # (the partial last wave of a GEMM, latency-bound attention). Measured +3.7 % over one stream;
    # a third stream added nothing.
    be = CudaBackend.from_synthetic(cfg, w.tensors, device=local, max_tokens=BATCH_TOKENS)
    be2 = CudaBackend.from_synthetic(cfg, w.tensors, device=local, max_tokens=BATCH_TOKENS)
    # load-time warm-up (the reference warms its length buckets at load): one captured graph per
    # packed-token bucket on each handle
    be.warmup()
    be2.warmup()
    log(f"[rank {rank}] model ready in {time.time() - t0:.1f}s: {be.name()} x 2 streams")
    # Dedicated (non-default) streams: each backend captures per-shape CUDA graphs on its own.
    stream = torch.cuda.Stream()
    stream2 = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    be.set_stream(stream.cuda_stream)
    be2.set_stream(stream2.cuda_stream)

    all_reqs, mine = workload(world, rank)
    batches = pack_batches(mine, BATCH_TOKENS)
    tokens_mine = sum(b.total for b in batches)
    # inputs resident in HBM before timing
    d_ids = [torch.from_numpy(b.ids.astype(np.int32)).cuda() for b in batches]
    max_n = max(b.n for b in batches)
    max_m = max(b.n * b.kmax for b in batches)
    outs = [(torch.empty(max(max_m, 1), dtype=torch.float32, device="cuda"),
             torch.empty(max_n * cfg.encoder.hidden_size, dtype=torch.float32, device="cuda")) for _ in range(2)]
    handles = (be, be2)
    launch_count = [0]

    def step(count=False):
        # every batch of the step enqueued back to back, alternating handles; one wait at the end
        for i, (b, ids) in enumerate(zip(batches, d_ids)):
            h = handles[i & 1]
            h.forward_device_async(b, ids.data_ptr(), outs[i & 1][0].data_ptr(), outs[i & 1][1].data_ptr())
            if count:
                launch_count[0] += h.last_launch_count()
        be.synchronize()
        be2.synchronize()

    def barrier():
        torch.cuda.synchronize()
        dist.barrier(world)
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        return dist.max_over_ranks(x, world, device="cuda")

    for _ in range(args.warmup):
        step()
    # ---- timed region: device-resident inputs --------------------------------------------
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        stream2.wait_event(e0)
        for _ in range(args.steps):
            step(count=True)
        e1.record(stream)  # both handles were synchronised at the end of the last step
        barrier()
    launches = launch_count[0]
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    per_rank = dist.gather_over_ranks([ms / args.steps, len(batches), tokens_mine], world, rank, device="cuda")
    tokens_total = sum(len(r.ids) for r in all_reqs)
    value = tokens_total * args.steps / (ms_max / 1e3)

    # ---- the same steps again with per-launch CUDA events (kernel shares, roofline) ---------
    be.profile(True)
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    for _ in range(args.steps):  # one handle, one stream: per-launch events see each kernel alone
        for b, ids in zip(batches, d_ids):
            be.forward_device_async(b, ids.data_ptr(), outs[0][0].data_ptr(), outs[0][1].data_ptr())
        be.synchronize()
    p1.record(stream)
    barrier()
    prof_ms = p0.elapsed_time(p1)
    prof = be.profile_report()
    be.profile(False)
    kernel_ms = sum(v["ms"] for v in prof.values()) / args.steps
    # ---- e2e: the serving API with host buffers, copies inside the timed region -------------
    # This rank's requests are submitted one by one to the serving queue (sys1rust_b200.server:
    # one native worker per handle, cross-request packing into <= BATCH_TOKENS varlen batches,
    # each batch's ids / metadata copied in and its logits / pooled rows copied back) and every
    # result is collected per request.
    from sys1rust_b200.server import Server
    be.set_stream(0)  # the backends' own streams
    be2.set_stream(0)
    # The timed steps' requests arrive as one stream, as under continuous load: step k + 1's
    # requests are queued while step k's are still being served, so the queue does not drain
    # between steps; every request's result is still collected.
    e2e_steps = max(1, min(args.steps, 3))
    with Server([be, be2], max_concurrent=e2e_steps * len(mine) + 1, max_batch_tokens=BATCH_TOKENS,
                linger_us=1000) as srv:
        def serve_all(steps):
            tk = [srv.submit(it) for _ in range(steps) for it in mine]
            for i, t in enumerate(tk):
                srv.wait(t, len(mine[i % len(mine)].markers))
        serve_all(1)  # warm-up pass
        barrier()
        t_e2e = time.perf_counter()
        serve_all(e2e_steps)
        e2e_s = max_over_ranks(time.perf_counter() - t_e2e)
        srv_stats = srv.stats()
    e2e_value = tokens_total * e2e_steps / e2e_s
    # bytes per step: each request's ids, marker positions, qtype, row offset and marker count in,
    # plus one closing offset per batch; its marker logits and pooled row out (the kmax padding of
    # a batch's logits rows is not counted)
    batches_per_step = int(srv_stats["batches"]) // (e2e_steps + 1)
    h2d = sum(4 * (len(it.ids) + len(it.markers) + 3) for it in mine) + 4 * batches_per_step
    d2h = sum(4 * (len(it.markers) + cfg.encoder.hidden_size) for it in mine)

    # ---- the same host-buffer path on pre-packed batches, one handle (s1c_forward_varlen) ----
    for b in batches[:2]:
        be.forward_varlen(b)
    barrier()
    t_b = time.perf_counter()
    for b in batches:
        be.forward_varlen(b)
    batched_s = max_over_ranks(time.perf_counter() - t_b)
    e2e_batched = {"value": tokens_total / batched_s, "unit": "tokens/s",
                   "path": "s1c_forward_varlen on the step's pre-packed batches, one handle"}

    # ---- latency of one 128-token request (cfg1), host API ---------------------------------
    lat = None
    one = Varlen.from_rows(cfg1())
    for _ in range(20):
        be.forward_varlen(one)
    ts = []
    for _ in range(100):
        t = time.perf_counter()
        be.forward_varlen(one)
        ts.append((time.perf_counter() - t) * 1e3)
    lat = {"p50_ms": float(np.median(ts)), "p90_ms": float(np.percentile(ts, 90)), "n": len(ts),
           "path": "s1c_forward_varlen, host buffers, copies included; the same request 100 times after 20"}
    # ---- latency over single requests whose shapes never repeat --------------------------
    from sys1rust_b200.latency import stream_latency
    from sys1rust_b200.workloads import latency_stream
    lat_stream = stream_latency(be, latency_stream(200))
    lat_stream.update({"workload": "200 single requests, lengths U[64, 200], 1-3 questions, no (length, "
                                   "marker count) repeated, each run once",
                       "path": "s1c_forward_varlen, host buffers, copies included; packed-token buckets "
                               "with graphs captured by warmup() at load"})

    # ---- cfg3: 64 requests U[64,512] in one varlen batch, device-resident -----------------
    c3 = Varlen.from_rows(cfg3())
    c3_ids = torch.from_numpy(c3.ids.astype(np.int32)).cuda()
    c3_l = torch.empty(c3.n * c3.kmax, dtype=torch.float32, device="cuda")
    c3_p = torch.empty(c3.n * cfg.encoder.hidden_size, dtype=torch.float32, device="cuda")
    be.set_stream(stream.cuda_stream)
    for _ in range(3):
        be.forward_device(c3, c3_ids.data_ptr(), c3_l.data_ptr(), c3_p.data_ptr())
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(10):
        be.forward_device(c3, c3_ids.data_ptr(), c3_l.data_ptr(), c3_p.data_ptr())
    a1.record(stream)
    torch.cuda.synchronize()
    cfg3_tps = c3.total * 10 / (a0.elapsed_time(a1) / 1e3)

    # ---- roofline of the dominant kernel ------------------------------------------------
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    total_ms = sum(v["ms"] for v in prof.values()) or 1.0
    dom_name, dom = max(prof.items(), key=lambda kv: kv[1]["ms"])
    per_launch_ms = dom["ms"] / dom["launches"]
    traffic = None
    if dom_name in DRAM_BYTES_PER_FLOP and dom["flops"] > 0:
        traffic = DRAM_BYTES_PER_FLOP[dom_name] * dom["flops"] / dom["launches"]
    if dom["flops"] > 0:
        achieved = dom["flops"] / dom["launches"] / (per_launch_ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops_sustained")
        roof = {"kernel": dom_name, "bound": "tensor", "achieved": achieved, "unit": "TFLOP/s",
                "peak": peak if peak else 1400.0, "peak_source": "measured (sustained)" if peak else "fallback",
                "frac": achieved / (peak if peak else 1400.0), "traffic": traffic,
                "flops_per_launch": dom["flops"] / dom["launches"], "ms_per_launch": per_launch_ms,
                "share_of_device_time": dom["ms"] / total_ms,
                "measured": "per-launch CUDA events on the launch stream over a second pass of the timed steps"}
    else:
        achieved = dom["bytes"] / dom["launches"] / (per_launch_ms / 1e3) / 1e9
        peak = peaks.get("hbm_gbs", 6650.0)
        roof = {"kernel": dom_name, "bound": "hbm", "achieved": achieved, "unit": "GB/s", "peak": peak,
                "frac": achieved / peak, "traffic": traffic, "share_of_device_time": dom["ms"] / total_ms}
    enc = [k for k in prof if k.startswith("gemm_")]
    enc_tflops = sum(prof[k]["flops"] for k in enc) / (sum(prof[k]["ms"] for k in enc) / 1e3) / 1e12 if enc else None
    kernels = {k: {"launches": v["launches"], "share": v["ms"] / total_ms,
                   "tflops": (v["flops"] / (v["ms"] / 1e3) / 1e12) if v["flops"] else None,
                   "gbs": (v["bytes"] / (v["ms"] / 1e3) / 1e9) if v["bytes"] else None}
               for k, v in sorted(prof.items(), key=lambda kv: -kv[1]["ms"])}

    # ---- CPU baseline (rank 0, N = 1) -----------------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = cpu_sample_requests()
        v, info = cpu_oracle_sample(cfg, w, sample, 30.0)
        vc, infoc = cpu_oracle_sample(cfg, w, sample, 30.0, kind="c")
        cpu = {"value": v, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
               "sample": f"{info['requests']} requests / {info['tokens']} tokens of this workload (cfg5 "
                         f"stratified by length, the reference arm's sample), one row per forward, "
                         f"{info['seconds']:.1f} s, torch fp32 oracle",
               "c_restatement": {"value": vc, "cores": infoc["cores"],
                                 "sample": f"{infoc['requests']} requests / {infoc['tokens']} tokens, "
                                           f"{infoc['seconds']:.1f} s, oracle/forward_ref.c (fp32, AVX2, OpenMP)"}}

    dist.barrier(world)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "value_per_gpu": value / world,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {**arm_config(world, tokens_total, len(batches)),
                       "value_reading": f"value is the whole job's tokens/s over all {world} GPU(s); per GPU "
                                        f"that is {value / world:.0f} tokens/s (value_per_gpu)"},
            "per_rank": [{"rank": r, "ms_per_step": p[0], "batches": int(p[1]), "tokens": int(p[2])}
                         for r, p in enumerate(per_rank)],
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
                    "path": "sys1rust_b200.server.Server (s1c_server_*): the step's requests submitted one by one "
                            "from host arrays, packed across requests by one native worker per handle (2 per "
                            "GPU), host -> device copies and logits / pooled rows back to host inside the timed "
                            "region, every result collected per request; the timed steps' requests form one "
                            "stream (no queue drain between steps)"},
            "e2e_batched": e2e_batched,
            "roofline": roof,
            "encoder_gemm_tflops": enc_tflops,
            "cpu_baseline": cpu,
            "latency_cfg1": lat,
            "latency_stream": lat_stream,
            "cfg3_tokens_per_s": cfg3_tps,
            "clocks": clk.summary(),
            "gpu_launches": int(launches),
            "profiled_pass_ms_per_step": prof_ms / args.steps,
            "kernel_ms_per_step": kernel_ms,
            "kernels": kernels,
        }
        print(json.dumps(line), flush=True)
    be.close()
    be2.close()
    dist.shutdown(world)


if __name__ == "__main__":
    main()
