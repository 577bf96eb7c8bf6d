"""The multi-GPU host logic on CPU: two gloo ranks (world size 2, 127.0.0.1) run the sharding and the
collectives ``bench.py`` uses at N > 1, and a rank that never joins makes the other's collective
fail within the process-group timeout instead of hanging.
"""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_req, out_dir):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    from sys1rust_b200 import dist
    from sys1rust_b200.workloads import cfg5_requests
    info = dist.env_rank()
    dist.init(info.world, backend="gloo", timeout_s=60)
    reqs = cfg5_requests(n=n_req, seed=1)
    mine = dist.shard_for_rank(reqs, info.world, info.rank)
    pos = {id(r): i for i, r in enumerate(reqs)}
    ids = [pos[id(r)] for r in mine]
    tokens = sum(len(r.ids) for r in mine)
    dist.barrier(info.world)
    mx = dist.max_over_ranks(float(tokens), info.world)
    tot = dist.sum_over_ranks(float(tokens), info.world)
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{tokens} {mx} {tot}\n" + " ".join(map(str, ids)) + "\n")
    dist.shutdown(info.world)


def test_two_gloo_ranks_shard_disjointly_and_reduce(tmp_path):
    world, n_req = 2, 96
    mp.start_processes(_rank_main, args=(world, _free_port(), n_req, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    from sys1rust_b200.workloads import cfg5_requests
    reqs = cfg5_requests(n=n_req, seed=1)
    seen, toks = [], []
    for r in range(world):
        head, idx = open(tmp_path / f"rank{r}.txt").read().splitlines()
        t = head.split()[0]
        toks.append(int(t))
        seen.append([int(i) for i in idx.split()])
    all_tok = sum(len(x.ids) for x in reqs)
    for r in range(world):
        head = open(tmp_path / f"rank{r}.txt").read().splitlines()[0].split()
        assert float(head[1]) == max(toks)
        assert float(head[2]) == all_tok
    # every request on exactly one rank, arrival order kept within a rank
    assert sorted(seen[0] + seen[1]) == list(range(n_req))
    assert all(s == sorted(s) for s in seen)
    # longest-first least-loaded: the imbalance is at most one request's length
    assert abs(toks[0] - toks[1]) <= max(len(x.ids) for x in reqs)


def _lonely_rank(rank, world, port, out_dir):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    import torch.distributed as tdist
    from sys1rust_b200 import dist
    if rank == 1:
        # this rank joins, then leaves between steps without entering the collective
        dist.init(world, backend="gloo", timeout_s=5)
        with open(os.path.join(out_dir, "rank1.txt"), "w") as f:
            f.write("left\n")
        return
    dist.init(world, backend="gloo", timeout_s=5)
    try:
        dist.max_over_ranks(1.0, world)
        msg = "completed"
    except Exception as e:  # the process-group timeout ends the collective with an error
        msg = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(msg + "\n")
    try:
        tdist.destroy_process_group()
    except Exception:
        pass


def test_rank_that_leaves_fails_the_others_collective(tmp_path):
    world = 2
    ctx = mp.start_processes(_lonely_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                             start_method="spawn", join=False)
    ctx.join(timeout=120)
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    out = open(tmp_path / "rank0.txt").read().strip()
    assert out.startswith("error"), out
