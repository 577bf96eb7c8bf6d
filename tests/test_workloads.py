"""Host logic of the benchmark workloads (CPU): the non-repeating latency stream, the batch packing
and the cost-balanced sharding the multi-GPU bench uses."""
import math

import numpy as np

from sys1rust_b200.dist import shard_for_rank
from sys1rust_b200.workloads import (cfg5_requests, encoder_flops, latency_stream, pack_batches, request_cost,
                                     shard_lpt)


def test_latency_stream_never_repeats_a_shape():
    reqs = latency_stream(200)
    shapes = [(len(r.ids), len(r.markers)) for r in reqs]
    assert len(shapes) == 200 and len(set(shapes)) == 200
    assert all(64 <= L <= 200 for L, _ in shapes)
    assert all(1 <= k <= 12 for _, k in shapes)  # 1-3 questions of 2-4 options
    assert latency_stream(200)[7].ids == reqs[7].ids  # seeded


def test_request_cost_is_one_row_of_encoder_flops():
    for L in (1, 32, 64, 65, 129, 700):
        assert math.isclose(request_cost(L), encoder_flops([L]), rel_tol=1e-12)


def test_packing_reaches_the_fewest_batches():
    reqs = cfg5_requests(n=1024, seed=1)
    batches = pack_batches(reqs, 16384)
    total = sum(len(r.ids) for r in reqs)
    assert len(batches) == math.ceil(total / 16384)
    assert all(b.total <= 16384 for b in batches)
    # every request exactly once, rows of a batch in arrival order
    seen = sorted(tuple(b.ids[b.cu_seqlens[i]: b.cu_seqlens[i + 1]]) for b in batches for i in range(b.n))
    assert seen == sorted(tuple(r.ids) for r in reqs)
    # a request longer than the limit runs alone
    big = cfg5_requests(n=3, seed=5)
    out = pack_batches(big, 10)
    assert len(out) == 3 and all(b.n == 1 for b in out)


def test_shards_balance_cost_and_batch_counts():
    for world in (2, 4, 8):
        reqs = cfg5_requests(n=1024 * world, seed=1)
        shards = [shard_for_rank(reqs, world, r) for r in range(world)]
        assert sorted(id(x) for s in shards for x in s) == sorted(id(x) for x in reqs)
        cost = [sum(request_cost(len(x.ids)) for x in s) for s in shards]
        assert max(cost) / min(cost) < 1.001
        assert len({len(pack_batches(s, 16384)) for s in shards}) == 1
    # the LPT order is by cost, which is increasing in length
    assert np.all(np.diff([request_cost(L) for L in range(1, 300)]) > 0)
    assert len(shard_lpt(cfg5_requests(n=10, seed=2), 3)) == 3
