"""The serving queue on the GPU: requests from many clients packed into shared varlen batches give,
per request, the outputs of that request run alone (to the rounding of differently grouped GEMM
sums, as ``test_rows_agree_alone_or_batched`` bounds it), on one worker and on workers sharing one
GPU; and the queue does pack (fewer forwards than requests).
"""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _items(n, seed, vocab):
    from sys1rust_b200.workloads import _row
    rng = np.random.default_rng(seed)
    return [_row(rng, vocab, int(rng.integers(8, 300)), [int(rng.integers(0, 3))]) for _ in range(n)]


@pytest.mark.parametrize("workers", [1, 2])
def test_served_requests_match_single_forwards(cuda_lib, workers):
    from sys1rust_b200.backend import CudaBackend
    from sys1rust_b200.batch import Varlen
    from sys1rust_b200.config import small_model
    from sys1rust_b200.server import Server
    from sys1rust_b200.weights import SyntheticWeights
    cfg = small_model()
    w = SyntheticWeights(cfg, seed=21)
    bes = [CudaBackend.from_synthetic(cfg, w.tensors) for _ in range(workers)]
    items = _items(40, 5, cfg.encoder.vocab_size)
    alone = [bes[0].forward_varlen(Varlen.from_rows([it])) for it in items]
    d = cfg.encoder.hidden_size
    with Server(bes, max_concurrent=64, max_batch_tokens=2048) as srv:
        results = [None] * len(items)

        def client(lo, hi):
            for i in range(lo, hi):
                results[i] = srv.predict(items[i])

        ts = [threading.Thread(target=client, args=(k * 10, k * 10 + 10)) for k in range(4)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        st = srv.stats()
    assert st["rows"] == len(items) and st["failed_batches"] == 0
    assert st["batches"] < len(items)
    for it, a, (lg, pl, ms) in zip(items, alone, results):
        k = len(it.markers)
        assert np.abs(lg - a.logits[:k]).max() < 2e-3
        assert np.linalg.norm(pl - a.pooled[:d]) / np.linalg.norm(a.pooled[:d]) < 1e-2
    for b in bes:
        b.close()
