"""One serving queue over handles on two GPUs (sys1rust's worker contract,
``runtime/crates/sys1rust/src/worker.rs:103-223``, with the batcher feeding several GPUs): requests
from several clients are served by workers on both devices, and every result equals the request's
own forward (to the rounding of differently grouped GEMM sums) and the CPU oracle on a sample.
Needs two GPUs; skipped on a one-GPU box."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_one_queue_serves_two_gpus(cuda_lib):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from sys1rust_b200.backend import CudaBackend
    from sys1rust_b200.batch import Varlen, collate_to
    from sys1rust_b200.config import small_model
    from sys1rust_b200.server import Server
    from sys1rust_b200.weights import SyntheticWeights
    from sys1rust_b200.workloads import _row
    from oracle.forward_ref import OracleModel

    cfg = small_model()
    w = SyntheticWeights(cfg, seed=23)
    bes = [CudaBackend.from_synthetic(cfg, w.tensors, device=dev) for dev in (0, 1, 0, 1)]
    rng = np.random.default_rng(9)
    items = [_row(rng, cfg.encoder.vocab_size, int(rng.integers(8, 400)), [int(rng.integers(0, 3))])
             for _ in range(96)]
    ref = CudaBackend.from_synthetic(cfg, w.tensors, device=0)
    alone = [ref.forward_varlen(Varlen.from_rows([it])) for it in items]
    d = cfg.encoder.hidden_size
    with Server(bes, max_concurrent=256, max_batch_tokens=1024) as srv:
        # the whole load queued at once (about 20 batches for 4 workers), then a second wave from
        # client threads while the first is still being served
        tickets = [srv.submit(it) for it in items]
        results = [srv.wait(t, len(it.markers)) for t, it in zip(tickets, items)]
        again = [None] * len(items)

        def client(lo, hi):
            for i in range(lo, hi):
                again[i] = srv.predict(items[i])

        ts = [threading.Thread(target=client, args=(k * 12, k * 12 + 12)) for k in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        st = srv.stats()
    assert st["rows"] == 2 * len(items) and st["failed_batches"] == 0 and st["workers_alive"] == 4
    # a handle's launch count is that of its last forward: a handle that ran no batch has 0
    assert any(b.last_launch_count() > 0 for b in bes[0::2]) and any(b.last_launch_count() > 0 for b in bes[1::2])
    for a, b in zip(results, again):
        assert np.abs(a[0] - b[0]).max() < 2e-3
    for it, a, (lg, pl, _) in zip(items, alone, results):
        k = len(it.markers)
        assert np.abs(lg - a.logits[:k]).max() < 2e-3
        assert np.linalg.norm(pl - a.pooled[:d]) / np.linalg.norm(a.pooled[:d]) < 1e-2
    om = OracleModel(cfg, w.tensors)
    for i in range(0, len(items), 16):
        lo, po, _ = om.forward(collate_to([items[i]], cfg.encoder.pad_token_id))
        lg, pl, _ = results[i]
        assert np.abs(lg - lo[: len(items[i].markers)]).max() < 5e-2
        assert np.linalg.norm(pl - po) / np.linalg.norm(po) < 5e-2
    for b in bes + [ref]:
        b.close()
