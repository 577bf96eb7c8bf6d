"""The native serving queue (``s1c_server_*``) on CPU, with a Python forward in place of the GPU:
cross-request packing within the token and row limits in arrival order, results routed to their
tickets, the reference's non-blocking admission (busy at the cap, worker.rs / http.rs:168-181),
cancelled requests dropped unrun (worker.rs:202-205), a failed forward failing only its batch,
several workers sharing the queue, and stop failing what is still queued.
"""
import threading
import time

import numpy as np
import pytest

from sys1rust_b200.backend import BackendError, S1C_ERR_ARG
from sys1rust_b200.batch import EncodedItem
from sys1rust_b200.server import Server, ServerBusy, WaitTimeout, WorkerNotRunning

HIDDEN = 8


def _item(i, L, n_markers=2, qtype=0):
    rng = np.random.default_rng(i)
    ids = rng.integers(4, 1000, size=L).tolist()
    markers = sorted(rng.choice(np.arange(1, L), size=min(n_markers, L - 1), replace=False).tolist()) if L > 1 else []
    return EncodedItem(ids, markers, qtype)


def _expect(item):
    s = float(sum(item.ids) % 997)
    return (np.array([s + m for m in item.markers], np.float32),
            np.array([len(item.ids) + 0.5 * j for j in range(HIDDEN)], np.float32))


class Fake:
    """Deterministic forward; records every batch; the first call can be held on a gate."""

    def __init__(self, hold_first=False, fail_if=None):
        self.batches = []
        self.gate = threading.Event()
        if not hold_first:
            self.gate.set()
        self.fail_if = fail_if
        self.lock = threading.Lock()

    def __call__(self, worker, n, kmax, ids, cu, mp, mc, qt):
        self.gate.wait(10)
        rows = [ids[cu[r]:cu[r + 1]].tolist() for r in range(n)]
        with self.lock:
            self.batches.append({"worker": worker, "rows": rows, "tokens": int(cu[-1]), "kmax": kmax})
        if self.fail_if and any(self.fail_if(r) for r in rows):
            raise RuntimeError("planted failure")
        km = max(kmax, 1)
        logits = np.full((n, km), -1e4, np.float32)
        for r in range(n):
            s = float(sum(rows[r]) % 997)
            for k in range(mc[r]):
                logits[r, k] = s + float(mp[r, k])
        pooled = np.array([[len(rows[r]) + 0.5 * j for j in range(HIDDEN)] for r in range(n)], np.float32)
        return logits, pooled


def _wait_queued(srv, n, timeout=5.0):
    """Until all n submitted requests are either queued or taken into a batch."""
    t0 = time.time()
    while time.time() - t0 < timeout:
        st = srv.stats()
        if st["queued"] + st["rows"] >= n:
            return
        time.sleep(0.005)


def test_requests_are_packed_in_arrival_order_within_limits():
    fake = Fake(hold_first=True)
    with Server(forward=fake, hidden=HIDDEN, max_concurrent=64, max_batch_tokens=300, max_batch_rows=4) as srv:
        items = [_item(i, L) for i, L in enumerate([50, 90, 120, 40, 30, 200, 10, 10, 10, 10, 10, 500, 60])]
        tickets = [srv.submit(it) for it in items]
        _wait_queued(srv, len(items))
        fake.gate.set()
        for it, t in zip(items, tickets):
            lg, pl, ms = srv.wait(t, len(it.markers))
            el, ep = _expect(it)
            assert np.array_equal(lg, el) and np.array_equal(pl, ep)
            assert ms >= 0
        st = srv.stats()
    order = [tuple(r) for b in fake.batches for r in b["rows"]]
    assert order == [tuple(it.ids) for it in items]  # every request once, arrival order
    for b in fake.batches:
        assert len(b["rows"]) <= 4
        assert b["tokens"] <= 300 or len(b["rows"]) == 1  # the 500-token request runs alone
        assert b["kmax"] == 2  # every test row has 2 markers
    # the held-back queue was packed: fewer batches than requests, each as full as the limits allow
    assert len(fake.batches) < len(items)
    for b, nxt in zip(fake.batches[1:], fake.batches[2:]):
        assert len(b["rows"]) == 4 or b["tokens"] + len(nxt["rows"][0]) > 300
    assert st["rows"] == len(items) and st["in_flight"] == 0


def test_admission_refuses_at_the_cap_without_queueing():
    fake = Fake(hold_first=True)
    with Server(forward=fake, hidden=HIDDEN, max_concurrent=3) as srv:
        items = [_item(i, 20) for i in range(4)]
        t = [srv.submit(it) for it in items[:3]]
        with pytest.raises(ServerBusy, match="server busy, try again later") as e:
            srv.submit(items[3])
        assert e.value.retry_after == 1
        assert srv.stats()["busy_rejections"] == 1
        fake.gate.set()
        srv.wait(t[0], 2)  # collecting a result frees a permit
        t.append(srv.submit(items[3]))
        for tk, it in zip(t[1:], items[1:]):
            assert np.array_equal(srv.wait(tk, 2)[0], _expect(it)[0])


def test_cancelled_requests_are_dropped_unrun():
    fake = Fake(hold_first=True)
    # one request per batch: while the first is held in the forward, the others stay queued
    with Server(forward=fake, hidden=HIDDEN, max_concurrent=8, max_batch_rows=1) as srv:
        items = [_item(i, 30) for i in range(5)]
        t = [srv.submit(it) for it in items]
        _wait_queued(srv, 5)
        srv.cancel(t[2])
        srv.cancel(t[3])
        fake.gate.set()
        for k in (0, 1, 4):
            srv.wait(t[k], 2)
        with pytest.raises(BackendError, match="unknown ticket"):
            srv.wait(t[2], 2)
        st = srv.stats()
    ran = {tuple(r) for b in fake.batches for r in b["rows"]}
    assert tuple(items[2].ids) not in ran and tuple(items[3].ids) not in ran
    assert st["cancelled_skipped"] == 2


def test_a_failed_forward_fails_only_its_batch():
    bad = _item(99, 25)
    fake = Fake(hold_first=True, fail_if=lambda row: row == bad.ids)
    with Server(forward=fake, hidden=HIDDEN, max_concurrent=8, max_batch_rows=2) as srv:
        items = [_item(0, 25), _item(1, 25), bad, _item(3, 25), _item(4, 25)]
        t = [srv.submit(it) for it in items]
        _wait_queued(srv, 5)
        fake.gate.set()
        failed = set()
        for tk, it in zip(t, items):
            try:
                srv.wait(tk, 2)
            except BackendError as e:
                assert "planted failure" in str(e)
                failed.add(tuple(it.ids))
        assert srv.stats()["failed_batches"] == 1
        # the server keeps serving after the failure
        after = _item(5, 25)
        assert np.array_equal(srv.predict(after)[0], _expect(after)[0])
    bad_batch = next(b for b in fake.batches if bad.ids in b["rows"])
    assert failed == {tuple(r) for r in bad_batch["rows"]}


def test_workers_share_the_queue():
    gate_all = threading.Event()

    class Slow(Fake):
        def __call__(self, *a):
            gate_all.wait(10)
            return super().__call__(*a)

    fake = Slow()
    with Server(forward=fake, n_workers=3, hidden=HIDDEN, max_concurrent=32, max_batch_rows=1) as srv:
        items = [_item(i, 15) for i in range(9)]
        t = [srv.submit(it) for it in items]
        time.sleep(0.2)  # every worker has taken a request and blocks in the forward
        gate_all.set()
        for tk, it in zip(t, items):
            assert np.array_equal(srv.wait(tk, 2)[1], _expect(it)[1])
        assert srv.stats()["workers_alive"] == 3
    assert len({b["worker"] for b in fake.batches}) == 3


def test_wait_timeout_keeps_the_ticket_and_stop_fails_the_queue():
    fake = Fake(hold_first=True)
    srv = Server(forward=fake, hidden=HIDDEN, max_concurrent=8, max_batch_rows=1)
    items = [_item(i, 12) for i in range(3)]
    t = [srv.submit(it) for it in items]
    _wait_queued(srv, 3)
    with pytest.raises(WaitTimeout):
        srv.wait(t[0], 2, timeout_ms=50)
    threading.Timer(0.2, fake.gate.set).start()
    srv.stop()  # the running batch finishes; the two queued requests fail
    assert np.array_equal(srv.wait(t[0], 2)[0], _expect(items[0])[0])
    for tk in t[1:]:
        with pytest.raises(WorkerNotRunning, match="inference worker is not running"):
            srv.wait(tk, 2)
    with pytest.raises(WorkerNotRunning):
        srv.submit(items[0])
    srv.close()


def test_malformed_rows_are_refused_at_submit():
    with Server(forward=Fake(), hidden=HIDDEN) as srv:
        with pytest.raises(BackendError) as e:
            srv.submit(EncodedItem([], [], 0))
        assert e.value.code == S1C_ERR_ARG
        with pytest.raises(BackendError, match="marker position 9 outside a row of 5 tokens"):
            srv.submit(EncodedItem([5, 6, 7, 8, 9], [9], 2))
        assert srv.stats()["in_flight"] == 0


def test_repeated_waves_stream_through_without_draining():
    """Three waves of the same requests queued back to back (the serving benchmark's stream): two
    workers pack across wave boundaries, and every ticket gets its own request's result even though
    the waves repeat the same contents."""
    fake = Fake()
    items = [_item(i, 5 + (7 * i) % 40, n_markers=1 + i % 3) for i in range(40)]
    waves = 3
    with Server(forward=fake, n_workers=2, hidden=HIDDEN, max_concurrent=waves * len(items) + 1,
                max_batch_tokens=200) as srv:
        tickets = [srv.submit(it) for _ in range(waves) for it in items]
        assert len(set(tickets)) == len(tickets)
        for i, tk in enumerate(tickets):
            it = items[i % len(items)]
            logits, pooled, _ = srv.wait(tk, len(it.markers))
            want_l, want_p = _expect(it)
            assert np.array_equal(logits, want_l) and np.array_equal(pooled, want_p)
        st = srv.stats()
        assert st["rows"] == waves * len(items) and st["failed_batches"] == 0
    # batches stayed within the token limit and every queued request ran exactly once
    assert all(b["tokens"] <= 200 or len(b["rows"]) == 1 for b in fake.batches)
    assert sum(len(b["rows"]) for b in fake.batches) == waves * len(items)
