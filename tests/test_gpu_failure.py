"""Device-side failure detection without a GPU fault: every wait in the kernels is bounded by the
globaltimer; when a wait runs out it records a status code, the kernel returns and the context stays
usable. ``s1c_selftest_wait_timeout`` makes both forms of the wait (the single-thread form of the
TMA / MMA roles and the warp form of the epilogue / softmax roles) wait on an mbarrier that nothing
completes, with a short budget."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_and_report(cuda_lib):
    from sys1rust_b200.backend import selftest_wait_timeout
    t = time.perf_counter()
    codes = selftest_wait_timeout(0, 50_000_000)
    dt = time.perf_counter() - t
    assert codes == [1, 4, 0, 0]  # DEV_TIMEOUT_PRODUCER, DEV_TIMEOUT_EPILOGUE, neither wait succeeded
    assert 0.04 < dt < 5.0


def test_context_is_usable_after_a_timeout(cuda_lib):
    from conftest import get_backend
    from sys1rust_b200.backend import selftest_wait_timeout
    from test_gpu_forward import make_rows
    from sys1rust_b200.batch import collate_to
    cfg, w, be = get_backend("small:3")
    batch = collate_to(make_rows(cfg, 51, [30, 70], [2, 3]), cfg.encoder.pad_token_id)
    before = be.forward(batch)
    assert selftest_wait_timeout(0, 20_000_000)[:2] == [1, 4]
    after = be.forward(batch)
    assert np.array_equal(before.logits, after.logits) and np.array_equal(before.pooled, after.pooled)


def test_budget_is_validated(cuda_lib):
    from sys1rust_b200.backend import BackendError, selftest_wait_timeout
    with pytest.raises(BackendError):
        selftest_wait_timeout(0, 10)
