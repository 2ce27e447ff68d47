"""Serve-path batching (host logic, CPU): concurrent predict() calls share batches, every caller gets
its own row, batches are padded to the fixed graph sizes, failures reach every caller of a batch."""

import concurrent.futures as cf
import threading
import time

import numpy as np
import pytest

from foidfinder_b200.serving import BatchingBackend, batch_sizes


def _fake(delay=0.01, fail=False):
    seen = []

    def run(imgs):
        seen.append(imgs.shape[0])
        time.sleep(delay)
        if fail:
            raise RuntimeError("device lost")
        return imgs.reshape(imgs.shape[0], -1)[:, :4].astype(np.float32) / 255.0

    return run, seen


def _prep(v):
    return np.full((8, 8, 3), v, np.uint8)


def test_batch_sizes():
    assert batch_sizes(1) == [1]
    assert batch_sizes(32) == [1, 2, 4, 8, 16, 32]
    assert batch_sizes(24) == [1, 2, 4, 8, 16, 24]


def test_single_request():
    run, seen = _fake()
    b = BatchingBackend(run, _prep, max_batch=8)
    try:
        out = b.predict(7)
        assert np.allclose(out, 7 / 255.0) and out.shape == (4,)
        assert seen == [1] and b.batches == [1]
    finally:
        b.close()


def test_concurrent_requests_share_batches():
    run, seen = _fake(delay=0.02)
    b = BatchingBackend(run, _prep, max_batch=16, max_wait_ms=5.0)
    try:
        with cf.ThreadPoolExecutor(32) as ex:
            vals = list(range(40))
            outs = list(ex.map(b.predict, vals))
        for v, o in zip(vals, outs):
            assert np.allclose(o, v / 255.0)
        assert sum(b.batches) == 40
        assert len(b.batches) < 40  # requests were coalesced
        assert all(s in batch_sizes(16) for s in seen)  # padded to graph sizes
        assert max(b.batches) <= 16
    finally:
        b.close()


def test_failure_reaches_every_caller():
    run, _ = _fake(fail=True)
    b = BatchingBackend(run, _prep, max_batch=4, max_wait_ms=20.0)
    try:
        futs = [b.submit(i) for i in range(3)]
        for f in futs:
            with pytest.raises(RuntimeError, match="device lost"):
                f.result(timeout=10)
    finally:
        b.close()


def test_close_stops_worker_and_rejects():
    run, _ = _fake()
    b = BatchingBackend(run, _prep)
    b.close()
    assert not b._worker.is_alive()
    with pytest.raises(RuntimeError):
        b.predict(1)
