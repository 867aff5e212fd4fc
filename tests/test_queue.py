"""The batching request queue (kk_queue) with a host executor: batch
formation, per-request ordering, limits, cancellation and error results,
from several submitting threads. No GPU: the executor is a Python function
called from the queue's worker threads."""
import threading
import time
from types import SimpleNamespace

import numpy as np
import pytest

import kokopop_b200 as kb


def _chunk(request, index, T):
    """A chunk whose style carries (request, index) and whose asr frames
    carry their position, so an executor can tell what it ran."""
    asr = np.zeros((T, 512), np.float32)
    asr[:, 0] = np.arange(T, dtype=np.float32) + 1000.0 * index
    style = np.zeros(128, np.float32)
    style[0], style[1] = request, index
    return SimpleNamespace(T=T, asr=asr, f0=np.full(2 * T, 100.0, np.float32), noise=np.zeros(2 * T, np.float32),
                           style=style)


class Recorder:
    """Executor: audio sample 600 t + k of a chunk = its asr[t, 0] + k / 1000;
    records the (request, index) pairs of each batch."""

    def __init__(self, fail_request=None, gate=None):
        self.batches = []
        self.lock = threading.Lock()
        self.fail_request = fail_request
        self.gate = gate

    def __call__(self, T, asr, f0, noise, style, audio):
        if self.gate is not None:
            self.gate.wait(10)
        pairs = [(int(style[128 * i]), int(style[128 * i + 1])) for i in range(len(T))]
        with self.lock:
            self.batches.append(pairs)
        if self.fail_request is not None and any(r == self.fail_request for r, _ in pairs):
            return 5
        off = 0
        for t in T:
            a = asr[off * 512:(off + t) * 512].reshape(t, 512)[:, 0]
            audio[600 * off:600 * (off + t)] = (a[:, None] + np.arange(600, dtype=np.float32)[None] / 1000.0).ravel()
            off += t
        return 0


def _expected(c):
    return (c.asr[:, 0][:, None] + np.arange(600, dtype=np.float32)[None] / 1000.0).ravel()


def test_results_reach_their_chunks():
    rec = Recorder()
    q = kb.Queue(executor=rec, n_workers=2, max_batch=8, max_batch_frames=4000, max_wait_us=5000)
    try:
        chunks = [_chunk(r, 0, 7 + 3 * r) for r in range(20)]
        tickets = [q.submit(r, c) for r, c in enumerate(chunks)]
        for t, c in zip(tickets, chunks):
            rc, audio = q.wait(t, 10000)
            assert rc == 0
            np.testing.assert_array_equal(audio, _expected(c))
        st = q.stats()
        assert st["jobs"] == 20 and st["max_batch"] <= 8 and st["batches"] >= 3
    finally:
        q.close()


def test_chunks_of_a_request_run_in_order_one_at_a_time():
    rec = Recorder()
    q = kb.Queue(executor=rec, n_workers=3, max_batch=16, max_batch_frames=10000, max_wait_us=1000)
    try:
        tickets = []
        for i in range(6):
            for r in range(5):
                tickets.append(q.submit(r, _chunk(r, i, 10)))
        assert all(q.wait(t, 10000)[0] == 0 for t in tickets)
    finally:
        q.close()
    last = {}
    for b in rec.batches:
        reqs = [r for r, _ in b]
        assert len(reqs) == len(set(reqs)), "two chunks of one request in one batch"
        for r, i in b:
            assert i == last.get(r, -1) + 1, "chunk out of order"
            last[r] = i
    assert all(last[r] == 5 for r in range(5))


def test_batch_limits():
    rec = Recorder(gate=threading.Event())
    q = kb.Queue(executor=rec, n_workers=1, max_batch=3, max_batch_frames=250, max_wait_us=0)
    try:
        tickets = [q.submit(r, _chunk(r, 0, 100)) for r in range(7)]
        rec.gate.set()
        assert all(q.wait(t, 10000)[0] == 0 for t in tickets)
    finally:
        q.close()
    assert all(len(b) <= 2 for b in rec.batches)  # 250 frames: two chunks of 100
    with pytest.raises(kb.KKError):
        kb.Queue(executor=rec, max_batch=0)


def test_cancel_and_errors():
    gate = threading.Event()
    rec = Recorder(fail_request=9, gate=gate)
    q = kb.Queue(executor=rec, n_workers=1, max_batch=1, max_batch_frames=1000, max_wait_us=0)
    try:
        first = q.submit(1, _chunk(1, 0, 5))  # holds the worker at the gate
        time.sleep(0.2)
        queued = [q.submit(2, _chunk(2, i, 5)) for i in range(3)]
        bad = q.submit(9, _chunk(9, 0, 5))
        assert q.cancel(2) == 3
        gate.set()
        assert q.wait(first, 10000)[0] == 0
        assert all(q.wait(t, 10000)[0] == kb.QUEUE_CANCELLED for t in queued)
        assert q.wait(bad, 10000)[0] == 5
        with pytest.raises(kb.KKError):
            q.wait(first, 0)  # already returned
    finally:
        q.close()


def test_many_submitting_threads():
    rec = Recorder()
    q = kb.Queue(executor=rec, n_workers=2, max_batch=32, max_batch_frames=100000, max_wait_us=2000)
    errors = []

    def client(k):
        try:
            cs = [_chunk(100 + k, i, 4 + (i % 5)) for i in range(15)]
            ts = [q.submit(100 + k, c) for c in cs]
            for t, c in zip(ts, cs):
                rc, audio = q.wait(t, 20000)
                assert rc == 0
                np.testing.assert_array_equal(audio, _expected(c))
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=client, args=(k,)) for k in range(6)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(60)
    q.close()
    assert not errors
    assert q.h.value is None
