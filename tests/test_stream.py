"""Streaming sessions (kk_stream) and the chunk post-processing they apply,
pinned against the reference's own functions: postprocess_chunk_audio and
apply_crossfade_smart (src/audio/audio_postprocess.cpp), compiled unmodified
into oracle/_ref/, composed as postprocess_and_crossfade composes them
(src/streaming/streaming.cpp:26-60). Bit-exact. No GPU: the sessions run
over a queue whose executor is a Python function."""
import threading
from types import SimpleNamespace

import numpy as np
import pytest

import kokopop_b200 as kb
from oracle import oracle as O

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")

BOUNDARIES = list(range(6))


def _cfgs():
    a, b = kb.StreamConfig.preset(0), kb.StreamConfig.preset(1)
    c = kb.StreamConfig.preset(0)
    c.trim_silence = 0
    d = kb.StreamConfig.preset(1)
    d.crossfade_ms = 0
    e = kb.StreamConfig.preset(0)  # a one-sample crossfade
    e.sample_rate, e.crossfade_ms = 1000, 1
    return [a, b, c, d, e]


def _audio(rng, n, lead, trail, amp=0.3):
    """n samples: `lead` near-silent samples (below the 0.01 threshold), a
    tone, `trail` near-silent samples."""
    body = max(0, n - lead - trail)
    t = np.arange(body, dtype=np.float32)
    tone = (amp * np.sin(0.013 * t) * (0.5 + 0.5 * rng.random(body))).astype(np.float32)
    quiet = lambda k: (0.009 * (rng.random(k) * 2 - 1)).astype(np.float32)
    return np.concatenate([quiet(lead), tone, quiet(trail)])[:n].astype(np.float32)


@needs_ref
def test_postprocess_matches_reference_bit_exact():
    rng = np.random.default_rng(5)
    cases = 0
    for cfg in _cfgs():
        for n, lead, trail in [(0, 0, 0), (1, 0, 0), (37, 10, 10), (600, 0, 0), (600, 600, 0), (24000, 3000, 5000),
                               (24000, 0, 4000), (50000, 20000, 1), (9000, 8999, 0), (30000, 100, 2900)]:
            a = _audio(rng, n, lead, trail)
            for b in BOUNDARIES:
                for first in (False, True):
                    for last in (False, True):
                        got = kb.postprocess_chunk(cfg, a, b, first, last)
                        want = O.ref_postprocess_chunk(a, b, first, last, cfg)
                        np.testing.assert_array_equal(got, want)
                        cases += 1
    assert cases == 5 * 10 * 6 * 4


@needs_ref
def test_crossfade_matches_reference_bit_exact():
    rng = np.random.default_rng(6)
    for cfg in _cfgs():
        n_cf = cfg.crossfade_ms * cfg.sample_rate // 1000
        for np_, nn in [(0, 0), (0, 5), (5, 0), (n_cf, n_cf), (max(n_cf - 1, 0), 3000), (3000, max(n_cf - 1, 0)),
                        (n_cf, 7000), (4000, 9000), (1, 1)]:
            p = rng.normal(0, 0.3, np_).astype(np.float32)
            q = rng.normal(0, 0.3, nn).astype(np.float32)
            for b in BOUNDARIES:
                got = kb.crossfade(cfg, p, q, b)
                want = O.ref_crossfade_smart(p, q, b, cfg.crossfade_ms, cfg.sample_rate)
                np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("mode", [0, 1])
def test_session_matches_golden_reference_outputs(mode):
    """tests/golden/stream_ref.npz: five raw chunks through the reference's
    own post-processing and crossfade (make_golden.py), against a session
    whose executor returns those raw chunks."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "stream_ref.npz"))
    lens = z["lens"].tolist()
    raws = np.split(z["raw"], np.cumsum(lens)[:-1])
    want = np.split(z[f"out_{mode}"], np.cumsum(z[f"out_lens_{mode}"])[:-1])
    by_id = {100 + i: r for i, r in enumerate(raws)}

    def ex(T, asr, f0, noise, style, audio):
        off = 0
        for i, t in enumerate(T):
            audio[600 * off:600 * (off + t)] = by_id[int(style[128 * i])]
            off += int(t)
        return kb.KK_OK

    q = kb.Queue(executor=ex, n_workers=1, max_wait_us=0)
    try:
        s = kb.Stream(q, kb.StreamConfig.preset(mode))
        got = _run(s, [(100 + i, n // 600) for i, n in enumerate(lens)], [int(b) for b in z["bounds"]])
        s.close()
    finally:
        q.close()
    assert len(got) == len(want)
    for (rc, samples, _), w in zip(got, want):
        assert rc == kb.KK_OK
        np.testing.assert_array_equal(samples, w)


# ---------------------------------------------------------------------------
# sessions over a queue with a host executor
# ---------------------------------------------------------------------------

def _raw(cid, T):
    """The raw audio the executor returns for chunk id `cid` of T frames."""
    rng = np.random.default_rng(1000 + cid)
    n = 600 * T
    return _audio(rng, n, (cid * 997) % (n // 3 + 1), (cid * 1499) % (n // 3 + 1), amp=0.2 + 0.05 * (cid % 5))


class RawExecutor:
    """Writes _raw(style[0], T) for each chunk; fails the chunk ids in
    `fail`; waits on `gate` (if given) before each batch."""

    def __init__(self, fail=(), gate=None):
        self.fail = set(fail)
        self.gate = gate
        self.batches = 0
        self.lock = threading.Lock()

    def __call__(self, T, asr, f0, noise, style, audio):
        if self.gate is not None:
            self.gate.wait(10)
        with self.lock:
            self.batches += 1
        off = 0
        for i, t in enumerate(T):
            cid = int(style[128 * i])
            if cid in self.fail:
                return kb.KK_ERROR_INFERENCE
            audio[600 * off:600 * (off + t)] = _raw(cid, int(t))
            off += int(t)
        return kb.KK_OK


def _chunk(cid, T):
    style = np.zeros(128, np.float32)
    style[0] = cid
    return SimpleNamespace(T=T, asr=np.zeros((T, 512), np.float32), f0=np.zeros(2 * T, np.float32),
                           noise=np.zeros(2 * T, np.float32), style=style)


def _run(stream, chunks, bounds):
    for k, ((cid, T), b) in enumerate(zip(chunks, bounds)):
        stream.push(_chunk(cid, T), b, k == len(chunks) - 1)
    got = []
    while True:
        rc, s, idx = stream.next(5000)
        if rc == kb.STREAM_END:
            return got
        got.append((rc, s, idx))


@needs_ref
@pytest.mark.parametrize("mode", [0, 1])
def test_session_equals_reference_pipeline(mode):
    cfg = kb.StreamConfig.preset(mode)
    q = kb.Queue(executor=RawExecutor(), n_workers=2, max_batch=8, max_batch_frames=4000, max_wait_us=500)
    try:
        chunks = [(11, 30), (12, 4), (13, 55), (14, 20), (15, 31), (16, 2)]
        bounds = [kb.BOUNDARY_CLAUSE_WEAK, kb.BOUNDARY_NONE, kb.BOUNDARY_SENTENCE, kb.BOUNDARY_CLAUSE_STRONG,
                  kb.BOUNDARY_PARAGRAPH, kb.BOUNDARY_NEWLINE]
        s = kb.Stream(q, cfg)
        got = _run(s, chunks, bounds)
        s.close()
        want = O.ref_stream([_raw(c, T) for c, T in chunks], bounds, cfg)
        assert [g[2] for g in got] == list(range(len(chunks)))
        for (rc, samples, _), w in zip(got, want):
            assert rc == kb.KK_OK
            np.testing.assert_array_equal(samples, w)
    finally:
        q.close()


@needs_ref
def test_failed_chunk_is_skipped_and_breaks_the_crossfade():
    """streaming.cpp:325-333: a failed chunk hands out nothing and the next
    chunk is not crossfaded onto the tail from before it."""
    cfg = kb.StreamConfig.preset(0)
    q = kb.Queue(executor=RawExecutor(fail={22}), n_workers=1, max_wait_us=0)
    try:
        chunks = [(21, 20), (22, 20), (23, 20), (24, 20)]
        bounds = [kb.BOUNDARY_NONE] * 4
        s = kb.Stream(q, cfg)
        got = _run(s, chunks, bounds)
        s.close()
        assert [g[0] for g in got] == [kb.KK_OK, kb.KK_ERROR_INFERENCE, kb.KK_OK, kb.KK_OK]
        assert got[1][1] is None
        # the reference's pipeline over the chunks that ran, restarted after the failure
        np.testing.assert_array_equal(got[0][1], O.ref_postprocess_chunk(_raw(21, 20), 0, True, False, cfg))
        c23 = O.ref_postprocess_chunk(_raw(23, 20), 0, False, False, cfg)
        np.testing.assert_array_equal(got[2][1], c23)  # no tail to crossfade onto
        ncf = cfg.crossfade_ms * cfg.sample_rate // 1000
        c24 = O.ref_crossfade_smart(c23[-ncf:], O.ref_postprocess_chunk(_raw(24, 20), 0, False, True, cfg), 0,
                                    cfg.crossfade_ms, cfg.sample_rate)
        np.testing.assert_array_equal(got[3][1], c24)
    finally:
        q.close()


def test_cancel_end_and_argument_errors():
    gate = threading.Event()
    q = kb.Queue(executor=RawExecutor(gate=gate), n_workers=1, max_batch=1, max_wait_us=0)
    try:
        s = kb.Stream(q)
        assert s.next(0)[0] == kb.QUEUE_PENDING  # nothing pushed yet
        for k in range(4):
            s.push(_chunk(30 + k, 10), kb.BOUNDARY_NONE, k == 3)
        with pytest.raises(kb.KKError):
            s.push(_chunk(99, 10))  # after the last chunk
        assert s.next(50)[0] == kb.QUEUE_PENDING  # the executor waits on the gate
        s.cancel()
        gate.set()
        got = []
        while True:
            rc, samples, idx = s.next(5000)
            if rc == kb.STREAM_END:
                break
            got.append((rc, idx))
        # the first chunk was dispatched before the cancel; the rest never ran
        assert got[0] == (kb.KK_OK, 0)
        assert [g[0] for g in got[1:]] == [kb.QUEUE_CANCELLED] * 3
        assert s.next(0)[0] == kb.STREAM_END
        s.close()
        # a session destroyed with chunks in flight waits for them
        gate.clear()
        s2 = kb.Stream(q)
        s2.push(_chunk(40, 5))
        threading.Timer(0.2, gate.set).start()
        s2.close()
    finally:
        gate.set()
        q.close()
    L = kb.load_library()
    bad = kb.StreamConfig.preset(0)
    bad.sample_rate = 0
    with pytest.raises(kb.KKError):
        kb.postprocess_chunk(bad, np.zeros(10, np.float32), 0, False, False)
    with pytest.raises(kb.KKError):
        kb.crossfade(kb.StreamConfig.preset(0), np.zeros(3, np.float32), np.zeros(3, np.float32), 9)
    assert L.kk_stream_preset(2, None) == kb.KK_ERROR_INVALID_ARGUMENT


@needs_ref
def test_many_sessions_share_batches_and_keep_their_order():
    """Eight sessions pushing from eight threads onto one queue: every
    session's output equals the reference pipeline over its own chunks,
    and chunks of different sessions share batches."""
    cfg = kb.StreamConfig.preset(0)
    ex = RawExecutor()
    q = kb.Queue(executor=ex, n_workers=2, max_batch=16, max_batch_frames=8000, max_wait_us=3000)
    results, errors = {}, []

    def client(k):
        try:
            rng = np.random.default_rng(k)
            chunks = [(100 * k + i, int(rng.integers(2, 40))) for i in range(6)]
            bounds = [int(b) for b in rng.integers(0, 6, size=6)]
            s = kb.Stream(q, cfg)
            got = _run(s, chunks, bounds)
            s.close()
            results[k] = (got, O.ref_stream([_raw(c, T) for c, T in chunks], bounds, cfg))
        except Exception as e:  # reported below
            errors.append(e)

    try:
        th = [threading.Thread(target=client, args=(k,)) for k in range(8)]
        for t in th:
            t.start()
        for t in th:
            t.join()
    finally:
        q.close()
    assert not errors, errors
    for got, want in results.values():
        assert len(got) == len(want)
        for (rc, samples, _), w in zip(got, want):
            assert rc == kb.KK_OK
            np.testing.assert_array_equal(samples, w)
    assert ex.batches < 48
