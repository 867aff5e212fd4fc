"""A streaming session over a GPU queue: each chunk's decoder audio comes
from the queue's batched forwards, then the session post-processes and
crossfades it. The result equals, bit for bit, the reference's
postprocess_and_crossfade (oracle/_ref's compiled audio_postprocess.cpp, or
the library's own bit-exact restatement where _ref is absent) applied to
the same chunks decoded one by one with kk_decoder_forward: batching changes
no bit of a chunk (tests/test_gpu_decoder.py), and the post-processing is
host arithmetic."""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _expected(raws, bounds, cfg):
    if O.ref_available():
        return O.ref_stream(raws, bounds, cfg)
    out, tail = [], np.zeros(0, np.float32)
    ncf = cfg.crossfade_ms * cfg.sample_rate // 1000
    for i, (r, b) in enumerate(zip(raws, bounds)):
        p = kb.postprocess_chunk(cfg, r, b, i == 0, i == len(raws) - 1)
        if len(tail) and len(p):
            p = kb.crossfade(cfg, tail, p, b)
        tail = p[max(0, len(p) - ncf):] if len(p) and ncf else np.zeros(0, np.float32)
        out.append(p)
    return out


@pytest.mark.parametrize("mode", [0, 1])
def test_stream_over_gpu_queue_equals_reference_postprocessing(mode):
    w = W.config2_weights()
    c = kb.Context(0)
    c.upload(w)
    rng = np.random.default_rng(40 + mode)
    chunks = [W.make_utterance(rng, t) for t in (37, 8, 90, 21, 3)]
    bounds = [kb.BOUNDARY_CLAUSE_WEAK, kb.BOUNDARY_NONE, kb.BOUNDARY_SENTENCE, kb.BOUNDARY_CLAUSE_STRONG,
              kb.BOUNDARY_NONE]
    raws = [c.decoder_forward([u])[0] for u in chunks]
    cfg = kb.StreamConfig.preset(mode)
    want = _expected(raws, bounds, cfg)
    q = kb.Queue(contexts=[c], max_batch=8, max_batch_frames=4000, max_wait_us=1000)
    try:
        s = kb.Stream(q, cfg)
        for i, (u, b) in enumerate(zip(chunks, bounds)):
            s.push(u, b, i == len(chunks) - 1)
        got = []
        while True:
            rc, samples, idx = s.next(30000)
            if rc == kb.STREAM_END:
                break
            assert rc == kb.KK_OK
            got.append((idx, samples))
        s.close()
    finally:
        q.close()
        c.close()
    assert [g[0] for g in got] == list(range(len(chunks)))
    for (_, g), w_ in zip(got, want):
        np.testing.assert_array_equal(g, w_)


def test_two_sessions_interleave_on_one_gpu_queue():
    """Two sessions whose chunks share batches: each gets its own chunks,
    in order, bit-exact."""
    w = W.config2_weights()
    c = kb.Context(0)
    c.upload(w)
    rng = np.random.default_rng(50)
    reqs = [[W.make_utterance(rng, t) for t in lens] for lens in ((12, 40, 7), (30, 5, 18, 9))]
    cfg = kb.StreamConfig.preset(0)
    wants = []
    for chunks in reqs:
        raws = [c.decoder_forward([u])[0] for u in chunks]
        wants.append(_expected(raws, [kb.BOUNDARY_CLAUSE_WEAK] * len(chunks), cfg))
    q = kb.Queue(contexts=[c], max_batch=8, max_batch_frames=4000, max_wait_us=3000)
    try:
        ss = [kb.Stream(q, cfg) for _ in reqs]
        for s, chunks in zip(ss, reqs):
            for i, u in enumerate(chunks):
                s.push(u, kb.BOUNDARY_CLAUSE_WEAK, i == len(chunks) - 1)
        for s, want in zip(ss, wants):
            for k, w_ in enumerate(want):
                rc, samples, idx = s.next(30000)
                assert rc == kb.KK_OK and idx == k
                np.testing.assert_array_equal(samples, w_)
            assert s.next(0)[0] == kb.STREAM_END
            s.close()
        assert q.stats()["batches"] < 7
    finally:
        q.close()
        c.close()
