"""The batching request queue over a real context: chunks submitted from
several threads, batched by the queue, give the same audio bit for bit as
direct single-utterance calls (the decoder's output does not depend on the
batch a chunk runs in)."""
import threading

import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W

pytestmark = pytest.mark.gpu


def test_queue_over_a_context_matches_direct_calls():
    c = kb.Context(0)
    try:
        c.upload(W.config2_weights())
        rng = np.random.default_rng(41)
        utts = [W.make_utterance(rng, t) for t in (30, 5, 77, 12, 41, 8, 64, 3, 19, 50)]
        want = [c.decoder_forward([u])[0] for u in utts]
        q = kb.Queue(contexts=[c], max_batch=4, max_batch_frames=160, max_wait_us=3000)
        got = [None] * len(utts)
        errors = []

        def client(k):
            try:
                idx = list(range(k, len(utts), 2))
                tickets = [(i, q.submit(i % 3, utts[i])) for i in idx]
                for i, t in tickets:
                    rc, audio = q.wait(t, 60000)
                    assert rc == 0
                    got[i] = audio
            except Exception as e:  # reported below
                errors.append(e)

        threads = [threading.Thread(target=client, args=(k,)) for k in range(2)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(120)
        st = q.stats()
        q.close()
        assert not errors
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w)
        assert st["jobs"] == len(utts) and st["max_batch"] <= 4
    finally:
        c.close()
