"""The device entry points composed as the reference's Kokoro pipeline runs
them for one chunk (kokoro.cpp:199-541, :669-763): token ids -> ALBERT +
bert_encoder -> duration encoder -> duration head -> (config 2's seeded
U[2, 10] duration override) -> alignment -> prosody F0 / N and the text
encoder's t_en -> decoder -> audio. Each stage's parity is tested on its
own; this checks that the layouts hand over (shapes, alignment, finite and
clamped audio) and that the text-encoder path equals the oracle's alignment."""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_front_end_to_audio():
    weights = {}
    weights.update(W.config2_frontend_weights())
    weights.update(W.prosody_weights(f16=True))
    weights.update(W.config2_weights())
    rng = np.random.default_rng(51)
    ids = W.token_ids(rng, 40)
    n = len(ids)
    style_p = rng.normal(0, 0.1, 128).astype(np.float32)
    style_d = rng.normal(0, 0.1, 128).astype(np.float32)
    c = kb.Context(0)
    try:
        c.upload(weights)
        bert = c.albert([ids])[0]
        d = c.duration_encoder([bert], [style_p])[0]
        dur = c.duration_head([d])[0]
        assert bert.shape == (n, 512) and d.shape == (n, 640) and dur.shape == (n,)
        assert np.all(np.isfinite(dur)) and np.all(dur > 0)
        dur = rng.integers(2, 11, size=n).astype(np.float32)  # the config's override
        frames, total, en = c.align_durations(dur, 1.0, d)
        np.testing.assert_array_equal(frames, dur.astype(np.int32))
        t_en = c.text_encoder([ids])[0]
        _, _, asr_fm = c.align_durations(dur, 1.0, t_en)
        want_fm = O.align_durations(dur, 1.0, t_en)[2]
        np.testing.assert_array_equal(asr_fm, want_fm)
        (f0, nn), = c.prosody_f0n([en], [style_p])
        assert f0.shape == (2 * total,) and nn.shape == (2 * total,)
        u = W.Utterance(T=int(total), asr=np.ascontiguousarray(asr_fm.T), f0=f0, noise=nn, style=style_d)
        audio = c.decoder_forward([u])[0]
        assert audio.shape == (600 * total,)
        assert np.all(np.isfinite(audio)) and np.abs(audio).max() <= 1.0
    finally:
        c.close()
