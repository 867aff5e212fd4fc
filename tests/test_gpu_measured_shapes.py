"""GPU parity at the shapes the benchmark measures, through the C ABI,
against the oracle on the same seeded inputs.

* The batched decoder workload (256 utterances, T ~ U[40, 800] asr frames,
  F16 weights seed 2, batch 64 per GPU): the pool's longest utterance
  (T close to 800: 480 000 samples, a 96 000-row stage-1 instance norm, the
  phase recurrence over 1 600 segments) against the oracle at the waveform
  bar of 1e-3 max-abs; and the full batch of 64 that holds it, whose
  outputs must equal single-utterance calls bit for bit for 8 of its
  utterances (the longest and shortest included).
* The LSTM stack (input 640, hidden 256, 3 layers, seed 1 U(-1/16, 1/16)) at
  its benchmarked lengths: one layer over L = 512 at B = 1, and the
  duration encoder at L = 512 (B = 4) and L = 64 (B = 32), with F32 and F16
  weights, under the tolerances of tests/test_gpu_lstm.py (5e-6 per layer;
  1e-4 for the encoder with F32 weights; 3e-3 max / 1e-4 mean with F16
  weights, where every layer input is rounded to half).
"""
import numpy as np
import pytest

from kokopop_b200 import shard
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

AUDIO_TOL = 1e-3
TOL_LAYER = 5e-6
TOL_ENCODER = 1e-4
TOL_ENCODER_F16 = 3e-3
TOL_ENCODER_F16_MEAN = 1e-4
PFX = "kokopop.predictor.text_encoder.lstms.0"


@pytest.fixture(scope="module")
def pool():
    return W.config3_utterances()


@pytest.fixture(scope="module")
def w16():
    return W.config2_weights()


def _longest(pool):
    return int(np.argmax([u.T for u in pool]))


def test_pool_longest_utterance_matches_oracle(ctx, w16, pool):
    i = _longest(pool)
    u = pool[i]
    assert u.T >= 790
    ctx.upload(w16)
    got = ctx.decoder_forward([u])[0]
    want = O.OracleModel(w16).decoder_forward(u.asr, u.f0, u.noise, u.style)
    assert got.shape == want.shape == (600 * u.T,)
    assert np.all(np.isfinite(got))
    err = float(np.abs(got - want).max())
    print(f"pool utterance {i} (T = {u.T}): max abs err vs oracle {err:.3g}")
    assert err < AUDIO_TOL


def test_pool_batch_of_64_equals_single_calls(ctx, w16, pool):
    """The batch of 64 that the benchmark runs with the longest utterance:
    packing changes nothing, bit for bit, for 8 of its utterances."""
    ctx.upload(w16)
    i_long = _longest(pool)
    nb = shard.n_blocks(len(pool), 64)
    idx = shard.block(len(pool), 64, i_long % nb)
    assert i_long in idx
    utts = [pool[i] for i in idx]
    batch = ctx.decoder_forward(utts)
    lens = [u.T for u in utts]
    pick = {int(np.argmax(lens)), int(np.argmin(lens))}
    rng = np.random.default_rng(64)
    while len(pick) < 8:
        pick.add(int(rng.integers(0, 64)))
    for j in sorted(pick):
        single = ctx.decoder_forward([utts[j]])[0]
        assert single.shape == batch[j].shape == (600 * utts[j].T,)
        np.testing.assert_array_equal(single, batch[j], err_msg=f"batch slot {j} (T = {utts[j].T})")


@pytest.fixture(scope="module")
def lstm32():
    import kokopop_b200 as kb
    wts = W.config1_weights(f16=False)
    c = kb.Context(0)
    c.upload(wts)
    yield c, O.OracleModel(wts)
    c.close()


@pytest.fixture(scope="module")
def lstm16():
    import kokopop_b200 as kb
    wts = W.config1_weights(f16=True)
    c = kb.Context(0)
    c.upload(wts)
    yield c, O.OracleModel(wts)
    c.close()


def _inputs(seed, lens, dim):
    rng = np.random.default_rng(seed)
    xs = [rng.normal(0.0, 1.0, size=(n, dim)).astype(np.float32) for n in lens]
    styles = [rng.normal(0.0, 1.0, size=128).astype(np.float32) for _ in lens]
    return xs, styles


def test_bilstm_layer_over_512_steps(lstm32):
    c, m = lstm32
    xs, _ = _inputs(512, [512], 640)
    got = c.bilstm(PFX, xs)[0]
    want = m.bilstm(PFX, xs[0])
    err = float(np.abs(got - want).max())
    print(f"biLSTM layer L = 512: max abs err {err:.3g}")
    assert err < TOL_LAYER


@pytest.mark.parametrize("L,B", [(512, 4), (64, 32)])
def test_duration_encoder_f32_at_benchmark_lengths(lstm32, L, B):
    c, m = lstm32
    xs, styles = _inputs(1000 + L + B, [L] * B, 512)
    got = c.duration_encoder(xs, styles)
    errs = [float(np.abs(g - m.duration_encoder(x, s)).max()) for g, x, s in zip(got, xs, styles)]
    print(f"duration encoder F32 L = {L}, B = {B}: max abs err {max(errs):.3g}")
    assert max(errs) < TOL_ENCODER


@pytest.mark.parametrize("L,B", [(512, 4), (64, 32)])
def test_duration_encoder_f16_at_benchmark_lengths(lstm16, L, B):
    c, m = lstm16
    xs, styles = _inputs(2000 + L + B, [L] * B, 512)
    got = c.duration_encoder(xs, styles)
    errs, means = [], []
    for g, x, s in zip(got, xs, styles):
        d = np.abs(g - m.duration_encoder(x, s))
        errs.append(float(d.max()))
        means.append(float(d.mean()))
    print(f"duration encoder F16 L = {L}, B = {B}: max abs err {max(errs):.3g}, mean {max(means):.3g}")
    assert max(errs) < TOL_ENCODER_F16 and max(means) < TOL_ENCODER_F16_MEAN
