"""GPU parity of the prosody predictor's F0 / N chain (kokoro.cpp:669-708:
the biLSTM kokopop.predictor.shared, three AdainResBlk1d per branch and the
1x1 projections) against the oracle, through the C ABI. Tolerances, max-abs
on the f0 / n curves (magnitude ~0.05 with these weights): 1e-4 with F32
weights; 1e-3 with F16 weights, whose half-rounded operands can land on the
other side of a rounding step than the oracle's."""
import numpy as np
import pytest

from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-4
TOL_F16 = 1e-3


@pytest.fixture(scope="module")
def wp32():
    return W.prosody_weights(f16=False)


@pytest.fixture(scope="module")
def wp16():
    return W.prosody_weights(f16=True)


def _inputs(rng, T):
    return (rng.normal(0.0, 1.0, size=(T, 640)).astype(np.float32),
            rng.normal(0.0, 0.1, size=128).astype(np.float32))


def _check(got, want, tol):
    assert got.shape == want.shape
    assert np.all(np.isfinite(got))
    err = float(np.abs(got - want).max())
    assert err < tol, f"max abs err {err}"


@pytest.mark.parametrize("T", [1, 7, 64])
def test_prosody_f32_matches_oracle(ctx, wp32, T):
    ctx.upload(wp32)
    o = O.OracleModel(wp32)
    en, st = _inputs(np.random.default_rng(300 + T), T)
    (f0, n), = ctx.prosody_f0n([en], [st])
    wf0, wn = o.prosody_f0n(en, st)
    _check(f0, wf0, TOL_F32)
    _check(n, wn, TOL_F32)


def test_prosody_f16_matches_oracle(ctx, wp16):
    ctx.upload(wp16)
    o = O.OracleModel(wp16)
    en, st = _inputs(np.random.default_rng(400), 45)
    (f0, n), = ctx.prosody_f0n([en], [st])
    wf0, wn = o.prosody_f0n(en, st)
    _check(f0, wf0, TOL_F16)
    _check(n, wn, TOL_F16)


def test_prosody_ragged_batch_equals_single_calls(ctx, wp16):
    """Packing utterances into one batch changes nothing, bit for bit."""
    ctx.upload(wp16)
    rng = np.random.default_rng(401)
    items = [_inputs(rng, T) for T in (5, 1, 33, 12)]
    batch = ctx.prosody_f0n([e for e, _ in items], [s for _, s in items])
    for (e, s), (bf0, bn) in zip(items, batch):
        (f0, n), = ctx.prosody_f0n([e], [s])
        np.testing.assert_array_equal(f0, bf0)
        np.testing.assert_array_equal(n, bn)


def test_prosody_needs_its_weights(ctx):
    """A weight set without the predictor reports a model error."""
    ctx.upload(W.config1_weights())
    en, st = _inputs(np.random.default_rng(402), 4)
    with pytest.raises(RuntimeError, match="prosody weights incomplete"):
        ctx.prosody_f0n([en], [st])
