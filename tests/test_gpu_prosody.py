"""GPU parity of the prosody predictor's F0 / N chain (kokoro.cpp:669-708:
the biLSTM kokopop.predictor.shared, three AdainResBlk1d per branch and the
1x1 projections) against the oracle, through the C ABI. Tolerances, max-abs
on the f0 / n curves (magnitude ~0.05 with these weights): 1e-6 with F32
weights (measured <= 3e-8); 1e-4 with F16 weights (measured <= 7e-6: the
half-rounded operands meet sums taken in another order than the oracle's)."""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-6
TOL_F16 = 1e-4


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


@pytest.mark.parametrize("f16", [False, True])
def test_prosody_short_call_after_long_call(ctx, wp32, wp16, f16):
    """A call after a longer one reads nothing the longer one left behind
    (the workspaces keep their contents between calls)."""
    w = wp16 if f16 else wp32
    ctx.upload(w)
    o = O.OracleModel(w)
    rng = np.random.default_rng(403)
    for T in (300, 1, 9):
        en, st = _inputs(rng, T)
        (f0, n), = ctx.prosody_f0n([en], [st])
        wf0, wn = o.prosody_f0n(en, st)
        _check(f0, wf0, TOL_F16 if f16 else TOL_F32)
        _check(n, wn, TOL_F16 if f16 else TOL_F32)


def test_prosody_needs_its_weights():
    """A context whose weights lack the predictor reports a model error
    naming the first missing tensor (uploads add to a context's weights, so
    this needs a context of its own)."""
    c = kb.Context(0)
    try:
        c.upload(W.config1_weights())
        en, st = _inputs(np.random.default_rng(402), 4)
        with pytest.raises(RuntimeError, match="prosody weights incomplete"):
            c.prosody_f0n([en], [st])
    finally:
        c.close()
