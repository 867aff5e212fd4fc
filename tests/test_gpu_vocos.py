"""GPU parity of the sanoTTS Vocos decoder (kk_vocos_forward) against the
oracle, through the C ABI, on seeded weights (seed 3) and inputs at the
stand-in dimensions of kokopop_b200.workload.VOCOS_DIMS.

Tolerances. The inverse FFT, the overlap-add and the DC blocker follow the
reference's operations one by one, and exp / cos / sin are correctly
rounded on both sides; what differs is the accumulation order of the dense
linears (tensor cores against the oracle's ascending sums), for F32
weights the split hi + lo products, and the GELU's erf (CUDA's erff, within
2 ulp, against the oracle's correctly rounded value). Measured differences are far below the
reference's own cross-backend gate for this decoder (RMS error 1e-3,
tests/test_sanotts_backends.cpp:61-100): the waveform is held to 1e-4
max-abs with F32 weights and 1e-3 with F16 weights (every linear's input is
rounded to half, so a last-bit difference can flip a half rounding). Ragged
batches equal single-chunk calls bit for bit.
"""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

D = W.VOCOS_DIMS
P = W.VOCOS_PREFIX
TOL_F32 = 1e-4
TOL_F16 = 1e-3


@pytest.fixture(scope="module")
def v32():
    w = W.vocos_weights(f16=False)
    c = kb.Context(0)
    c.upload(w)
    yield c, O.OracleModel(w)
    c.close()


@pytest.fixture(scope="module")
def v16():
    w = W.vocos_weights(f16=True)
    c = kb.Context(0)
    c.upload(w)
    yield c, O.OracleModel(w)
    c.close()


def _chunks(seed, lens):
    rng = np.random.default_rng(seed)
    return [W.vocos_inputs(rng, f) for f in lens]


@pytest.mark.parametrize("lens", [[2], [38], [938], [120, 2, 57]])
def test_vocos_f32_matches_oracle(v32, lens):
    c, m = v32
    ins = _chunks(400 + sum(lens), lens)
    got = c.vocos_forward(P, D, [a for a, _ in ins], [b for _, b in ins])
    err = 0.0
    for g, (mel, noise), f in zip(got, ins, lens):
        want = m.vocos(P, D, mel, noise)
        assert g.shape == want.shape == (D["hop"] * (f - 1),)
        assert np.all(np.isfinite(g))
        err = max(err, float(np.abs(g - want).max()))
    print(f"vocos F32 lens={lens}: max abs err {err:.3g}")
    assert err < TOL_F32


def test_vocos_f16_matches_oracle(v16):
    c, m = v16
    lens = [200, 31]
    ins = _chunks(500, lens)
    got = c.vocos_forward(P, D, [a for a, _ in ins], [b for _, b in ins])
    err = max(float(np.abs(g - m.vocos(P, D, mel, noise)).max()) for g, (mel, noise) in zip(got, ins))
    print(f"vocos F16: max abs err {err:.3g}")
    assert err < TOL_F16


def test_vocos_reference_noise_draw(v32):
    """The decoder fed with the reference's own noise stream
    (sano::seeded_noise, compiled from the reference into oracle/_ref/)."""
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    c, m = v32
    F = 96
    mel = np.random.default_rng(9).normal(0.0, 1.0, size=(D["mels"], F)).astype(np.float32)
    noise = O.ref_sano_noise(0x5EED, D["noise_ch"], F)
    got = c.vocos_forward(P, D, [mel], [noise])[0]
    assert float(np.abs(got - m.vocos(P, D, mel, noise)).max()) < TOL_F32


def test_vocos_ragged_batch_equals_single_calls(v32):
    c, _ = v32
    lens = [64, 7, 300, 2, 45]
    ins = _chunks(600, lens)
    batch = c.vocos_forward(P, D, [a for a, _ in ins], [b for _, b in ins])
    for (mel, noise), b in zip(ins, batch):
        np.testing.assert_array_equal(c.vocos_forward(P, D, [mel], [noise])[0], b)


def test_vocos_device_variant_equals_host_variant(v32):
    import torch
    c, _ = v32
    lens = [50, 80]
    ins = _chunks(700, lens)
    want = np.concatenate(c.vocos_forward(P, D, [a for a, _ in ins], [b for _, b in ins]))
    mel = torch.from_numpy(np.concatenate([a.reshape(-1) for a, _ in ins])).cuda()
    noise = torch.from_numpy(np.concatenate([b.reshape(-1) for _, b in ins])).cuda()
    out = torch.zeros(len(want), device="cuda")
    stream = torch.cuda.Stream()
    c.vocos_forward_device(P, D, np.array(lens, np.int32), mel.data_ptr(), noise.data_ptr(), out.data_ptr(),
                           stream.cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_vocos_rejects_bad_parameters(v32):
    c, _ = v32
    mel, noise = W.vocos_inputs(np.random.default_rng(1), 10)
    for bad in ({"n_fft": 1000}, {"hop": 0}, {"dc_pole": 1.0}, {"dw_kernel": 6}, {"mag_clip": -1.0}):
        d = dict(D)
        d.update(bad)
        with pytest.raises(kb.KKError) as e:
            c.vocos_forward(P, d, [mel], [noise])
        assert e.value.code == kb.KK_ERROR_INVALID_ARGUMENT
    with pytest.raises(kb.KKError) as e:
        c.vocos_forward(P, D, [mel[:, :1]], [noise[:, :1]])
    assert e.value.code == kb.KK_ERROR_INVALID_ARGUMENT
    with pytest.raises(kb.KKError) as e:
        c.vocos_forward("kokopop.sanotts.voice.9.", D, [mel], [noise])
    assert e.value.code == kb.KK_ERROR_MODEL
    d = dict(D)
    d["mels"] = 81  # disagrees with the stem weight's shape
    with pytest.raises(kb.KKError) as e:
        c.vocos_forward(P, d, [np.zeros((81, 10), np.float32)], [noise])
    assert e.value.code == kb.KK_ERROR_MODEL
