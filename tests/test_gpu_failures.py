"""Failure detection without a GPU fault: the failures are made on the host
(a non-finite input, an allocation that fails, a wait on a flag nothing
sets), each call returns a status with a message, and the context stays
usable for the next call, which must give the same bits as before."""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def w16():
    return W.config2_weights()


def _utts(seed, lens):
    rng = np.random.default_rng(seed)
    return [W.make_utterance(rng, t) for t in lens]


@pytest.mark.parametrize("field,label", [("asr", "asr"), ("f0", "f0"), ("noise", "noise")])
def test_non_finite_input_is_reported_and_context_stays_usable(ctx, w16, field, label):
    """all_finite (kokoro.cpp:91-99): the first non-finite value of the
    first tensor in the reference's order, indexed as the caller packed it."""
    ctx.upload(w16)
    utts = _utts(71, [9, 14])
    want = ctx.decoder_forward(utts)
    bad = _utts(71, [9, 14])
    arr = getattr(bad[1], field)
    flat = arr.reshape(-1)
    flat[7] = np.nan
    flat[11] = np.inf
    offset = getattr(bad[0], field).size  # the second utterance follows the first
    with pytest.raises(kb.KKError) as e:
        ctx.decoder_forward(bad)
    assert e.value.code == kb.KK_ERROR_INFERENCE
    assert f"non-finite Kokoro {label} value at index {offset + 7}" in str(e.value)
    again = ctx.decoder_forward(utts)
    for a, b in zip(again, want):
        np.testing.assert_array_equal(a, b)


def test_non_finite_style_is_reported_after_the_decoder_output(ctx, w16):
    """A NaN style value makes every AdaIN's gamma / beta NaN, but the
    LeakyReLU after each AdaIN maps NaN to 0 (ggml_vec_leaky_relu_f32's
    (x > 0 ? x : 0) + slope (x < 0 ? x : 0), restated exactly), so the
    decoder output stays finite and, as in the reference's check order
    (kokoro.cpp:933-940), the style itself is reported."""
    ctx.upload(w16)
    bad = _utts(72, [6])
    bad[0].style[3] = np.nan
    with pytest.raises(kb.KKError) as e:
        ctx.decoder_forward(bad)
    assert e.value.code == kb.KK_ERROR_INFERENCE
    assert "non-finite Kokoro decoder style value at index 3" in str(e.value)
    assert ctx.decoder_forward(_utts(72, [6]))[0].shape == (3600,)


def test_allocation_failure_is_reported_and_context_recovers(w16):
    """A workspace that cannot grow: KK_ERROR_INFERENCE naming cudaMalloc;
    the next call allocates again and computes the same bits as a context
    that never failed."""
    L = kb.load_library()
    small, big = _utts(73, [4]), _utts(74, [120, 60])
    c, ref = kb.Context(0), kb.Context(0)
    try:
        c.upload(w16)
        ref.upload(w16)
        c.decoder_forward(small)  # workspaces sized for a small batch
        assert L.kk_inject_allocation_failures(1) == kb.KK_OK
        with pytest.raises(kb.KKError) as e:
            c.decoder_forward(big)
        assert e.value.code == kb.KK_ERROR_INFERENCE and "cudaMalloc" in str(e.value)
        assert L.kk_inject_allocation_failures(0) == kb.KK_OK
        got = c.decoder_forward(big)
        want = ref.decoder_forward(big)
        for a, b in zip(got, want):
            np.testing.assert_array_equal(a, b)
    finally:
        L.kk_inject_allocation_failures(0)
        c.close()
        ref.close()


def test_bounded_wait_runs_out_and_context_stays_usable(ctx, w16):
    """The tensor-core kernels' bounded mbarrier wait, on a barrier nothing
    arrives at (2 ms): the kernel gives up, the host reads the code, and
    the context runs the next forward normally."""
    L = kb.load_library()
    ctx.upload(w16)
    utts = _utts(75, [11])
    want = ctx.decoder_forward(utts)[0]
    rc = L.kk_wait_selftest(ctx.h, 2000)
    assert rc == kb.KK_ERROR_INFERENCE
    assert "bounded wait ran out" in L.kk_last_error().decode()
    np.testing.assert_array_equal(ctx.decoder_forward(utts)[0], want)


def test_device_variant_reports_a_non_finite_input_on_the_next_synchronising_call(ctx, w16):
    import torch
    ctx.upload(w16)
    bad = _utts(76, [8])
    bad[0].asr[0, 5] = np.nan
    n, asr, f0, noise, style = W.pack(bad)
    t = lambda a: torch.from_numpy(a).cuda()
    d_asr, d_f0, d_noise, d_style = t(asr), t(f0), t(noise), t(style)
    out = torch.empty(600 * int(n.sum()), device="cuda")
    ctx.decoder_forward_device(n, d_asr.data_ptr(), d_f0.data_ptr(), d_noise.data_ptr(), d_style.data_ptr(),
                               out.data_ptr())
    with pytest.raises(kb.KKError) as e:
        ctx.decoder_forward(_utts(77, [3]))
    assert "non-finite Kokoro asr value at index 5" in str(e.value)
    assert ctx.decoder_forward(_utts(77, [3]))[0].shape == (1800,)
