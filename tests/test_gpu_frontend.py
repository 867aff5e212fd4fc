"""GPU parity of the text encoder (graph_ops.cpp:1578-1624, up to its
biLSTM) and the duration head (kokoro.cpp:343-355, :469-516), through the C
ABI, against the oracle on the same seeded inputs.

Tolerances. The text encoder ends in a biLSTM whose output h lies in
[-1, 1]; with F32 weights the convs run as split F32 GEMMs on the tensor
cores and the LSTM's input projection likewise, so h differs from the
oracle by the accumulation order only: 5e-6 max-abs, the LSTM layer bound.
With F16 weights each conv rounds its input to half; a last-bit difference
in the LayerNorm input of a layer can flip one half rounding of the next
conv's input, so that case is held to 1e-4. Durations are sums of 50
logistic terms (about 25 here): 1e-4 max-abs, and the frames derived from
them equal. The projection and bucket sum alone, given the same h, run the
reference's double arithmetic in its order: bit-exact.
"""
import numpy as np
import pytest

import kokopop_b200 as kb
from kokopop_b200 import workload as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_TE_F32 = 5e-6
TOL_TE_F16 = 1e-4
TOL_DUR = 1e-4


@pytest.fixture(scope="module", params=[False, True], ids=["f32", "f16"])
def setup(request):
    wts = W.frontend_weights(f16=request.param)
    c = kb.Context(0)
    c.upload(wts)
    yield c, O.OracleModel(wts), request.param
    c.close()


def _ids(seed, lens):
    rng = np.random.default_rng(seed)
    return [W.token_ids(rng, n - 2) for n in lens]


def test_text_encoder_matches_oracle(setup):
    c, m, f16 = setup
    ids = _ids(21, [130, 7, 64])
    got = c.text_encoder(ids)
    err = max(float(np.abs(g - m.text_encoder(i)).max()) for g, i in zip(got, ids))
    print(f"text encoder {'f16' if f16 else 'f32'}: max abs err {err:.3g}")
    assert all(g.shape == (len(i), 512) for g, i in zip(got, ids))
    assert err < (TOL_TE_F16 if f16 else TOL_TE_F32)


def test_text_encoder_batch_equals_single_calls(setup):
    """Packing sequences into one batch changes nothing, bit for bit."""
    c, _, _ = setup
    ids = _ids(22, [40, 3, 90, 12])
    batch = c.text_encoder(ids)
    for i, b in zip(ids, batch):
        np.testing.assert_array_equal(c.text_encoder([i])[0], b)


def test_text_encoder_rejects_bad_ids(setup):
    c, _, _ = setup
    with pytest.raises(kb.KKError):
        c.text_encoder([np.array([0, 5, 178, 0], np.int32)])
    with pytest.raises(kb.KKError):
        c.text_encoder([np.array([0, -1, 0], np.int32)])
    # the context stays usable
    assert c.text_encoder(_ids(23, [5]))[0].shape == (5, 512)


def test_text_encoder_device_entry_matches_host_entry(setup):
    import torch

    c, _, _ = setup
    ids = _ids(24, [33, 18])
    want = np.concatenate(c.text_encoder(ids))
    lens = np.array([len(i) for i in ids], np.int32)
    d_ids = torch.from_numpy(np.concatenate(ids)).cuda()
    out = torch.empty(int(lens.sum()), 512, device="cuda")
    c.text_encoder_device(lens, d_ids.data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_duration_head_matches_oracle(setup):
    c, m, f16 = setup
    rng = np.random.default_rng(25)
    ds = [rng.normal(0.0, 1.0, size=(n, 640)).astype(np.float32) for n in (130, 9, 47)]
    got = c.duration_head(ds)
    for g, d in zip(got, ds):
        want = m.duration_head(d)
        err = float(np.abs(g - want).max())
        print(f"duration head {'f16' if f16 else 'f32'} N={len(d)}: max abs err {err:.3g}")
        assert g.shape == want.shape and err < TOL_DUR
        fg, tg, _ = O.align_durations(g, 1.0)
        fw, tw, _ = O.align_durations(want, 1.0)
        np.testing.assert_array_equal(fg, fw)


def test_duration_proj_bit_exact(setup):
    """Given the same biLSTM output, the projection and the bucket sum in
    double equal the oracle's (the reference's host loop) bit for bit,
    including large pre-activations on both sides of the logistic branch."""
    c, m, _ = setup
    rng = np.random.default_rng(26)
    h = rng.uniform(-1.0, 1.0, size=(300, 512)).astype(np.float32)
    h[:20] *= 400.0  # |acc| up to ~40: both logistic branches, saturated terms
    np.testing.assert_array_equal(c.duration_proj(h), m.duration_proj(h))


# ALBERT + bert_encoder: twelve passes of LayerNorm-ed residual layers. With
# F32 weights the linears run as split F32 GEMMs and the attention, softmax
# and GELU follow the oracle's order and roundings, so the output (values
# around 0.1) differs by accumulation order only: 1e-5. With F16 weights every
# linear rounds its input to half, and a last-bit difference can flip one such
# rounding, which the following layers carry: 2e-3 max-abs, 1e-4 mean-abs.
# The oracle's ALBERT is unpinned (its ggml GELU / softmax / norm semantics
# are restated from the public ggml source), so these bound the CUDA path
# against the restatement only.
TOL_AL_F32 = 1e-5
TOL_AL_F16 = 2e-3
TOL_AL_F16_MEAN = 1e-4


@pytest.fixture(scope="module", params=[False, True], ids=["f32", "f16"])
def albert_setup(request):
    wts = W.albert_weights(f16=request.param)
    c = kb.Context(0)
    c.upload(wts)
    yield c, O.OracleModel(wts), request.param
    c.close()


def test_albert_matches_oracle(albert_setup):
    c, m, f16 = albert_setup
    ids = _ids(31, [40, 5, 23])
    got = c.albert(ids)
    errs = [np.abs(g - m.albert(i)) for g, i in zip(got, ids)]
    err = max(float(e.max()) for e in errs)
    mean = max(float(e.mean()) for e in errs)
    print(f"albert {'f16' if f16 else 'f32'}: max abs err {err:.3g}, mean {mean:.3g}")
    assert all(g.shape == (len(i), 512) for g, i in zip(got, ids))
    if f16:
        assert err < TOL_AL_F16 and mean < TOL_AL_F16_MEAN
    else:
        assert err < TOL_AL_F32


def test_albert_batch_equals_single_calls(albert_setup):
    c, _, _ = albert_setup
    ids = _ids(32, [17, 64, 2])
    batch = c.albert(ids)
    for i, b in zip(ids, batch):
        np.testing.assert_array_equal(c.albert([i])[0], b)


def test_albert_rejects_bad_input(albert_setup):
    c, _, _ = albert_setup
    with pytest.raises(kb.KKError):
        c.albert([np.array([0, 178, 0], np.int32)])
    with pytest.raises(kb.KKError):
        c.albert([np.zeros(513, np.int32)])
    assert c.albert(_ids(33, [4]))[0].shape == (4, 512)
