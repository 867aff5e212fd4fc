"""kk_istft_static, the iSTFT entry point that allocates no device memory,
checked through the C ABI against kk_istft (the context-based entry point)
on the same inputs. The file name sorts last so that the GPU test also runs
after every other test of a session; it passes on its own as well."""
import ctypes

import numpy as np
import pytest

import kokopop_b200 as kb

_f32p = ctypes.POINTER(ctypes.c_float)


def _istft_static(L, post: np.ndarray, device: int = 0) -> np.ndarray:
    post = np.ascontiguousarray(post, np.float32)
    n = post.shape[1]
    audio = np.full(max(1, (n - 1) * 5), np.nan, np.float32)  # NaN: any sample left unwritten shows
    rc = L.kk_istft_static(device, n, post.ctypes.data_as(_f32p), audio.ctypes.data_as(_f32p), None)
    assert rc == kb.KK_OK, L.kk_last_error().decode()
    return audio[: max(0, (n - 1) * 5)]


def test_static_istft_rejects_oversize_and_bad_arguments():
    """Argument checks come before any CUDA call: no GPU needed."""
    L = kb.load_library()
    n_max = 32768  # KK_ISTFT_STATIC_MAX_FRAMES
    one = np.zeros(22, np.float32)
    rc = L.kk_istft_static(0, n_max + 1, one.ctypes.data_as(_f32p), one.ctypes.data_as(_f32p), None)
    assert rc == kb.KK_ERROR_INVALID_ARGUMENT
    msg = L.kk_last_error().decode()
    assert "static scratch" in msg and str(n_max) in msg
    assert L.kk_istft_static(0, 5, None, None, None) == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_istft_static(0, -1, None, None, None) == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_istft_static(-1, 5, one.ctypes.data_as(_f32p), one.ctypes.data_as(_f32p), None) == \
        kb.KK_ERROR_INVALID_ARGUMENT
    # 0 or 1 frame: no samples, nothing to do
    assert L.kk_istft_static(0, 1, one.ctypes.data_as(_f32p), one.ctypes.data_as(_f32p), None) == kb.KK_OK


@pytest.mark.gpu
def test_static_istft_matches_kk_istft_on_two_calls_in_a_row(ctx):
    """Two calls in a row, the second shorter than the first (stale data of
    the first call in the shared scratch would show), then the maximum size
    twice. Same kernel as kk_istft, so the samples agree to well inside the
    tolerance (1e-6 absolute on samples clamped to +-1)."""
    L = kb.load_library()
    rng = np.random.default_rng(2024)
    tol = 1e-6
    cases = [rng.normal(0.0, 3.0, size=(22, 4001)).astype(np.float32),
             rng.normal(0.0, 3.0, size=(22, 257)).astype(np.float32),
             rng.normal(0.0, 3.0, size=(22, 32768)).astype(np.float32)]
    cases.append(cases[-1])
    for post in cases:
        want = ctx.istft(post)
        got = _istft_static(L, post)
        assert got.shape == want.shape
        assert np.all(np.isfinite(got))
        np.testing.assert_allclose(got, want, rtol=0, atol=tol)
