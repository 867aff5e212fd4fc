"""kk_istft_static, the iSTFT entry point that allocates no device memory,
checked through the C ABI against kk_istft (the context-based entry point)
on the same inputs. It serves callers that cannot allocate mid-run: a
real-time audio thread (cudaMalloc / cudaFree can synchronise the whole
device) or a process that fixes its device-memory budget at start-up. The
file name sorts last so that the GPU test also runs after every other test
of a session; it passes on its own as well."""
import ctypes
import os
import re

import numpy as np
import pytest

import kokopop_b200 as kb

_f32p = ctypes.POINTER(ctypes.c_float)
CSRC = os.path.join(os.path.dirname(kb.__file__), "csrc")


def _istft_static(L, post: np.ndarray, device: int = 0) -> np.ndarray:
    post = np.ascontiguousarray(post, np.float32)
    n = post.shape[1]
    audio = np.full(max(1, (n - 1) * 5), np.nan, np.float32)  # NaN: any sample left unwritten shows
    rc = L.kk_istft_static(device, n, post.ctypes.data_as(_f32p), audio.ctypes.data_as(_f32p), None)
    assert rc == kb.KK_OK, L.kk_last_error().decode()
    return audio[: max(0, (n - 1) * 5)]


def _allocations(L) -> int:
    n = ctypes.c_uint64(0)
    assert L.kk_allocation_count(ctypes.byref(n)) == kb.KK_OK
    return n.value


def test_static_istft_rejects_oversize_and_bad_arguments():
    """Size and pointer checks come before any CUDA call: no GPU needed."""
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
    # a device index past the device count (any index on a machine without one)
    assert L.kk_istft_static(1 << 20, 5, one.ctypes.data_as(_f32p), one.ctypes.data_as(_f32p), None) == \
        kb.KK_ERROR_INVALID_ARGUMENT
    assert "out of range" in L.kk_last_error().decode()


def test_every_allocation_goes_through_the_counted_wrappers():
    """kk_allocation_count only means something if no source allocates
    around it: the one raw cudaMalloc / cudaMallocHost is inside the
    counting wrappers."""
    raw = re.compile(r"\b(cudaMalloc|cudaMallocHost|cudaHostAlloc|cudaMallocAsync|cudaMallocManaged|"
                     r"cudaMallocPitch|cudaMalloc3D|cudaMallocArray)\s*\(")
    hits = []
    for f in sorted(os.listdir(CSRC)):
        if not f.endswith((".cu", ".cpp", ".cuh", ".h")):
            continue
        for i, line in enumerate(open(os.path.join(CSRC, f)), 1):
            code = line.split("//")[0]
            if raw.search(code):
                hits.append(f"{f}:{i}: {line.strip()}")
    assert len(hits) == 2 and all(h.startswith("kk_host.cpp:") for h in hits), hits


@pytest.mark.gpu
def test_static_istft_matches_kk_istft_on_two_calls_in_a_row(ctx):
    """A 0-frame call first (the set-up call that reserves the array on this
    device), then two calls in a row, the second shorter than the first
    (stale data of the first call in the shared scratch would show), then
    the maximum size twice. Same kernel as kk_istft, so the samples agree to
    well inside the tolerance (1e-6 absolute on samples clamped to +-1).
    The static calls make no allocation of the library's."""
    L = kb.load_library()
    assert L.kk_istft_static(0, 0, None, None, None) == kb.KK_OK, L.kk_last_error().decode()
    assert L.kk_istft_static(0, 1, None, None, None) == kb.KK_OK, L.kk_last_error().decode()
    # a failed call leaves no pending error that a later valid call would report
    one = np.zeros(22 * 5, np.float32)
    assert L.kk_istft_static(1 << 20, 5, one.ctypes.data_as(_f32p), one.ctypes.data_as(_f32p), None) == \
        kb.KK_ERROR_INVALID_ARGUMENT
    rng = np.random.default_rng(2024)
    tol = 1e-6
    cases = [rng.normal(0.0, 3.0, size=(22, 4001)).astype(np.float32),
             rng.normal(0.0, 3.0, size=(22, 257)).astype(np.float32),
             rng.normal(0.0, 3.0, size=(22, 32768)).astype(np.float32)]
    cases.append(cases[-1])
    want = [ctx.istft(post) for post in cases]  # the context's buffers grow here, before counting
    before = _allocations(L)
    for post, w in zip(cases, want):
        got = _istft_static(L, post)
        assert got.shape == w.shape
        assert np.all(np.isfinite(got))
        np.testing.assert_allclose(got, w, rtol=0, atol=tol)
    assert _allocations(L) == before
