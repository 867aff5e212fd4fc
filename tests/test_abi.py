"""CPU checks of the C ABI: the library loads, exports every symbol that
include/kokopop_b200.h declares, and rejects bad arguments without touching
a GPU."""
import ctypes

import numpy as np
import pytest

import kokopop_b200 as kb


def test_library_exports_every_declared_symbol():
    L = kb.load_library()
    syms = kb.declared_symbols()
    assert len(syms) >= 8
    for s in syms:
        assert hasattr(L, s), s


def test_null_context_is_invalid_argument_with_message():
    L = kb.load_library()
    n = np.array([4], np.int32)
    z = np.zeros(4096, np.float32)
    f = ctypes.POINTER(ctypes.c_float)
    rc = L.kk_decoder_forward(None, 1, n.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), *(z.ctypes.data_as(f),) * 5)
    assert rc == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_last_error().decode()
    assert L.kk_istft(None, 3, z.ctypes.data_as(f), z.ctypes.data_as(f)) == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_weights_upload(None, None, 0) == kb.KK_ERROR_INVALID_ARGUMENT
    i32p = ctypes.POINTER(ctypes.c_int32)
    assert L.kk_bilstm_forward(None, b"p", 1, n.ctypes.data_as(i32p), 640, z.ctypes.data_as(f), z.ctypes.data_as(f)) \
        == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_duration_encoder_forward(None, 1, n.ctypes.data_as(i32p), *(z.ctypes.data_as(f),) * 3) \
        == kb.KK_ERROR_INVALID_ARGUMENT
    tot = ctypes.c_int64(0)
    assert L.kk_align_durations(None, 1, z.ctypes.data_as(f), 1.0, n.ctypes.data_as(i32p), ctypes.byref(tot),
                                None, 0, None, 0) == kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_ctx_create(0, None) == kb.KK_ERROR_INVALID_ARGUMENT
    L.kk_ctx_destroy(None)  # no-op


def test_error_slot_is_thread_local():
    import threading
    L = kb.load_library()
    L.kk_ctx_create(0, None)
    seen = {}

    def other():
        seen["msg"] = L.kk_last_error().decode()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert L.kk_last_error().decode() != ""


def test_front_end_and_queue_entry_points_reject_bad_arguments():
    """The front-end entry points and the queue validate their arguments
    before touching a device."""
    L = kb.load_library()
    n = np.array([4], np.int32)
    ids = np.zeros(4, np.int32)
    z = np.zeros(4096, np.float32)
    f = ctypes.POINTER(ctypes.c_float)
    i32p = ctypes.POINTER(ctypes.c_int32)
    ip, fp = n.ctypes.data_as(i32p), z.ctypes.data_as(f)
    idp = ids.ctypes.data_as(i32p)
    E = kb.KK_ERROR_INVALID_ARGUMENT
    assert L.kk_text_encoder_forward(None, 1, ip, idp, fp) == E
    assert L.kk_albert_forward(None, 1, ip, idp, fp) == E
    assert L.kk_duration_head_forward(None, 1, ip, fp, fp) == E
    assert L.kk_duration_proj(None, 4, fp, fp) == E
    assert L.kk_prosody_f0n(None, 1, ip, fp, fp, fp, fp) == E
    q = ctypes.c_void_p()
    assert L.kk_queue_create(None, 1, 64, 1000, 0, ctypes.byref(q)) == E
    assert L.kk_queue_create_exec(kb.QUEUE_EXEC_FN(0), None, 1, 64, 1000, 0, ctypes.byref(q)) == E
    assert L.kk_queue_last_error().decode()
    t = ctypes.c_uint64()
    assert L.kk_queue_submit(None, 0, 4, fp, fp, fp, fp, fp, ctypes.byref(t)) == E
    assert L.kk_queue_wait(None, 1, 0) == E
    L.kk_queue_destroy(None)  # no-op
    # one context listed twice would give two workers the same workspaces;
    # the check runs before any context is touched, so any non-null handle serves
    fake = ctypes.c_void_p(0x1000)
    ctxs = (ctypes.c_void_p * 2)(fake, fake)
    assert L.kk_queue_create(ctxs, 2, 64, 1000, 0, ctypes.byref(q)) == E
    assert "twice" in L.kk_queue_last_error().decode()
    n = ctypes.c_uint64(0)
    assert L.kk_allocation_count(ctypes.byref(n)) == kb.KK_OK
    assert L.kk_allocation_count(None) == E
    # failure injection and the wait self-test validate before any CUDA call
    assert L.kk_inject_allocation_failures(-1) == E
    assert L.kk_inject_allocation_failures(0) == kb.KK_OK
    assert L.kk_wait_selftest(None, 1000) == E
    pv = kb.VocosParams.of(dict(dim=8, blocks=1, pw_hidden=8, dw_kernel=7, embed_kernel=7, noise_ch=4, mels=8,
                                n_fft=64, hop=16, dc_pole=0.9, mag_clip=100.0))
    assert L.kk_vocos_forward(None, b"p", ctypes.byref(pv), 1, ip, fp, fp, fp) == E


def test_queue_rejects_out_of_range_chunks_and_limits():
    ok = kb.Queue(executor=lambda *a: 0, max_batch=2, max_batch_frames=100, max_wait_us=0)
    try:
        from types import SimpleNamespace
        big = SimpleNamespace(T=101, asr=np.zeros((512, 101), np.float32), f0=np.zeros(202, np.float32),
                              noise=np.zeros(202, np.float32), style=np.zeros(128, np.float32))
        with pytest.raises(kb.KKError):
            ok.submit(1, big)
    finally:
        ok.close()
    for kw in ({"max_batch": 0}, {"max_batch_frames": 0}, {"max_wait_us": -1}):
        with pytest.raises(kb.KKError):
            kb.Queue(executor=lambda *a: 0, **kw)
