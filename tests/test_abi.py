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
