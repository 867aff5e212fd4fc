"""ctypes access to the oracle (oracle/_build/libkk_oracle.so) and to the
reference's own compiled iSTFT / LSTM (oracle/_ref/libkk_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, always as the checker or the timed CPU
reference, never as the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Callable, Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkk_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libkk_ref.so")

_f32p = ctypes.POINTER(ctypes.c_float)


class TensorDesc(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("dtype", ctypes.c_int32),
        ("n_dims", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("data", ctypes.c_void_p),
    ]


def build() -> None:
    """Builds the oracle and, where the reference checkout exists (the
    KOKOPOP_REFERENCE environment variable, else /root/reference), the
    reference's own host-side sources into _ref/."""
    ref = os.environ.get("KOKOPOP_REFERENCE", "/root/reference")
    args = ["make", "-s", "-C", HERE]
    if os.path.isdir(os.path.join(ref, "src")):
        args.append(f"REF={ref}")
    subprocess.run(args, check=True)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def descs_for(weights) -> tuple:
    """kk_tensor_desc array for a {name: workload.Tensor} dict. The returned
    tuple keeps the name buffers and arrays alive."""
    items = list(weights.values())
    arr = (TensorDesc * len(items))()
    keep = []
    for i, t in enumerate(items):
        nm = t.name.encode()
        keep.append(nm)
        data = np.ascontiguousarray(t.data)
        keep.append(data)
        arr[i].name = nm
        arr[i].dtype = t.dtype
        arr[i].n_dims = len(t.ne)
        for d in range(4):
            arr[i].ne[d] = t.ne[d] if d < len(t.ne) else 1
        arr[i].data = data.ctypes.data
    return arr, keep


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.kko_model_create.restype = ctypes.c_void_p
        L.kko_model_create.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.kko_model_free.argtypes = [ctypes.c_void_p]
        L.kko_last_error.restype = ctypes.c_char_p
        L.kko_round_f16.restype = ctypes.c_float
        L.kko_round_f16.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


class VocosDims(ctypes.Structure):
    """kko_vocos_dims."""
    _int_names = ("dim", "blocks", "pw_hidden", "dw_kernel", "embed_kernel", "noise_ch", "mels", "n_fft", "hop")
    _fields_ = [(n, ctypes.c_int32) for n in _int_names] + [("dc_pole", ctypes.c_float),
                                                              ("mag_clip", ctypes.c_float)]


def istft_r2(re: np.ndarray, im: np.ndarray, n_fft: int, hop: int) -> np.ndarray:
    """kko_istft_r2: frame-major re / im [F, n_fft/2 + 1] -> audio [hop (F - 1)]."""
    re = np.ascontiguousarray(re, np.float32)
    im = np.ascontiguousarray(im, np.float32)
    F = re.shape[0]
    audio = np.zeros(max(1, hop * (F - 1)), np.float32)
    n = ctypes.c_int64(0)
    L = lib()
    L.kko_istft_r2.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p,
                               ctypes.POINTER(ctypes.c_int64)]
    if L.kko_istft_r2(_ptr(re), _ptr(im), F, n_fft, hop, _ptr(audio), ctypes.byref(n)) != 0:
        raise RuntimeError(L.kko_last_error().decode())
    return audio[: n.value]


def dc_block(audio: np.ndarray, pole: float) -> np.ndarray:
    a = np.array(audio, np.float32, copy=True)
    L = lib()
    L.kko_dc_block.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float]
    L.kko_dc_block.restype = None
    L.kko_dc_block(_ptr(a), len(a), ctypes.c_float(pole))
    return a


TAP_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p)


class OracleModel:
    """The oracle over one weight set."""

    def __init__(self, weights):
        self.L = lib()
        arr, self._keep = descs_for(weights)
        self.h = self.L.kko_model_create(ctypes.cast(arr, ctypes.c_void_p), len(arr))
        if not self.h:
            raise RuntimeError("kko_model_create failed")
        self._tap_cb = None
        self.taps: Dict[str, np.ndarray] = {}

    def __del__(self):
        try:
            if self.h:
                self.L.kko_model_free(ctypes.c_void_p(self.h))
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != 0:
            raise RuntimeError(self.L.kko_last_error().decode())

    def set_source_libm(self, use_libm: bool):
        """True: the harmonic source uses the C library's float tanhf/sinf/cosf
        (the reference's literal calls); False (default): correctly rounded."""
        self.L.kko_set_source_libm(ctypes.c_void_p(self.h), 1 if use_libm else 0)

    def record_taps(self, enable: bool = True):
        self.taps = {}
        if enable:
            def cb(name, data, ne0, ne1, user):
                self.taps[name.decode()] = np.ctypeslib.as_array(data, shape=(ne1, ne0)).copy()
            self._tap_cb = TAP_FN(cb)
            self.L.kko_set_tap(ctypes.c_void_p(self.h), self._tap_cb, None)
        else:
            self.L.kko_set_tap(ctypes.c_void_p(self.h), TAP_FN(), None)

    def harmonic_stft(self, f0: np.ndarray, target_frames: int):
        f0 = np.ascontiguousarray(f0, dtype=np.float32)
        har = np.zeros((22, target_frames), np.float32)
        src = np.zeros(len(f0) * 300, np.float32)
        self._check(self.L.kko_harmonic_stft(ctypes.c_void_p(self.h), _ptr(f0), ctypes.c_int64(len(f0)),
                                             ctypes.c_int64(target_frames), _ptr(har), _ptr(src)))
        return har, src

    def generator(self, decoder: np.ndarray, f0: np.ndarray, style: np.ndarray, want_post: bool = False):
        decoder = np.ascontiguousarray(decoder, dtype=np.float32)
        L = decoder.shape[1]
        audio = np.zeros(L * 300, np.float32)
        post = np.zeros((22, 60 * L + 1), np.float32) if want_post else None
        self._check(self.L.kko_generator(ctypes.c_void_p(self.h), ctypes.c_int64(L), _ptr(decoder),
                                         _ptr(np.ascontiguousarray(f0, np.float32)),
                                         _ptr(np.ascontiguousarray(style, np.float32)), _ptr(audio),
                                         _ptr(post) if post is not None else None))
        return (audio, post) if want_post else audio

    def decoder(self, asr, f0, noise, style):
        T = asr.shape[1]
        out = np.zeros((512, 2 * T), np.float32)
        self._check(self.L.kko_decoder(ctypes.c_void_p(self.h), ctypes.c_int64(T),
                                       _ptr(np.ascontiguousarray(asr, np.float32)),
                                       _ptr(np.ascontiguousarray(f0, np.float32)),
                                       _ptr(np.ascontiguousarray(noise, np.float32)),
                                       _ptr(np.ascontiguousarray(style, np.float32)), _ptr(out)))
        return out

    def decoder_forward(self, asr, f0, noise, style):
        T = asr.shape[1]
        audio = np.zeros(600 * T, np.float32)
        self._check(self.L.kko_decoder_forward(ctypes.c_void_p(self.h), ctypes.c_int64(T),
                                               _ptr(np.ascontiguousarray(asr, np.float32)),
                                               _ptr(np.ascontiguousarray(f0, np.float32)),
                                               _ptr(np.ascontiguousarray(noise, np.float32)),
                                               _ptr(np.ascontiguousarray(style, np.float32)), _ptr(audio)))
        return audio

    def bilstm(self, prefix: str, x: np.ndarray, hidden: int = 256):
        x = np.ascontiguousarray(x, dtype=np.float32)
        N, D = x.shape
        out = np.zeros((N, 2 * hidden), np.float32)
        self._check(self.L.kko_bilstm(ctypes.c_void_p(self.h), prefix.encode(), ctypes.c_int64(N),
                                      ctypes.c_int64(D), _ptr(x), _ptr(out)))
        return out

    def duration_encoder(self, x: np.ndarray, style: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        N = x.shape[0]
        out = np.zeros((N, 640), np.float32)
        self._check(self.L.kko_duration_encoder(ctypes.c_void_p(self.h), ctypes.c_int64(N), _ptr(x),
                                                _ptr(np.ascontiguousarray(style, np.float32)), _ptr(out)))
        return out


    def prosody_f0n(self, en: np.ndarray, style: np.ndarray):
        """kko_prosody_f0n: en [T, 640], style [128] -> (f0 [2T], n [2T])."""
        en = np.ascontiguousarray(en, dtype=np.float32)
        T = en.shape[0]
        f0 = np.zeros(2 * T, np.float32)
        nn = np.zeros(2 * T, np.float32)
        self._check(self.L.kko_prosody_f0n(ctypes.c_void_p(self.h), ctypes.c_int64(T), _ptr(en),
                                           _ptr(np.ascontiguousarray(style, np.float32)), _ptr(f0), _ptr(nn)))
        return f0, nn

    def text_encoder(self, ids: np.ndarray):
        """kko_text_encoder: token ids [N] -> [N, 512] (the biLSTM output)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        N = len(ids)
        out = np.zeros((N, 512), np.float32)
        self._check(self.L.kko_text_encoder(ctypes.c_void_p(self.h), ctypes.c_int64(N),
                                            ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _ptr(out)))
        return out

    def albert(self, ids: np.ndarray):
        """kko_albert: token ids [N] -> [N, 512] (ALBERT + bert_encoder)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((len(ids), 512), np.float32)
        self._check(self.L.kko_albert(ctypes.c_void_p(self.h), ctypes.c_int64(len(ids)),
                                      ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), _ptr(out)))
        return out

    def duration_head(self, d: np.ndarray):
        """kko_duration_head: the duration encoder output [N, 640] -> durations [N]."""
        d = np.ascontiguousarray(d, dtype=np.float32)
        out = np.zeros(d.shape[0], np.float32)
        self._check(self.L.kko_duration_head(ctypes.c_void_p(self.h), ctypes.c_int64(d.shape[0]), _ptr(d),
                                             _ptr(out)))
        return out

    def vocos(self, prefix: str, dims, mel: np.ndarray, noise: np.ndarray) -> np.ndarray:
        """kko_vocos: mel [mels, F], noise [noise_ch, F] -> audio [hop (F - 1)]."""
        d = VocosDims(*(int(dims[n]) for n in VocosDims._int_names), float(dims["dc_pole"]),
                      float(dims["mag_clip"]))
        mel = np.ascontiguousarray(mel, np.float32)
        noise = np.ascontiguousarray(noise, np.float32)
        F = mel.shape[1]
        audio = np.zeros(max(1, int(dims["hop"]) * (F - 1)), np.float32)
        n = ctypes.c_int64(0)
        self._check(self.L.kko_vocos(ctypes.c_void_p(self.h), prefix.encode(), ctypes.byref(d), ctypes.c_int64(F),
                                     _ptr(mel), _ptr(noise), _ptr(audio), ctypes.byref(n)))
        return audio[: n.value]

    def duration_proj(self, h: np.ndarray):
        """kko_duration_proj: the predictor biLSTM output [N, 512] -> durations [N]."""
        h = np.ascontiguousarray(h, dtype=np.float32)
        out = np.zeros(h.shape[0], np.float32)
        self._check(self.L.kko_duration_proj(ctypes.c_void_p(self.h), ctypes.c_int64(h.shape[0]), _ptr(h),
                                             _ptr(out)))
        return out


def istft(post: np.ndarray) -> np.ndarray:
    post = np.ascontiguousarray(post, dtype=np.float32)
    n = post.shape[1]
    audio = np.zeros(max(0, (n - 1) * 5), np.float32)
    n_out = ctypes.c_int64(0)
    rc = lib().kko_istft(_ptr(post), ctypes.c_int64(n), _ptr(audio) if audio.size else None, ctypes.byref(n_out))
    if rc != 0:
        raise RuntimeError(lib().kko_last_error().decode())
    return audio[: n_out.value]


def lstm_direction(pre: np.ndarray, w_hh_rowwise: np.ndarray, b_hh: np.ndarray, reverse: bool) -> np.ndarray:
    pre = np.ascontiguousarray(pre, np.float32)
    N, H4 = pre.shape
    H = H4 // 4
    out = np.zeros((N, H), np.float32)
    lib().kko_lstm_direction(_ptr(pre), _ptr(np.ascontiguousarray(w_hh_rowwise, np.float32)),
                             _ptr(np.ascontiguousarray(b_hh, np.float32)), ctypes.c_int64(H),
                             ctypes.c_int64(N), ctypes.c_int(1 if reverse else 0), _ptr(out))
    return out


def align_durations(durations: np.ndarray, speed: float, hidden: Optional[np.ndarray] = None):
    d = np.ascontiguousarray(durations, np.float32)
    n = len(d)
    frames = np.zeros(n, np.int32)
    total = ctypes.c_int64(0)
    L = lib()
    L.kko_align_durations.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float, ctypes.POINTER(ctypes.c_int32),
                                      ctypes.POINTER(ctypes.c_int64), _f32p, ctypes.c_int64, _f32p, ctypes.c_int64]
    if hidden is None:
        rc = L.kko_align_durations(_ptr(d), n, ctypes.c_float(speed),
                                   frames.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(total),
                                   None, 0, None, 0)
        if rc != 0:
            raise RuntimeError(L.kko_last_error().decode())
        return frames, total.value, None
    hidden = np.ascontiguousarray(hidden, np.float32)
    cap = 50 * n
    en = np.zeros((cap, hidden.shape[1]), np.float32)
    rc = L.kko_align_durations(_ptr(d), n, ctypes.c_float(speed),
                               frames.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(total),
                               _ptr(hidden), hidden.shape[1], _ptr(en), cap)
    if rc != 0:
        raise RuntimeError(L.kko_last_error().decode())
    return frames, total.value, en[: total.value]


# --- the reference's own compiled code (oracle/_ref) ----------------------

_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_PATH)
        R.kkref_istft_kokoro.argtypes = [_f32p, ctypes.c_int64, _f32p, ctypes.POINTER(ctypes.c_int64)]
        R.kkref_lstm_direction.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _f32p]
        R.kkref_harmonic_stft.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, _f32p, ctypes.c_float, _f32p, _f32p]
        R.kkref_duration_to_frames.argtypes = [ctypes.c_float, ctypes.c_float]
        R.kkref_duration_mask.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int64, ctypes.c_int64, _f32p]
        R.kkref_postprocess_chunk.argtypes = [_f32p, ctypes.c_int64] + [ctypes.c_int] * 10 + [_f32p, ctypes.c_int64]
        R.kkref_postprocess_chunk.restype = ctypes.c_int64
        R.kkref_crossfade_smart.argtypes = [_f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, _f32p, ctypes.c_int64]
        R.kkref_crossfade_smart.restype = ctypes.c_int64
        R.kkref_istft_complex.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p,
                                          ctypes.POINTER(ctypes.c_int64)]
        R.kkref_dc_block.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float]
        R.kkref_dc_block.restype = None
        R.kkref_bin_mask.argtypes = [ctypes.c_uint32, _f32p]
        R.kkref_bin_mask.restype = None
        R.kkref_sano_noise.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, _f32p]
        _ref = R
    return _ref


def ref_istft_complex(re: np.ndarray, im: np.ndarray, n_fft: int, hop: int) -> np.ndarray:
    """The reference's istft() (src/audio/istft.cpp) on a frame-major
    spectrum [F, n_fft/2 + 1], centred."""
    re = np.ascontiguousarray(re, np.float32)
    im = np.ascontiguousarray(im, np.float32)
    F = re.shape[0]
    audio = np.zeros(max(1, hop * (F - 1)), np.float32)
    n = ctypes.c_int64(0)
    if ref().kkref_istft_complex(_ptr(re), _ptr(im), F, n_fft, hop, _ptr(audio), ctypes.byref(n)) != 0:
        raise RuntimeError("reference istft failed")
    return audio[: n.value]


def ref_dc_block(audio: np.ndarray, pole: float) -> np.ndarray:
    """The reference's dc_block (src/arch/sanotts/sano_vocos.cpp:81-92)."""
    a = np.array(audio, np.float32, copy=True)
    ref().kkref_dc_block(_ptr(a), len(a), ctypes.c_float(pole))
    return a


def ref_postprocess_chunk(audio: np.ndarray, boundary: int, is_first: bool, is_last: bool, cfg) -> np.ndarray:
    """The reference's postprocess_chunk_audio (src/audio/audio_postprocess.cpp:
    260-307) with cfg's post-processing fields (a kokopop_b200.StreamConfig
    or any object with those attributes)."""
    R = ref()
    a = np.ascontiguousarray(audio, np.float32)
    cap = len(a) + max(cfg.paragraph_pause_ms, cfg.sentence_pause_ms, cfg.comma_pause_ms, 0) * cfg.sample_rate // 1000 + 1
    out = np.zeros(cap, np.float32)
    n = R.kkref_postprocess_chunk(_ptr(a), len(a), boundary, int(is_first), int(is_last), cfg.comma_pause_ms,
                                  cfg.sentence_pause_ms, cfg.paragraph_pause_ms, cfg.crossfade_ms,
                                  int(cfg.trim_silence), cfg.max_silence_trim_ms, cfg.sample_rate, _ptr(out), cap)
    assert n <= cap
    return out[:n].copy()


def ref_crossfade_smart(prev: np.ndarray, nxt: np.ndarray, boundary: int, crossfade_ms: int,
                        sample_rate: int) -> np.ndarray:
    """The reference's apply_crossfade_smart (audio_postprocess.cpp:94-202)."""
    R = ref()
    p = np.ascontiguousarray(prev, np.float32)
    q = np.ascontiguousarray(nxt, np.float32)
    cap = len(p) + len(q)
    out = np.zeros(max(cap, 1), np.float32)
    n = R.kkref_crossfade_smart(_ptr(p), len(p), _ptr(q), len(q), boundary, crossfade_ms, sample_rate, _ptr(out),
                                cap)
    assert n <= cap
    return out[:n].copy()


def ref_stream(raw_chunks, boundaries, cfg):
    """postprocess_and_crossfade (src/streaming/streaming.cpp:26-60) over a
    request's raw chunk audio, in order, with the reference's own functions:
    the list of post-processed, crossfaded chunks it hands to its callback."""
    out, tail = [], np.zeros(0, np.float32)
    n = len(raw_chunks)
    ncf = cfg.crossfade_ms * cfg.sample_rate // 1000 if cfg.crossfade_ms > 0 else 0
    for i, (raw, b) in enumerate(zip(raw_chunks, boundaries)):
        p = ref_postprocess_chunk(raw, b, i == 0, i == n - 1, cfg)
        if len(tail) and len(p):
            p = ref_crossfade_smart(tail, p, b, cfg.crossfade_ms, cfg.sample_rate)
        tail = p[max(0, len(p) - ncf):].copy() if len(p) and ncf > 0 else np.zeros(0, np.float32)
        out.append(p)
    return out


def ref_bin_mask(bins: int) -> np.ndarray:
    m = np.zeros(bins, np.float32)
    ref().kkref_bin_mask(bins, _ptr(m))
    return m


def ref_sano_noise(seed: int, channels: int, frames: int) -> np.ndarray:
    """The reference's sano::seeded_noise: [channels, frames]."""
    out = np.zeros((channels, frames), np.float32)
    if ref().kkref_sano_noise(seed, channels, frames, _ptr(out)) != 0:
        raise RuntimeError("reference seeded_noise failed")
    return out


def ref_harmonic_stft(f0: np.ndarray, target_frames: int, merge_w: np.ndarray, merge_b: float):
    """The reference's fill_harmonic_stft (audio_utils.cpp:120-422, compiled
    unchanged): har [22, target_frames] and the sine source [300 len(f0)]."""
    f0 = np.ascontiguousarray(f0, np.float32)
    mw = np.ascontiguousarray(np.asarray(merge_w, np.float32).ravel())
    har = np.zeros((22, target_frames), np.float32)
    src = np.zeros(300 * len(f0), np.float32)
    if ref().kkref_harmonic_stft(_ptr(f0), len(f0), target_frames, _ptr(mw), float(merge_b), _ptr(har),
                                 _ptr(src)) != 0:
        raise RuntimeError("reference fill_harmonic_stft failed")
    return har, src


def ref_duration_frames(durations: np.ndarray, speed: float) -> np.ndarray:
    """The reference's duration_to_frames(value, speed) (kokoro.cpp:181-193)
    per token."""
    R = ref()
    return np.array([R.kkref_duration_to_frames(float(v), float(speed)) for v in
                     np.asarray(durations, np.float32)], np.int32)


def ref_duration_mask(frames: np.ndarray) -> np.ndarray:
    """The reference's build_duration_mask (kokoro.cpp:115-152): [tokens,
    total frames], 1 where a frame belongs to the token."""
    fr = np.ascontiguousarray(frames, np.int32)
    total = int(fr.sum())
    mask = np.zeros((len(fr), total), np.float32)
    if ref().kkref_duration_mask(fr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(fr), total,
                                 _ptr(mask)) != 0:
        raise RuntimeError("reference build_duration_mask failed")
    return mask


def ref_istft(post: np.ndarray) -> np.ndarray:
    post = np.ascontiguousarray(post, np.float32)
    n = post.shape[1]
    audio = np.zeros(max(1, (n - 1) * 5), np.float32)
    n_out = ctypes.c_int64(0)
    if ref().kkref_istft_kokoro(_ptr(post), n, _ptr(audio), ctypes.byref(n_out)) != 0:
        raise RuntimeError("reference istft failed")
    return audio[: n_out.value]


def ref_lstm_direction(pre: np.ndarray, w_hh_rowwise: np.ndarray, b_hh: np.ndarray, reverse: bool) -> np.ndarray:
    pre = np.ascontiguousarray(pre, np.float32)
    N, H4 = pre.shape
    H = H4 // 4
    out = np.full((N, H), -99.0, np.float32)
    ref().kkref_lstm_direction(_ptr(pre), _ptr(np.ascontiguousarray(w_hh_rowwise, np.float32)),
                               _ptr(np.ascontiguousarray(b_hh, np.float32)), H, N, 1 if reverse else 0, _ptr(out))
    return out
