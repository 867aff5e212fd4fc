"""kokopop_b200 — B200 (sm_100a) Kokoro-82M synthesis hot path.

Python access to the C ABI of include/kokopop_b200.h through ctypes. The
product is the in-tree shared library libkokopop_b200.so (CUDA kernels plus
the C++ host layer); this module only marshals arguments. There is no CPU
fallback: without the library, or without a B200, every call raises.
"""
from __future__ import annotations

import ctypes
import threading
import os
from typing import Dict, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkokopop_b200.so")
HEADER = os.path.join(HERE, "..", "include", "kokopop_b200.h")

KK_OK = 0
KK_ERROR_INVALID_ARGUMENT = 1
KK_ERROR_IO = 2
KK_ERROR_MODEL = 3
KK_ERROR_INFERENCE = 5

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


class TensorDesc(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("dtype", ctypes.c_int32),
        ("n_dims", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("data", ctypes.c_void_p),
    ]


class Profile(ctypes.Structure):
    _fields_ = [
        ("launches", ctypes.c_uint64),
        ("conv_launches", ctypes.c_uint64),
        ("conv_ms", ctypes.c_double),
        ("conv_flop", ctypes.c_double),
    ]


class VocosParams(ctypes.Structure):
    """kk_vocos_params."""
    _fields_ = [(n, ctypes.c_int32) for n in ("dim", "blocks", "pw_hidden", "dw_kernel", "embed_kernel",
                                                 "noise_ch", "mels", "n_fft", "hop")] + \
               [("dc_pole", ctypes.c_float), ("mag_clip", ctypes.c_float)]

    @classmethod
    def of(cls, d: Dict) -> "VocosParams":
        return cls(*(int(d[n]) for n in ("dim", "blocks", "pw_hidden", "dw_kernel", "embed_kernel", "noise_ch",
                                         "mels", "n_fft", "hop")), float(d["dc_pole"]), float(d["mag_clip"]))


class ProfileRecord(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("taps", ctypes.c_int32),
        ("ms", ctypes.c_double),
        ("flop", ctypes.c_double),
        ("bytes", ctypes.c_double),
    ]


# kinds of timed launches (KK_PROF_*)
PROF_KINDS = ["conv", "operand", "stats", "istft", "source", "lstm", "other"]


class KKError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def load_library():
    """Loads libkokopop_b200.so and declares its signatures. Raises when the
    library has not been built (python -m kokopop_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m kokopop_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    vp = ctypes.c_void_p
    L.kk_last_error.restype = ctypes.c_char_p
    L.kk_ctx_create.argtypes = [ctypes.c_int, ctypes.POINTER(vp)]
    L.kk_ctx_destroy.argtypes = [vp]
    L.kk_ctx_destroy.restype = None
    L.kk_weights_upload.argtypes = [vp, vp, ctypes.c_size_t]
    L.kk_decoder_forward.argtypes = [vp, ctypes.c_int32, _i32p, _f32p, _f32p, _f32p, _f32p, _f32p]
    L.kk_decoder_forward_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp, vp, vp, vp]
    L.kk_generator_forward.argtypes = [vp, ctypes.c_int32, _i32p, _f32p, _f32p, _f32p, _f32p]
    L.kk_istft.argtypes = [vp, ctypes.c_int64, _f32p, _f32p]
    L.kk_istft_static.argtypes = [ctypes.c_int, ctypes.c_int64, _f32p, _f32p, vp]
    L.kk_bilstm_forward.argtypes = [vp, ctypes.c_char_p, ctypes.c_int32, _i32p, ctypes.c_int64, _f32p, _f32p]
    L.kk_duration_encoder_forward.argtypes = [vp, ctypes.c_int32, _i32p, _f32p, _f32p, _f32p]
    L.kk_duration_encoder_forward_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp, vp]
    L.kk_prosody_f0n.argtypes = [vp, ctypes.c_int32, _i32p, _f32p, _f32p, _f32p, _f32p]
    L.kk_prosody_f0n_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp, vp, vp]
    L.kk_text_encoder_forward.argtypes = [vp, ctypes.c_int32, _i32p, _i32p, _f32p]
    L.kk_text_encoder_forward_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp]
    L.kk_albert_forward.argtypes = [vp, ctypes.c_int32, _i32p, _i32p, _f32p]
    L.kk_albert_forward_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp]
    L.kk_duration_head_forward.argtypes = [vp, ctypes.c_int32, _i32p, _f32p, _f32p]
    L.kk_duration_head_forward_device.argtypes = [vp, ctypes.c_int32, _i32p, vp, vp, vp]
    L.kk_duration_proj.argtypes = [vp, ctypes.c_int64, _f32p, _f32p]
    L.kk_align_durations.argtypes = [vp, ctypes.c_int64, _f32p, ctypes.c_float, _i32p,
                                     ctypes.POINTER(ctypes.c_int64), _f32p, ctypes.c_int64, _f32p, ctypes.c_int64]
    L.kk_queue_create.argtypes = [ctypes.POINTER(vp), ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                  ctypes.POINTER(vp)]
    L.kk_queue_create_exec.argtypes = [QUEUE_EXEC_FN, ctypes.POINTER(vp), ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int64, ctypes.c_int32, ctypes.POINTER(vp)]
    L.kk_queue_submit.argtypes = [vp, ctypes.c_uint64, ctypes.c_int32, _f32p, _f32p, _f32p, _f32p, _f32p,
                                  ctypes.POINTER(ctypes.c_uint64)]
    L.kk_queue_wait.argtypes = [vp, ctypes.c_uint64, ctypes.c_int32]
    L.kk_queue_cancel.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_int32)]
    L.kk_queue_stats.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                 ctypes.POINTER(ctypes.c_uint64)]
    L.kk_queue_last_error.restype = ctypes.c_char_p
    L.kk_queue_destroy.argtypes = [vp]
    L.kk_queue_destroy.restype = None
    L.kk_profile_enable.argtypes = [vp, ctypes.c_int]
    L.kk_profile_read.argtypes = [vp, ctypes.POINTER(Profile), ctypes.c_int]
    L.kk_allocation_count.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
    L.kk_inject_allocation_failures.argtypes = [ctypes.c_int32]
    L.kk_wait_selftest.argtypes = [vp, ctypes.c_int64]
    L.kk_vocos_forward.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(VocosParams), ctypes.c_int32, _i32p, _f32p,
                                   _f32p, _f32p]
    L.kk_vocos_forward_device.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(VocosParams), ctypes.c_int32, _i32p,
                                          vp, vp, vp, vp]
    L.kk_profile_records.argtypes = [vp, ctypes.POINTER(ProfileRecord), ctypes.c_size_t,
                                     ctypes.POINTER(ctypes.c_size_t)]
    i64p = ctypes.POINTER(ctypes.c_int64)
    cfgp = ctypes.POINTER(StreamConfig)
    L.kk_stream_preset.argtypes = [ctypes.c_int32, cfgp]
    L.kk_postprocess_chunk.argtypes = [cfgp, _f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       _f32p, ctypes.c_int64, i64p]
    L.kk_crossfade.argtypes = [cfgp, _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int32, _f32p,
                               ctypes.c_int64, i64p]
    L.kk_stream_create.argtypes = [vp, cfgp, ctypes.POINTER(vp)]
    L.kk_stream_push.argtypes = [vp, ctypes.c_int32, _f32p, _f32p, _f32p, _f32p, ctypes.c_int32, ctypes.c_int32]
    L.kk_stream_next.argtypes = [vp, ctypes.c_int32, ctypes.POINTER(_f32p), i64p, ctypes.POINTER(ctypes.c_int32)]
    L.kk_stream_cancel.argtypes = [vp]
    L.kk_stream_destroy.argtypes = [vp]
    L.kk_stream_destroy.restype = None
    _lib = L
    return L


def declared_symbols() -> List[str]:
    """Every kk_* function declared in include/kokopop_b200.h."""
    import re
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(kk_[a-z0-9_]+)\s*\(", src)))


# kk_queue_exec_fn
QUEUE_EXEC_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                                 ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
                                 ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
                                 ctypes.POINTER(ctypes.c_float))
QUEUE_PENDING = -1
QUEUE_CANCELLED = -2
STREAM_END = -3

# chunk boundaries (KK_BOUNDARY_*)
BOUNDARY_NONE, BOUNDARY_CLAUSE_WEAK, BOUNDARY_CLAUSE_STRONG, BOUNDARY_SENTENCE, BOUNDARY_NEWLINE, \
    BOUNDARY_PARAGRAPH = range(6)


class StreamConfig(ctypes.Structure):
    """kk_stream_config: the post-processing fields of the reference's
    ChunkConfig. preset(0) is the adaptative preset, preset(1) long-form."""
    _fields_ = [
        ("comma_pause_ms", ctypes.c_int32),
        ("sentence_pause_ms", ctypes.c_int32),
        ("paragraph_pause_ms", ctypes.c_int32),
        ("crossfade_ms", ctypes.c_int32),
        ("trim_silence", ctypes.c_int32),
        ("max_silence_trim_ms", ctypes.c_int32),
        ("sample_rate", ctypes.c_int32),
    ]

    @classmethod
    def preset(cls, mode: int = 0) -> "StreamConfig":
        c = cls()
        L = load_library()
        rc = L.kk_stream_preset(mode, ctypes.byref(c))
        if rc != 0:
            raise KKError(rc, L.kk_queue_last_error().decode())
        return c


def postprocess_chunk(cfg: StreamConfig, audio: np.ndarray, boundary_after: int, is_first: bool,
                      is_last: bool) -> np.ndarray:
    """kk_postprocess_chunk (the reference's postprocess_chunk_audio)."""
    L = load_library()
    a = np.ascontiguousarray(audio, np.float32)
    longest_pause_ms = max(cfg.paragraph_pause_ms, cfg.sentence_pause_ms, cfg.comma_pause_ms, 0)
    cap = len(a) + longest_pause_ms * cfg.sample_rate // 1000 + 1
    out = np.zeros(cap, np.float32)
    n = ctypes.c_int64()
    rc = L.kk_postprocess_chunk(ctypes.byref(cfg), _ptr(a), len(a), boundary_after, int(is_first), int(is_last),
                                _ptr(out), cap, ctypes.byref(n))
    if rc != 0:
        raise KKError(rc, L.kk_queue_last_error().decode())
    return out[:n.value].copy()


def crossfade(cfg: StreamConfig, prev: np.ndarray, nxt: np.ndarray, boundary: int) -> np.ndarray:
    """kk_crossfade (the reference's apply_crossfade_smart)."""
    L = load_library()
    p = np.ascontiguousarray(prev, np.float32)
    q = np.ascontiguousarray(nxt, np.float32)
    cap = len(p) + len(q)
    out = np.zeros(max(cap, 1), np.float32)
    n = ctypes.c_int64()
    rc = L.kk_crossfade(ctypes.byref(cfg), _ptr(p), len(p), _ptr(q), len(q), boundary, _ptr(out), cap,
                        ctypes.byref(n))
    if rc != 0:
        raise KKError(rc, L.kk_queue_last_error().decode())
    return out[:n.value].copy()


def _ptr(a: Optional[np.ndarray], t=_f32p):
    return None if a is None else a.ctypes.data_as(t)


def _descs(weights) -> tuple:
    items = list(weights.values())
    arr = (TensorDesc * len(items))()
    keep = []
    for i, t in enumerate(items):
        nm = t.name.encode()
        data = np.ascontiguousarray(t.data)
        keep += [nm, data]
        arr[i].name = nm
        arr[i].dtype = t.dtype
        arr[i].n_dims = len(t.ne)
        for d in range(4):
            arr[i].ne[d] = t.ne[d] if d < len(t.ne) else 1
        arr[i].data = data.ctypes.data
    return arr, keep


class Context:
    """One kk_ctx: a CUDA device, its stream and the uploaded weights."""

    def __init__(self, device: int = 0):
        self.L = load_library()
        h = ctypes.c_void_p()
        self._check(self.L.kk_ctx_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            self.L.kk_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != KK_OK:
            raise KKError(rc, self.L.kk_last_error().decode())

    def upload(self, weights) -> None:
        arr, keep = _descs(weights)
        self._check(self.L.kk_weights_upload(self.h, ctypes.cast(arr, ctypes.c_void_p), len(arr)))
        del keep

    def decoder_forward(self, utts: Sequence) -> List[np.ndarray]:
        """Decoder + generator + iSTFT for a ragged batch of workload.Utterance."""
        from .workload import pack
        n_frames, asr, f0, noise, style = pack(utts)
        audio = np.zeros(600 * int(n_frames.sum()), np.float32)
        self._check(self.L.kk_decoder_forward(self.h, len(utts), _ptr(n_frames, _i32p), _ptr(asr), _ptr(f0),
                                              _ptr(noise), _ptr(style), _ptr(audio)))
        out, o = [], 0
        for t in n_frames:
            out.append(audio[o:o + 600 * int(t)])
            o += 600 * int(t)
        return out

    def decoder_forward_packed(self, n_frames, asr, f0, noise, style, audio) -> None:
        """Host-buffer call on pre-packed arrays (the bench's end-to-end leg)."""
        self._check(self.L.kk_decoder_forward(self.h, len(n_frames), _ptr(n_frames, _i32p), _ptr(asr), _ptr(f0),
                                              _ptr(noise), _ptr(style), _ptr(audio)))

    def decoder_forward_device(self, n_frames: np.ndarray, asr_ptr: int, f0_ptr: int, noise_ptr: int,
                               style_ptr: int, audio_ptr: int, stream: int = 0) -> None:
        n_frames = np.ascontiguousarray(n_frames, np.int32)
        self._check(self.L.kk_decoder_forward_device(self.h, len(n_frames), _ptr(n_frames, _i32p), asr_ptr, f0_ptr,
                                                     noise_ptr, style_ptr, audio_ptr, stream or None))

    def generator_forward(self, decoders: Sequence[np.ndarray], f0s: Sequence[np.ndarray],
                          styles: Sequence[np.ndarray]) -> List[np.ndarray]:
        lens = np.array([d.shape[1] for d in decoders], np.int32)
        dec = np.concatenate([np.ascontiguousarray(d, np.float32).reshape(-1) for d in decoders])
        f0 = np.concatenate([np.asarray(f, np.float32) for f in f0s])
        style = np.concatenate([np.asarray(s, np.float32)[:128] for s in styles])
        audio = np.zeros(300 * int(lens.sum()), np.float32)
        self._check(self.L.kk_generator_forward(self.h, len(lens), _ptr(lens, _i32p), _ptr(dec), _ptr(f0),
                                                _ptr(style), _ptr(audio)))
        out, o = [], 0
        for t in lens:
            out.append(audio[o:o + 300 * int(t)])
            o += 300 * int(t)
        return out

    def profile_enable(self, on: bool = True) -> None:
        self._check(self.L.kk_profile_enable(self.h, 1 if on else 0))

    def profile_read(self, reset: bool = False) -> Dict[str, float]:
        p = Profile()
        self._check(self.L.kk_profile_read(self.h, ctypes.byref(p), 1 if reset else 0))
        return {"launches": int(p.launches), "conv_launches": int(p.conv_launches),
                "conv_ms": float(p.conv_ms), "conv_flop": float(p.conv_flop)}

    def vocos_forward(self, prefix: str, dims: Dict, mels: Sequence[np.ndarray],
                      noises: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_vocos_forward over chunks: mels[u] [mels, F_u], noises[u]
        [noise_ch, F_u] (time-fastest) -> audio [hop (F_u - 1)] each."""
        p = VocosParams.of(dims)
        lens = np.array([m.shape[1] for m in mels], np.int32)
        mel = np.concatenate([np.ascontiguousarray(m, np.float32).reshape(-1) for m in mels])
        noise = np.concatenate([np.ascontiguousarray(z, np.float32).reshape(-1) for z in noises])
        hop = int(dims["hop"])
        audio = np.zeros(max(1, int((hop * (lens - 1)).sum())), np.float32)
        self._check(self.L.kk_vocos_forward(self.h, prefix.encode(), ctypes.byref(p), len(lens), _ptr(lens, _i32p),
                                            _ptr(mel), _ptr(noise), _ptr(audio)))
        out, o = [], 0
        for f in lens:
            n = hop * (int(f) - 1)
            out.append(audio[o:o + n])
            o += n
        return out

    def vocos_forward_device(self, prefix: str, dims: Dict, lens: np.ndarray, mel_ptr: int, noise_ptr: int,
                             audio_ptr: int, stream: int = 0) -> None:
        p = VocosParams.of(dims)
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_vocos_forward_device(self.h, prefix.encode(), ctypes.byref(p), len(lens),
                                                   _ptr(lens, _i32p), mel_ptr, noise_ptr, audio_ptr, stream or None))

    def profile_records(self) -> List[Dict[str, float]]:
        """The timed launches since the last reset: kind (PROF_KINDS), taps,
        device ms, algorithmic FLOPs and DRAM bytes."""
        n = ctypes.c_size_t(0)
        self._check(self.L.kk_profile_records(self.h, None, 0, ctypes.byref(n)))
        arr = (ProfileRecord * max(1, n.value))()
        self._check(self.L.kk_profile_records(self.h, arr, n.value, ctypes.byref(n)))
        return [{"kind": PROF_KINDS[r.kind], "taps": int(r.taps), "ms": float(r.ms), "flop": float(r.flop),
                 "bytes": float(r.bytes)} for r in arr[: n.value]]

    def istft(self, post: np.ndarray) -> np.ndarray:
        post = np.ascontiguousarray(post, np.float32)
        n = post.shape[1]
        audio = np.zeros(max(1, (n - 1) * 5), np.float32)
        self._check(self.L.kk_istft(self.h, n, _ptr(post), _ptr(audio)))
        return audio[: max(0, (n - 1) * 5)]

    # ---- LSTM stack and durations ----

    def bilstm(self, prefix: str, xs: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_bilstm_forward over sequences xs[b] of shape [N_b, in_dim];
        returns [N_b, 512] each (forward h, then backward h)."""
        xs = [np.ascontiguousarray(x, np.float32) for x in xs]
        lens = np.array([x.shape[0] for x in xs], np.int32)
        x = np.concatenate(xs, axis=0)
        out = np.zeros((int(lens.sum()), 512), np.float32)
        self._check(self.L.kk_bilstm_forward(self.h, prefix.encode(), len(xs), _ptr(lens, _i32p), x.shape[1],
                                             _ptr(x), _ptr(out)))
        return np.split(out, np.cumsum(lens)[:-1])

    def duration_encoder(self, xs: Sequence[np.ndarray], styles: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_duration_encoder_forward: xs[b] [N_b, 512], styles[b] [128] ->
        [N_b, 640] each."""
        xs = [np.ascontiguousarray(x, np.float32) for x in xs]
        lens = np.array([x.shape[0] for x in xs], np.int32)
        x = np.concatenate(xs, axis=0)
        st = np.ascontiguousarray(np.stack(styles), np.float32)
        out = np.zeros((int(lens.sum()), 640), np.float32)
        self._check(self.L.kk_duration_encoder_forward(self.h, len(xs), _ptr(lens, _i32p), _ptr(x), _ptr(st),
                                                       _ptr(out)))
        return np.split(out, np.cumsum(lens)[:-1])

    def prosody_f0n(self, ens: Sequence[np.ndarray], styles: Sequence[np.ndarray]):
        """kk_prosody_f0n: ens[b] [T_b, 640] (aligned duration-encoder
        output), styles[b] [128] -> (f0 [2 T_b], n [2 T_b]) per utterance."""
        ens = [np.ascontiguousarray(e, np.float32) for e in ens]
        lens = np.array([e.shape[0] for e in ens], np.int32)
        en = np.concatenate(ens, axis=0)
        st = np.ascontiguousarray(np.stack(styles), np.float32)
        f0 = np.zeros(2 * int(lens.sum()), np.float32)
        nn = np.zeros(2 * int(lens.sum()), np.float32)
        self._check(self.L.kk_prosody_f0n(self.h, len(ens), _ptr(lens, _i32p), _ptr(en), _ptr(st), _ptr(f0),
                                          _ptr(nn)))
        cuts = np.cumsum(2 * lens)[:-1]
        return list(zip(np.split(f0, cuts), np.split(nn, cuts)))

    def prosody_f0n_device(self, lens: np.ndarray, en_ptr: int, style_ptr: int, f0_ptr: int, n_ptr: int,
                           stream: int = 0) -> None:
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_prosody_f0n_device(self.h, len(lens), _ptr(lens, _i32p), en_ptr, style_ptr, f0_ptr,
                                                 n_ptr, stream))

    def duration_encoder_device(self, lens: np.ndarray, x_ptr: int, style_ptr: int, out_ptr: int,
                                stream: int = 0) -> None:
        """kk_duration_encoder_forward_device on device pointers (asynchronous)."""
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_duration_encoder_forward_device(self.h, len(lens), _ptr(lens, _i32p), x_ptr,
                                                              style_ptr, out_ptr, stream or None))

    def text_encoder(self, ids: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_text_encoder_forward: ids[b] int32 [N_b] -> [N_b, 512] each
        (the text encoder's biLSTM output)."""
        ids = [np.ascontiguousarray(i, np.int32) for i in ids]
        lens = np.array([len(i) for i in ids], np.int32)
        flat = np.concatenate(ids) if ids else np.zeros(0, np.int32)
        out = np.zeros((int(lens.sum()), 512), np.float32)
        self._check(self.L.kk_text_encoder_forward(self.h, len(ids), _ptr(lens, _i32p), _ptr(flat, _i32p),
                                                   _ptr(out)))
        return np.split(out, np.cumsum(lens)[:-1])

    def text_encoder_device(self, lens: np.ndarray, ids_ptr: int, out_ptr: int, stream: int = 0) -> None:
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_text_encoder_forward_device(self.h, len(lens), _ptr(lens, _i32p), ids_ptr, out_ptr,
                                                          stream))

    def albert(self, ids: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_albert_forward: ids[b] int32 [N_b] -> [N_b, 512] each (ALBERT +
        bert_encoder, the duration encoder's input)."""
        ids = [np.ascontiguousarray(i, np.int32) for i in ids]
        lens = np.array([len(i) for i in ids], np.int32)
        out = np.zeros((int(lens.sum()), 512), np.float32)
        self._check(self.L.kk_albert_forward(self.h, len(ids), _ptr(lens, _i32p), _ptr(np.concatenate(ids), _i32p),
                                             _ptr(out)))
        return np.split(out, np.cumsum(lens)[:-1])

    def albert_device(self, lens: np.ndarray, ids_ptr: int, out_ptr: int, stream: int = 0) -> None:
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_albert_forward_device(self.h, len(lens), _ptr(lens, _i32p), ids_ptr, out_ptr, stream))

    def duration_head(self, ds: Sequence[np.ndarray]) -> List[np.ndarray]:
        """kk_duration_head_forward: ds[b] [N_b, 640] (duration encoder
        output) -> durations [N_b] each."""
        ds = [np.ascontiguousarray(d, np.float32) for d in ds]
        lens = np.array([d.shape[0] for d in ds], np.int32)
        out = np.zeros(int(lens.sum()), np.float32)
        self._check(self.L.kk_duration_head_forward(self.h, len(ds), _ptr(lens, _i32p), _ptr(np.concatenate(ds)),
                                                    _ptr(out)))
        return np.split(out, np.cumsum(lens)[:-1])

    def duration_head_device(self, lens: np.ndarray, d_ptr: int, out_ptr: int, stream: int = 0) -> None:
        lens = np.ascontiguousarray(lens, np.int32)
        self._check(self.L.kk_duration_head_forward_device(self.h, len(lens), _ptr(lens, _i32p), d_ptr, out_ptr,
                                                           stream))

    def duration_proj(self, h: np.ndarray) -> np.ndarray:
        """kk_duration_proj: the predictor biLSTM output [N, 512] -> durations [N]."""
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros(h.shape[0], np.float32)
        self._check(self.L.kk_duration_proj(self.h, h.shape[0], _ptr(h), _ptr(out)))
        return out

    def align_durations(self, durations: np.ndarray, speed: float, hidden: Optional[np.ndarray] = None):
        """kk_align_durations: (frames int32 [n], total, en [total, D] or None)."""
        d = np.ascontiguousarray(durations, np.float32)
        n = len(d)
        frames = np.zeros(max(n, 1), np.int32)
        total = ctypes.c_int64(0)
        if hidden is None:
            self._check(self.L.kk_align_durations(self.h, n, _ptr(d), speed, _ptr(frames, _i32p),
                                                  ctypes.byref(total), None, 0, None, 0))
            return frames[:n], total.value, None
        hidden = np.ascontiguousarray(hidden, np.float32)
        cap = 50 * max(n, 1)
        en = np.zeros((cap, hidden.shape[1]), np.float32)
        self._check(self.L.kk_align_durations(self.h, n, _ptr(d), speed, _ptr(frames, _i32p), ctypes.byref(total),
                                              _ptr(hidden), hidden.shape[1], _ptr(en), cap))
        return frames[:n], total.value, en[: total.value]


class Queue:
    """kk_queue: batches decoder chunks from any number of threads onto the
    workers (one per Context, or `n_workers` calling `executor`). A chunk is
    a workload.Utterance-like object (asr [T, 512] time-fastest as in
    workload.pack, f0, noise, style); results come back by ticket."""

    def __init__(self, contexts: Optional[Sequence["Context"]] = None, executor=None, n_workers: int = 1,
                 max_batch: int = 64, max_batch_frames: int = 64 * 800, max_wait_us: int = 2000):
        self.L = load_library()
        self.h = ctypes.c_void_p()
        self._keep = {}
        self._lock = threading.Lock()
        if contexts is not None:
            arr = (ctypes.c_void_p * len(contexts))(*[c.h.value for c in contexts])
            rc = self.L.kk_queue_create(arr, len(contexts), max_batch, max_batch_frames, max_wait_us,
                                        ctypes.byref(self.h))
        else:
            def call(user, n, T, asr, f0, noise, style, audio):
                try:
                    t = np.ctypeslib.as_array(T, shape=(n,)).copy()
                    fr = int(t.sum())
                    return int(executor(t, np.ctypeslib.as_array(asr, shape=(fr * 512,)),
                                        np.ctypeslib.as_array(f0, shape=(2 * fr,)),
                                        np.ctypeslib.as_array(noise, shape=(2 * fr,)),
                                        np.ctypeslib.as_array(style, shape=(n * 128,)),
                                        np.ctypeslib.as_array(audio, shape=(600 * fr,))))
                except Exception:
                    return 5
            self._fn = QUEUE_EXEC_FN(call)
            rc = self.L.kk_queue_create_exec(self._fn, None, n_workers, max_batch, max_batch_frames, max_wait_us,
                                             ctypes.byref(self.h))
        if rc != 0:
            raise KKError(rc, self.L.kk_queue_last_error().decode())

    def submit(self, request: int, u, out: Optional[np.ndarray] = None) -> int:
        """Queues chunk u; `out` (float32, 600 T samples) receives its audio,
        a new array when not given."""
        asr = np.ascontiguousarray(u.asr, np.float32)
        f0 = np.ascontiguousarray(u.f0, np.float32)
        noise = np.ascontiguousarray(u.noise, np.float32)
        style = np.ascontiguousarray(u.style, np.float32)
        if out is not None:
            if out.dtype != np.float32 or not out.flags.c_contiguous or out.size != 600 * int(u.T):
                raise KKError(KK_ERROR_INVALID_ARGUMENT, "out must be contiguous float32 of 600 T samples")
            audio = out
        else:
            audio = np.zeros(600 * int(u.T), np.float32)
        ticket = ctypes.c_uint64()
        with self._lock:
            rc = self.L.kk_queue_submit(self.h, request, int(u.T), _ptr(asr), _ptr(f0), _ptr(noise), _ptr(style),
                                        _ptr(audio), ctypes.byref(ticket))
            if rc != 0:
                raise KKError(rc, self.L.kk_queue_last_error().decode())
            self._keep[ticket.value] = (asr, f0, noise, style, audio)
        return ticket.value

    def wait(self, ticket: int, timeout_ms: int = -1):
        """(result, audio): result 0 (audio valid), a KK_ERROR_* code,
        QUEUE_CANCELLED, or QUEUE_PENDING on timeout (audio None)."""
        rc = self.L.kk_queue_wait(self.h, ticket, timeout_ms)
        if rc == QUEUE_PENDING:
            return rc, None
        with self._lock:
            bufs = self._keep.pop(ticket, None)
        if rc == 1 and bufs is None:
            raise KKError(rc, self.L.kk_queue_last_error().decode())
        return rc, (bufs[4] if bufs is not None and rc == 0 else None)

    def cancel(self, request: int) -> int:
        n = ctypes.c_int32()
        self.L.kk_queue_cancel(self.h, request, ctypes.byref(n))
        return n.value

    def stats(self):
        b, j, m = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self.L.kk_queue_stats(self.h, ctypes.byref(b), ctypes.byref(j), ctypes.byref(m))
        return {"batches": b.value, "jobs": j.value, "max_batch": m.value}

    def close(self):
        if self.h:
            self.L.kk_queue_destroy(self.h)
            self.h = ctypes.c_void_p()


class Stream:
    """kk_stream: one request's chunks through a Queue, returned in order,
    post-processed and crossfaded as the reference's stream_synthesize
    does. push() takes a workload.Utterance-like chunk; next() returns
    (status, samples or None, chunk index)."""

    def __init__(self, queue: "Queue", cfg: Optional[StreamConfig] = None):
        self.L = load_library()
        self.q = queue
        self.cfg = cfg if cfg is not None else StreamConfig.preset(0)
        self.h = ctypes.c_void_p()
        rc = self.L.kk_stream_create(queue.h, ctypes.byref(self.cfg), ctypes.byref(self.h))
        if rc != 0:
            raise KKError(rc, self.L.kk_queue_last_error().decode())

    def push(self, u, boundary_after: int = BOUNDARY_NONE, is_last: bool = False) -> None:
        a = [np.ascontiguousarray(x, np.float32) for x in (u.asr, u.f0, u.noise, u.style)]
        rc = self.L.kk_stream_push(self.h, int(u.T), *[_ptr(x) for x in a], boundary_after, int(is_last))
        if rc != 0:
            raise KKError(rc, self.L.kk_queue_last_error().decode())

    def next(self, timeout_ms: int = -1):
        p = _f32p()
        n = ctypes.c_int64()
        idx = ctypes.c_int32()
        rc = self.L.kk_stream_next(self.h, timeout_ms, ctypes.byref(p), ctypes.byref(n), ctypes.byref(idx))
        if rc == 0:
            out = np.ctypeslib.as_array(p, shape=(n.value,)).copy() if n.value else np.zeros(0, np.float32)
            return rc, out, idx.value
        if rc == 1:
            raise KKError(rc, self.L.kk_queue_last_error().decode())
        return rc, None, idx.value

    def cancel(self) -> None:
        self.L.kk_stream_cancel(self.h)

    def close(self) -> None:
        if self.h:
            self.L.kk_stream_destroy(self.h)
            self.h = ctypes.c_void_p()
