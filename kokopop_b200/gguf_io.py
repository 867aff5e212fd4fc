"""GGUF files in the Kokoro converter's layout, for kk_weights_upload.

The reference ships its weights as a GGUF v3 file written by
tools/convert_kokoro_to_gguf.py and loads it with src/model/model.cpp. This
module writes and reads that layout with the `gguf` package, so that a
weight set can travel as the same kind of file the reference loads:

* tensor data in ggml order: a numpy array of shape (ne[n-1], ..., ne[0]),
  dims written reversed (convert_kokoro_to_gguf.py:274-276); F16 tensors as
  IEEE half, F32 as float (the converter's F16 / F32 policy is the caller's,
  kokopop_b200.workload applies it);
* physical tensor names: a logical name of 64 bytes or more, or one already
  used, is stored as "kt." + the 12-byte BLAKE2s hex digest of the logical
  name (convert_kokoro_to_gguf.py:389-407), and the two string arrays
  kokopop.tensor.logical_names / kokopop.tensor.physical_names record the
  mapping (:456-459; voice tensors keep their name and are not listed);
* metadata: kokopop.kokoro.version = 4 (the loader's gate,
  src/arch/kokoro/kokoro_arch.cpp:230-233), kokopop.arch = "kokoro-82m",
  kokopop.mock = false, kokopop.sample_rate = 24000 and the other keys of
  convert_kokoro_to_gguf.py:757-779 that do not need the original checkpoint.

read_kokoro_gguf is the loader's side: it applies the version gate and the
tensor-type gate (F32 / F16 for this path; model.cpp:390-401 also admits
quantised types, which the B200 path does not take) and maps physical names
back to logical ones (model.cpp:371-379).
"""
from __future__ import annotations

import hashlib
from typing import Dict, Iterable, Optional

import numpy as np

from .workload import Tensor

KOKORO_GGUF_VERSION = 4
ARCH = "kokoro-82m"
NAME_LIMIT = 64  # bytes; longer (or repeated) logical names are hashed


def physical_name(logical: str, used: set) -> str:
    """The converter's physical name for `logical` (registers it in used)."""
    if len(logical.encode("utf-8")) < NAME_LIMIT and logical not in used:
        used.add(logical)
        return logical
    physical = "kt." + hashlib.blake2s(logical.encode("utf-8"), digest_size=12).hexdigest()
    if physical in used:
        raise ValueError(f"tensor name hash collision for {logical}")
    used.add(physical)
    return physical


def write_kokoro_gguf(path: str, weights: Dict[str, Tensor], vocab: Optional[Iterable[str]] = None,
                      voices: Iterable[str] = (), extra_u32: Optional[Dict[str, int]] = None) -> Dict[str, str]:
    """Writes `weights` (logical name -> Tensor) to `path`; returns the
    logical -> physical name map."""
    import gguf

    w = gguf.GGUFWriter(path, arch=ARCH)
    w.add_uint32("kokopop.kokoro.version", KOKORO_GGUF_VERSION)
    w.add_bool("kokopop.mock", False)
    w.add_uint32("kokopop.sample_rate", 24000)
    w.add_string("kokopop.arch", ARCH)
    w.add_string("kokopop.tensor_layout", "runtime-v3")
    w.add_string("kokopop.quantization", "f16")
    w.add_array("tokenizer.ggml.tokens", list(vocab) if vocab is not None else ["$"] + [f"t{i}" for i in range(1, 178)])
    w.add_array("kokopop.voices", list(voices) if voices else ["af_synthetic"])
    for k, v in (extra_u32 or {}).items():
        w.add_uint32(k, int(v))
    used: set = set()
    mapping: Dict[str, str] = {}
    logical, physical = [], []
    for name, t in weights.items():
        p = physical_name(name, used)
        mapping[name] = p
        logical.append(name)
        physical.append(p)
        data = np.ascontiguousarray(t.data)
        if data.dtype not in (np.float32, np.float16):
            raise ValueError(f"{name}: only F32 / F16 tensors are written")
        expect = tuple(int(v) for v in t.ne[::-1])
        w.add_tensor(p, data.reshape(expect))
    w.add_array("kokopop.tensor.logical_names", logical)
    w.add_array("kokopop.tensor.physical_names", physical)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return mapping


def _field(reader, key):
    f = reader.get_field(key)
    return None if f is None else f.contents()


def read_kokoro_gguf(path: str) -> Dict[str, Tensor]:
    """Reads a Kokoro GGUF: version and type gates, physical -> logical
    names. Returns logical name -> Tensor (data copied out of the file)."""
    import gguf

    r = gguf.GGUFReader(path)
    version = _field(r, "kokopop.kokoro.version")
    if version != KOKORO_GGUF_VERSION:
        raise ValueError(f"unsupported Kokoro GGUF version {version} (want {KOKORO_GGUF_VERSION})")
    arch = _field(r, "kokopop.arch")
    if arch != ARCH:
        raise ValueError(f"not a {ARCH} GGUF: kokopop.arch = {arch!r}")
    logical = _field(r, "kokopop.tensor.logical_names") or []
    physical = _field(r, "kokopop.tensor.physical_names") or []
    to_logical = dict(zip(physical, logical)) if len(logical) == len(physical) else {}
    out: Dict[str, Tensor] = {}
    for t in r.tensors:
        name = to_logical.get(t.name, t.name)
        if t.tensor_type == gguf.GGMLQuantizationType.F32:
            dt = np.float32
        elif t.tensor_type == gguf.GGMLQuantizationType.F16:
            dt = np.float16
        else:
            raise ValueError(f"{name}: tensor type {t.tensor_type.name} is not F32 / F16")
        ne = tuple(int(v) for v in t.shape)
        data = np.array(t.data, dtype=dt, copy=True).reshape(ne[::-1])
        out[name] = Tensor(name, ne, np.ascontiguousarray(data))
    return out
