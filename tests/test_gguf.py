"""GGUF files in the reference converter's layout (kokopop_b200.gguf_io):
write, read back, name hashing and the loader's gates, on CPU; on the GPU,
weights loaded from the file give the same audio, bit for bit, as the
in-memory weight set they were written from."""
import hashlib

import numpy as np
import pytest

from kokopop_b200 import gguf_io as G
from kokopop_b200 import workload as W


@pytest.fixture(scope="module")
def decoder_file(tmp_path_factory):
    ws = W.config2_weights()
    path = str(tmp_path_factory.mktemp("gguf") / "kokoro-decoder.gguf")
    mapping = G.write_kokoro_gguf(path, ws)
    return ws, path, mapping


def test_round_trip_is_bit_exact(decoder_file):
    ws, path, _ = decoder_file
    back = G.read_kokoro_gguf(path)
    assert set(back) == set(ws)
    for name, t in ws.items():
        b = back[name]
        assert b.ne == tuple(t.ne) and b.data.dtype == t.data.dtype, name
        np.testing.assert_array_equal(b.data.view(np.uint8), np.ascontiguousarray(t.data).view(np.uint8))


def test_long_and_repeated_names_are_hashed_like_the_converter():
    """convert_kokoro_to_gguf.py:389-407: 64 bytes or more (or a name used
    before) -> "kt." + BLAKE2s-96 hex digest of the logical name."""
    used = set()
    short = "kokopop.decoder.F0_conv.bias"
    assert G.physical_name(short, used) == short
    long_name = "kokopop.albert.encoder.albert_layer_groups.0.albert_layers.0.attention.dense.weight"
    want = "kt." + hashlib.blake2s(long_name.encode(), digest_size=12).hexdigest()
    assert G.physical_name(long_name, used) == want
    exactly_64 = "x" * 64
    assert G.physical_name(exactly_64, used).startswith("kt.")
    assert G.physical_name("y" * 63, used) == "y" * 63
    assert G.physical_name(short, used) == "kt." + hashlib.blake2s(short.encode(), digest_size=12).hexdigest()


def test_front_end_names_map_back_to_logical(tmp_path):
    ws = W.albert_weights(f16=True)
    path = str(tmp_path / "albert.gguf")
    mapping = G.write_kokoro_gguf(path, ws)
    hashed = {k: v for k, v in mapping.items() if k != v}
    assert len(hashed) >= 10 and all(v.startswith("kt.") for v in hashed.values())
    import gguf
    r = gguf.GGUFReader(path)
    stored = {t.name for t in r.tensors}
    assert set(hashed.values()) <= stored and not (set(hashed) & stored)
    assert r.get_field("kokopop.kokoro.version").contents() == 4
    assert r.get_field("kokopop.arch").contents() == "kokoro-82m"
    back = G.read_kokoro_gguf(path)
    assert set(back) == set(ws)


def test_loader_gates(tmp_path):
    """The version gate (kokoro_arch.cpp:230-233) and the F32 / F16 type gate."""
    import gguf
    p3 = str(tmp_path / "v3.gguf")
    w = gguf.GGUFWriter(p3, arch="kokoro-82m")
    w.add_uint32("kokopop.kokoro.version", 3)
    w.add_string("kokopop.arch", "kokoro-82m")
    w.add_tensor("kokopop.decoder.F0_conv.bias", np.zeros(1, np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="version"):
        G.read_kokoro_gguf(p3)
    pi = str(tmp_path / "int.gguf")
    w = gguf.GGUFWriter(pi, arch="kokoro-82m")
    w.add_uint32("kokopop.kokoro.version", 4)
    w.add_string("kokopop.arch", "kokoro-82m")
    w.add_tensor("kokopop.decoder.F0_conv.bias", np.zeros(4, np.int32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="F32 / F16"):
        G.read_kokoro_gguf(pi)
    with pytest.raises(ValueError, match="only F32 / F16"):
        G.write_kokoro_gguf(str(tmp_path / "bad.gguf"),
                            {"a": W.Tensor("a", (2,), np.zeros(2, np.int32))})


@pytest.mark.gpu
def test_gguf_loaded_weights_give_identical_audio(decoder_file):
    import kokopop_b200 as kb
    ws, path, _ = decoder_file
    utts = [W.make_utterance(np.random.default_rng(61), t) for t in (25, 3, 60)]
    c = kb.Context(0)
    try:
        c.upload(ws)
        want = c.decoder_forward(utts)
        c.upload(G.read_kokoro_gguf(path))
        got = c.decoder_forward(utts)
    finally:
        c.close()
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)
