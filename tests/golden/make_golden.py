"""Generates the golden fixtures in tests/golden/.

  istft_ref.npz   seeded Kokoro post tensors and the iSTFT output of the
                  reference's own src/audio/istft.cpp (compiled unchanged into
                  oracle/_ref/ by oracle/Makefile), incl. the 3-frame known
                  answer of tests/test_audio_utils.cpp:371-399
  lstm_ref.npz    the deterministic inputs of tests/test_lstm_fused.cpp:64-73
                  (H=33, N=9, forward and reverse) plus a seeded H=64 case,
                  with outputs of the reference's own lstm_fused.cpp
  harmonic_ref.npz  seeded F0 curves (voiced, unvoiced spans, all unvoiced)
                  with the harmonic source and its STFT from the reference's
                  own fill_harmonic_stft (src/arch/kokoro/audio_utils.cpp,
                  compiled unchanged), which calls the C library's float
                  sin / cos / tanh / atan2
  align_ref.npz   edge-case durations at several speeds with the frame counts
                  of the reference's duration_to_frames and the mask of its
                  build_duration_mask (src/arch/kokoro/kokoro.cpp)
  vocos_ref.npz   seeded frame-major spectra with the output of the
                  reference's istft() (its radix-2 path at n_fft 1024 / hop
                  256, and n_fft 64), the reference's DC blocker
                  (src/arch/sanotts/sano_vocos.cpp) on a seeded signal, and
                  its DC / Nyquist bin mask
  oracle_small.npz  regression vectors of the oracle itself (decoder + generator
                  at T=3 for the F32 and F16 weight sets); these are NOT
                  reference outputs (the reference's generator needs ggml,
                  which is absent), they pin the restatement against drift.

Run from the repository root with the reference tree present:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from kokopop_b200 import workload as W  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def lstm_inputs(H, N):
    i = np.arange(4 * H * N, dtype=np.float32)
    pre = (np.float32(0.17) * np.sin(i * np.float32(0.37)) + np.float32(0.05) * np.cos(i * np.float32(0.11)))
    j = np.arange(4 * H * H, dtype=np.float32)
    w_hh = np.float32(0.08) * np.sin(j * np.float32(0.19))
    k = np.arange(4 * H, dtype=np.float32)
    b_hh = np.float32(0.03) * np.cos(k * np.float32(0.23))
    # w_hh is ggml [H, 4H] (w[k + H*j]); the rowwise copy has the same layout
    return pre.astype(np.float32).reshape(N, 4 * H), w_hh.astype(np.float32).reshape(4 * H, H), b_hh.astype(np.float32)


def main():
    if not O.ref_available():
        O.build()
    rng = np.random.default_rng(7)
    ist = {}
    known = np.full((22, 3), -20.0, np.float32)
    known[1, :] = 0.0
    known[11:, :] = 0.0
    ist["known_post"] = known
    ist["known_audio"] = O.ref_istft(known)
    for n in (2, 3, 17, 50):
        post = rng.normal(0.0, 2.0, size=(22, n)).astype(np.float32)
        ist[f"post_{n}"] = post
        ist[f"audio_{n}"] = O.ref_istft(post)
    np.savez_compressed(os.path.join(OUT, "istft_ref.npz"), **ist)

    ls = {}
    for rev in (0, 1):
        pre, w, b = lstm_inputs(33, 9)
        ls[f"h33_pre"], ls[f"h33_w"], ls[f"h33_b"] = pre, w, b
        ls[f"h33_out_{rev}"] = O.ref_lstm_direction(pre, w, b, bool(rev))
    pre = rng.normal(0.0, 3.0, size=(12, 256)).astype(np.float32)
    w = rng.uniform(-0.5, 0.5, size=(256, 64)).astype(np.float32)
    b = rng.uniform(-1 / 16, 1 / 16, size=256).astype(np.float32)
    ls["h64_pre"], ls["h64_w"], ls["h64_b"] = pre, w, b
    ls["h64_out_0"] = O.ref_lstm_direction(pre, w, b, False)
    ls["h64_out_1"] = O.ref_lstm_direction(pre, w, b, True)
    np.savez_compressed(os.path.join(OUT, "lstm_ref.npz"), **ls)

    wts = W.config0_weights()
    mw = wts["kokopop.decoder.generator.m_source.l_linear.weight"].data.astype(np.float32).ravel()
    mb = float(wts["kokopop.decoder.generator.m_source.l_linear.bias"].data.ravel()[0])
    hs = {"merge_w": mw, "merge_b": np.float32(mb)}
    curves = {
        "voiced": W.make_utterance(np.random.default_rng(31), 8).f0,
        "gaps": np.array([0, 0, 180, 181.5, 0, 95, 300, 300, 12, 0, 250, 251], np.float32),
        "unvoiced": np.zeros(6, np.float32),
    }
    for k, f0 in curves.items():
        f0 = np.ascontiguousarray(f0, np.float32)
        har, src = O.ref_harmonic_stft(f0, 60 * len(f0) + 1, mw, mb)
        hs[f"f0_{k}"], hs[f"har_{k}"], hs[f"src_{k}"] = f0, har, src
    np.savez_compressed(os.path.join(OUT, "harmonic_ref.npz"), **hs)

    edge = np.array([0.0, 0.4, 0.5, 1.5, 2.5, 2.5000002, 3.49, 49.5, 50.5, 1e9, np.inf, -np.inf, np.nan, -3.0,
                     3e9, 1e30, -1e30, 0.49999997, 7.5, 8.5], np.float32)
    dur = np.concatenate([edge, np.random.default_rng(17).uniform(0.0, 30.0, 60).astype(np.float32)])
    al = {"durations": dur}
    for i, sp in enumerate((1.0, 2.0, 0.7, -1.0, float("nan"), float("inf"), 0.0)):
        al[f"speed_{i}"] = np.float32(sp)
        al[f"frames_{i}"] = O.ref_duration_frames(dur, sp)
    al["mask_frames"] = al["frames_0"][:24]
    al["mask"] = O.ref_duration_mask(al["mask_frames"])
    np.savez_compressed(os.path.join(OUT, "align_ref.npz"), **al)

    vs = {}
    for F, n, hop in ((5, 1024, 256), (3, 64, 16)):
        bins = n // 2 + 1
        re = rng.normal(0.0, 1.0, size=(F, bins)).astype(np.float32)
        im = rng.normal(0.0, 1.0, size=(F, bins)).astype(np.float32)
        vs[f"re_{n}"], vs[f"im_{n}"] = re, im
        vs[f"hop_{n}"] = np.int32(hop)
        vs[f"audio_{n}"] = O.ref_istft_complex(re, im, n, hop)
    x = rng.normal(0.0, 1.0, size=3000).astype(np.float32)
    vs["dc_in"], vs["dc_out"] = x, O.ref_dc_block(x, 0.9973)
    vs["mask_513"] = O.ref_bin_mask(513)
    np.savez_compressed(os.path.join(OUT, "vocos_ref.npz"), **vs)

    # streaming: raw chunks (a tone between near-silent stretches) through
    # the reference's postprocess_chunk_audio + apply_crossfade_smart, as
    # postprocess_and_crossfade composes them, for both presets
    import kokopop_b200 as kb
    srng = np.random.default_rng(23)
    lens = [600 * T for T in (4, 2, 6, 3, 5)]
    raws = []
    for n in lens:
        lead, trail = int(srng.integers(0, n // 3)), int(srng.integers(0, n // 3))
        body = n - lead - trail
        tone = (0.3 * np.sin(0.013 * np.arange(body)) * (0.5 + 0.5 * srng.random(body))).astype(np.float32)
        quiet = lambda k: (0.009 * (srng.random(k) * 2 - 1)).astype(np.float32)
        raws.append(np.concatenate([quiet(lead), tone, quiet(trail)]).astype(np.float32))
    bounds = np.array([1, 0, 3, 2, 5], np.int32)
    st = {"raw": np.concatenate(raws), "lens": np.array(lens, np.int64), "bounds": bounds}
    for mode in (0, 1):
        cfg = kb.StreamConfig.preset(mode)
        outs = O.ref_stream(raws, [int(b) for b in bounds], cfg)
        st[f"out_{mode}"] = np.concatenate(outs)
        st[f"out_lens_{mode}"] = np.array([len(o) for o in outs], np.int64)
    np.savez_compressed(os.path.join(OUT, "stream_ref.npz"), **st)

    sm = {}
    u = W.make_utterance(np.random.default_rng(11), 3)
    sm["asr"], sm["f0"], sm["noise"], sm["style"] = u.asr, u.f0, u.noise, u.style
    for tag, wts in (("f32", W.config0_weights()), ("f16", W.config2_weights())):
        m = O.OracleModel(wts)
        sm[f"audio_{tag}"] = m.decoder_forward(u.asr, u.f0, u.noise, u.style)
    np.savez_compressed(os.path.join(OUT, "oracle_small.npz"), **sm)
    print("wrote", sorted(os.listdir(OUT)))


if __name__ == "__main__":
    main()
