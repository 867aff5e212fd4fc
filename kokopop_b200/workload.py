"""Synthetic Kokoro-82M weights and inputs for the hot path.

No checkpoint or dataset is available, so every run uses seeded random-init
weights with the real Kokoro-82M tensor names and shapes, and seeded inputs
with the shapes and value ranges the workloads specify:

  * weights are laid out exactly as the reference's converter writes them
    (tools/convert_kokoro_to_gguf.py): dims reversed to ggml order, regular
    Conv1d weights reshaped [OC, IC, K] -> [OC, IC*K] (:67-84, :376-378),
    ConvTranspose (``.ups.``) and ``.pool.`` kept 3-D (:112-116), AdaIN ``fc``
    split into ``.fc.gamma.*`` / ``.fc.beta.*`` (:502-509), LSTMs in PyTorch
    packed gate order i, f, g, o (:479-499);
  * F16 models follow the converter's type policy (:140-177): tensors of two
    or more dims become F16, 1-D tensors and Snake ``.alpha*`` stay F32.

Shapes come from the Kokoro-82M module definitions (ISTFTNet generator:
upsample rates 10/6, kernels 20/12, initial channels 512, resblock kernels
3/7/11 with dilations 1/3/5, n_fft 20, hop 5; decoder: AdainResBlk1d encode
514->1024, decode 1090->1024 x3 and 1090->512 with upsample; prosody duration
encoder: 3 x (biLSTM 640->2x256 + AdaLayerNorm(128, 512))).
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Sequence, Tuple

import numpy as np

STYLE_DIM = 128
HIDDEN = 512          # decoder input channels (asr features)
GEN_CH = (256, 128)   # generator channels after ups.0 / ups.1
RES_KERNELS = (3, 7, 11)

F32 = 0
F16 = 1


@dataclasses.dataclass
class Tensor:
    name: str
    ne: Tuple[int, ...]   # ggml order, ne[0] fastest
    data: np.ndarray      # float32 or float16, C-contiguous, shape = ne[::-1]

    @property
    def dtype(self) -> int:
        return F16 if self.data.dtype == np.float16 else F32


def _adain(prefix: str, channels: int) -> List[Tuple[str, Tuple[int, ...]]]:
    return [
        (f"{prefix}.norm.weight", (channels,)),
        (f"{prefix}.norm.bias", (channels,)),
        (f"{prefix}.fc.gamma.weight", (STYLE_DIM, channels)),
        (f"{prefix}.fc.gamma.bias", (channels,)),
        (f"{prefix}.fc.beta.weight", (STYLE_DIM, channels)),
        (f"{prefix}.fc.beta.bias", (channels,)),
    ]


def _gen_resblock(prefix: str, ch: int, k: int) -> List[Tuple[str, Tuple[int, ...]]]:
    out: List[Tuple[str, Tuple[int, ...]]] = []
    for i in range(3):
        out += [
            (f"{prefix}.convs1.{i}.weight", (ch * k, ch)),
            (f"{prefix}.convs1.{i}.bias", (ch,)),
            (f"{prefix}.convs2.{i}.weight", (ch * k, ch)),
            (f"{prefix}.convs2.{i}.bias", (ch,)),
            (f"{prefix}.alpha1.{i}", (1, ch, 1)),
            (f"{prefix}.alpha2.{i}", (1, ch, 1)),
        ]
        out += _adain(f"{prefix}.adain1.{i}", ch)
        out += _adain(f"{prefix}.adain2.{i}", ch)
    return out


def _adain_resblk(prefix: str, cin: int, cout: int, upsample: bool) -> List[Tuple[str, Tuple[int, ...]]]:
    out = [
        (f"{prefix}.conv1.weight", (cin * 3, cout)),
        (f"{prefix}.conv1.bias", (cout,)),
        (f"{prefix}.conv2.weight", (cout * 3, cout)),
        (f"{prefix}.conv2.bias", (cout,)),
    ]
    out += _adain(f"{prefix}.norm1", cin)
    out += _adain(f"{prefix}.norm2", cout)
    if cin != cout:
        out.append((f"{prefix}.conv1x1.weight", (cin, cout)))
    if upsample:
        out += [(f"{prefix}.pool.weight", (3, 1, cin)), (f"{prefix}.pool.bias", (cin,))]
    return out


def decoder_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """Tensors read by the decoder encode/decode blocks and the generator."""
    p = "kokopop.decoder"
    g = f"{p}.generator"
    spec: List[Tuple[str, Tuple[int, ...]]] = [
        (f"{p}.F0_conv.weight", (3, 1)),
        (f"{p}.F0_conv.bias", (1,)),
        (f"{p}.N_conv.weight", (3, 1)),
        (f"{p}.N_conv.bias", (1,)),
        (f"{p}.asr_res.0.weight", (HIDDEN, 64)),
        (f"{p}.asr_res.0.bias", (64,)),
    ]
    spec += _adain_resblk(f"{p}.encode", HIDDEN + 2, 1024, False)
    for i in range(3):
        spec += _adain_resblk(f"{p}.decode.{i}", 1024 + 66, 1024, False)
    spec += _adain_resblk(f"{p}.decode.3", 1024 + 66, HIDDEN, True)
    spec += [
        (f"{g}.m_source.l_linear.weight", (9, 1)),
        (f"{g}.m_source.l_linear.bias", (1,)),
        (f"{g}.noise_convs.0.weight", (22 * 12, GEN_CH[0])),
        (f"{g}.noise_convs.0.bias", (GEN_CH[0],)),
        (f"{g}.noise_convs.1.weight", (22, GEN_CH[1])),
        (f"{g}.noise_convs.1.bias", (GEN_CH[1],)),
        (f"{g}.ups.0.weight", (20, GEN_CH[0], HIDDEN)),
        (f"{g}.ups.0.bias", (GEN_CH[0],)),
        (f"{g}.ups.1.weight", (12, GEN_CH[1], GEN_CH[0])),
        (f"{g}.ups.1.bias", (GEN_CH[1],)),
        (f"{g}.conv_post.weight", (GEN_CH[1] * 7, 22)),
        (f"{g}.conv_post.bias", (22,)),
    ]
    spec += _gen_resblock(f"{g}.noise_res.0", GEN_CH[0], 7)
    spec += _gen_resblock(f"{g}.noise_res.1", GEN_CH[1], 11)
    for s in range(2):
        for j, k in enumerate(RES_KERNELS):
            spec += _gen_resblock(f"{g}.resblocks.{s * 3 + j}", GEN_CH[s], k)
    return spec


def lstm_spec(prefix: str, in_dim: int, hidden: int = 256) -> List[Tuple[str, Tuple[int, ...]]]:
    out = []
    for sfx in ("", "_reverse"):
        out += [
            (f"{prefix}.weight_ih_l0{sfx}", (in_dim, 4 * hidden)),
            (f"{prefix}.weight_hh_l0{sfx}", (hidden, 4 * hidden)),
            (f"{prefix}.bias_ih_l0{sfx}", (4 * hidden,)),
            (f"{prefix}.bias_hh_l0{sfx}", (4 * hidden,)),
        ]
    return out


def duration_encoder_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """predictor.text_encoder: 3 x (biLSTM 640 -> 2x256, AdaLayerNorm(128, 512))."""
    p = "kokopop.predictor.text_encoder.lstms"
    spec: List[Tuple[str, Tuple[int, ...]]] = []
    for blk in range(3):
        spec += lstm_spec(f"{p}.{2 * blk}", HIDDEN + STYLE_DIM)
        spec += [
            (f"{p}.{2 * blk + 1}.fc.gamma.weight", (STYLE_DIM, HIDDEN)),
            (f"{p}.{2 * blk + 1}.fc.gamma.bias", (HIDDEN,)),
            (f"{p}.{2 * blk + 1}.fc.beta.weight", (STYLE_DIM, HIDDEN)),
            (f"{p}.{2 * blk + 1}.fc.beta.bias", (HIDDEN,)),
        ]
    return spec


def prosody_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """The prosody predictor's F0 / N chain (kokoro.cpp:669-708): the shared
    biLSTM 640 -> 2 x 256, then per branch AdainResBlk1d(512, 512),
    (512, 256, x2 upsample), (256, 256) and the 1x1 projection 256 -> 1."""
    p = "kokopop.predictor"
    spec: List[Tuple[str, Tuple[int, ...]]] = lstm_spec(f"{p}.shared", HIDDEN + STYLE_DIM)
    for br in ("F0", "N"):
        spec += _adain_resblk(f"{p}.{br}.0", HIDDEN, HIDDEN, False)
        spec += _adain_resblk(f"{p}.{br}.1", HIDDEN, HIDDEN // 2, True)
        spec += _adain_resblk(f"{p}.{br}.2", HIDDEN // 2, HIDDEN // 2, False)
        spec += [(f"{p}.{br}_proj.weight", (HIDDEN // 2, 1)), (f"{p}.{br}_proj.bias", (1,))]
    return spec


VOCAB = 178  # Kokoro's token vocabulary (pad 0, phonemes 1..177)


def text_encoder_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """The text encoder up to its biLSTM (graph_ops.cpp:1578-1624): the
    embedding [512, vocab], three k = 5 convs 512 -> 512 (weights stored 2-D,
    innermost IC * K, as the converter writes them) with their LayerNorm
    gamma / beta, and the biLSTM 512 -> 2 x 256."""
    p = "kokopop.text_encoder"
    spec: List[Tuple[str, Tuple[int, ...]]] = [(f"{p}.embedding.weight", (HIDDEN, VOCAB))]
    for i in range(3):
        spec += [
            (f"{p}.cnn.{i}.0.weight", (HIDDEN * 5, HIDDEN)),
            (f"{p}.cnn.{i}.0.bias", (HIDDEN,)),
            (f"{p}.cnn.{i}.1.gamma", (HIDDEN,)),
            (f"{p}.cnn.{i}.1.beta", (HIDDEN,)),
        ]
    spec += lstm_spec(f"{p}.lstm", HIDDEN)
    return spec


def duration_head_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """predictor.lstm (biLSTM 640 -> 2 x 256) and the duration projection
    512 -> 50 buckets (kokoro.cpp:343-355, :469-516)."""
    p = "kokopop.predictor"
    return lstm_spec(f"{p}.lstm", HIDDEN + STYLE_DIM) + [
        (f"{p}.duration_proj.linear_layer.weight", (HIDDEN, 50)),
        (f"{p}.duration_proj.linear_layer.bias", (50,)),
    ]


ALBERT_EMBED = 128
ALBERT_HIDDEN = 768
ALBERT_FFN = 2048
ALBERT_POSITIONS = 512


def albert_spec() -> List[Tuple[str, Tuple[int, ...]]]:
    """ALBERT (embed 128, hidden 768, one shared layer of 12 heads, FFN 2048)
    and bert_encoder 768 -> 512 (kokoro.cpp:52-81, :213-224)."""
    e = "kokopop.albert.embeddings"
    lay = "kokopop.albert.encoder.albert_layer_groups.0.albert_layers.0"
    E, H, F = ALBERT_EMBED, ALBERT_HIDDEN, ALBERT_FFN
    spec: List[Tuple[str, Tuple[int, ...]]] = [
        (f"{e}.word_embeddings.weight", (E, VOCAB)),
        (f"{e}.position_embeddings.weight", (E, ALBERT_POSITIONS)),
        (f"{e}.token_type_embeddings.weight", (E, 2)),
        (f"{e}.LayerNorm.weight", (E,)),
        (f"{e}.LayerNorm.bias", (E,)),
        ("kokopop.albert.encoder.embedding_hidden_mapping_in.weight", (E, H)),
        ("kokopop.albert.encoder.embedding_hidden_mapping_in.bias", (H,)),
        ("kokopop.bert_encoder.weight", (H, HIDDEN)),
        ("kokopop.bert_encoder.bias", (HIDDEN,)),
    ]
    for n in ("query", "key", "value", "dense"):
        spec += [(f"{lay}.attention.{n}.weight", (H, H)), (f"{lay}.attention.{n}.bias", (H,))]
    spec += [
        (f"{lay}.attention.LayerNorm.weight", (H,)),
        (f"{lay}.attention.LayerNorm.bias", (H,)),
        (f"{lay}.ffn.weight", (H, F)),
        (f"{lay}.ffn.bias", (F,)),
        (f"{lay}.ffn_output.weight", (F, H)),
        (f"{lay}.ffn_output.bias", (H,)),
        (f"{lay}.full_layer_layer_norm.weight", (H,)),
        (f"{lay}.full_layer_layer_norm.bias", (H,)),
    ]
    return spec


def albert_weights(f16: bool = False) -> Dict[str, Tensor]:
    """ALBERT + bert_encoder weights: seed 2, N(0, 0.02) (config 2's draw),
    F16 under the converter's policy when f16, else F32."""
    return make_weights(albert_spec(), seed=2, dist="normal", scale=0.02, f16=f16)


def frontend_weights(f16: bool = False) -> Dict[str, Tensor]:
    """Text encoder + duration head weights: seed 2, N(0, 0.02) (config 2's
    draw), F16 under the converter's policy when f16, else F32."""
    return make_weights(text_encoder_spec() + duration_head_spec(), seed=2, dist="normal", scale=0.02, f16=f16)


def config2_frontend_weights() -> Dict[str, Tensor]:
    """Config 2's front end up to the durations and t_en: ALBERT +
    bert_encoder, the duration encoder, the duration head and the text
    encoder, seed 2, N(0, 0.02), F16 under the converter's policy."""
    spec = albert_spec() + duration_encoder_spec() + duration_head_spec() + text_encoder_spec()
    return make_weights(spec, seed=2, dist="normal", scale=0.02, f16=True)


def token_ids(rng: np.random.Generator, n: int) -> np.ndarray:
    """n phoneme ids uniform over 1..177 wrapped in the pad id 0 (n + 2 ids)."""
    return np.concatenate([[0], rng.integers(1, VOCAB, size=n), [0]]).astype(np.int32)


def prosody_weights(f16: bool = False) -> Dict[str, Tensor]:
    """Prosody F0 / N chain weights: seed 2, N(0, 0.02) (config 2's
    draw), F16 under the converter's policy when f16, else F32."""
    return make_weights(prosody_spec(), seed=2, dist="normal", scale=0.02, f16=f16)


# --------------------------------------------------------------------------
# sanoTTS Vocos decoder
# --------------------------------------------------------------------------

# Tensor prefix of voice 0 in a sanoTTS GGUF (sano_arch.cpp:47).
VOCOS_PREFIX = "kokopop.sanotts.voice.0."

# The `heart` voice's decoder dimensions come from an upstream header
# (nano_q8_meta.h, read by tools/convert_sanotts_to_gguf.py:2226-2291) that
# is not available here; these stand in for them. n_fft 1024 / hop 256, the
# DC pole 0.9973 and mag_clip 100 are the converter's own values
# (:2362-2381), four noise channels the noise adapter's (sano_noise.h).
VOCOS_DIMS = dict(dim=256, blocks=8, pw_hidden=768, dw_kernel=7, embed_kernel=7, noise_ch=4, mels=80,
                  n_fft=1024, hop=256, dc_pole=0.9973, mag_clip=100.0)


def vocos_spec(prefix: str = VOCOS_PREFIX, dims: Dict = VOCOS_DIMS) -> List[Tuple[str, Tuple[int, ...]]]:
    """Tensor names and ggml shapes the loader expects (load_vocos,
    sano_arch.cpp:1138-1177)."""
    d = dims
    D, H, bins = d["dim"], d["pw_hidden"], d["n_fft"] // 2 + 1
    p = prefix + "dec."
    spec = [(p + "embed.weight", (d["mels"] * d["embed_kernel"], D)), (p + "embed.bias", (D,)),
            (p + "noise.weight", (d["noise_ch"] * d["embed_kernel"], D)), (p + "noise.bias", (D,)),
            (p + "norm.weight", (D,)), (p + "norm.bias", (D,)),
            (p + "final_norm.weight", (D,)), (p + "final_norm.bias", (D,)),
            (p + "head.weight", (D, 2 * bins)), (p + "head.bias", (2 * bins,))]
    for i in range(d["blocks"]):
        b = f"{p}blocks.{i}."
        spec += [(b + "dw.weight", (d["dw_kernel"], D)), (b + "dw.bias", (D,)), (b + "norm.weight", (D,)),
                 (b + "norm.bias", (D,)), (b + "pw0.weight", (D, H)), (b + "pw0.bias", (H,)),
                 (b + "pw1.weight", (H, D)), (b + "pw1.bias", (D,)), (b + "gamma", (D,))]
    return spec


def vocos_weights(f16: bool = False, seed: int = 3, prefix: str = VOCOS_PREFIX, dims: Dict = VOCOS_DIMS):
    """The Vocos decoder: seed 3, N(0, 0.02); the LayerNorm weights drawn
    around 1 (N(1, 0.02)) so that the normalised activations keep their
    scale. F32 (the configuration's), or F16 for the multi-dimensional
    tensors."""
    w = make_weights(vocos_spec(prefix, dims), seed=seed, dist="normal", scale=0.02, f16=f16)
    for name, t in w.items():
        if name.endswith("norm.weight"):
            t.data[...] = (t.data.astype(np.float32) + np.float32(1.0)).astype(t.data.dtype)
    return w


def vocos_inputs(rng: np.random.Generator, frames: int, dims: Dict = VOCOS_DIMS):
    """One chunk's mel features [mels, frames] ~ N(0, 1) and noise
    [noise_ch, frames] ~ N(0, 1) (time-fastest, the ggml [frames, C])."""
    mel = rng.normal(0.0, 1.0, size=(dims["mels"], frames)).astype(np.float32)
    noise = rng.normal(0.0, 1.0, size=(dims["noise_ch"], frames)).astype(np.float32)
    return mel, noise


def _is_f16_under_converter_policy(name: str, ne: Sequence[int]) -> bool:
    """_target_type (tools/convert_kokoro_to_gguf.py:140-177) for these tensors."""
    if len(ne) <= 1:
        return False
    if ".alpha" in name and ".weight" not in name:
        return False
    # embedding lookup tables stay F32 (indexed, never multiplied)
    if name.endswith(".weight") and (".embeddings." in name or ".embedding.weight" in name):
        return False
    return True


def make_weights(spec: Sequence[Tuple[str, Tuple[int, ...]]], seed: int, dist: str = "normal",
                 scale: float = 0.02, f16: bool = False) -> Dict[str, Tensor]:
    """Seeded random-init weights, drawn in sorted-name order.

    dist "normal": N(0, scale); dist "uniform": U(-scale, scale). Snake alphas
    are kept away from exactly 0 (the reference computes 1/alpha,
    graph_ops.cpp:425).
    """
    rng = np.random.default_rng(seed)
    out: Dict[str, Tensor] = {}
    for name, ne in sorted(spec):
        shape = tuple(reversed(ne))
        if dist == "normal":
            v = rng.normal(0.0, scale, size=shape).astype(np.float32)
        else:
            v = rng.uniform(-scale, scale, size=shape).astype(np.float32)
        if ".alpha" in name:
            v = np.where(np.abs(v) < 1e-6, np.float32(1e-6), v).astype(np.float32)
        if f16 and _is_f16_under_converter_policy(name, ne):
            v = v.astype(np.float16)
        out[name] = Tensor(name, tuple(ne), np.ascontiguousarray(v))
    return out


def config0_weights() -> Dict[str, Tensor]:
    """Decoder weights: seed 0, N(0, 0.02), all F32."""
    return make_weights(decoder_spec(), seed=0, dist="normal", scale=0.02, f16=False)


def config2_weights() -> Dict[str, Tensor]:
    """Decoder weights: seed 2, N(0, 0.02), F16 under the converter's policy."""
    return make_weights(decoder_spec(), seed=2, dist="normal", scale=0.02, f16=True)


def config1_weights(f16: bool = False) -> Dict[str, Tensor]:
    """Duration-encoder LSTM stack: seed 1, U(-1/16, 1/16)."""
    return make_weights(duration_encoder_spec(), seed=1, dist="uniform", scale=1.0 / 16.0, f16=f16)


# --------------------------------------------------------------------------
# inputs
# --------------------------------------------------------------------------

def f0_curve(rng: np.random.Generator, n: int) -> np.ndarray:
    """Smooth random walk in 80-300 Hz with ~20% of frames zeroed in
    contiguous spans (<= 10 Hz is unvoiced, audio_utils.cpp:179)."""
    f = np.empty(n, dtype=np.float64)
    v = rng.uniform(80.0, 300.0)
    for i in range(n):
        v += rng.normal(0.0, 3.0)
        if v < 80.0:
            v = 160.0 - v
        if v > 300.0:
            v = 600.0 - v
        f[i] = v
    zero = np.zeros(n, dtype=bool)
    target = int(round(0.2 * n))
    guard = 0
    while zero.sum() < target and guard < 10000:
        guard += 1
        span = int(rng.integers(3, max(4, min(30, n // 4 + 4))))
        start = int(rng.integers(0, max(1, n - span + 1)))
        zero[start:start + span] = True
    f[zero] = 0.0
    return f.astype(np.float32)


@dataclasses.dataclass
class Utterance:
    T: int                 # asr frames
    asr: np.ndarray        # [512, T] time-fastest (torch [1, 512, T])
    f0: np.ndarray         # [2T]
    noise: np.ndarray      # [2T]
    style: np.ndarray      # [128] decoder style


def make_utterance(rng: np.random.Generator, T: int, style_dim: int = STYLE_DIM) -> Utterance:
    asr = rng.normal(0.0, 1.0, size=(HIDDEN, T)).astype(np.float32)
    f0 = f0_curve(rng, 2 * T)
    noise = rng.normal(0.0, 0.5, size=2 * T).astype(np.float32)
    style = rng.normal(0.0, 0.1, size=style_dim).astype(np.float32)
    return Utterance(T, asr, f0, noise, np.ascontiguousarray(style[:STYLE_DIM]))


def config0_inputs(T: int = 200) -> Utterance:
    """T=200 frames (5 s, 120000 samples), input seed 100."""
    return make_utterance(np.random.default_rng(100), T)


def config3_utterances(n: int = 256, t_min: int = 40, t_max: int = 800, seed: int = 103) -> List[Utterance]:
    """256 independent utterances, T ~ U[40, 800]; style is the decoder half
    ([0:128]) of a 256-d N(0, 0.1) voice row."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(t_min, t_max + 1, size=n)
    return [make_utterance(rng, int(t), style_dim=256) for t in lens]


def pack(utts: Sequence[Utterance]):
    """Concatenate a ragged batch into the C ABI's back-to-back layout."""
    n_frames = np.array([u.T for u in utts], dtype=np.int32)
    asr = np.concatenate([u.asr.reshape(-1) for u in utts]).astype(np.float32)
    f0 = np.concatenate([u.f0 for u in utts]).astype(np.float32)
    noise = np.concatenate([u.noise for u in utts]).astype(np.float32)
    style = np.concatenate([u.style for u in utts]).astype(np.float32)
    return n_frames, asr, f0, noise, style
