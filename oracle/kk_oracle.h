/*
 * The oracle: a CPU restatement of the Kokoro-82M synthesis hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or
 * calls this code. Only the parity tests, the smoke check and the bench's CPU
 * baseline leg use it, and only as the checker / the timed CPU reference.
 *
 * Every function restates the reference's scalar (no AVX2 / NEON) x86-64 code
 * path, which is what the reference's own translation units compile to with
 * its flags (`-O3 -DNDEBUG`, no `-march`, no FMA contraction; reference
 * CMakeLists.txt:38-40). ggml op semantics that are not in the reference tree
 * (ggml v0.28.0 is fetched at configure time) are restated from the public
 * ggml CPU implementation and marked "ggml semantics" where used.
 *
 * Tensor layout is ggml's: ne[0] is the fastest axis. An activation [L, C]
 * (time-fastest) is stored as x[c * L + t], as in CpuTensor::at
 * (src/arch/kokoro/kokoro.h:200-212).
 */
#ifndef KK_ORACLE_H
#define KK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/kokopop_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kko_model kko_model;

/* Copies (and dequantises to F32) every tensor; the dtype is kept because it
 * selects ggml's F16 or F32 arithmetic for the ops that consume the tensor. */
kko_model *kko_model_create(const kk_tensor_desc *descs, size_t n);
void kko_model_free(kko_model *m);

/* Optional observer for intermediate tensors (mirrors the reference's
 * KOKOPOP_POST_STATS / KOKOPOP_DUMP_DIR taps, audio_utils.cpp:945-1041). */
typedef void (*kko_tap_fn)(const char *name, const float *data, int64_t ne0,
                           int64_t ne1, void *user);
void kko_set_tap(kko_model *m, kko_tap_fn fn, void *user);

/* 1: evaluate the harmonic source's tanh / sin / cos with the C library's
 * float functions, exactly the calls the reference makes; 0 (default): the
 * correctly rounded values (see kk_oracle.c). */
void kko_set_source_libm(kko_model *m, int use_libm);

/* Last error message of the calling thread ("" when none). */
const char *kko_last_error(void);

/* ---- R1: harmonic source + forward STFT (audio_utils.cpp:120-422) ----
 * f0: [n_f0] frames at 80 Hz-equivalent resolution (300 samples each).
 * har: [22, target_frames] -> har[r * target_frames + frame].
 * source (optional): [n_f0 * 300]. */
int kko_harmonic_stft(kko_model *m, const float *f0, int64_t n_f0,
                      int64_t target_frames, float *har, float *source);

/* ---- R9: Kokoro iSTFT (audio_utils.cpp:462-532 + src/audio/istft.cpp) ----
 * post: [22, n_frames]; audio: [(n_frames - 1) * 5] samples, clamped to +-1.
 * Returns the number of samples written in *n_out. */
int kko_istft(const float *post, int64_t n_frames, float *audio, int64_t *n_out);

/* ---- R10: generator (audio_utils.cpp:594-1051) ----
 * decoder: [L, 512] time-fastest (L = 2T decoder frames); f0: [L]; style: [128].
 * audio: [L * 300] samples. post_out (optional): [22, 60 L + 1]. */
int kko_generator(kko_model *m, int64_t L, const float *decoder, const float *f0,
                  const float *style, float *audio, float *post_out);

/* ---- R6: decoder encode/decode (kokoro.cpp:716-763) ----
 * asr: [T, 512] time-fastest; f0, noise: [2T]; style: [128].
 * decoder_out: [2T, 512] time-fastest. */
int kko_decoder(kko_model *m, int64_t T, const float *asr, const float *f0,
                const float *noise, const float *style, float *decoder_out);

/* decoder + generator + iSTFT for one utterance: audio [600 T]. */
int kko_decoder_forward(kko_model *m, int64_t T, const float *asr, const float *f0,
                        const float *noise, const float *style, float *audio);

/* ---- R7: one LSTM direction (lstm_fused.cpp:200-247) ----
 * pre_gates: [N, 4H] (pre[t * 4H + j]); w_hh_rowwise: [4H, H]; b_hh: [4H];
 * out: [N, H]. */
void kko_lstm_direction(const float *pre_gates, const float *w_hh_rowwise,
                        const float *b_hh, int64_t H, int64_t N, int reverse,
                        float *out);

/* ---- R8: bidirectional LSTM (graph_ops.cpp:1439-1529) ----
 * x: [N, in_dim] (feature-fastest); out: [N, 2H] (forward half first). */
int kko_bilstm(kko_model *m, const char *prefix, int64_t N, int64_t in_dim,
               const float *x, float *out);

/* ---- R8: prosody duration encoder (graph_ops.cpp:1535-1576) ----
 * x: [N, 512]; style: [128]; out: [N, 640]. */
int kko_duration_encoder(kko_model *m, int64_t N, const float *x,
                         const float *style, float *out);

/* ---- prosody predictor F0 / N chain (kokoro.cpp:669-708) ----
 * en: [T, 640] (the aligned duration-encoder output, frame-major);
 * style: [128] (prosody half); f0, n: [2T]. */
int kko_prosody_f0n(kko_model *m, int64_t T, const float *en, const float *style,
                    float *f0, float *n);

/* ---- R11: durations -> frames and the alignment (kokoro.cpp:115-193, :669-674)
 * frames[i] = clamp(lrint(d[i] / speed), 1, 50); *total = sum(frames).
 * If hidden != NULL: en[f, :] = hidden[token(f), :] for every frame f
 * (the one-hot matmul d . mask), en: [total, hidden_dim]. */
int kko_align_durations(const float *durations, int64_t n_tokens, float speed,
                        int32_t *frames, int64_t *total, const float *hidden,
                        int64_t hidden_dim, float *en, int64_t en_capacity);

/* ---- text encoder (graph_ops.cpp:1578-1624, up to the biLSTM) ----
 * ids: [N] token ids, 0 <= id < vocab; out: [N, 512] feature-fastest (the
 * biLSTM kokopop.text_encoder.lstm, forward half first), the t_en that the
 * duration alignment multiplies by the one-hot mask. */
int kko_text_encoder(kko_model *m, int64_t N, const int32_t *ids, float *out);

/* ---- duration head (kokoro.cpp:343-355, :469-516) ----
 * d: [N, 640] (the duration encoder output) -> the biLSTM
 * kokopop.predictor.lstm -> per token the sum over the projection buckets of
 * sigmoid(linear), in double; durations: [N]. */
int kko_duration_head(kko_model *m, int64_t N, const float *d, float *durations);

/* The duration head's last step alone, from the biLSTM output h [N, P]
 * (P = the projection's input size). */
int kko_duration_proj(kko_model *m, int64_t N, const float *h, float *durations);

/* ---- ALBERT + bert_encoder (kokoro.cpp:279-337) ----
 * ids: [N] token ids (positions 0..N-1, token type 0); out: [N, 512]
 * feature-fastest, the bert_encoder output that the duration encoder
 * reads. PARITY UNPINNED: ggml_gelu, ggml_soft_max_ext and ggml_norm are
 * restated from the public ggml CPU source (v0.28.0, not in the reference
 * tree); exp and tanh are taken correctly rounded (see kk_oracle.c). */
int kko_albert(kko_model *m, int64_t N, const int32_t *ids, float *out);

/* ---- sanoTTS Vocos decoder (src/arch/sanotts/sano_vocos.cpp:94-230) ----
 * The voice's decoder hyper-parameters (its GGUF dec.* keys,
 * src/arch/sanotts/sano_arch.cpp:1081-1096). */
typedef struct kko_vocos_dims {
    int32_t dim, blocks, pw_hidden, dw_kernel, embed_kernel, noise_ch, mels, n_fft, hop;
    float dc_pole, mag_clip;
} kko_vocos_dims;

/* mel [mels][frames], noise [noise_ch][frames] (time-fastest) -> audio
 * [hop * (frames - 1)]; weights "<prefix>dec.embed.weight", ... PARITY
 * UNPINNED for the trunk (ggml ops); the iSTFT restatement is pinned
 * against the reference's compiled istft.cpp. */
int kko_vocos(kko_model *m, const char *prefix, const kko_vocos_dims *d, int64_t frames, const float *mel,
              const float *noise, float *audio, int64_t *n_out);

/* The RealRadix2 iSTFT (power-of-two n_fft >= 64, center): re / im
 * frame-major [frames][n_fft / 2 + 1] -> audio [hop * (frames - 1)]. */
int kko_istft_r2(const float *re, const float *im, int64_t frames, int n_fft, int hop, float *audio,
                 int64_t *n_out);

/* The DC blocker y[n] = x[n] - x[n-1] + pole y[n-1], in place. */
void kko_dc_block(float *audio, int64_t n, float pole);

/* Single-op entry points used by the unit tests. */
void kko_norm_time(const float *x, int64_t C, int64_t L, float eps, float *y);
float kko_round_f16(float x);

#ifdef __cplusplus
}
#endif

#endif /* KK_ORACLE_H */
