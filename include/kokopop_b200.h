/*
 * kokopop_b200 — C ABI of the B200 (sm_100a) Kokoro-82M synthesis hot path.
 *
 * This is the thin layer that kokopop's C++ host code calls in place of the
 * ggml graph for the hot-path ops only. Everything above it (include/kokopop.h,
 * the session / streaming layer, the GGUF loader) is unchanged.
 *
 * Conventions (mirroring the reference's C API, include/kokopop.h:125-132 and
 * src/kokopop.cpp:38-59):
 *   - every call returns a KK_* status; on failure a message is stored in a
 *     thread-local slot read by kk_last_error() (src/core/error.cpp:4-15);
 *   - no C++ exception and no CUDA error crosses this boundary;
 *   - a kk_ctx owns one CUDA stream and all device memory it uses; it is not
 *     thread-safe, exactly like a kokopop_model (docs/c-api.md:284-286);
 *   - pointers are plain host pointers unless the name ends in _device, in
 *     which case they are device pointers on the context's device and the
 *     call is asynchronous on `stream` (NULL = the context's own stream):
 *     it stages its small tables in pinned memory and returns without
 *     waiting for the GPU;
 *   - calls on one context reuse its workspaces, so the device runs them in
 *     the order they were made, also when they name different streams: a
 *     call waits (on the device, not the host) for the previous call of the
 *     context to finish. Calls on different contexts are independent.
 *
 * Layouts follow ggml (ne[0] fastest). Per utterance, an activation written
 * "[L, C]" is time-fastest: x[c * L + t] (src/arch/kokoro/kokoro.h:200-212).
 * Ragged batches are the per-utterance arrays concatenated back to back.
 */
#ifndef KOKOPOP_B200_H
#define KOKOPOP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same numeric values as KOKOPOP_OK .. KOKOPOP_ERROR_INFERENCE
 * (include/kokopop.h:125-132), so the host can return them unchanged. */
enum {
    KK_OK = 0,
    KK_ERROR_INVALID_ARGUMENT = 1,
    KK_ERROR_IO = 2,
    KK_ERROR_MODEL = 3,
    KK_ERROR_INFERENCE = 5
};

/* Same numeric values as GGML_TYPE_F32 / GGML_TYPE_F16. */
enum { KK_DTYPE_F32 = 0, KK_DTYPE_F16 = 1 };

/* One weight tensor as the reference's loader holds it: logical GGUF name
 * (tools/convert_kokoro_to_gguf.py layout, dims already reversed to ggml
 * order), type and host data. Replaces the weight upload of
 * src/model/model.cpp:429-443 for the tensors the hot path reads. */
typedef struct kk_tensor_desc {
    const char *name;
    int32_t dtype;     /* KK_DTYPE_F32 or KK_DTYPE_F16 (raw IEEE half bits) */
    int32_t n_dims;
    int64_t ne[4];     /* unused trailing dims = 1 */
    const void *data;  /* host pointer, copied during the call */
} kk_tensor_desc;

typedef struct kk_ctx kk_ctx;

/* Creates a context on CUDA device `device` (the value KOKOPOP_CUDA_DEVICE
 * selects in src/backend/cuda.cpp:38-45). Fails on a device that is not
 * sm_100. */
int kk_ctx_create(int device, kk_ctx **out);
void kk_ctx_destroy(kk_ctx *ctx);

/* Uploads the hot-path weights once (replaces KokoroArch::preload_tensor_cache,
 * src/arch/kokoro/kokoro_arch.cpp:389-607, for these tensors). Tensors the hot
 * path does not read are ignored. May be called again to replace weights. */
int kk_weights_upload(kk_ctx *ctx, const kk_tensor_desc *descs, size_t n);

/* Thread-local message of the last failed call on this thread. */
const char *kk_last_error(void);

/* Decoder encode/decode + ISTFTNet generator + iSTFT for a ragged batch of
 * independent utterances. Replaces, per utterance, the decoder sub-graph of
 * run_kokoro_generation_probe (src/arch/kokoro/kokoro.cpp:716-763) followed by
 * ggml_generator (src/arch/kokoro/audio_utils.cpp:594-1051).
 *   n_frames[u] = T_u (asr frames, 40 per second of audio), 1 <= T_u <= 8192
 *   asr   : per utterance [T_u, 512]   (time-fastest)
 *   f0    : per utterance [2 T_u]      (F0 curve, Hz)
 *   noise : per utterance [2 T_u]      (N curve)
 *   style : per utterance [128]        (decoder half of the voice row)
 *   audio : per utterance [600 T_u]    samples at 24 kHz, clamped to +-1
 * Like the reference (all_finite, src/arch/kokoro/kokoro.cpp:91-99,
 * :933-940), a non-finite f0, noise or asr value, decoder output or style
 * value is KK_ERROR_INFERENCE with "non-finite Kokoro <name> value at index
 * <i>" (the first such tensor in that order, its smallest index; inputs are
 * indexed as passed). The context stays usable.
 */
int kk_decoder_forward(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames,
                       const float *asr, const float *f0, const float *noise,
                       const float *style, float *audio);

/* Same as kk_decoder_forward with device-resident inputs and output; the
 * lengths stay on the host. Asynchronous on `stream`; a non-finite value is
 * reported by the next call of this context that synchronises. */
int kk_decoder_forward_device(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames,
                              const float *asr, const float *f0,
                              const float *noise, const float *style,
                              float *audio, void *stream);

/* The ggml_generator seam (src/arch/kokoro/kokoro.h:214-219) for a ragged
 * batch: decoder output [L_u, 512] with L_u = 2 T_u, f0 [L_u], style [128]
 * -> audio [300 L_u]. Host buffers. */
int kk_generator_forward(kk_ctx *ctx, int32_t n_utts, const int32_t *n_decoder_frames,
                         const float *decoder, const float *f0, const float *style,
                         float *audio);

/* The Kokoro iSTFT seam (cpu_istft, src/arch/kokoro/audio_utils.cpp:462-536):
 * post [n_frames, 22] (bin-major: post[r * n_frames + t]) -> audio
 * [(n_frames - 1) * 5], clamped to +-1. n_frames may be 0 or 1 (no samples). */
int kk_istft(kk_ctx *ctx, int64_t n_frames, const float *post, float *audio);

/* Bidirectional LSTM layer `prefix` (weights prefix.weight_ih_l0[_reverse],
 * .weight_hh_l0[_reverse], .bias_ih_l0[_reverse], .bias_hh_l0[_reverse];
 * hidden size 256) over a ragged batch. Replaces bidirectional_lstm
 * (src/arch/kokoro/graph_ops.cpp:1514-1529): the input projection of
 * lstm_direction (:1439-1512) and the fused recurrence cpu_lstm_contiguous
 * (src/arch/kokoro/lstm_fused.cpp:200-247), gate order i, f, g, o.
 *   n_steps[b] = N_b in [1, 65536]
 *   x   : per sequence [N_b, in_dim] (feature-fastest), back to back
 *   out : per sequence [N_b, 512]: forward h in [0, 256), backward in [256, 512)
 * Host buffers. */
int kk_bilstm_forward(kk_ctx *ctx, const char *prefix, int32_t n_seqs, const int32_t *n_steps, int64_t in_dim,
                      const float *x, float *out);

/* The prosody duration encoder (duration_encoder,
 * src/arch/kokoro/graph_ops.cpp:1535-1576): 3 x (concat style -> biLSTM
 * kokopop.predictor.text_encoder.lstms.{0,2,4} -> AdaLayerNorm
 * ...lstms.{1,3,5}), output concatenated with the style once more.
 *   x     : per sequence [N_b, 512]
 *   style : per sequence [128] (the prosody half of the voice row)
 *   out   : per sequence [N_b, 640]
 * Host buffers. */
int kk_duration_encoder_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_steps, const float *x,
                                const float *style, float *out);

/* Same with device-resident x, style and out; the lengths stay on the host.
 * Asynchronous on `stream` (NULL = the context's stream). */
int kk_duration_encoder_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_steps, const float *x,
                                       const float *style, float *out, void *stream);

/* The prosody predictor's F0 / N chain (src/arch/kokoro/kokoro.cpp:669-708,
 * replacing the ggml sub-graph from the aligned `en` to f0_curve / n_curve):
 * the biLSTM kokopop.predictor.shared (640 -> 2 x 256) over the T_b frames,
 * then for each of F0 and N three adain_resblk1d
 * kokopop.predictor.{F0,N}.{0,1,2} (graph_ops.cpp:996-1065; the second
 * upsamples x2) with the prosody style, and the 1x1 conv {F0,N}_proj + bias.
 * Ragged batch; per utterance b:
 *   n_frames[b] = T_b, at most 8192
 *   en    : [T_b, 640], frame-major (the aligned duration-encoder output,
 *           as kk_align_durations writes it)
 *   style : [128] (the prosody half of the voice row)
 *   f0, n : [2 T_b]
 * Host buffers. */
int kk_prosody_f0n(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *en, const float *style,
                   float *f0, float *n);

/* Same with device-resident en, style, f0 and n (lengths on the host).
 * Asynchronous on `stream` (NULL = the context's stream). */
int kk_prosody_f0n_device(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *en,
                          const float *style, float *f0, float *n, void *stream);

/* The text encoder up to its biLSTM (text_encoder,
 * src/arch/kokoro/graph_ops.cpp:1578-1624, replacing the ggml sub-graph from
 * the token ids to the biLSTM output that the duration mask then multiplies):
 * the embedding lookup, three times conv1d_chfirst k = 5 (pad 2) + bias ->
 * LayerNorm over the 512 channels (eps 1e-5) * gamma + beta -> LeakyReLU
 * 0.2, then the biLSTM kokopop.text_encoder.lstm (512 -> 2 x 256). Ragged
 * batch; per sequence b:
 *   n_tokens[b] = N_b, at most 8192
 *   ids : int32 [N_b], concatenated over the sequences, 0 <= id < vocab
 *   out : [N_b, 512], token-major (forward half first)
 * Host buffers; an id out of range is KK_ERROR_INVALID_ARGUMENT. */
int kk_text_encoder_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out);

/* Same with device-resident ids and out (lengths on the host). Asynchronous
 * on `stream` (NULL = the context's stream); an id out of range gives a zero
 * embedding row and is reported (KK_ERROR_INVALID_ARGUMENT) by the next call
 * of this context that synchronises. */
int kk_text_encoder_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids,
                                   float *out, void *stream);

/* ALBERT and bert_encoder (src/arch/kokoro/kokoro.cpp:279-337, replacing the
 * frontend graph from the token ids to `cur = linear(enc_w, enc_b, cur)`):
 * word + position (0..N_b - 1) + token-type-0 embeddings, LayerNorm (eps
 * 1e-12), the 128 -> 768 mapping, twelve passes of the shared layer (12
 * heads of 64, softmax(q k / 8) v, dense + residual -> LayerNorm, ffn ->
 * GELU -> ffn_output + residual -> LayerNorm), then bert_encoder 768 -> 512.
 * Ragged batch; per sequence b: n_tokens[b] = N_b, at most 512 (the position
 * table); ids int32 [N_b] concatenated; out [N_b, 512] token-major (the
 * duration encoder's input). Host buffers; an id out of range is
 * KK_ERROR_INVALID_ARGUMENT. */
int kk_albert_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out);

/* Same with device-resident ids and out (lengths on the host), asynchronous
 * on `stream` (NULL = the context's stream); a bad id as in
 * kk_text_encoder_forward_device. */
int kk_albert_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out,
                             void *stream);

/* The duration head (src/arch/kokoro/kokoro.cpp:343-355 and :469-516,
 * replacing the predictor.lstm graph node and the host loop over the
 * duration_proj buckets): the biLSTM kokopop.predictor.lstm (640 -> 2 x 256)
 * over the duration encoder output, then per token
 *   durations[t] = (float) sum over buckets n of sigmoid((float) acc_n),
 *   acc_n = bias[n] + sum over k of w[n][k] h[k]
 * in double, as the reference computes it on the host. Ragged batch;
 * per sequence b: n_tokens[b] = N_b (at most 65536), d: [N_b, 640]
 * token-major, durations: [N_b]. Host buffers. */
int kk_duration_head_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const float *d,
                             float *durations);

/* Same with device-resident d and durations (lengths on the host).
 * Asynchronous on `stream` (NULL = the context's stream). */
int kk_duration_head_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const float *d,
                                    float *durations, void *stream);

/* The duration head's projection and bucket sum alone (kokoro.cpp:469-516),
 * from the predictor biLSTM output h: [n_rows, 512] token-major, durations:
 * [n_rows]; at most 65536 rows. Host buffers. */
int kk_duration_proj(kk_ctx *ctx, int64_t n_rows, const float *h, float *durations);

/* ---- Batching request queue (the per-GPU counterpart of the reference's
 * SynthesisScheduler, src/http/synthesis_scheduler.cpp:15-209, which runs
 * one chunk of one request at a time, round-robin over the requests) ----
 * Workers (one per GPU context, or per caller executor) each run a ragged
 * batch per call: the oldest pending chunk of each request, in arrival
 * order, at most max_batch chunks and max_batch_frames frames, after waiting
 * up to max_wait_us from the oldest chunk's arrival for the batch to fill. A
 * request has at most one chunk dispatched at a time, so its chunks finish
 * in submission order. Results: KK_* statuses, or these. */
enum { KK_QUEUE_PENDING = -1, KK_QUEUE_CANCELLED = -2 };

typedef struct kk_queue kk_queue;

/* A batch executor with the arguments of kk_decoder_forward (host buffers);
 * returns a KK_* status. Called from the queue's worker threads. */
typedef int (*kk_queue_exec_fn)(void *user, int32_t n_utts, const int32_t *n_frames, const float *asr,
                                const float *f0, const float *noise, const float *style, float *audio);

/* One worker per context (each with the decoder weights uploaded, used by
 * that worker only while the queue lives). The worker stages a batch in
 * pinned memory and runs it with kk_decoder_forward_device on its own
 * stream, packing the next batch while the GPU runs. */
int kk_queue_create(kk_ctx *const *ctxs, int32_t n_ctx, int32_t max_batch, int64_t max_batch_frames,
                    int32_t max_wait_us, kk_queue **out);

/* One worker per users[i] (NULL users: n_workers workers with user NULL),
 * each calling fn(users[i], ...) for its batches. */
int kk_queue_create_exec(kk_queue_exec_fn fn, void *const *users, int32_t n_workers, int32_t max_batch,
                         int64_t max_batch_frames, int32_t max_wait_us, kk_queue **out);

/* Queues one decoder chunk of request `request` (any caller-chosen id):
 * asr [T, 512], f0 / noise [2 T], style [128], audio [600 T], as for
 * kk_decoder_forward; the buffers stay the caller's and must stay valid
 * until the ticket's result is returned. 1 <= T <= min(8192,
 * max_batch_frames). Thread-safe. */
int kk_queue_submit(kk_queue *q, uint64_t request, int32_t n_frames, const float *asr, const float *f0,
                    const float *noise, const float *style, float *audio, uint64_t *ticket);

/* Waits up to timeout_ms (< 0: without limit) for a ticket. Returns
 * KK_QUEUE_PENDING on timeout; otherwise the chunk's result (KK_OK, a
 * KK_ERROR_*, or KK_QUEUE_CANCELLED), after which the ticket is forgotten
 * (waiting on it again is KK_ERROR_INVALID_ARGUMENT). Thread-safe. */
int kk_queue_wait(kk_queue *q, uint64_t ticket, int32_t timeout_ms);

/* Cancels the chunks of `request` not yet dispatched (the reference's
 * cancelled flag); *n_cancelled (optional) = how many. */
int kk_queue_cancel(kk_queue *q, uint64_t request, int32_t *n_cancelled);

/* Batches and chunks run so far, and the largest batch. */
int kk_queue_stats(kk_queue *q, uint64_t *batches, uint64_t *jobs, uint64_t *max_batch_seen);

/* Message of the last failed kk_queue_* call on this thread. */
const char *kk_queue_last_error(void);

/* Cancels the pending chunks, lets the dispatched batches finish and stops
 * the workers. Call it once every kk_queue_wait has returned. */
void kk_queue_destroy(kk_queue *q);

/* ---- Streaming sessions over the queue ----
 * The reference streams a request chunk by chunk (stream_synthesize,
 * src/streaming/streaming.cpp:252-360): each chunk's raw audio is
 * post-processed (postprocess_chunk_audio, src/audio/audio_postprocess.cpp:
 * 260-307: silence trim and the boundary pause) and crossfaded onto the
 * previous chunk's tail (postprocess_and_crossfade, streaming.cpp:26-60;
 * apply_crossfade_smart, audio_postprocess.cpp:94-202), then handed to the
 * caller in order. A kk_stream does the same over a kk_queue: kk_stream_push
 * submits a chunk's decoder inputs at once (so the chunks of many sessions
 * share GPU batches), kk_stream_next returns the chunks in push order, each
 * post-processed and crossfaded as the reference does. The chunker and the
 * phonemizer stay outside (their outputs are the pushed inputs). */

/* Chunk boundaries (Boundary, src/synthesis/chunker/chunker.h:14-21). */
enum {
    KK_BOUNDARY_NONE = 0,
    KK_BOUNDARY_CLAUSE_WEAK = 1,
    KK_BOUNDARY_CLAUSE_STRONG = 2,
    KK_BOUNDARY_SENTENCE = 3,
    KK_BOUNDARY_NEWLINE = 4,
    KK_BOUNDARY_PARAGRAPH = 5
};

/* kk_stream_next after the last chunk has been returned. */
enum { KK_STREAM_END = -3 };

/* The post-processing fields of ChunkConfig (chunker.h:26-51). */
typedef struct kk_stream_config {
    int32_t comma_pause_ms;
    int32_t sentence_pause_ms;
    int32_t paragraph_pause_ms;
    int32_t crossfade_ms;
    int32_t trim_silence;        /* 0 or 1 */
    int32_t max_silence_trim_ms;
    int32_t sample_rate;         /* 24000 for Kokoro */
} kk_stream_config;

/* The reference's presets (make_adaptative_config / make_long_form_config,
 * src/synthesis/chunker/chunker.cpp:16-48): mode 0 adaptative, 1 long-form;
 * sample_rate 24000. */
int kk_stream_preset(int32_t mode, kk_stream_config *out);

/* postprocess_chunk_audio on a host buffer: out gets at most `capacity`
 * samples, *n_out the processed length (also when capacity is too small,
 * then KK_ERROR_INVALID_ARGUMENT). Bit-exact with the reference. */
int kk_postprocess_chunk(const kk_stream_config *cfg, const float *audio, int64_t n, int32_t boundary_after,
                         int32_t is_first, int32_t is_last, float *out, int64_t capacity, int64_t *n_out);

/* apply_crossfade_smart(prev, next, boundary, crossfade_ms, sample_rate) on
 * host buffers, the same capacity rule. Bit-exact with the reference. */
int kk_crossfade(const kk_stream_config *cfg, const float *prev, int64_t n_prev, const float *next, int64_t n_next,
                 int32_t boundary, float *out, int64_t capacity, int64_t *n_out);

typedef struct kk_stream kk_stream;

/* A session on q (its own request id); the config is copied. */
int kk_stream_create(kk_queue *q, const kk_stream_config *cfg, kk_stream **out);

/* Queues the next chunk (inputs as for kk_queue_submit; they are copied, so
 * the caller may reuse them on return). is_last marks the final chunk: no
 * pause after it, and kk_stream_next returns KK_STREAM_END once it has been
 * returned. No push after is_last. */
int kk_stream_push(kk_stream *s, int32_t n_frames, const float *asr, const float *f0, const float *noise,
                   const float *style, int32_t boundary_after, int32_t is_last);

/* The next chunk in push order, waiting up to timeout_ms (< 0: without
 * limit): KK_OK with *samples / *n_samples (owned by the session, valid
 * until the next call) and *chunk_index; KK_QUEUE_PENDING on timeout, or
 * when nothing has been pushed yet; KK_STREAM_END after the last chunk. A
 * chunk that failed returns its status with no samples, and the next chunk
 * is not crossfaded onto the tail from before it (streaming.cpp:325-333);
 * a cancelled chunk returns KK_QUEUE_CANCELLED. Not thread-safe per
 * session; sessions are independent. */
int kk_stream_next(kk_stream *s, int32_t timeout_ms, const float **samples, int64_t *n_samples,
                   int32_t *chunk_index);

/* Cancels the session's chunks not yet dispatched (the reference's stopped
 * flag); the dispatched ones finish and are still returned by
 * kk_stream_next. */
int kk_stream_cancel(kk_stream *s);

/* Waits for the session's chunks in flight, then frees it. */
void kk_stream_destroy(kk_stream *s);

/* Durations -> frames and the alignment (duration_to_frames,
 * src/arch/kokoro/kokoro.cpp:181-193; build_duration_mask :115-152 and
 * en = d . mask :669-674): frames[i] = clamp(int(lrint(d[i] / speed)), 1, 50)
 * (non-finite -> 1; a non-finite or non-positive speed counts as 1),
 * *total = sum(frames). If hidden != NULL (then en != NULL): en[f, :] =
 * hidden[token(f), :] for every frame f, en holding en_capacity rows of
 * hidden_dim. At most 65535 tokens. Host buffers. */
int kk_align_durations(kk_ctx *ctx, int64_t n_tokens, const float *durations, float speed, int32_t *frames,
                       int64_t *total, const float *hidden, int64_t hidden_dim, float *en, int64_t en_capacity);

/* ---- sanoTTS Vocos decoder ----
 * The hyper-parameters of one voice's decoder: its GGUF keys dec.dim,
 * dec.blocks, dec.pw_hidden, dec.dw_kernel, dec.embed_kernel, dec.noise_ch,
 * dec.mels, dec.n_fft, dec.hop, dec.dc_pole, dec.mag_clip
 * (src/arch/sanotts/sano_arch.cpp:1081-1096; dec.bins = n_fft / 2 + 1). */
typedef struct kk_vocos_params {
    int32_t dim, blocks, pw_hidden, dw_kernel, embed_kernel, noise_ch, mels, n_fft, hop;
    float dc_pole, mag_clip;
} kk_vocos_params;

/* sano_run_vocos (src/arch/sanotts/sano_vocos.cpp:94-230) for a ragged batch
 * of chunks of one voice: the two 7-tap stem convs (mel, noise), LayerNorm,
 * `blocks` ConvNeXt1D blocks (depthwise conv, LayerNorm, pw0, exact GELU,
 * pw1, layer scale, residual), LayerNorm, the magnitude / phase head, the
 * iSTFT (n_fft, hop, centred) and the DC blocker. Weights are read under
 * `prefix` (e.g. "kokopop.sanotts.voice.0." + "dec.embed.weight"); the
 * pointwise / stem / head weights all F16 or all F32. The noise input is the
 * caller's (sano::seeded_noise in the reference). Per chunk u:
 *   n_frames[u] = F_u frames, 2 <= F_u <= 8192
 *   mel   : [F_u, mels]      (time-fastest: mel[c * F_u + t])
 *   noise : [F_u, noise_ch]  (time-fastest)
 *   audio : [hop (F_u - 1)] samples
 * n_fft must be a power of two in [64, 2048], dim and pw_hidden at most
 * 1024, the kernels odd. Host buffers. */
int kk_vocos_forward(kk_ctx *ctx, const char *prefix, const kk_vocos_params *params, int32_t n_chunks,
                     const int32_t *n_frames, const float *mel, const float *noise, float *audio);

/* Same with device-resident mel, noise and audio (lengths on the host).
 * Asynchronous on `stream` (NULL = the context's stream). */
int kk_vocos_forward_device(kk_ctx *ctx, const char *prefix, const kk_vocos_params *params, int32_t n_chunks,
                            const int32_t *n_frames, const float *mel, const float *noise, float *audio,
                            void *stream);

/* kk_istft without any device allocation (no counterpart in the reference,
 * whose iSTFT runs on the host). Same arguments and results as kk_istft, but
 * no kk_ctx: input, output, tables and descriptor are staged in one static
 * device array of the library (about 3.5 MB per device), so the call never
 * allocates or frees device memory itself. For callers that cannot allocate
 * mid-run: a real-time audio thread (cudaMalloc / cudaFree can synchronise
 * the whole device) or a process that fixes its device-memory budget up
 * front.
 *   device   CUDA device to run on (made current for the call, then
 *            restored); an index past the device count is
 *            KK_ERROR_INVALID_ARGUMENT
 *   stream   a stream of that device, or NULL for its legacy default stream;
 *            the call returns after the stream has finished the copy back
 *   n_frames at most KK_ISTFT_STATIC_MAX_FRAMES; larger inputs are rejected
 *            with KK_ERROR_INVALID_ARGUMENT (use kk_istft for them)
 * Set-up: with CUDA's default lazy module loading, the array's memory is
 * reserved when the first call on a device looks up its address, so that
 * first call can fail for lack of device memory or stall while the module
 * loads. Make one call with n_frames = 0 (or 1) on each device at start-up,
 * before any stream capture: it does that set-up and nothing else. (With
 * CUDA_MODULE_LOADING=EAGER the array is reserved when the context is
 * created.) The device then holds the array until the process exits.
 * Nothing in the array has to start at zero. Calls that overlap in time on
 * one device (from several threads, or on several streams) share the array
 * and overwrite each other's data: serialise them. */
#define KK_ISTFT_STATIC_MAX_FRAMES 32768
int kk_istft_static(int device, int64_t n_frames, const float *post, float *audio, void *stream);

/* Counters of a context, for measurement (no counterpart in the reference,
 * which prints ggml_time_us stage timings under KOKOPOP_GEN_PROFILE,
 * src/arch/kokoro/audio_utils.cpp:834-893). */
typedef struct kk_profile {
    uint64_t launches;       /* kernels this context launched */
    uint64_t conv_launches;  /* dense-convolution launches timed */
    double conv_ms;          /* their summed device time (CUDA events) */
    double conv_flop;        /* their algorithmic FLOPs: 2*OC*IC*K per valid position */
} kk_profile;

/* When enabled, every launch of the kinds below is bracketed by CUDA events
 * on its stream and recorded with its algorithmic work. */
int kk_profile_enable(kk_ctx *ctx, int enable);
/* Reads (after synchronising the context's work) and optionally resets the
 * counters and the records. */
int kk_profile_read(kk_ctx *ctx, kk_profile *out, int reset);

/* Kinds of timed launches. */
enum {
    KK_PROF_CONV = 0,     /* dense convolution (tensor or CUDA cores), its statistics epilogue included */
    KK_PROF_OPERAND = 1,  /* AdaIN / activation operand pass (instance norm applied, Snake or LeakyReLU) */
    KK_PROF_STATS = 2,    /* instance-norm statistics pass over an activation */
    KK_PROF_ISTFT = 3,    /* conv_post magnitude / phase -> inverse DFT -> overlap-add */
    KK_PROF_SOURCE = 4,   /* harmonic source and its STFT (side stream) */
    KK_PROF_LSTM = 5,     /* LSTM recurrence */
    KK_PROF_OTHER = 6     /* packing, upsampling, the ConvTranspose edge row */
};

/* One timed launch: its kind, the convolution's taps (0 for other kinds),
 * its device time and its algorithmic work: FLOPs (2 per multiply-add) and
 * DRAM bytes (every input element read once, every output written once). */
typedef struct kk_profile_record {
    int32_t kind;
    int32_t taps;
    double ms;
    double flop;
    double bytes;
} kk_profile_record;

/* The records since the last reset, in launch order per stream (after
 * synchronising): copies min(cap, *n) of them to out; *n = how many exist. */
int kk_profile_records(kk_ctx *ctx, kk_profile_record *out, size_t cap, size_t *n);

/* How many device or pinned-host allocations the library has made in this
 * process, over all contexts and queues (no counterpart in the reference).
 * Lets a caller check that a path allocates nothing once warm. */
int kk_allocation_count(uint64_t *out);

/* ---- failure injection and self-tests (no counterpart in the reference) ----
 * The next n device or pinned-host allocations of the library fail as out of
 * memory (0 clears), so that a caller can test its handling of
 * KK_ERROR_INFERENCE from a workspace that cannot grow. A call that fails
 * this way leaves its context usable: the next call allocates again. */
int kk_inject_allocation_failures(int32_t n);

/* Runs the bounded wait of the tensor-core kernels on an mbarrier that
 * nothing arrives at, for limit_us microseconds (at most 2 s), on the
 * context's stream. Returns KK_ERROR_INFERENCE with the wait's code in
 * kk_last_error(): the path a real expiry takes (the kernel gives up and
 * returns, the host reports it); the context stays usable. */
int kk_wait_selftest(kk_ctx *ctx, int64_t limit_us);

#ifdef __cplusplus
}
#endif

#endif /* KOKOPOP_B200_H */
