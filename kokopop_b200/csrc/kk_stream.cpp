// Streaming sessions over the batching queue: the reference's per-chunk
// post-processing and crossfade (src/audio/audio_postprocess.cpp:18-307,
// src/streaming/streaming.cpp:26-60) around chunks that run in the queue's
// ragged GPU batches.
//
// A session pushes every chunk of its request into the queue at once (the
// reference keeps one chunk of lookahead on a worker thread,
// streaming.cpp:252-360; here the queue's workers run the chunks of many
// sessions together), and kk_stream_next hands them back in push order. Each
// returned chunk is post-processed (leading / trailing silence trim and the
// boundary pause) and crossfaded onto the tail kept from the previous one,
// the same operations, in the same order, as postprocess_and_crossfade.
#include "../../include/kokopop_b200.h"
#include "kk_host.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <deque>
#include <exception>
#include <vector>

namespace {

constexpr float kSilence = 0.01f;  // SILENCE_THRESHOLD (audio_postprocess.cpp:18)

// ms_to_samples (audio_postprocess.h:22-25)
size_t samples_of(int ms, int rate) {
    if (ms <= 0 || rate <= 0) return 0;
    return (size_t)(((int64_t)ms * rate) / 1000);
}

bool loud(const float *p, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (std::fabs(p[i]) > kSilence) return true;
    return false;
}

// The first sample of the first 50 ms window (stepped by a quarter window)
// that holds a sample above the threshold, within the first `limit` samples;
// `limit` (clipped to n) when there is none (scan_leading_edge, :46-61).
size_t lead_edge(const float *p, size_t n, size_t limit, int rate) {
    const size_t check = std::min(n, limit);
    if (check == 0) return 0;
    const size_t win = samples_of(50, rate);
    const size_t step = std::max<size_t>(1, win / 4);
    for (size_t i = 0; i < check; i += step)
        if (loud(p + i, std::min(win, check - i))) return i;
    return check;
}

// One past the last sample above the threshold among the last `limit`
// samples; n - limit (or 0) when they are all silent; n when n or limit is 0
// (scan_trailing_edge, :63-81; its block walk finds the same sample).
size_t trail_edge(const float *p, size_t n, size_t limit) {
    if (n == 0 || limit == 0) return n;
    const size_t floor = n > limit ? n - limit : 0;
    for (size_t i = n; i > floor; --i)
        if (std::fabs(p[i - 1]) > kSilence) return i;
    return floor;
}

// pause_for_boundary (:242-258)
int pause_ms(int boundary, const kk_stream_config &c) {
    switch (boundary) {
        case KK_BOUNDARY_PARAGRAPH: return c.paragraph_pause_ms;
        case KK_BOUNDARY_NEWLINE: return c.paragraph_pause_ms / 2;
        case KK_BOUNDARY_SENTENCE: return c.sentence_pause_ms;
        case KK_BOUNDARY_CLAUSE_STRONG: return (int)((float)c.sentence_pause_ms * 0.7f);
        case KK_BOUNDARY_CLAUSE_WEAK: return c.comma_pause_ms;
        default: return 0;
    }
}

// postprocess_chunk_audio (:260-307)
void postprocess(const kk_stream_config &c, const float *a, size_t n, int boundary, bool first, bool last,
                 std::vector<float> &out) {
    out.clear();
    if (n == 0) return;
    size_t start = 0, end = n;
    if (c.trim_silence) {
        // no leading trim on the first chunk (its natural intro stays)
        if (!first) start = lead_edge(a, n, samples_of(c.max_silence_trim_ms, c.sample_rate), c.sample_rate);
        int trim = c.max_silence_trim_ms;
        if (boundary != KK_BOUNDARY_NONE) trim = std::max(1, trim / 2);
        end = start + trail_edge(a + start, n - start, samples_of(trim, c.sample_rate));
    }
    size_t pause = 0;
    const int pm = pause_ms(boundary, c);
    if (pm > 0 && !last) pause = samples_of(pm, c.sample_rate);
    const size_t body = end > start ? end - start : 0;
    out.assign(body + pause, 0.0f);
    if (body) std::memcpy(out.data(), a + start, body * sizeof(float));
}

// apply_crossfade (:94-182): the tail of prev and the head of next blended
// over n samples with t = i / (n - 1); concatenation when either is shorter
// than n (or n is 0).
void crossfade_linear(const float *prev, size_t np, const float *next, size_t nn, int ms, int rate,
                      std::vector<float> &out) {
    out.clear();
    if (np == 0) {
        out.assign(next, next + nn);
        return;
    }
    if (nn == 0) {
        out.assign(prev, prev + np);
        return;
    }
    const size_t n = samples_of(ms, rate);
    if (n == 0 || np < n || nn < n) {
        out.reserve(np + nn);
        out.insert(out.end(), prev, prev + np);
        out.insert(out.end(), next, next + nn);
        return;
    }
    out.resize(np + nn - n);
    std::memcpy(out.data(), prev, (np - n) * sizeof(float));
    float *o = out.data() + (np - n);
    if (n == 1) {
        o[0] = next[0];
    } else {
        const float inv = 1.0f / (float)(n - 1);
        const float *tail = prev + (np - n);
        for (size_t i = 0; i < n; ++i) {
            const float t = (float)i * inv;
            const float a = tail[i] * (1.0f - t);
            const float b = next[i] * t;
            o[i] = a + b;
        }
    }
    std::memcpy(o + n, next + n, (nn - n) * sizeof(float));
}

// apply_crossfade_smart (:184-202): after a sentence, newline or paragraph
// boundary the two are concatenated (the pause stands), else crossfaded.
void crossfade_smart(const kk_stream_config &c, const float *prev, size_t np, const float *next, size_t nn,
                     int boundary, std::vector<float> &out) {
    if (boundary == KK_BOUNDARY_SENTENCE || boundary == KK_BOUNDARY_PARAGRAPH || boundary == KK_BOUNDARY_NEWLINE) {
        out.clear();
        out.reserve(np + nn);
        out.insert(out.end(), prev, prev + np);
        out.insert(out.end(), next, next + nn);
        return;
    }
    crossfade_linear(prev, np, next, nn, c.crossfade_ms, c.sample_rate, out);
}

bool config_ok(const kk_stream_config *c) {
    return c && c->sample_rate > 0 && c->crossfade_ms >= 0 && c->max_silence_trim_ms >= 0 &&
           c->comma_pause_ms >= 0 && c->sentence_pause_ms >= 0 && c->paragraph_pause_ms >= 0 &&
           (c->trim_silence == 0 || c->trim_silence == 1);
}

bool boundary_ok(int32_t b) { return b >= KK_BOUNDARY_NONE && b <= KK_BOUNDARY_PARAGRAPH; }

int copy_out(const std::vector<float> &v, float *out, int64_t capacity, int64_t *n_out) {
    *n_out = (int64_t)v.size();
    if ((int64_t)v.size() > capacity) return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "output capacity too small");
    if (!v.empty()) std::memcpy(out, v.data(), v.size() * sizeof(float));
    return KK_OK;
}

template <typename F>
int s_guard(F &&f) noexcept {
    try {
        return f();
    } catch (const std::exception &e) {
        return kk::queue_error(KK_ERROR_INFERENCE, e.what());
    } catch (...) {
        return kk::queue_error(KK_ERROR_INFERENCE, "unknown C++ exception");
    }
}

}  // namespace

// One pushed chunk: its inputs (copied), the raw audio the queue writes, and
// its ticket.
struct KkStreamChunk {
    uint64_t ticket = 0;
    int32_t T = 0, boundary = 0, index = 0;
    bool first = false, last = false;
    std::vector<float> in;     // asr [T][512] | f0 [2T] | noise [2T] | style [128]
    std::vector<float> audio;  // [600 T]
};

struct kk_stream {
    kk_queue *q = nullptr;
    kk_stream_config cfg{};
    uint64_t request = 0;
    std::deque<KkStreamChunk> chunks;  // pushed, not yet returned (element addresses are stable)
    int32_t n_pushed = 0;
    bool pushed_last = false, returned_last = false;
    std::vector<float> tail, out, tmp;
};

namespace {
// Request ids of the sessions: a range callers of kk_queue_submit are unlikely
// to pick, one id per session.
std::atomic<uint64_t> g_stream_ids{0xC000000000000000ull};
}  // namespace

extern "C" {

int kk_stream_preset(int32_t mode, kk_stream_config *out) {
    if (!out || (mode != 0 && mode != 1)) return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "unknown preset");
    kk_stream_config c{};
    if (mode == 0) {  // adaptative
        c.comma_pause_ms = 70;
        c.sentence_pause_ms = 170;
        c.paragraph_pause_ms = 350;
        c.crossfade_ms = 25;
        c.max_silence_trim_ms = 120;
    } else {  // long-form
        c.comma_pause_ms = 90;
        c.sentence_pause_ms = 220;
        c.paragraph_pause_ms = 450;
        c.crossfade_ms = 35;
        c.max_silence_trim_ms = 160;
    }
    c.trim_silence = 1;
    c.sample_rate = 24000;
    *out = c;
    return KK_OK;
}

int kk_postprocess_chunk(const kk_stream_config *cfg, const float *audio, int64_t n, int32_t boundary_after,
                         int32_t is_first, int32_t is_last, float *out, int64_t capacity, int64_t *n_out) {
    if (!config_ok(cfg) || (!audio && n > 0) || n < 0 || !boundary_ok(boundary_after) || !n_out ||
        (!out && capacity > 0) || capacity < 0)
        return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "invalid post-processing arguments");
    return s_guard([&] {
        std::vector<float> v;
        postprocess(*cfg, audio, (size_t)n, boundary_after, is_first != 0, is_last != 0, v);
        return copy_out(v, out, capacity, n_out);
    });
}

int kk_crossfade(const kk_stream_config *cfg, const float *prev, int64_t n_prev, const float *next, int64_t n_next,
                 int32_t boundary, float *out, int64_t capacity, int64_t *n_out) {
    if (!config_ok(cfg) || n_prev < 0 || n_next < 0 || (!prev && n_prev > 0) || (!next && n_next > 0) ||
        !boundary_ok(boundary) || !n_out || (!out && capacity > 0) || capacity < 0)
        return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "invalid crossfade arguments");
    return s_guard([&] {
        std::vector<float> v;
        crossfade_smart(*cfg, prev, (size_t)n_prev, next, (size_t)n_next, boundary, v);
        return copy_out(v, out, capacity, n_out);
    });
}

int kk_stream_create(kk_queue *q, const kk_stream_config *cfg, kk_stream **out) {
    if (out) *out = nullptr;
    if (!q || !out || !config_ok(cfg)) return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "invalid stream arguments");
    return s_guard([&] {
        kk_stream *s = new kk_stream();
        s->q = q;
        s->cfg = *cfg;
        s->request = g_stream_ids.fetch_add(1);
        *out = s;
        return (int)KK_OK;
    });
}

int kk_stream_push(kk_stream *s, int32_t n_frames, const float *asr, const float *f0, const float *noise,
                   const float *style, int32_t boundary_after, int32_t is_last) {
    if (!s || !asr || !f0 || !noise || !style || !boundary_ok(boundary_after))
        return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "invalid stream push arguments");
    if (s->pushed_last) return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "push after the last chunk");
    if (n_frames < 1 || n_frames > kk::kMaxFrames)
        return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "chunk length out of range");
    return s_guard([&] {
        const size_t T = (size_t)n_frames;
        KkStreamChunk c;
        c.T = n_frames;
        c.boundary = boundary_after;
        c.index = s->n_pushed;
        c.first = s->n_pushed == 0;
        c.last = is_last != 0;
        c.in.resize(T * 512 + 4 * T + 128);
        std::memcpy(c.in.data(), asr, T * 512 * sizeof(float));
        std::memcpy(c.in.data() + T * 512, f0, 2 * T * sizeof(float));
        std::memcpy(c.in.data() + T * 514, noise, 2 * T * sizeof(float));
        std::memcpy(c.in.data() + T * 516, style, 128 * sizeof(float));
        c.audio.resize(600 * T);
        s->chunks.push_back(std::move(c));
        KkStreamChunk &b = s->chunks.back();
        const float *p = b.in.data();
        const int rc = kk_queue_submit(s->q, s->request, n_frames, p, p + T * 512, p + T * 514, p + T * 516,
                                       b.audio.data(), &b.ticket);
        if (rc != KK_OK) {
            s->chunks.pop_back();
            return rc;  // the queue's message stands
        }
        ++s->n_pushed;
        if (b.last) s->pushed_last = true;
        return (int)KK_OK;
    });
}

int kk_stream_next(kk_stream *s, int32_t timeout_ms, const float **samples, int64_t *n_samples,
                   int32_t *chunk_index) {
    if (!s || !samples || !n_samples || !chunk_index)
        return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "invalid stream next arguments");
    *samples = nullptr;
    *n_samples = 0;
    *chunk_index = -1;
    if (s->chunks.empty()) return s->returned_last ? (int)KK_STREAM_END : (int)KK_QUEUE_PENDING;
    return s_guard([&] {
        KkStreamChunk &c = s->chunks.front();
        const int rc = kk_queue_wait(s->q, c.ticket, timeout_ms);
        if (rc == KK_QUEUE_PENDING) return rc;  // the ticket stays live
        *chunk_index = c.index;
        const bool last = c.last;
        if (rc != KK_OK) {
            // a failed or cancelled chunk: nothing to hand out, and the next
            // chunk is not crossfaded onto the tail from before it
            s->tail.clear();
            s->chunks.pop_front();
            if (last) s->returned_last = true;
            return rc;
        }
        // postprocess_and_crossfade (streaming.cpp:26-60)
        postprocess(s->cfg, c.audio.data(), c.audio.size(), c.boundary, c.first, c.last, s->tmp);
        if (!s->tail.empty() && !s->tmp.empty())
            crossfade_smart(s->cfg, s->tail.data(), s->tail.size(), s->tmp.data(), s->tmp.size(), c.boundary,
                            s->out);
        else
            s->out.swap(s->tmp);
        const size_t ncf = samples_of(s->cfg.crossfade_ms, s->cfg.sample_rate);
        if (!s->out.empty() && ncf > 0) {
            const size_t from = s->out.size() > ncf ? s->out.size() - ncf : 0;
            s->tail.assign(s->out.begin() + (ptrdiff_t)from, s->out.end());
        } else {
            s->tail.clear();
        }
        s->chunks.pop_front();
        if (last) s->returned_last = true;
        *samples = s->out.data();
        *n_samples = (int64_t)s->out.size();
        return (int)KK_OK;
    });
}

int kk_stream_cancel(kk_stream *s) {
    if (!s) return kk::queue_error(KK_ERROR_INVALID_ARGUMENT, "null stream");
    return kk_queue_cancel(s->q, s->request, nullptr);
}

void kk_stream_destroy(kk_stream *s) {
    if (!s) return;
    // the queue may still write into the chunks' buffers: undispatched ones
    // are cancelled, the others are waited for
    kk_queue_cancel(s->q, s->request, nullptr);
    for (KkStreamChunk &c : s->chunks) kk_queue_wait(s->q, c.ticket, -1);
    delete s;
}

}  // extern "C"
