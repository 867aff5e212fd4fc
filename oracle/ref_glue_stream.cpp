/*
 * extern "C" entry points over the reference's own, unmodified chunk
 * post-processing (src/audio/audio_postprocess.cpp), compiled into
 * oracle/_ref/ by oracle/Makefile. TEST INFRASTRUCTURE ONLY: the tests pin
 * the library's kk_postprocess_chunk / kk_crossfade / kk_stream against
 * postprocess_chunk_audio and apply_crossfade_smart bit for bit.
 *
 * The translation unit is compiled with the reference's flags (-O3, no
 * -march): its NEON / AVX2 branches are not taken, as in the reference's own
 * x86-64 build.
 */
#include "audio/audio_postprocess.h"

#include <cstring>

#define KKREF_API __attribute__((visibility("default")))

extern "C" {

/* postprocess_chunk_audio with a ChunkConfig holding the given post-
 * processing fields (the rest at their defaults); returns the processed
 * length, copying at most `capacity` samples. */
KKREF_API int64_t kkref_postprocess_chunk(const float *audio, int64_t n, int boundary, int is_first, int is_last,
                                          int comma_ms, int sentence_ms, int paragraph_ms, int crossfade_ms,
                                          int trim, int max_trim_ms, int sample_rate, float *out,
                                          int64_t capacity) {
    using namespace kokopop;
    ChunkConfig cfg;
    cfg.comma_pause_ms = comma_ms;
    cfg.sentence_pause_ms = sentence_ms;
    cfg.paragraph_pause_ms = paragraph_ms;
    cfg.crossfade_ms = crossfade_ms;
    cfg.trim_silence = trim != 0;
    cfg.max_silence_trim_ms = max_trim_ms;
    Chunk chunk;
    chunk.boundary_after = static_cast<Boundary>(boundary);
    chunk.is_first = is_first != 0;
    chunk.is_last = is_last != 0;
    std::vector<float> a(audio, audio + n);
    const std::vector<float> r = postprocess_chunk_audio(a, chunk, 0, 1, cfg, sample_rate);
    const int64_t m = static_cast<int64_t>(r.size());
    if (m <= capacity && m > 0) std::memcpy(out, r.data(), r.size() * sizeof(float));
    return m;
}

/* apply_crossfade_smart(prev, next, boundary, crossfade_ms, sample_rate). */
KKREF_API int64_t kkref_crossfade_smart(const float *prev, int64_t n_prev, const float *next, int64_t n_next,
                                        int boundary, int crossfade_ms, int sample_rate, float *out,
                                        int64_t capacity) {
    using namespace kokopop;
    std::vector<float> p(prev, prev + n_prev), q(next, next + n_next);
    const std::vector<float> r = apply_crossfade_smart(p, q, static_cast<Boundary>(boundary), crossfade_ms,
                                                       sample_rate);
    const int64_t m = static_cast<int64_t>(r.size());
    if (m <= capacity && m > 0) std::memcpy(out, r.data(), r.size() * sizeof(float));
    return m;
}

}  // extern "C"
