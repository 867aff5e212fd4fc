/*
 * extern "C" entry points over the reference's own, unmodified
 * src/arch/kokoro/kokoro.cpp, compiled into oracle/_ref/ by oracle/Makefile.
 * TEST INFRASTRUCTURE ONLY: the tests use them to pin the oracle's duration
 * rounding and alignment (R11) against the reference's real code.
 *
 * The file is included whole, so that build_duration_mask (:115-152, in an
 * anonymous namespace) can be called from this translation unit;
 * duration_to_frames (:181-193) is an external function. The ggml headers
 * are the declaration-only stand-ins of oracle/ref_shim/, and everything
 * that would build a ggml graph is dropped at link time (hidden visibility,
 * --gc-sections).
 */
#include "arch/kokoro/kokoro.cpp"

#define KKREF_API __attribute__((visibility("default")))

extern "C" {

/* duration_to_frames(value, speed). */
KKREF_API int kkref_duration_to_frames(float value, float speed) { return kokopop::duration_to_frames(value, speed); }

/* build_duration_mask: frames [n_tokens] -> mask [n_tokens, total_frames]
 * (mask[token * total_frames + frame] = 1 where the frame belongs to the
 * token). Returns 0, or -1 when the reference reports an error. */
KKREF_API int kkref_duration_mask(const int32_t *frames, int64_t n_tokens, int64_t total_frames, float *mask) {
    std::vector<int> d(frames, frames + n_tokens);
    std::vector<float> m;
    std::string error;
    if (!kokopop::build_duration_mask(d, total_frames, n_tokens, m, error)) return -1;
    std::copy(m.begin(), m.begin() + static_cast<ptrdiff_t>(total_frames * n_tokens), mask);
    return 0;
}

}  // extern "C"
