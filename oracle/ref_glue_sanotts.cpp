/*
 * extern "C" entry points over the reference's own, unmodified sanoTTS and
 * iSTFT sources, compiled into oracle/_ref/ by oracle/Makefile. TEST
 * INFRASTRUCTURE ONLY: the tests use them to pin the oracle's Vocos
 * restatement (its radix-2 iSTFT at n_fft 1024 and its DC blocker) and to
 * draw the decoder's noise input exactly as the reference draws it.
 *
 * src/arch/sanotts/sano_vocos.cpp is included whole so that its file-local
 * dc_block (:81-92) and bin_mask (:72-78) can be called; everything that
 * would build a ggml graph is dropped at link time (hidden visibility,
 * --gc-sections). src/arch/sanotts/sano_noise.cpp (no ggml) is compiled
 * beside it. src/audio/istft.cpp is the same translation unit the Kokoro
 * glue uses.
 */
#include "arch/sanotts/sano_vocos.cpp"

#include <algorithm>

#define KKREF_API __attribute__((visibility("default")))

extern "C" {

/* istft() with a plan for (n_fft, hop, center): re / im frame-major
 * [frames][n_fft / 2 + 1] (the view sano_run_vocos builds, :217-223) ->
 * audio (capacity hop * (frames - 1)); *n_out = samples. 0 or -1. */
KKREF_API int kkref_istft_complex(const float *re, const float *im, int64_t frames, int n_fft, int hop,
                                  float *audio, int64_t *n_out) {
    using namespace kokopop;
    *n_out = 0;
    IstftPlan plan;
    std::string error;
    if (!IstftPlan::create(IstftConfig{static_cast<uint32_t>(n_fft), static_cast<uint32_t>(hop), true}, plan,
                           error))
        return -1;
    ComplexSpectrumView view;
    view.real = re;
    view.imag = im;
    view.bins = plan.bins();
    view.frames = static_cast<size_t>(frames);
    view.bin_stride = 1;
    view.frame_stride = static_cast<ptrdiff_t>(plan.bins());
    IstftWorkspace ws;
    std::vector<float> out;
    if (!istft(plan, ws, view, out, error)) return -1;
    std::copy(out.begin(), out.end(), audio);
    *n_out = static_cast<int64_t>(out.size());
    return 0;
}

/* dc_block(audio, pole), in place. */
KKREF_API void kkref_dc_block(float *audio, int64_t n, float pole) {
    std::vector<float> a(audio, audio + n);
    kokopop::dc_block(a, pole);
    std::copy(a.begin(), a.end(), audio);
}

/* bin_mask(bins) -> mask [bins]. */
KKREF_API void kkref_bin_mask(uint32_t bins, float *mask) {
    const std::vector<float> m = kokopop::bin_mask(bins);
    std::copy(m.begin(), m.end(), mask);
}

/* sano::seeded_noise(seed, channels, frames) -> noise [channels][frames];
 * 0 or -1 (fewer than 16 values). */
KKREF_API int kkref_sano_noise(uint64_t seed, int64_t channels, int64_t frames, float *noise) {
    std::vector<float> out;
    std::string error;
    if (!kokopop::sano::seeded_noise(seed, static_cast<size_t>(channels), static_cast<size_t>(frames), out, error))
        return -1;
    std::copy(out.begin(), out.end(), noise);
    return 0;
}

}  // extern "C"
