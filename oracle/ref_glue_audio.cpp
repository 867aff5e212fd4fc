/*
 * extern "C" entry points over the reference's own, unmodified
 * src/arch/kokoro/audio_utils.cpp, compiled into oracle/_ref/ by
 * oracle/Makefile. TEST INFRASTRUCTURE ONLY: the tests use them to pin the
 * oracle's harmonic source + STFT (R1) and its Kokoro iSTFT conversion (R9)
 * against the reference's real code.
 *
 * The file is included whole, so that its file-local functions
 * fill_harmonic_stft (:120-422) and cpu_istft_data (:462-532) can be called
 * from this translation unit. The ggml headers it needs are the
 * declaration-only stand-ins of oracle/ref_shim/; everything that would build
 * a ggml graph is dropped at link time (hidden visibility, --gc-sections).
 * What those two functions still reference is defined below as stubs that
 * report failure: the KokoroArch member functions (whose real definitions
 * live in kokoro_arch.cpp, which is not compiled here) and tensor_to_f32
 * (src/model/model.cpp). require_tensor comes from kokoro.cpp, compiled in
 * ref_glue_kokoro.cpp, and finds no tensor through the cached_tensor stub.
 * fill_harmonic_stft never reaches those lookups here,
 * because the glue hands it the merge weights already loaded
 * (harmonic_source_loaded = true), exactly as the reference's second and
 * later calls see them.
 */
#include "arch/kokoro/audio_utils.cpp"

#define KKREF_API __attribute__((visibility("default")))

namespace kokopop {

bool KokoroArch::load(Model &, std::string &error) {
    error = "oracle stub";
    return false;
}
const VoiceDesc *KokoroArch::find_voice(std::string_view) const { return nullptr; }
const VoiceDesc *KokoroArch::default_voice() const { return nullptr; }
bool KokoroArch::phonemize(const std::string &, const VoiceDesc &, std::string &, std::string &error) const {
    error = "oracle stub";
    return false;
}
bool KokoroArch::tokenize(const std::string &, const VoiceDesc &, std::vector<uint32_t> &,
                          std::string &error) const {
    error = "oracle stub";
    return false;
}
ChunkConfig KokoroArch::adjust_chunk_config(ChunkConfig cfg, const VoiceDesc &) const { return cfg; }
bool KokoroArch::synthesize(Model &, const std::vector<uint32_t> &, const VoiceDesc &, float,
                            const SynthesisExtras &, std::vector<float> &, std::string &error) {
    error = "oracle stub";
    return false;
}
ggml_tensor *KokoroArch::cached_tensor(const std::string &) const { return nullptr; }
bool tensor_to_f32(Backend &, ggml_tensor *, std::vector<float> &) { return false; }

}  // namespace kokopop

extern "C" {

/* fill_harmonic_stft on host buffers: f0 [n_f0] (Hz), the nine
 * m_source.l_linear weights and its bias; har [22, target_frames]
 * (bin-major), source [300 n_f0] (the tanh-merged sine source). Returns 0,
 * or -1 with nothing written. */
KKREF_API int kkref_harmonic_stft(const float *f0, int64_t n_f0, int64_t target_frames, const float *merge_w,
                                  float merge_b, float *har, float *source) {
    using namespace kokopop;
    KokoroArch model;
    model.harmonic_merge_w.assign(merge_w, merge_w + KOKOPOP_HARMONIC_COUNT);
    model.harmonic_merge_b = merge_b;
    model.harmonic_source_loaded = true;
    const std::vector<float> f(f0, f0 + n_f0);
    std::vector<float> h;
    std::string error;
    if (!fill_harmonic_stft(model, f, target_frames, h, error)) return -1;
    std::copy(h.begin(), h.end(), har);
    const size_t n_src = static_cast<size_t>(n_f0) * KOKOPOP_UPSAMPLE;
    std::copy(model.tmp_stft_source_f32.begin(), model.tmp_stft_source_f32.begin() + n_src, source);
    return 0;
}

/* cpu_istft_data: post [22, n_frames] (bin-major) -> audio
 * [(n_frames - 1) * 5], clamped to +-1; *n_out = samples written. */
KKREF_API int kkref_istft_kokoro(const float *post, int64_t n_frames, float *audio, int64_t *n_out) {
    using namespace kokopop;
    *n_out = 0;
    KokoroArch model;
    std::vector<float> out;
    if (!cpu_istft_data(model, post, n_frames, out) && n_frames > 1) return -1;
    std::copy(out.begin(), out.end(), audio);
    *n_out = static_cast<int64_t>(out.size());
    return 0;
}

}  // extern "C"
