/*
 * extern "C" entry points over the reference's own, unmodified sources
 * (src/audio/istft.cpp and src/arch/kokoro/lstm_fused.cpp), compiled into
 * oracle/_ref/ by oracle/Makefile. TEST INFRASTRUCTURE ONLY: the tests use it
 * to pin the oracle's restatement against the reference's real code.
 */
#include "audio/istft.h"
#include "arch/kokoro/lstm_fused.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

extern "C" {

/* cpu_istft_data (src/arch/kokoro/audio_utils.cpp:462-532): the Kokoro
 * log-magnitude / sin-phase conversion (restated here: that file needs ggml)
 * followed by the reference's own istft() and the +-1 clamp. */
int kkref_istft_kokoro(const float *post, int64_t n_frames, float *audio, int64_t *n_out) {
    using namespace kokopop;
    *n_out = 0;
    if (n_frames <= 0) return 0;
    IstftPlan plan;
    std::string error;
    if (!IstftPlan::create(IstftConfig{20, 5, true}, plan, error)) return -1;
    const size_t bins = plan.bins();
    const size_t frames = static_cast<size_t>(n_frames);
    std::vector<float> real(bins * frames), imag(bins * frames);
    for (size_t k = 0; k < bins; ++k) {
        for (size_t t = 0; t < frames; ++t) {
            const float mag = std::exp(std::clamp(post[k * frames + t], -20.0f, 8.0f));
            const float phase = std::sin(post[(k + 11) * frames + t]);
            real[k * frames + t] = mag * std::cos(phase);
            imag[k * frames + t] = mag * std::sin(phase);
        }
    }
    ComplexSpectrumView spectrum;
    spectrum.real = real.data();
    spectrum.imag = imag.data();
    spectrum.bins = bins;
    spectrum.frames = frames;
    spectrum.bin_stride = static_cast<ptrdiff_t>(frames);
    spectrum.frame_stride = 1;
    IstftWorkspace ws;
    std::vector<float> out;
    if (!istft(plan, ws, spectrum, out, error)) return -1;
    for (size_t i = 0; i < out.size(); ++i) audio[i] = std::clamp(out[i], -1.0f, 1.0f);
    *n_out = static_cast<int64_t>(out.size());
    return 0;
}

/* lstm_fused_callback (src/arch/kokoro/lstm_fused.cpp:339-378) on host
 * buffers: pre_gates [N, 4H], w_hh ggml [H, 4H] (= rowwise), b_hh [4H],
 * out [N, H]. */
void kkref_lstm_direction(const float *pre_gates, const float *w_hh, const float *b_hh,
                          int64_t H, int64_t N, int reverse, float *out) {
    using namespace kokopop;
    ggml_tensor pre{};
    pre.type = GGML_TYPE_F32;
    pre.ne[0] = 4 * H; pre.ne[1] = N; pre.ne[2] = pre.ne[3] = 1;
    pre.nb[0] = sizeof(float); pre.nb[1] = 4 * H * sizeof(float);
    pre.nb[2] = pre.nb[3] = pre.nb[1] * N;
    pre.data = const_cast<float *>(pre_gates);
    ggml_tensor dst{};
    dst.type = GGML_TYPE_F32;
    dst.ne[0] = H; dst.ne[1] = N; dst.ne[2] = dst.ne[3] = 1;
    dst.nb[0] = sizeof(float); dst.nb[1] = H * sizeof(float);
    dst.nb[2] = dst.nb[3] = dst.nb[1] * N;
    dst.data = out;
    LstmCustomParams p{};
    p.opencl.magic = kLstmOpenclParamsMagic;
    p.opencl.w_hh_f32 = w_hh;
    p.opencl.b_hh = b_hh;
    p.opencl.hidden = H;
    p.opencl.n_steps = N;
    p.opencl.reverse = reverse ? 1 : 0;
    p.w_hh_rowwise = w_hh;
    p.metal_kernel = nullptr;
    p.whh_key = nullptr;
    lstm_fused_callback(&dst, nullptr, &pre, 0, 1, &p);
}

} // extern "C"
