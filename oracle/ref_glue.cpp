/*
 * extern "C" entry point over the reference's own, unmodified
 * src/arch/kokoro/lstm_fused.cpp, compiled into oracle/_ref/ by
 * oracle/Makefile. TEST INFRASTRUCTURE ONLY: the tests use it to pin the
 * oracle's restatement against the reference's real code. The other entry
 * points of oracle/_ref/ are in ref_glue_audio.cpp and ref_glue_kokoro.cpp.
 */
#include "arch/kokoro/lstm_fused.h"

#include <cstring>

#define KKREF_API __attribute__((visibility("default")))

extern "C" {

/* lstm_fused_callback (src/arch/kokoro/lstm_fused.cpp:339-378) on host
 * buffers: pre_gates [N, 4H], w_hh ggml [H, 4H] (= rowwise), b_hh [4H],
 * out [N, H]. */
KKREF_API void kkref_lstm_direction(const float *pre_gates, const float *w_hh, const float *b_hh, int64_t H,
                                    int64_t N, int reverse, float *out) {
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
