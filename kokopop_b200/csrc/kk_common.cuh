// Shared device-side definitions of the Kokoro-82M hot path (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace kk {

// Constants of the reference's src/core/constants.h.
constexpr int kStftN = 20;
constexpr int kHop = 5;
constexpr int kBins = kStftN / 2 + 1;
constexpr int kHarmonics = 9;
constexpr int kUpsample = 300;  // samples per F0 frame
constexpr int kStyle = 128;

// A ragged batch is packed along time: utterance u of a level with
// multiplier m occupies rows [m * offT[u], m * offT[u] + len) of a [C, R]
// channel-major buffer (time-fastest within a channel, like ggml's [T, C]).
// The rows between utterances are gaps that conv operands keep at zero, so
// one convolution over the whole buffer equals per-utterance zero-padded
// convolutions.
struct Batch {
    int n;                   // utterances
    const int32_t *T;        // [n] length in base units (device)
    const int64_t *offT;     // [n] row offset at the base level (device)
};

// Round-to-nearest-even float -> half -> float, as ggml's F16 im2col does.
__device__ __forceinline__ float round_f16(float x) {
    return __half2float(__float2half_rn(x));
}

// Leaky ReLU exactly as ggml_vec_leaky_relu_f32:
// (x > 0 ? x : 0) + slope * (x < 0 ? x : 0).
__device__ __forceinline__ float leaky(float x, float slope) {
    return __fadd_rn(x > 0.f ? x : 0.f, __fmul_rn(slope, x < 0.f ? x : 0.f));
}

// sin for the Snake activation. Its arguments v * alpha are small in
// practice, where the odd Taylor polynomial of sin to x^9 (Horner in x^2)
// is accurate to float rounding: the first omitted term x^11/11! is below
// 3e-9 relative for |x| <= pi/4. Larger arguments take the library sinf.
constexpr float kSnakeSmall = 0.78539816f;  // pi / 4: the polynomial's range

// The polynomial alone, for |x| <= kSnakeSmall.
__device__ __forceinline__ float snake_sin_small(float x) {
    const float x2 = x * x;
    float p = 2.7557319e-06f;         // 1/9!
    p = fmaf(p, x2, -1.9841270e-04f);  // -1/7!
    p = fmaf(p, x2, 8.3333333e-03f);   // 1/5!
    p = fmaf(p, x2, -1.6666667e-01f);  // -1/3!
    return fmaf(x * x2, p, x);
}

__device__ __forceinline__ float snake_sin(float x) {
    if (fabsf(x) <= kSnakeSmall) return snake_sin_small(x);
    return sinf(x);
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace kk
