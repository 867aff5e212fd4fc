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

// Exact GELU as ggml_vec_gelu_erf_f32 evaluates it, left to right:
// (0.5f * x) * (1.0f + erff(x * SQRT_2_INV)), each operation rounded once.
// erff is CUDA's single-precision erf (at most 2 ulp from the exact value,
// like a C library's); the oracle takes it correctly rounded.
__device__ __forceinline__ float gelu_erf(float x) {
    const float t = __fmul_rn(x, 0.70710678118654752440f);
    const float e = erff(t);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, e));
}

// sin^2 for the Snake activation v + sin^2(v alpha) / alpha. sin^2 has
// period pi: with k the integer nearest y * 2/pi and r = y - k pi/2
// (|r| <= pi/4), sin^2 y = sin^2 r for even k and cos^2 r = 1 - sin^2 r for
// odd k. sin^2 r is its Taylor series
//   sum_{n >= 1} (-1)^(n+1) 2^(2n-1) r^(2n) / (2n)!  =  r^2 P(r^2),
// P to the r^10 term (Horner); the first omitted term is below 6e-9 of the
// value on |r| <= pi/4. The reduction is Cody-Waite with pi/2 split into two
// floats (r exact to about 2e-11 for |y| <= kSnakeReduce); k is rounded by
// the 1.5 * 2^23 addend, whose low mantissa bit is k's parity. Against
// sin^2 in double precision: within 2 ulp for |y| <= 0.78, within 3.6 ulp
// (or 1.1e-7 absolute near the zeros) up to kSnakeReduce, 0.38-0.46 ulp on
// average (a C library's sinf, squared and rounded, averages 0.52-0.57).
// Larger arguments take the library sinf, squared.
constexpr float kSnakeFast = 0.77f;       // |y| < kSnakeFast: k = 0 and r = y
constexpr float kSnakeReduce = 8192.0f;  // the two-constant reduction's range

// r^2 P(r^2) given r2 = r * r.
__device__ __forceinline__ float snake_p(float r2) {
    float p = -4.2755596e-06f;          // -2 / 467775     (n = 6)
    p = fmaf(p, r2, 1.4109348e-04f);    //  2 / 14175      (n = 5)
    p = fmaf(p, r2, -3.1746032e-03f);   // -1 / 315        (n = 4)
    p = fmaf(p, r2, 4.4444446e-02f);    //  2 / 45         (n = 3)
    p = fmaf(p, r2, -3.3333334e-01f);   // -1 / 3          (n = 2)
    p = fmaf(p, r2, 1.0f);              //  1              (n = 1)
    return __fmul_rn(r2, p);
}

// |y| <= kSnakeReduce. For |y| < kSnakeFast this is snake_p(y * y) bit for
// bit (k = +0: both fmas return y unchanged, and the parity bit is 0).
__device__ __forceinline__ float snake_sin2_reduced(float y) {
    const float t = fmaf(y, 0.63661975f, 12582912.0f);  // 2/pi; 1.5 * 2^23
    const float k = __fsub_rn(t, 12582912.0f);
    float r = fmaf(-k, 1.5707964f, y);    // float(pi/2)
    r = fmaf(-k, -4.371139e-08f, r);      // pi/2 - float(pi/2)
    const float s2 = snake_p(__fmul_rn(r, r));
    return (__float_as_int(t) & 1) ? __fsub_rn(1.0f, s2) : s2;
}

// Arguments past the reduction's range (and non-finite ones), out of line so
// that the unrolled element loops stay small.
static __device__ __noinline__ float snake_sin2_huge(float y) {
    const float s = sinf(y);
    return __fmul_rn(s, s);
}

__device__ __forceinline__ float snake_sin2(float y) {
    return fabsf(y) <= kSnakeReduce ? snake_sin2_reduced(y) : snake_sin2_huge(y);
}

// Packed FP32 pairs (sm_100 f32x2): two lanes of IEEE round-to-nearest
// arithmetic per instruction, each the same value as the scalar operation.
// The assembler contracts a packed mul.rn feeding a packed add.rn into one
// fused multiply-add (measured on B200: about 15 % of random operand pairs
// then differ from the separately rounded scalar ops). f2mul is written as
// fma.rn(a, b, -0), the product rounded once (-0 is the identity of addition
// for every product, signed zeros included), but where a product feeds an
// add whose rounding must match a reference, use the scalar _rn intrinsics:
// a chain of such packed ops still differed from them in about 4e-5 of the
// results on B200.
__device__ __forceinline__ float2 f2add(float2 a, float2 b) {
    float2 r;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
    float2 r;
    asm("{\n .reg .b64 ra, rb, rz, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mov.b64 rz, {%6, %6};\n fma.rn.f32x2 rd, ra, rb, rz;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(-0.0f));
    return r;
}
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}

// FP32 pairs held in one 64-bit register from load to store (no packing
// moves between operations); products as fma(a, b, z) with z a packed -0
// from a kernel parameter, so each step keeps its own rounding.
typedef unsigned long long p2_t;
__device__ __forceinline__ p2_t p2_bc(float v) {
    p2_t d;
    asm("mov.b64 %0, {%1, %1};" : "=l"(d) : "f"(v));
    return d;
}
__device__ __forceinline__ p2_t p2_pack(float lo, float hi) {
    p2_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ float2 p2_unpack(p2_t a) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(a));
    return r;
}
__device__ __forceinline__ p2_t p2_add(p2_t a, p2_t b) {
    p2_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ p2_t p2_fma(p2_t a, p2_t b, p2_t c) {
    p2_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Split F32 operands for the half tensor cores: v = hi + lo with hi = half(v)
// and lo = half(v - hi) (the difference is exact in F32). A product of two
// splits summed as hi*hi' + hi*lo' + lo*hi' carries about 22 significant
// bits; the omitted lo*lo' is below 2^-22 of |v v'| (less where lo falls in
// the half subnormal range, below 2^-14, where its absolute error is 2^-25).
__device__ __forceinline__ __half split_lo(float v, __half hi) {
    return __float2half_rn(__fsub_rn(v, __half2float(hi)));
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Instance-norm terms from the double sums over an utterance's n valid rows,
// ggml_norm semantics (eps 1e-5): mean = (float)S1 / n; the two-pass variance
// sum((x - mean)^2) / n with the float mean, expanded as
// (S2 - 2 mean S1 + n mean^2) / n in double; scale = 1 / sqrtf(var + eps).
__device__ __forceinline__ float2 norm_from_sums(double s1, double s2, int64_t n) {
    const float mean = __fdiv_rn((float)s1, (float)n);
    const double md = (double)mean;
    double q = s2 - 2.0 * md * s1 + (double)n * md * md;
    if (q < 0.0) q = 0.0;
    const float var = (float)(q / (double)n);
    return make_float2(mean, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f))));
}

// The utterance whose slot holds row q of level m: the last u with
// m * offT[u] <= q, or 0 when q lies before the first utterance (such rows,
// and the gap rows after an utterance, fall outside that utterance's
// [m * offT[u], m * offT[u] + m * T[u] + extra) and are not counted).
__device__ __forceinline__ int utt_of_row(const Batch &b, int m, int64_t q) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((int64_t)m * __ldg(b.offT + mid) <= q)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

}  // namespace kk
