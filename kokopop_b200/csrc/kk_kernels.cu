// Memory-bound and small kernels of the Kokoro-82M hot path (sm_100a):
// harmonic source + STFT, instance-norm statistics, the AdaIN / Snake /
// LeakyReLU operand prologue, ConvTranspose upsampling, the depthwise pool,
// F0/N convs and the fused iSTFT. Dense convolutions live in kk_conv*.cu.
//
// Element-wise arithmetic uses the _rn intrinsics wherever the reference
// rounds each operation separately (its translation units build without FMA
// contraction), so these kernels reproduce the reference's rounding exactly
// except inside the transcendental functions.
#include "kk_kernels.h"

#include <math.h>

namespace kk {

// ---------------------------------------------------------------------------
// packing helpers
// ---------------------------------------------------------------------------

// Copies per-utterance [C, m*T + extra] tensors (concatenated back to back,
// src offset C * (m*cumT + extra*u)) into the packed [C, R] buffer.
__global__ void k_scatter(const float *__restrict__ src, float *__restrict__ dst, int64_t R, int C,
                          int m, int extra, Batch b, const int64_t *__restrict__ cumT) {
    const int u = blockIdx.z;
    const int c = blockIdx.y;
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const float *s = src + (int64_t)C * ((int64_t)m * cumT[u] + (int64_t)extra * u) + (int64_t)c * len;
    float *d = dst + (int64_t)c * R + (int64_t)m * b.offT[u];
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < len;
         t += (int64_t)gridDim.x * blockDim.x)
        d[t] = s[t];
}

// all_finite (src/arch/kokoro/kokoro.cpp:91-99) on the device: the smallest
// index of a non-finite value, and the error word if nothing set it before.
__global__ void k_check_finite(const float *__restrict__ x, int64_t n, int label, DevStatus *status) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (!isfinite(x[i])) {
            atomicMin(&status->first[label], (unsigned long long)i);
            atomicCAS(&status->code, 0, kErrNonFinite + label);
        }
    }
}

void check_finite(const float *x, int64_t n, int label, DevStatus *status, cudaStream_t st) {
    if (n <= 0) return;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 1184) blocks = 1184;  // 8 per SM
    k_check_finite<<<(unsigned)blocks, 256, 0, st>>>(x, n, label, status);
}

void scatter(const float *src, float *dst, int64_t R, int C, int m, int extra, const Batch &b,
             const int64_t *cumT, int max_len, cudaStream_t st) {
    dim3 grid((unsigned)((max_len + 255) / 256 < 64 ? (max_len + 255) / 256 : 64), C, b.n);
    k_scatter<<<grid, 256, 0, st>>>(src, dst, R, C, m, extra, b, cumT);
}

// The inverse of k_scatter: the packed [C, R] rows of each utterance back to
// per-utterance [C, m*T + extra] tensors, concatenated.
__global__ void k_gather(const float *__restrict__ src, float *__restrict__ dst, int64_t R, int C, int m,
                         int extra, Batch b, const int64_t *__restrict__ cumT) {
    const int u = blockIdx.z;
    const int c = blockIdx.y;
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const float *s = src + (int64_t)c * R + (int64_t)m * b.offT[u];
    float *d = dst + (int64_t)C * ((int64_t)m * cumT[u] + (int64_t)extra * u) + (int64_t)c * len;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < len;
         t += (int64_t)gridDim.x * blockDim.x)
        d[t] = s[t];
}

void gather(const float *src, float *dst, int64_t R, int C, int m, int extra, const Batch &b,
            const int64_t *cumT, int max_len, cudaStream_t st) {
    dim3 grid((unsigned)((max_len + 255) / 256 < 64 ? (max_len + 255) / 256 : 64), C, b.n);
    k_gather<<<grid, 256, 0, st>>>(src, dst, R, C, m, extra, b, cumT);
}

// ---------------------------------------------------------------------------
// AdaIN affine terms: gamma = Wg . style + bg, beta = Wb . style + bb
// (linear(), graph_ops.cpp:636-654). Sequential F32 sum over the 128 style
// features; ggml converts the style to half when the weight is F16.
// ---------------------------------------------------------------------------

__global__ void k_adain_affine(const AdainSite *__restrict__ sites, const float *__restrict__ style,
                               int n_utts) {
    const AdainSite s = sites[blockIdx.x];
    const int u = blockIdx.y;
    __shared__ float st[kStyle];
    for (int i = threadIdx.x; i < kStyle; i += blockDim.x) {
        const float v = style[(int64_t)u * kStyle + i];
        st[i] = s.f16 ? round_f16(v) : v;
    }
    __syncthreads();
    // weights transposed at upload ([128][C]) so the threads of a warp read
    // consecutive channels; the sum over the style features stays sequential
    for (int c = threadIdx.x; c < s.C; c += blockDim.x) {
        float g = 0.f, be = 0.f;
        for (int i = 0; i < kStyle; ++i) {
            g = __fadd_rn(g, __fmul_rn(s.gw[(int64_t)i * s.C + c], st[i]));
            be = __fadd_rn(be, __fmul_rn(s.bw[(int64_t)i * s.C + c], st[i]));
        }
        s.gamma[(int64_t)u * s.C + c] = __fadd_rn(g, s.gb[c]);
        s.beta[(int64_t)u * s.C + c] = __fadd_rn(be, s.bb[c]);
    }
}

void adain_affine(const AdainSite *sites_dev, int n_sites, const float *style, int n_utts,
                  cudaStream_t st) {
    if (n_sites == 0 || n_utts == 0) return;
    k_adain_affine<<<dim3(n_sites, n_utts), 256, 0, st>>>(sites_dev, style, n_utts);
}

// ---------------------------------------------------------------------------
// Instance-norm statistics, ggml_norm semantics (eps 1e-5): per (channel,
// utterance), mean = (float)sum_double / n, var = sum_double((x-mean)^2) / n,
// scale = 1 / sqrtf(var + eps) (ggml's norm, restated in the oracle).
// ---------------------------------------------------------------------------

template <int NT>
__device__ double block_sum_double(double v, double *red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x < 32) {
        r = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.0;
        r = warp_sum(r);
        if (threadIdx.x == 0) red[0] = r;
    }
    __syncthreads();
    return red[0];
}

// One pass: sum and sum of squares in double, then the (mean, scale) pair.
__global__ void __launch_bounds__(256) k_stats(const float *__restrict__ x, int64_t R, int C, int m,
                                               int extra, Batch b, float2 *__restrict__ ms) {
    __shared__ double red[32];
    const int c = blockIdx.x, u = blockIdx.y;
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const float *p = x + (int64_t)c * R + (int64_t)m * b.offT[u];
    double s1 = 0.0, s2 = 0.0;
    for (int64_t t = threadIdx.x; t < len; t += 256) {
        const double v = (double)p[t];
        s1 += v;
        s2 += v * v;
    }
    s1 = block_sum_double<256>(s1, red);
    s2 = block_sum_double<256>(s2, red);
    if (threadIdx.x == 0) ms[(int64_t)u * C + c] = norm_from_sums(s1, s2, len);
}

// One warp per (channel, utterance), for the decoder levels (m <= 2) where an
// utterance has a few hundred to ~1600 rows and a block per pair would wait
// on its barriers: lane l sums rows l, l + 32, ... in double, then the lanes
// combine in a fixed butterfly. The order depends only on the length, never
// on the rest of the batch.
__global__ void __launch_bounds__(256) k_stats_w(const float *__restrict__ x, int64_t R, int C, int m, int extra,
                                                 Batch b, float2 *__restrict__ ms) {
    const int c = blockIdx.x * 8 + (threadIdx.x >> 5), u = blockIdx.y, lane = threadIdx.x & 31;
    if (c >= C) return;  // the whole warp
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const float *p = x + (int64_t)c * R + (int64_t)m * b.offT[u];
    double s1 = 0.0, s2 = 0.0;
#pragma unroll 4
    for (int64_t t = lane; t < len; t += 32) {
        const double v = (double)p[t];
        s1 += v;
        s2 += v * v;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) ms[(int64_t)u * C + c] = norm_from_sums(s1, s2, len);
}

void stats(const float *x, int64_t R, int C, int m, int extra, const Batch &b, float2 *ms,
           cudaStream_t st) {
    if (m <= 2)
        k_stats_w<<<dim3((C + 7) / 8, b.n), 256, 0, st>>>(x, R, C, m, extra, b, ms);
    else
        k_stats<<<dim3(C, b.n), 256, 0, st>>>(x, R, C, m, extra, b, ms);
}

// The same terms from 32-row block partials part[c * NB + row / 32] = (S, M2)
// (S the block's sum over its k valid rows, M2 = sum (v - S / k)^2), written
// by the tensor-core convolution while it stores the tensor. Every utterance
// starts on a block boundary, so block i of utterance u holds its rows
// 32 i .. 32 i + k - 1 whatever the packing, and the fixed summation order
// below makes the result independent of the batch the utterance is in:
// S1 = sum S, S2 = sum (M2 + S^2 / k), in double.
// One warp per (utterance, channel); 8 per block.
__global__ void __launch_bounds__(256) k_stats_blocks(const float2 *__restrict__ part, int64_t NB, int C, int m,
                                                      int extra, Batch b, float2 *__restrict__ ms) {
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.x * 8 + (threadIdx.x >> 5), u = blockIdx.y;
    if (c >= C) return;
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const int64_t b0 = (int64_t)m * b.offT[u] / 32;
    const int64_t nb = (len + 31) / 32;
    const float2 *p = part + (int64_t)c * NB + b0;
    double s1 = 0.0, s2 = 0.0;
    if (b0 + nb <= NB) {
        // full blocks four at a time per lane, then the last (partial) block
        const int64_t nfull = len / 32;
        int64_t i = lane;
        for (; i + 96 < nfull; i += 128) {
            float2 q[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) q[k] = p[i + 32 * k];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const double S = (double)q[k].x;
                s1 += S;
                s2 += (double)q[k].y + S * S * (1.0 / 32.0);
            }
        }
        for (; i < nb; i += 32) {
            const float2 q = p[i];
            const int64_t k = len - 32 * i < 32 ? len - 32 * i : 32;
            const double S = (double)q.x;
            s1 += S;
            s2 += (double)q.y + S * S / (double)k;
        }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) ms[(int64_t)u * C + c] = norm_from_sums(s1, s2, len);
}

void stats_blocks(const float2 *part, int64_t NB, int C, int m, int extra, const Batch &b, float2 *ms,
                  cudaStream_t st) {
    k_stats_blocks<<<dim3((C + 7) / 8, b.n), 256, 0, st>>>(part, NB, C, m, extra, b, ms);
}

// ---------------------------------------------------------------------------
// Operand prologue: y = act(adain(x)), written only on valid rows (gaps of
// the operand buffer stay zero). adain_1d (graph_ops.cpp:888-907):
//   cur = ((x - mean) * scale) * norm_w + norm_b; cur = cur + cur * gamma;
//   cur = cur + beta
// act: none, LeakyReLU(slope) or Snake (graph_ops.cpp:392-497):
//   y = v + sinf(v * alpha)^2 * (1 / alpha)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) k_prologue(const float *__restrict__ x, float *__restrict__ y,
                                                  int64_t R, int C, int m, int extra, Batch b,
                                                  PrologueArgs a) {
    const int u = blockIdx.z, c = blockIdx.y;
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const int64_t base = (int64_t)c * R + (int64_t)m * b.offT[u];
    float mean = 0.f, scale = 1.f, nw = 1.f, nb = 0.f, g = 0.f, be = 0.f;
    if (a.norm) {
        const float2 s = a.ms[(int64_t)u * C + c];
        mean = s.x;
        scale = s.y;
        nw = a.norm_w[c];
        nb = a.norm_b[c];
        g = a.gamma[(int64_t)u * C + c];
        be = a.beta[(int64_t)u * C + c];
    }
    float alpha = 0.f, inv_a = 0.f;
    if (a.act == ACT_SNAKE) {
        alpha = a.alpha[c];
        inv_a = __fdiv_rn(1.0f, alpha);
    }
    for (int64_t t = blockIdx.x * 256 + threadIdx.x; t < len; t += (int64_t)gridDim.x * 256) {
        float v = x[base + t];
        if (a.x2) v = __fmul_rn(__fadd_rn(__fadd_rn(v, a.x2[base + t]), a.x3[base + t]), a.sum_scale);
        if (a.norm) {
            v = __fmul_rn(__fsub_rn(v, mean), scale);
            v = __fadd_rn(__fmul_rn(v, nw), nb);
            v = __fadd_rn(v, __fmul_rn(v, g));
            v = __fadd_rn(v, be);
        }
        if (a.act == ACT_LEAKY) {
            v = leaky(v, a.slope);
        } else if (a.act == ACT_SNAKE) {
            v = __fadd_rn(v, __fmul_rn(snake_sin2(__fmul_rn(v, alpha)), inv_a));
        }
        if (a.round16) v = round_f16(v);
        y[base + t] = v;
    }
}

void prologue(const float *x, float *y, int64_t R, int C, int m, int extra, const Batch &b,
              int max_len, const PrologueArgs &a, cudaStream_t st) {
    int bx = (max_len + 255) / 256;
    if (bx > 32) bx = 32;
    k_prologue<<<dim3(bx, C, b.n), 256, 0, st>>>(x, y, R, C, m, extra, b, a);
}

// ---------------------------------------------------------------------------
// ConvTranspose row 0 under the left reflect pad of stage 1
// (ggml_pad_reflect_1d(x, 1, 0), audio_utils.cpp:750-752): out'[0] = out'[2]
// = the cropped conv-transpose output at position 1. The phase convolutions
// write every other row; this fills row 0 of each utterance:
// (dot(x[0], W[:, oc, 1 + crop]) + bias) + noise[0]. Only tap t_in = 0
// contributes because 1 + crop < s.
// ---------------------------------------------------------------------------

__global__ void k_convt_row0(ConvTRow0Args a, Batch b) {
    const int u = blockIdx.y;
    const int oc = blockIdx.x * blockDim.x + threadIdx.x;
    if (oc >= a.OC) return;
    const int64_t in_row = (int64_t)a.m_in * b.offT[u];
    const int64_t out_row = (int64_t)a.m_out * b.offT[u];
    const int k = 1 + a.crop;
    float acc = 0.f;
    for (int ic = 0; ic < a.IC; ++ic) {
        float x;
        if (a.in_h) {
            const int64_t o = (((int64_t)(ic >> 3)) * a.R_in + in_row) * 8 + (ic & 7);
            x = __half2float(a.in_h[o]);
            if (a.lo_off > 0) x = __fadd_rn(x, __half2float(a.in_h[o + a.lo_off]));
        } else {
            x = a.in[(int64_t)ic * a.R_in + in_row];
            if (a.round16) x = round_f16(x);
        }
        acc += x * a.w[((int64_t)ic * a.OC + oc) * a.K + k];
    }
    float v = __fadd_rn(acc, a.bias[oc]);
    const int64_t o = (int64_t)oc * a.R_out + out_row;
    v = __fadd_rn(v, a.add[o]);
    a.out[o] = v;
}

void convt_row0(const ConvTRow0Args &a, const Batch &b, cudaStream_t st) {
    k_convt_row0<<<dim3((a.OC + 127) / 128, b.n), 128, 0, st>>>(a, b);
}

// Half chunk-major variant of the prologue, the operand of the tensor-core
// convolution: y[(c/8 * Ry + row) * 8 + c%8]. Same arithmetic as k_prologue,
// then the round-to-nearest-even to half that ggml's F16 im2col applies.
// A thread produces 4 consecutive rows x 8 channels: eight 16-byte loads
// (one float4 per channel) and four contiguous 16-byte stores, so enough
// bytes are in flight to stream at HBM rate. Rows of the 4-row group that
// fall past the utterance are written as zero (they are gap rows); channels
// past C take the neutral terms below, which give zero. The normalisation
// and the activation are template parameters so that each variant keeps
// only the registers it needs (3 blocks per SM).
//
// The pass is bound by instruction issue as much as by HBM, so the work per
// element is kept to the arithmetic itself: the block's 8 channel terms are
// formed once in shared memory (1/alpha included) and read from there each
// pass, and one warp-wide test selects straight-line code for the common
// cases (all Snake arguments in the polynomial's k = 0 range; no row past
// the utterance).
template <bool NORM, int ACT, bool SPLIT>
__global__ void __launch_bounds__(256, SPLIT ? 2 : 3) k_prologue_h(const float *__restrict__ x, __half *__restrict__ y,
                                                       int64_t R, int64_t Ry, int C, int m, int extra, Batch b,
                                                       PrologueArgs a) {
    // per channel e: {mean, scale, norm_w, norm_b}, {gamma, beta, alpha,
    // 1/alpha}, and lim: |v| < lim keeps |v * alpha| below kSnakeFast
    __shared__ float4 prm0[8], prm1[8];
    __shared__ float lim[8];
    const int u = blockIdx.z, ch = blockIdx.y;
    if (threadIdx.x < 8) {
        const int e = threadIdx.x, c = ch * 8 + e;
        float4 p0 = make_float4(0.f, 1.f, 1.f, 0.f), p1 = make_float4(0.f, 0.f, 0.f, 0.f);
        float l = INFINITY;
        if (c < C) {
            if (NORM) {
                const float2 s = a.ms[(int64_t)u * C + c];
                p0 = make_float4(s.x, s.y, a.norm_w[c], a.norm_b[c]);
                p1.x = a.gamma[(int64_t)u * C + c];
                p1.y = a.beta[(int64_t)u * C + c];
            }
            if (ACT == ACT_SNAKE) {
                p1.z = a.alpha[c];
                p1.w = __fdiv_rn(1.0f, p1.z);
                l = __fdiv_rz(kSnakeFast, fabsf(p1.z));
            }
        }
        prm0[e] = p0;
        prm1[e] = p1;
        lim[e] = l;
    }
    __syncthreads();
    const int64_t len = (int64_t)m * b.T[u] + extra;
    const int64_t row0 = (int64_t)m * b.offT[u];  // a multiple of 4
    const float *xc = x + (int64_t)ch * 8 * R + row0;
    const int nc = C - ch * 8 < 8 ? C - ch * 8 : 8;
    for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; t < len;
         t += (int64_t)gridDim.x * blockDim.x * 4) {
        float4 v4[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
            v4[e] = e < nc ? *reinterpret_cast<const float4 *>(xc + e * R + t) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (!NORM && a.x2) {
            // average of the three branches, in the reference's order
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                if (e >= nc) continue;
                const int64_t o = (int64_t)(ch * 8 + e) * R + row0 + t;
                const float4 b2 = *reinterpret_cast<const float4 *>(a.x2 + o);
                const float4 b3 = *reinterpret_cast<const float4 *>(a.x3 + o);
                const float s3 = a.sum_scale;
                v4[e].x = __fmul_rn(__fadd_rn(__fadd_rn(v4[e].x, b2.x), b3.x), s3);
                v4[e].y = __fmul_rn(__fadd_rn(__fadd_rn(v4[e].y, b2.y), b3.y), s3);
                v4[e].z = __fmul_rn(__fadd_rn(__fadd_rn(v4[e].z, b2.z), b3.z), s3);
                v4[e].w = __fmul_rn(__fadd_rn(__fadd_rn(v4[e].w, b2.w), b3.w), s3);
            }
        }
        float v[4][8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float in[4] = {v4[e].x, v4[e].y, v4[e].z, v4[e].w};
            const float4 p0 = prm0[e], p1 = prm1[e];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float w = in[i];
                if (NORM) {
                    w = __fmul_rn(__fsub_rn(w, p0.x), p0.y);
                    w = __fadd_rn(__fmul_rn(w, p0.z), p0.w);
                    w = __fadd_rn(w, __fmul_rn(w, p1.x));
                    w = __fadd_rn(w, p1.y);
                }
                if (ACT == ACT_LEAKY) w = leaky(w, a.slope);
                if (ACT == ACT_GELU) w = gelu_erf(w);
                v[i][e] = w;
            }
        }
        if (ACT == ACT_SNAKE) {
            // One warp-wide test instead of a branch per element: when every
            // argument is in the k = 0 range the 32 elements run as
            // straight-line polynomials (snake_sin2 gives the same values).
            bool fast = true;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float l = lim[e];
#pragma unroll
                for (int i = 0; i < 4; ++i) fast = fast && fabsf(v[i][e]) < l;
            }
            if (__all_sync(__activemask(), fast)) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float4 p1 = prm1[e];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float yv = __fmul_rn(v[i][e], p1.z);
                        v[i][e] = __fadd_rn(v[i][e], __fmul_rn(snake_p(__fmul_rn(yv, yv)), p1.w));
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float4 p1 = prm1[e];
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        v[i][e] = __fadd_rn(v[i][e], __fmul_rn(snake_sin2(__fmul_rn(v[i][e], p1.z)), p1.w));
                }
            }
        }
        const int64_t off = ((int64_t)ch * Ry + row0 + t) * 8;
        uint4 *dst = reinterpret_cast<uint4 *>(y + off);
        const bool whole = t + 4 <= len;
        if (SPLIT) {
            // hi and lo halves of each row: [hi chunks | lo chunks]
            uint4 *dlo = reinterpret_cast<uint4 *>(y + off + a.lo_off);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                __align__(16) __half hh[8], ll[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    hh[e] = __float2half_rn(v[i][e]);
                    ll[e] = split_lo(v[i][e], hh[e]);
                }
                const bool keep = whole || t + i < len;
                dst[i] = keep ? *reinterpret_cast<const uint4 *>(hh) : make_uint4(0u, 0u, 0u, 0u);
                dlo[i] = keep ? *reinterpret_cast<const uint4 *>(ll) : make_uint4(0u, 0u, 0u, 0u);
            }
        } else {
            uint4 h4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                __align__(16) __half2 p[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) p[j] = __floats2half2_rn(v[i][2 * j], v[i][2 * j + 1]);
                h4[i] = *reinterpret_cast<const uint4 *>(p);
            }
            if (whole) {
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = h4[i];
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = t + i < len ? h4[i] : make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
}

template <bool SPLIT>
static void prologue_h_launch(dim3 grid, int nt, const float *x, __half *y, int64_t R, int64_t Ry, int C, int m,
                              int extra, const Batch &b, const PrologueArgs &a, cudaStream_t st) {
    if (a.norm) {
        if (a.act == ACT_SNAKE)
            k_prologue_h<true, ACT_SNAKE, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
        else if (a.act == ACT_LEAKY)
            k_prologue_h<true, ACT_LEAKY, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
        else
            k_prologue_h<true, ACT_NONE, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
    } else {
        if (a.act == ACT_SNAKE)
            k_prologue_h<false, ACT_SNAKE, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
        else if (a.act == ACT_LEAKY)
            k_prologue_h<false, ACT_LEAKY, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
        else if (a.act == ACT_GELU)
            k_prologue_h<false, ACT_GELU, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
        else
            k_prologue_h<false, ACT_NONE, SPLIT><<<grid, nt, 0, st>>>(x, y, R, Ry, C, m, extra, b, a);
    }
}

void prologue_h(const float *x, __half *y, int64_t R, int64_t Ry, int C, int m, int extra, const Batch &b,
                int mean_len, const PrologueArgs &a, cudaStream_t st) {
    // about three passes per thread over an utterance of the mean length, so
    // the per-channel set-up of a thread is spread over several; blocks of
    // 64 threads (256 rows a pass): at batch 64 they made the generator's
    // stage-1 passes 8 % and its stage-0 passes 6 % faster than blocks of 256
    // (128: in between)
    const int nt = 64;
    int bx = (mean_len + 3 * 4 * nt - 1) / (3 * 4 * nt);
    if (bx > 64) bx = 64;
    if (bx < 1) bx = 1;
    const dim3 grid(bx, (C + 7) / 8, b.n);
    if (a.lo_off > 0)
        prologue_h_launch<true>(grid, nt, x, y, R, Ry, C, m, extra, b, a, st);
    else
        prologue_h_launch<false>(grid, nt, x, y, R, Ry, C, m, extra, b, a, st);
}

// Depthwise x2 pool (see k_pool_up) written as the half chunk-major operand
// of the following F16 convolution (its input is rounded to half there).
__global__ void k_pool_up_h(const float *__restrict__ x, __half *__restrict__ y, int64_t R_in, int64_t Ry_out,
                            int C, const float *__restrict__ w, const float *__restrict__ bias, Batch b,
                            int64_t lo_off) {
    const int u = blockIdx.z, ch = blockIdx.y;
    const int64_t L = b.T[u];
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < 2 * L;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = t + 1;
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int c = ch * 8 + e;
            float v = 0.f;
            if (c < C) {
                const float *xp = x + (int64_t)c * R_in + b.offT[u];
                float acc = 0.f;
                const int64_t q = j >> 1;
                if (j & 1) {
                    if (q < L) acc = __fadd_rn(acc, __fmul_rn(w[c * 3 + 1], xp[q]));
                } else {
                    if (q - 1 >= 0 && q - 1 < L) acc = __fadd_rn(acc, __fmul_rn(w[c * 3 + 2], xp[q - 1]));
                    if (q < L) acc = __fadd_rn(acc, __fmul_rn(w[c * 3 + 0], xp[q]));
                }
                v = __fadd_rn(acc, bias[c]);
            }
            h[e] = __float2half_rn(v);
            l[e] = split_lo(v, h[e]);
        }
        __half *dst = y + ((int64_t)ch * Ry_out + 2 * b.offT[u] + t) * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        if (lo_off > 0) *reinterpret_cast<uint4 *>(dst + lo_off) = *reinterpret_cast<const uint4 *>(l);
    }
}

void pool_up_h(const float *x, __half *y, int64_t R_in, int64_t Ry_out, int C, const float *w, const float *bias,
               const Batch &b, int max_T, int64_t lo_off, cudaStream_t st) {
    int bx = (2 * max_T + 255) / 256;
    if (bx > 16) bx = 16;
    k_pool_up_h<<<dim3(bx, (C + 7) / 8, b.n), 256, 0, st>>>(x, y, R_in, Ry_out, C, w, bias, b, lo_off);
}

// The same pool of LeakyReLU(AdaIN(x)): the AdaIN + LeakyReLU of k_prologue
// (the same operations and roundings) applied to each input value as it is
// read, in place of a separate F32 pass over the frame level. A thread takes
// input rows q0 .. q0 + 3 of 8 channels (one float4 each, plus row q0 + 4)
// and writes the output rows 2 q0 .. 2 q0 + 7 they produce: 128 contiguous
// bytes of the half chunk-major operand. Input row q gives output row 2 q
// (w1 x[q]) and 2 q + 1 (w2 x[q], then + w0 x[q + 1] when q + 1 < T), each
// summed from +0 in that order and + bias, as in k_pool_up_h.
__global__ void __launch_bounds__(64) k_pool_up_adain_h(const float *__restrict__ x, __half *__restrict__ y,
                                                        int64_t R_in, int64_t Ry_out, int C,
                                                        const float *__restrict__ w, const float *__restrict__ bias,
                                                        Batch b, int64_t lo_off, PrologueArgs a) {
    const int u = blockIdx.z, ch = blockIdx.y;
    const int64_t L = b.T[u];
    const int64_t off = b.offT[u];  // a multiple of 4
    float mean[8], scale[8], nw[8], nb[8], g[8], be[8], w0[8], w1[8], w2[8], bs[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int c = ch * 8 + e;
        mean[e] = 0.f, scale[e] = 1.f, nw[e] = 1.f, nb[e] = 0.f, g[e] = 0.f, be[e] = 0.f;
        w0[e] = w1[e] = w2[e] = bs[e] = 0.f;
        if (c >= C) continue;
        const float2 s = a.ms[(int64_t)u * C + c];
        mean[e] = s.x;
        scale[e] = s.y;
        nw[e] = a.norm_w[c];
        nb[e] = a.norm_b[c];
        g[e] = a.gamma[(int64_t)u * C + c];
        be[e] = a.beta[(int64_t)u * C + c];
        w0[e] = w[c * 3 + 0];
        w1[e] = w[c * 3 + 1];
        w2[e] = w[c * 3 + 2];
        bs[e] = bias[c];
    }
    const int nc = C - ch * 8 < 8 ? C - ch * 8 : 8;
    auto act = [&](float v, int e) {
        v = __fmul_rn(__fsub_rn(v, mean[e]), scale[e]);
        v = __fadd_rn(__fmul_rn(v, nw[e]), nb[e]);
        v = __fadd_rn(v, __fmul_rn(v, g[e]));
        v = __fadd_rn(v, be[e]);
        return leaky(v, a.slope);
    };
    for (int64_t q0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; q0 < L;
         q0 += (int64_t)gridDim.x * blockDim.x * 4) {
        float av[5][8];  // activations of input rows q0 .. q0 + 4 (0 past T, never used)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            if (e < nc) {
                const float *xp = x + (int64_t)(ch * 8 + e) * R_in + off + q0;
                const float4 v = *reinterpret_cast<const float4 *>(xp);
                av[0][e] = act(v.x, e), av[1][e] = act(v.y, e), av[2][e] = act(v.z, e), av[3][e] = act(v.w, e);
                av[4][e] = q0 + 4 < L ? act(xp[4], e) : 0.f;
            } else {
#pragma unroll
                for (int i = 0; i < 5; ++i) av[i][e] = 0.f;
            }
        }
        __half *dst = y + ((int64_t)ch * Ry_out + 2 * off + 2 * q0) * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (q0 + i >= L) break;
            __align__(16) __half h0[8], l0[8], h1[8], l1[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float v0 = 0.f, v1 = 0.f;
                if (e < nc) {
                    v0 = __fadd_rn(__fadd_rn(0.f, __fmul_rn(w1[e], av[i][e])), bs[e]);
                    float acc = __fadd_rn(0.f, __fmul_rn(w2[e], av[i][e]));
                    if (q0 + i + 1 < L) acc = __fadd_rn(acc, __fmul_rn(w0[e], av[i + 1][e]));
                    v1 = __fadd_rn(acc, bs[e]);
                }
                h0[e] = __float2half_rn(v0);
                l0[e] = split_lo(v0, h0[e]);
                h1[e] = __float2half_rn(v1);
                l1[e] = split_lo(v1, h1[e]);
            }
            *reinterpret_cast<uint4 *>(dst + 16 * i) = *reinterpret_cast<const uint4 *>(h0);
            *reinterpret_cast<uint4 *>(dst + 16 * i + 8) = *reinterpret_cast<const uint4 *>(h1);
            if (lo_off > 0) {
                *reinterpret_cast<uint4 *>(dst + 16 * i + lo_off) = *reinterpret_cast<const uint4 *>(l0);
                *reinterpret_cast<uint4 *>(dst + 16 * i + 8 + lo_off) = *reinterpret_cast<const uint4 *>(l1);
            }
        }
    }
}

void pool_up_adain_h(const float *x, __half *y, int64_t R_in, int64_t Ry_out, int C, const float *w,
                     const float *bias, const Batch &b, int max_T, int64_t lo_off, const PrologueArgs &a,
                     cudaStream_t st) {
    // 64 threads cover 256 input rows
    int bx = (max_T + 255) / 256;
    if (bx > 16) bx = 16;
    if (bx < 1) bx = 1;
    k_pool_up_adain_h<<<dim3(bx, (C + 7) / 8, b.n), 64, 0, st>>>(x, y, R_in, Ry_out, C, w, bias, b, lo_off, a);
}

// Space-to-depth operand of the stride-6 noise convolution: every packed row
// t' of the stage-0 level gets the 132 channels x[r * 22 + ic] =
// half(har[ic][6 t' + r - 3]), r = 0..5, so that the k=12 / stride-6 / pad-3
// convolution becomes a stride-1 convolution with 2 taps. All rows are
// written: outside an utterance they read the zero gaps of har.
__global__ void k_har_s2d(const float *__restrict__ har, int64_t R_har, __half *__restrict__ y, int64_t R,
                          int64_t Ry, int64_t lo_off) {
    const int ch = blockIdx.y;  // output chunk of 8 (24 chunks = 192 padded channels)
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < R; t += (int64_t)gridDim.x * blockDim.x) {
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int c6 = ch * 8 + e;
            float v = 0.f;
            if (c6 < 132) {
                const int r = c6 / 22, ic = c6 % 22;
                const int64_t row = 6 * t + r - 3;
                if (row >= 0 && row < R_har) v = har[(int64_t)ic * R_har + row];
            }
            h[e] = __float2half_rn(v);
            l[e] = split_lo(v, h[e]);
        }
        __half *dst = y + ((int64_t)ch * Ry + t) * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(h);
        if (lo_off > 0) *reinterpret_cast<uint4 *>(dst + lo_off) = *reinterpret_cast<const uint4 *>(l);
    }
}

void har_s2d(const float *har, int64_t R_har, __half *y, int64_t R, int64_t Ry, int64_t lo_off, cudaStream_t st) {
    int bx = (int)((R + 255) / 256);
    if (bx > 2048) bx = 2048;
    k_har_s2d<<<dim3(bx, 24), 256, 0, st>>>(har, R_har, y, R, Ry, lo_off);
}

// ---------------------------------------------------------------------------
// Depthwise x2 pool upsample (depthwise_pool_upsample, audio_utils.cpp:
// 73-114): the dense [3, C, C] expansion through the F32 conv-transpose path
// reduces to out[j] = sum over t_in ascending of w[c][k] * x[c][t_in]
// (j + 1 = 2 t_in + k), + bias. Output length 2T.
// ---------------------------------------------------------------------------

__global__ void k_pool_up(const float *__restrict__ x, float *__restrict__ y, int64_t R_in,
                          int64_t R_out, int C, const float *__restrict__ w,
                          const float *__restrict__ bias, Batch b, int round16) {
    const int u = blockIdx.z, c = blockIdx.y;
    const int64_t L = b.T[u];
    const float *xp = x + (int64_t)c * R_in + b.offT[u];
    float *yp = y + (int64_t)c * R_out + 2 * b.offT[u];
    const float w0 = w[c * 3 + 0], w1 = w[c * 3 + 1], w2 = w[c * 3 + 2], bc = bias[c];
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < 2 * L;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = t + 1;
        float acc = 0.f;
        if (j & 1) {
            const int64_t q = j >> 1;  // k = 1
            if (q < L) acc = __fadd_rn(acc, __fmul_rn(w1, xp[q]));
        } else {
            const int64_t q = j >> 1;
            if (q - 1 >= 0 && q - 1 < L) acc = __fadd_rn(acc, __fmul_rn(w2, xp[q - 1]));  // k = 2
            if (q < L) acc = __fadd_rn(acc, __fmul_rn(w0, xp[q]));                        // k = 0
        }
        float v = __fadd_rn(acc, bc);
        if (round16) v = round_f16(v);
        yp[t] = v;
    }
}

void pool_up(const float *x, float *y, int64_t R_in, int64_t R_out, int C, const float *w,
             const float *bias, const Batch &b, int max_T, int round16, cudaStream_t st) {
    int bx = (2 * max_T + 255) / 256;
    if (bx > 16) bx = 16;
    k_pool_up<<<dim3(bx, C, b.n), 256, 0, st>>>(x, y, R_in, R_out, C, w, bias, b, round16);
}

// ---------------------------------------------------------------------------
// F0_conv / N_conv (kokoro.cpp:751-752): Conv1d(1, 1, k=3, stride 2, pad 1)
// from 2T to T frames. Its weight has ne[0] == K, so the reference takes
// ggml_conv_1d, whose im2col is F16: input and weights rounded to half.
// ---------------------------------------------------------------------------

__global__ void k_f0n_conv(const float *__restrict__ in, int64_t R_in, float *__restrict__ out0,
                           float *__restrict__ out1, int64_t R_out, const float *__restrict__ w,
                           const float *__restrict__ bias, Batch b) {
    const int u = blockIdx.y;
    const int64_t T = b.T[u];
    const float *xp = in + 2 * b.offT[u];
    const float w0 = round_f16(w[0]), w1 = round_f16(w[1]), w2 = round_f16(w[2]);
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < T;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i0 = 2 * t - 1;
        const float x0 = i0 >= 0 ? round_f16(xp[i0]) : 0.f;
        const float x1 = round_f16(xp[i0 + 1]);
        const float x2 = i0 + 2 < 2 * T ? round_f16(xp[i0 + 2]) : 0.f;
        float acc = __fmul_rn(w0, x0);
        acc = __fadd_rn(acc, __fmul_rn(w1, x1));
        acc = __fadd_rn(acc, __fmul_rn(w2, x2));
        const float v = __fadd_rn(acc, bias[0]);
        out0[b.offT[u] + t] = v;
        if (out1) out1[b.offT[u] + t] = v;
    }
    (void)R_in;
    (void)R_out;
}

void f0n_conv(const float *in, int64_t R_in, float *out0, float *out1, int64_t R_out, const float *w,
              const float *bias, const Batch &b, int max_T, cudaStream_t st) {
    int bx = (max_T + 255) / 256;
    k_f0n_conv<<<dim3(bx, b.n), 256, 0, st>>>(in, R_in, out0, out1, R_out, w, bias, b);
}

// ---------------------------------------------------------------------------
// Harmonic source (fill_harmonic_stft, audio_utils.cpp:120-353, scalar
// path). tanh, sin and cos are the correctly rounded float values (double
// evaluation, rounded once): the generator output depends on the last bit of
// the source through the phases of near-silent STFT bins, and only the
// correctly rounded values are reproducible across implementations. Lanes
// 0..8 each carry one harmonic's phasor sequentially through all voiced
// segments (rotation by (cos d, sin d) with each product rounded
// separately) and stage the 300 new sines of a segment in shared memory;
// merged = b + sum_h w_h * 0.1 * sin_h is formed in harmonic order and
// tanh'd. Unvoiced segments (f0 <= 10) hold tanh(b) (computed once on the
// host) and leave the phases untouched. The phasors are renormalised after
// every voiced segment whose index + 1 is a multiple of 16.
// ---------------------------------------------------------------------------

// One block of 4 warps per utterance, the segments pipelined: in step s,
// warp 0 carries the 9 phasors (lanes 0..8) through segment s into one half
// of a double buffer while warps 1..3 merge segment s - 1 from the other
// half; one block barrier per step. The arithmetic and its order are those
// of a single warp doing both in turn.
// (Half segments, 10.8 KB of shared memory so that a block shares an SM with
// a persistent conv CTA, made the batch-64 forward 2.3 ms slower: the source
// then runs longer beside the decoder and the generator waits for it.)
// A block carries kSineGroups utterances, one group of 4 warps each with its
// own named barrier and buffer, so the source occupies n / kSineGroups SMs
// while it runs beside the decoder (sinegen_blocks), not one per utterance:
// the decoder's persistent convolutions keep the other SMs (their CTAs take
// tiles in dynamic order, so one that starts late takes fewer). Measured at
// batch 64 (whole forwards, the conv grids then capped at the SMs the source
// left): one utterance per block 62.2-63.0 ms, two 60.9-61.3 ms, four
// 63.2-63.9 ms (the source itself slower).
// Two more measures keep the recurrence, the source's critical path, short
// (batch 64: the source 4.75 -> 3.37 ms beside the decoder, which waited for
// it, the forward -0.6 ms): each group's recurrence warp is a different warp
// of the block modulo 4, so the two recurrences run on different warp
// schedulers; and the block reserves the SM's shared memory, so that no
// block of another kernel (the issue-heavy operand pass) shares its SM.
// (Computing every segment's rotation beforehand in a parallel kernel, which
// leaves the recurrence warp the rotations alone, changed nothing.)
constexpr int kSineThreads = 128;  // per utterance
constexpr int kSineGroups = 2;
constexpr int kSineSmem = kSineGroups * 2 * kHarmonics * kUpsample * 4;  // used
constexpr int kSineBlockSmem = 227 * 1024;                              // reserved
static_assert(kSineSmem <= kSineBlockSmem, "source buffers");

__global__ void __launch_bounds__(kSineThreads *kSineGroups) k_sinegen(const float *__restrict__ f0, int mf,
                                                                       float *__restrict__ source, Batch b,
                                                                       const int64_t *__restrict__ cumT,
                                                                       SineArgs a) {
    extern __shared__ float sine_smem[];
    const int grp = threadIdx.x / kSineThreads;
    const int u = blockIdx.x * kSineGroups + grp;
    if (u >= b.n) return;  // the whole group (it syncs on its own barrier only)
    float(*sbuf)[kHarmonics][kUpsample] =
        reinterpret_cast<float(*)[kHarmonics][kUpsample]>(sine_smem + grp * 2 * kHarmonics * kUpsample);
    const int tid = threadIdx.x % kSineThreads, lane = tid & 31, warp = tid >> 5;
    const int cw = grp & 3;                             // this group's recurrence warp
    const int mt = ((warp - cw - 1) & 3) * 32 + lane;  // the merge warps' thread index, 0..95
    const int64_t nseg = (int64_t)mf * b.T[u];
    const float *fp = f0 + (int64_t)mf * b.offT[u];
    float *src = source + (int64_t)kUpsample * mf * cumT[u];
    float ps = 0.f, pc = 1.f;
    const bool chain = warp == cw && lane < kHarmonics;
    for (int64_t step = 0; step <= nseg; ++step) {
        if (warp == cw) {
            // the phasors through segment `step`
            if (step < nseg && chain) {
                const float base_f0 = fp[step];
                if (base_f0 > 10.0f) {
                    // delta = (float)(2 pi f0 (h+1) / 24000) evaluated in double
                    const float delta = (float)(2.0 * 3.14159265358979323846 * (double)base_f0 *
                                                (double)(lane + 1) / 24000.0);
                    const float sd = (float)sin((double)delta);
                    const float cd = (float)cos((double)delta);
                    float *row = sbuf[step & 1][lane];
                    for (int j = 0; j < kUpsample; ++j) {
                        const float ns = __fadd_rn(__fmul_rn(ps, cd), __fmul_rn(pc, sd));
                        const float nc = __fsub_rn(__fmul_rn(pc, cd), __fmul_rn(ps, sd));
                        ps = ns;
                        pc = nc;
                        row[j] = ns;
                    }
                    if ((step + 1) % 16 == 0) {
                        const float norm = __fsqrt_rn(__fadd_rn(__fmul_rn(ps, ps), __fmul_rn(pc, pc)));
                        if (norm > 0.0f) {
                            ps = __fdiv_rn(ps, norm);
                            pc = __fdiv_rn(pc, norm);
                        }
                    }
                }
            }
        } else if (step > 0) {
            // segment step - 1: merged = b + sum_h w_h * 0.1 * sin_h in
            // harmonic order, tanh; unvoiced segments hold tanh(b)
            const int64_t seg = step - 1;
            float *out = src + seg * kUpsample;
            if (fp[seg] > 10.0f) {
                const float(*sb)[kUpsample] = sbuf[seg & 1];
                for (int j = mt; j < kUpsample; j += kSineThreads - 32) {
                    float merged = a.mb;
#pragma unroll
                    for (int h = 0; h < kHarmonics; ++h) merged = __fadd_rn(merged, __fmul_rn(a.mw_scaled[h], sb[h][j]));
                    out[j] = (float)tanh((double)merged);
                }
            } else {
                for (int j = mt; j < kUpsample; j += kSineThreads - 32) out[j] = a.unvoiced;
            }
        }
        // this group's barrier (ids 1 .. kSineGroups; 0 is __syncthreads)
        asm volatile("bar.sync %0, %1;" ::"r"(grp + 1), "r"(kSineThreads) : "memory");
    }
}

int sinegen_blocks(int n_utts) { return (n_utts + kSineGroups - 1) / kSineGroups; }

void sinegen(const float *f0, int mf, float *source, const Batch &b, const int64_t *cumT,
             const SineArgs &a, cudaStream_t st) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaFuncSetAttribute(k_sinegen, cudaFuncAttributeMaxDynamicSharedMemorySize, kSineBlockSmem);
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    k_sinegen<<<sinegen_blocks(b.n), kSineThreads * kSineGroups, kSineBlockSmem, st>>>(f0, mf, source, b, cumT, a);
}

// Forward STFT of the source (audio_utils.cpp:381-419): Hann-20 window, hop
// 5, center padding 10 with the reference's edge rule (src < 0 -> -src - 1,
// src >= n -> 2n - src - 1), 11-bin DFT accumulated over n in order with
// separately rounded products; rows 0..10 = |X|, rows 11..21 = atan2(im, re).
__global__ void k_stft(const float *__restrict__ source, float *__restrict__ har, int64_t R, int mf,
                       Batch b, const int64_t *__restrict__ cumT, const StftTables *__restrict__ tab) {
    __shared__ float tc[kStftN][kBins], ts[kStftN][kBins], win[kStftN];
    for (int i = threadIdx.x; i < kStftN * kBins; i += blockDim.x) {
        tc[i / kBins][i % kBins] = tab->c[i / kBins][i % kBins];
        ts[i / kBins][i % kBins] = tab->s[i / kBins][i % kBins];
    }
    for (int i = threadIdx.x; i < kStftN; i += blockDim.x) win[i] = tab->window[i];
    __syncthreads();
    const int u = blockIdx.y;
    const int64_t n_samples = (int64_t)kUpsample * mf * b.T[u];
    const int64_t frames = 60 * (int64_t)mf * b.T[u] + 1;
    const float *src = source + (int64_t)kUpsample * mf * cumT[u];
    const int64_t out_base = 60 * (int64_t)mf * b.offT[u];
    for (int64_t f = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; f < frames;
         f += (int64_t)gridDim.x * blockDim.x) {
        float ws[kStftN];
        const int64_t first = f * kHop - kStftN / 2;
#pragma unroll
        for (int n = 0; n < kStftN; ++n) {
            int64_t si = first + n;
            if (si < 0) si = -si - 1;
            else if (si >= n_samples) si = 2 * n_samples - si - 1;
            ws[n] = (si >= 0 && si < n_samples) ? __fmul_rn(src[si], win[n]) : 0.f;
        }
        float re[kBins], im[kBins];
#pragma unroll
        for (int k = 0; k < kBins; ++k) re[k] = im[k] = 0.f;
#pragma unroll
        for (int n = 0; n < kStftN; ++n) {
#pragma unroll
            for (int k = 0; k < kBins; ++k) {
                re[k] = __fadd_rn(re[k], __fmul_rn(ws[n], tc[n][k]));
                im[k] = __fsub_rn(im[k], __fmul_rn(ws[n], ts[n][k]));
            }
        }
#pragma unroll
        for (int k = 0; k < kBins; ++k) {
            har[(int64_t)k * R + out_base + f] =
                __fsqrt_rn(__fadd_rn(__fmul_rn(re[k], re[k]), __fmul_rn(im[k], im[k])));
            har[(int64_t)(k + kBins) * R + out_base + f] = atan2f(im[k], re[k]);
        }
    }
}

void stft(const float *source, float *har, int64_t R, int mf, const Batch &b, const int64_t *cumT,
          const StftTables *tab, int max_T, cudaStream_t st) {
    const int64_t frames = 60 * (int64_t)mf * max_T + 1;
    int bx = (int)((frames + 127) / 128);
    k_stft<<<dim3(bx, b.n), 128, 0, st>>>(source, har, R, mf, b, cumT, tab);
}

// ---------------------------------------------------------------------------
// iSTFT (cpu_istft_data, audio_utils.cpp:462-532, and the DirectDft path of
// src/audio/istft.cpp:334-523): per frame mag = exp(clamp(p, -20, 8)),
// phase = sin(p'), X = mag (cos phase, sin phase); frame[i] = X0 +- X10 then
// += (2 re_k) cos - (2 im_k) sin for k = 1..9; * (1/20) * window; overlap-add
// in ascending frame order with the window-square envelope; out = env > 1e-8
// ? ola / env : 0; trim 10 samples each side; clamp to +-1.
// Block: 256 frames of one utterance (+3 frames of left context).
// ---------------------------------------------------------------------------

constexpr int IS_FB = 256;

__global__ void __launch_bounds__(256) k_istft(const float *__restrict__ post, int64_t R, int a_nf,
                                               float *__restrict__ audio, Batch b,
                                               const int64_t *__restrict__ cumT,
                                               const IstftTables *__restrict__ tab) {
    __shared__ float fr[(IS_FB + 3) * kStftN];
    __shared__ float dc[kBins][kStftN], ds[kBins][kStftN], win[kStftN], win2[kStftN];
    for (int i = threadIdx.x; i < kBins * kStftN; i += blockDim.x) {
        dc[i / kStftN][i % kStftN] = tab->c[i / kStftN][i % kStftN];
        ds[i / kStftN][i % kStftN] = tab->s[i / kStftN][i % kStftN];
    }
    for (int i = threadIdx.x; i < kStftN; i += blockDim.x) {
        win[i] = tab->window[i];
        win2[i] = tab->window_sq[i];
    }
    __syncthreads();
    const int u = blockIdx.y;
    const int64_t nf = (int64_t)a_nf * b.T[u] + 1;
    const int64_t f0 = (int64_t)blockIdx.x * IS_FB;
    // output j = p - 10 reaches p = 5 nf + 4, so the block starting at
    // f0 = nf (when nf is a multiple of the block) still has samples to write
    if (f0 > nf) return;
    const int64_t base = (int64_t)a_nf * b.offT[u];
    // frames f0-3 .. f0+FB-1
    for (int q = threadIdx.x; q < IS_FB + 3; q += blockDim.x) {
        const int64_t f = f0 - 3 + q;
        float *o = fr + q * kStftN;
        if (f < 0 || f >= nf) {
            for (int i = 0; i < kStftN; ++i) o[i] = 0.f;
            continue;
        }
        float re[kBins], im[kBins];
#pragma unroll
        for (int k = 0; k < kBins; ++k) {
            float v = post[(int64_t)k * R + base + f];
            v = fminf(fmaxf(v, -20.0f), 8.0f);
            const float mag = expf(v);
            const float ph = sinf(post[(int64_t)(k + kBins) * R + base + f]);
            re[k] = __fmul_rn(mag, cosf(ph));
            im[k] = __fmul_rn(mag, sinf(ph));
        }
        float x[kStftN];
        const float d0 = re[0], ny = re[kBins - 1];
#pragma unroll
        for (int i = 0; i < kStftN; i += 2) {
            x[i] = __fadd_rn(d0, ny);
            x[i + 1] = __fsub_rn(d0, ny);
        }
#pragma unroll
        for (int k = 1; k < kStftN / 2; ++k) {
            const float cr = __fmul_rn(2.0f, re[k]), ci = __fmul_rn(2.0f, im[k]);
#pragma unroll
            for (int i = 0; i < kStftN; ++i)
                x[i] = __fadd_rn(x[i], __fsub_rn(__fmul_rn(cr, dc[k][i]), __fmul_rn(ci, ds[k][i])));
        }
#pragma unroll
        for (int i = 0; i < kStftN; ++i) o[i] = __fmul_rn(__fmul_rn(x[i], 0.05f), win[i]);
    }
    __syncthreads();
    // padded positions p in [5 f0, 5 (f0 + FB)), output j = p - 10 in [0, 600 T)
    const int64_t n_out = 5 * (int64_t)a_nf * b.T[u];
    float *out = audio + 5 * (int64_t)a_nf * cumT[u];
    for (int q = threadIdx.x; q < IS_FB * kHop; q += blockDim.x) {
        const int64_t p = 5 * f0 + q;
        const int64_t j = p - 10;
        if (j < 0 || j >= n_out) continue;
        const int64_t fhi = p / 5;
        float ola = 0.f, env = 0.f;
        for (int64_t f = fhi - 3; f <= fhi; ++f) {
            if (f < 0 || f >= nf) continue;
            const int i = (int)(p - 5 * f);
            ola = __fadd_rn(ola, fr[(f - (f0 - 3)) * kStftN + i]);
            env = __fadd_rn(env, win2[i]);
        }
        float v = env > 1e-8f ? __fdiv_rn(ola, env) : 0.0f;
        out[j] = fminf(fmaxf(v, -1.0f), 1.0f);
    }
}

void istft(const float *post, int64_t R, int a_nf, float *audio, const Batch &b, const int64_t *cumT,
           const IstftTables *tab, int max_T, cudaStream_t st) {
    const int64_t nf = (int64_t)a_nf * max_T + 1;
    k_istft<<<dim3((unsigned)(nf / IS_FB + 1), b.n), 256, 0, st>>>(post, R, a_nf, audio, b, cumT,
                                                                            tab);
}

}  // namespace kk
