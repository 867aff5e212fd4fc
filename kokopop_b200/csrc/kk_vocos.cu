// The sanoTTS Vocos decoder's own kernels (sano_run_vocos,
// src/arch/sanotts/sano_vocos.cpp:94-230). Its convolutions and pointwise
// linears run on the tensor-core conv kernels and its LayerNorms on
// layer_norm_ch; what is specific to Vocos is here:
//   dw_layer_norm   the ConvNeXt block's depthwise conv over time + bias,
//                   then LayerNorm over the channels of each frame, written
//                   as the half operand of the first pointwise linear
//   vocos_spectrum  the head's log-magnitude / phase -> complex half-spectrum
//                   -> inverse real FFT (radix 2) -> windowed frame
//   vocos_ola       overlap-add of the windowed frames, 1 / sum(w^2), trim
//   dc_block        the first-order DC blocker, in sample order
// Activations are F32 channel-major [C][R] over the packed frames of a
// ragged batch (level 1 of its plan); every arithmetic step is one rounded
// F32 operation in the reference's order (src/audio/istft.cpp:186-375 and
// the scalar kernels of src/audio/istft_kernels.h), so the inverse FFT and
// the overlap-add reproduce the reference's istft() exactly on the same
// spectrum.
#include "kk_kernels.h"

#include <atomic>

namespace kk {

// ---------------------------------------------------------------------------
// depthwise conv + LayerNorm over channels
// ---------------------------------------------------------------------------

// A block of 128 threads takes 32 frames (rows): for each channel c the
// depthwise conv r[c][q] = sum_k w[c][k] x[c][q - K/2 + k] (taps outside the
// utterance are zero padding, ascending k) + bias[c] is staged in shared
// memory; then, as layer_norm_ch, warp 0 (lane = row) forms ggml_norm's
// mean and scale with double sums in channel order, and every (8-channel
// chunk, row) writes half(v) (and the lo half at lo_off for split operands)
// of v = (r - mean) * scale * gamma + beta, valid rows only.
constexpr int kDwMaxC = 1024;

__global__ void __launch_bounds__(128) k_dw_layer_norm(const float *__restrict__ x, int64_t R, int C, int K,
                                                       const float *__restrict__ dw_w, const float *__restrict__ dw_b,
                                                       const float *__restrict__ gamma,
                                                       const float *__restrict__ beta, float eps, Batch b,
                                                       __half *__restrict__ yh, int64_t Ryh, int64_t lo_off) {
    extern __shared__ float tile[];  // [C][32]
    __shared__ float stat[2][32];
    __shared__ int live_s[32];
    __shared__ int64_t lo_s[32], hi_s[32];  // the utterance's rows [lo, hi)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t q0 = (int64_t)blockIdx.x * 32;
    if (warp == 0) {
        const int64_t q = q0 + lane;
        int live = 0;
        int64_t lo = 0, hi = 0;
        if (q < R) {
            const int u = utt_of_row(b, 1, q);
            lo = b.offT[u];
            hi = lo + b.T[u];
            live = q >= lo && q < hi;
        }
        live_s[lane] = live;
        lo_s[lane] = lo;
        hi_s[lane] = hi;
    }
    __syncthreads();
    const int pad = K / 2;
    for (int i = tid; i < C * 32; i += 128) {
        const int c = i >> 5, r = i & 31;
        float acc = 0.0f;
        if (live_s[r]) {
            const int64_t q = q0 + r;
            const float *xc = x + (int64_t)c * R;
            const float *wc = dw_w + (int64_t)c * K;
            for (int k = 0; k < K; ++k) {
                const int64_t t = q - pad + k;
                if (t >= lo_s[r] && t < hi_s[r]) acc = __fadd_rn(acc, __fmul_rn(xc[t], __ldg(wc + k)));
            }
            acc = __fadd_rn(acc, __ldg(dw_b + c));
        }
        tile[i] = acc;
    }
    __syncthreads();
    if (warp == 0) {
        const float *xr = tile + lane;
        double s = 0.0;
        for (int c = 0; c < C; ++c) s = __dadd_rn(s, (double)xr[c * 32]);
        const float mean = __fdiv_rn((float)s, (float)C);
        double s2 = 0.0;
        for (int c = 0; c < C; ++c) {
            const float v = __fsub_rn(xr[c * 32], mean);
            s2 = __dadd_rn(s2, (double)__fmul_rn(v, v));
        }
        const float var = (float)__ddiv_rn(s2, (double)C);
        stat[0][lane] = mean;
        stat[1][lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const int nch = (C + 7) / 8;
    for (int i = tid; i < nch * 32; i += 128) {
        const int ck = i >> 5, r = i & 31;
        if (q0 + r >= R || !live_s[r]) continue;
        __align__(16) __half hh[8], ll[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int c = ck * 8 + e;
            float v = 0.0f;
            if (c < C) {
                v = __fmul_rn(__fsub_rn(tile[c * 32 + r], stat[0][r]), stat[1][r]);
                v = __fadd_rn(__fmul_rn(v, gamma[c]), beta[c]);
            }
            hh[e] = __float2half_rn(v);
            ll[e] = split_lo(v, hh[e]);
        }
        __half *dst = yh + ((int64_t)ck * Ryh + q0 + r) * 8;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(hh);
        if (lo_off > 0) *reinterpret_cast<uint4 *>(dst + lo_off) = *reinterpret_cast<const uint4 *>(ll);
    }
}

cudaError_t dw_layer_norm(const float *x, int64_t R, int C, int K, const float *dw_w, const float *dw_b,
                          const float *gamma, const float *beta, float eps, const Batch &b, __half *yh, int64_t Ryh,
                          int64_t lo_off, cudaStream_t st) {
    static std::atomic<bool> attr[64];
    if (C < 1 || C > kDwMaxC || K < 1) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(k_dw_layer_norm, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kDwMaxC * 32 * sizeof(float)));
        if (e != cudaSuccess) return e;
        attr[dev].store(true, std::memory_order_release);
    }
    const size_t smem = (size_t)C * 32 * sizeof(float);
    k_dw_layer_norm<<<(unsigned)((R + 31) / 32), 128, smem, st>>>(x, R, C, K, dw_w, dw_b, gamma, beta, eps, b, yh,
                                                                  Ryh, lo_off);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// spectrum -> inverse real FFT -> windowed frame
// ---------------------------------------------------------------------------

constexpr int kSpecFrames = 8;  // frames (rows) per block, one warp each

// One block takes 8 consecutive rows of the head output h [2 bins][R]:
// all threads form the complex spectrum of the 8 frames in shared memory
// (sano_vocos.cpp:165-181: magnitude min(exp(clamp(lm, +-60)), mag_clip),
// the DC and Nyquist bins times zero, real = mag cos(phase), imag =
// mag sin(phase); exp / cos / sin correctly rounded), then warp w runs the
// inverse transform of frame w exactly as istft()'s RealRadix2 path:
// hermitian_split with the 0.5 / half scale, the bit-reversal permutation,
// the pair stage and the radix-2 stages h = 2 .. half / 2, and
// interleave_windowed; the windowed frame goes to fr[q][0 .. n).
__global__ void __launch_bounds__(256) k_vocos_spectrum(const float *__restrict__ h, int64_t R, int n, float mag_clip,
                                                        Batch b, R2Tables tab, float *__restrict__ fr) {
    extern __shared__ float sm[];
    const int half = n / 2, bins = half + 1;
    float *Xr = sm;                          // [8][bins]
    float *Xi = Xr + kSpecFrames * bins;     // [8][bins]
    float *Z = Xi + kSpecFrames * bins;      // [8][2][half]
    __shared__ int live_s[kSpecFrames];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t q0 = (int64_t)blockIdx.x * kSpecFrames;
    if (tid < kSpecFrames) {
        const int64_t q = q0 + tid;
        int live = 0;
        if (q < R) {
            const int u = utt_of_row(b, 1, q);
            live = q >= b.offT[u] && q < b.offT[u] + b.T[u];
        }
        live_s[tid] = live;
    }
    for (int i = tid; i < kSpecFrames * bins; i += blockDim.x) {
        const int k = i / kSpecFrames, f = i % kSpecFrames;
        const int64_t q = q0 + f;
        float re = 0.0f, im = 0.0f;
        if (q < R) {
            const float lm = h[(int64_t)k * R + q];
            const float ph = h[(int64_t)(bins + k) * R + q];
            const float v = fminf(fmaxf(lm, -60.0f), 60.0f);
            float mag = __double2float_rn(exp((double)v));
            mag = fminf(fmaxf(mag, 0.0f), mag_clip);
            if (k == 0 || k == bins - 1) mag = __fmul_rn(mag, 0.0f);
            re = __fmul_rn(mag, __double2float_rn(cos((double)ph)));
            im = __fmul_rn(mag, __double2float_rn(sin((double)ph)));
        }
        Xr[f * bins + k] = re;
        Xi[f * bins + k] = im;
    }
    __syncthreads();
    if (warp >= kSpecFrames || !live_s[warp]) return;
    const float *xr = Xr + warp * bins, *xi = Xi + warp * bins;
    float *zr = Z + warp * 2 * half, *zi = zr + half;
    const float scale = __fdiv_rn(0.5f, (float)half);
    for (int k = lane; k < half; k += 32) {
        const float ar = xr[k], ai = xi[k], mr = xr[half - k], mi = xi[half - k];
        const float er = __fmul_rn(scale, __fadd_rn(ar, mr)), ei = __fmul_rn(scale, __fsub_rn(ai, mi));
        const float dr = __fmul_rn(scale, __fsub_rn(ar, mr)), di = __fmul_rn(scale, __fadd_rn(ai, mi));
        const float sc = tab.split_cos[k], ss = tab.split_sin[k];
        // the bit-reversal swaps place index k at rev[k]
        const int d = tab.rev[k];
        zr[d] = __fsub_rn(er, __fadd_rn(__fmul_rn(dr, ss), __fmul_rn(di, sc)));
        zi[d] = __fadd_rn(ei, __fsub_rn(__fmul_rn(dr, sc), __fmul_rn(di, ss)));
    }
    __syncwarp();
    for (int i = 2 * lane; i < half; i += 64) {
        const float ar = zr[i], ai = zi[i], br = zr[i + 1], bi = zi[i + 1];
        zr[i] = __fadd_rn(ar, br);
        zi[i] = __fadd_rn(ai, bi);
        zr[i + 1] = __fsub_rn(ar, br);
        zi[i + 1] = __fsub_rn(ai, bi);
    }
    __syncwarp();
    for (int hh = 2; hh < half; hh <<= 1) {
        const float *wc = tab.stage_cos + (hh - 1), *ws = tab.stage_sin + (hh - 1);
        for (int j = lane; j < half / 2; j += 32) {
            const int kk = j % hh;
            const int a = (j / hh) * 2 * hh + kk, bb = a + hh;
            const float c = wc[kk], s = ws[kk];
            const float brr = __fsub_rn(__fmul_rn(zr[bb], c), __fmul_rn(zi[bb], s));
            const float bii = __fadd_rn(__fmul_rn(zr[bb], s), __fmul_rn(zi[bb], c));
            const float arr = zr[a], aii = zi[a];
            zr[bb] = __fsub_rn(arr, brr);
            zi[bb] = __fsub_rn(aii, bii);
            zr[a] = __fadd_rn(arr, brr);
            zi[a] = __fadd_rn(aii, bii);
        }
        __syncwarp();
    }
    float2 *out = reinterpret_cast<float2 *>(fr + (q0 + warp) * (int64_t)n);
    for (int m = lane; m < half; m += 32)
        out[m] = make_float2(__fmul_rn(zr[m], tab.window[2 * m]), __fmul_rn(zi[m], tab.window[2 * m + 1]));
}

constexpr int kSpecMaxN = 2048;  // 8 frames of spectrum + FFT buffers: 131 KB of shared memory

cudaError_t vocos_spectrum(const float *h, int64_t R, int n, float mag_clip, const Batch &b, const R2Tables &tab,
                           float *fr, cudaStream_t st) {
    if (n < 64 || n > kSpecMaxN || (n & (n - 1))) return cudaErrorInvalidValue;
    static std::atomic<bool> attr[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t smem = (size_t)kSpecFrames * (2 * (n / 2 + 1) + n) * sizeof(float);
    if (!attr[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(k_vocos_spectrum, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kSpecFrames * (2 * (kSpecMaxN / 2 + 1) + kSpecMaxN) * sizeof(float)));
        if (e != cudaSuccess) return e;
        attr[dev].store(true, std::memory_order_release);
    }
    k_vocos_spectrum<<<(unsigned)((R + kSpecFrames - 1) / kSpecFrames), 256, smem, st>>>(h, R, n, mag_clip, b, tab,
                                                                                        fr);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// overlap-add, normalisation, trim
// ---------------------------------------------------------------------------

// Output sample j of utterance u (padded position p = j + n / 2): the frames
// f that cover p are added in ascending order, as istft()'s ring receives
// them, the window squares likewise; out = env > 1e-8 ? ola / env : 0.
__global__ void k_vocos_ola(const float *__restrict__ fr, int n, int hop, Batch b, const int64_t *__restrict__ cum,
                            const float *__restrict__ window_sq, float *__restrict__ audio) {
    const int u = blockIdx.y;
    const int64_t T = b.T[u];
    const int64_t len = (int64_t)hop * (T - 1);
    const int64_t row0 = b.offT[u];
    float *out = audio + cum[u];
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < len; j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = j + n / 2;
        int64_t f_lo = p - n + 1 > 0 ? (p - n + 1 + hop - 1) / hop : 0;
        int64_t f_hi = p / hop;
        if (f_hi > T - 1) f_hi = T - 1;
        float ola = 0.0f, env = 0.0f;
        for (int64_t f = f_lo; f <= f_hi; ++f) {
            const int i = (int)(p - f * hop);
            ola = __fadd_rn(ola, fr[(row0 + f) * (int64_t)n + i]);
            env = __fadd_rn(env, __ldg(window_sq + i));
        }
        out[j] = env > 1e-8f ? __fdiv_rn(ola, env) : 0.0f;
    }
}

void vocos_ola(const float *fr, int n, int hop, const Batch &b, const int64_t *cum, const float *window_sq,
               int64_t max_len, float *audio, cudaStream_t st) {
    int64_t bx = (max_len + 255) / 256;
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_vocos_ola<<<dim3((unsigned)bx, (unsigned)b.n), 256, 0, st>>>(fr, n, hop, b, cum, window_sq, audio);
}

// ---------------------------------------------------------------------------
// DC blocker
// ---------------------------------------------------------------------------

// One warp per utterance. The samples move through shared memory in chunks
// of 1024: the warp loads chunk c + 1 into registers while lane 0 runs the
// recurrence y = (x - x_prev) + pole * y_prev over chunk c in sample order
// (each operation rounded once, as the reference's scalar loop).
constexpr int kDcChunk = 1024;

__global__ void __launch_bounds__(32) k_dc_block(float *__restrict__ audio, const int64_t *__restrict__ cum,
                                                 const int64_t *__restrict__ len, float pole) {
    __shared__ float buf[kDcChunk];
    const int u = blockIdx.x, lane = threadIdx.x;
    float *a = audio + cum[u];
    const int64_t n = len[u];
    float pin = 0.0f, pout = 0.0f;
    float nxt[kDcChunk / 32];
    for (int i = 0; i < kDcChunk / 32; ++i) {
        const int64_t s = (int64_t)i * 32 + lane;
        nxt[i] = s < n ? a[s] : 0.0f;
    }
    for (int64_t c0 = 0; c0 < n; c0 += kDcChunk) {
        for (int i = 0; i < kDcChunk / 32; ++i) buf[i * 32 + lane] = nxt[i];
        __syncwarp();
        const int64_t c1 = c0 + kDcChunk;
        for (int i = 0; i < kDcChunk / 32; ++i) {
            const int64_t s = c1 + (int64_t)i * 32 + lane;
            nxt[i] = s < n ? a[s] : 0.0f;
        }
        if (lane == 0) {
            const int m = n - c0 < kDcChunk ? (int)(n - c0) : kDcChunk;
            for (int s = 0; s < m; ++s) {
                const float in = buf[s];
                const float o = __fadd_rn(__fsub_rn(in, pin), __fmul_rn(pole, pout));
                pin = in;
                pout = o;
                buf[s] = o;
            }
        }
        __syncwarp();
        for (int i = 0; i < kDcChunk / 32; ++i) {
            const int64_t s = c0 + (int64_t)i * 32 + lane;
            if (s < n) a[s] = buf[i * 32 + lane];
        }
        __syncwarp();
    }
}

void dc_block(float *audio, const int64_t *cum, const int64_t *len, int n_utts, float pole, cudaStream_t st) {
    k_dc_block<<<(unsigned)n_utts, 32, 0, st>>>(audio, cum, len, pole);
}

}  // namespace kk
