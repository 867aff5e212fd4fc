// Bidirectional LSTM stack (prosody duration encoder) and the durations ->
// frames alignment.
//
// Layout: the sequences of a batch are packed time-major, row = t * B + b
// (B sequences, t < max length), channel-major [C][R] like every other
// activation of the library, so the input projection W_ih x + b_ih is one
// K = 1 convolution over all rows and both directions (output channels
// [forward 4H | backward 4H]) on the existing convolution kernels.
//
// Recurrence (cpu_lstm_contiguous, src/arch/kokoro/lstm_fused.cpp:200-247):
// one thread-block cluster of 8 CTAs per (direction, group of Bc sequences).
// CTA r of the cluster owns hidden units [32 r, 32 r + 32) and their four
// gate rows of W_hh (128 rows x 256, F32, 128 KB) in shared memory for the
// whole sequence. Per step every CTA computes its 128 gate rows for the
// group's sequences, updates its 32 cells, and writes the new h values into
// the h buffer of every CTA of the cluster (distributed shared memory); one
// cluster barrier per step publishes them. The dot products keep the
// reference's scalar order (k ascending, separate multiply and add), and the
// gate sum is (b_hh + pre) + dot as in the reference.
#include "kk_kernels.h"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace kk {

constexpr int kLstmH = 256;        // hidden units per direction
constexpr int kLstmCl = 8;         // CTAs per cluster
constexpr int kLstmUnits = 32;     // hidden units per CTA
constexpr int kLstmRows = 128;     // gate rows per CTA (4 gates x 32 units)
constexpr int kLstmThreads = 256;

size_t lstm_rec_smem(int Bc) {
    return sizeof(float) * ((size_t)kLstmH * kLstmRows + 2 * (size_t)kLstmH * Bc + (size_t)kLstmRows * Bc +
                            (size_t)kLstmUnits * Bc);
}

// exp / tanh correctly rounded to float (through double)
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float tanh_cr(float x) { return (float)tanh((double)x); }

// lstm_fused.cpp:60-68: branch-stable logistic
__device__ __forceinline__ float sigmoid_stable(float x) {
    if (x >= 0.0f) {
        const float z = exp_cr(-x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
    }
    const float z = exp_cr(x);
    return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

// non-finite -> 0, clamp to +-lim
__device__ __forceinline__ float sanitize(float x, float lim) {
    if (!isfinite(x)) return 0.0f;
    return fminf(fmaxf(x, -lim), lim);
}

template <int RPT, int SPT>
__global__ void __cluster_dims__(kLstmCl, 1, 1) __launch_bounds__(kLstmThreads, 1)
    k_lstm_rec(const LstmRecArgs a) {
    cg::cluster_group cluster = cg::this_cluster();
    const int cr = (int)cluster.block_rank();
    const int cid = blockIdx.x / kLstmCl;
    const int d = cid & 1, grp = cid >> 1;
    const int Bc = a.Bc;
    const int b0 = grp * Bc;
    extern __shared__ __align__(16) float sm[];
    float *Wt = sm;                                  // [256 k][128 local rows]
    float *hb = Wt + kLstmH * kLstmRows;             // [2][256][Bc]
    float *gb = hb + 2 * kLstmH * Bc;                // [128][Bc]
    float *cs = gb + kLstmRows * Bc;                 // [32][Bc]
    const float *whh = d ? a.whh[1] : a.whh[0];
    const float *bhh = d ? a.bhh[1] : a.bhh[0];
    // local row lr = q * 32 + uu <-> gate row j = q * 256 + 32 cr + uu
    for (int idx = threadIdx.x; idx < kLstmRows * kLstmH; idx += kLstmThreads) {
        const int lr = idx / kLstmH, k = idx % kLstmH;
        const int j = (lr / kLstmUnits) * kLstmH + kLstmUnits * cr + (lr % kLstmUnits);
        Wt[k * kLstmRows + lr] = whh[(int64_t)j * kLstmH + k];
    }
    for (int idx = threadIdx.x; idx < kLstmH * Bc; idx += kLstmThreads) hb[idx] = 0.0f;
    for (int idx = threadIdx.x; idx < kLstmUnits * Bc; idx += kLstmThreads) cs[idx] = 0.0f;
    cluster.sync();

    constexpr int NRB = kLstmRows / RPT;
    const int rb = threadIdx.x % NRB, sb = threadIdx.x / NRB;
    const bool active = sb * SPT < Bc;
    int jg[RPT];
    float bias[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int lr = rb * RPT + i;
        jg[i] = (lr / kLstmUnits) * kLstmH + kLstmUnits * cr + (lr % kLstmUnits);
        bias[i] = bhh[jg[i]];
    }
    int len[SPT];
#pragma unroll
    for (int jj = 0; jj < SPT; ++jj) {
        const int b = b0 + sb * SPT + jj;
        len[jj] = (active && b < a.B) ? a.len[b] : 0;
    }
    const float *pre = a.pre + (int64_t)d * 4 * kLstmH * a.R;

    for (int s = 0; s < a.max_len; ++s) {
        const float *hp = hb + (s & 1) * kLstmH * Bc;
        float *hn = hb + ((s + 1) & 1) * kLstmH * Bc;
        if (active) {
            float pg[RPT][SPT];
#pragma unroll
            for (int jj = 0; jj < SPT; ++jj) {
                const int b = b0 + sb * SPT + jj;
                const bool live = s < len[jj];
                const int t = d ? len[jj] - 1 - s : s;
                const int64_t row = (int64_t)t * a.B + b;
#pragma unroll
                for (int i = 0; i < RPT; ++i) pg[i][jj] = live ? pre[(int64_t)jg[i] * a.R + row] : 0.0f;
            }
            float acc[RPT][SPT];
#pragma unroll
            for (int i = 0; i < RPT; ++i)
#pragma unroll
                for (int jj = 0; jj < SPT; ++jj) acc[i][jj] = 0.0f;
#pragma unroll 4
            for (int k = 0; k < kLstmH; ++k) {
                float w[RPT], h[SPT];
#pragma unroll
                for (int i = 0; i < RPT; ++i) w[i] = Wt[k * kLstmRows + rb * RPT + i];
#pragma unroll
                for (int jj = 0; jj < SPT; ++jj) h[jj] = hp[k * Bc + sb * SPT + jj];
#pragma unroll
                for (int i = 0; i < RPT; ++i)
#pragma unroll
                    for (int jj = 0; jj < SPT; ++jj) acc[i][jj] = __fadd_rn(acc[i][jj], __fmul_rn(w[i], h[jj]));
            }
#pragma unroll
            for (int i = 0; i < RPT; ++i)
#pragma unroll
                for (int jj = 0; jj < SPT; ++jj)
                    gb[(rb * RPT + i) * Bc + sb * SPT + jj] = __fadd_rn(__fadd_rn(bias[i], pg[i][jj]), acc[i][jj]);
        }
        __syncthreads();
        // the four gate activations of every live cell, spread over the
        // threads (in place: i, f, o logistic, g tanh)
        for (int idx = threadIdx.x; idx < kLstmRows * Bc; idx += kLstmThreads) {
            const int lr = idx / Bc, bl = idx % Bc, b = b0 + bl;
            if (b >= a.B || s >= a.len[b]) continue;
            const float x = sanitize(gb[idx], 80.0f);
            gb[idx] = lr / kLstmUnits == 2 ? tanh_cr(x) : sigmoid_stable(x);
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < kLstmUnits * Bc; idx += kLstmThreads) {
            const int uu = idx / Bc, bl = idx % Bc, b = b0 + bl;
            if (b >= a.B) continue;
            const int L = a.len[b];
            if (s >= L) continue;
            const float ig = gb[(0 * kLstmUnits + uu) * Bc + bl];
            const float fg = gb[(1 * kLstmUnits + uu) * Bc + bl];
            const float gg = gb[(2 * kLstmUnits + uu) * Bc + bl];
            const float og = gb[(3 * kLstmUnits + uu) * Bc + bl];
            const float cn = sanitize(__fadd_rn(__fmul_rn(fg, cs[uu * Bc + bl]), __fmul_rn(ig, gg)), 50.0f);
            cs[uu * Bc + bl] = cn;
            float hv = __fmul_rn(og, tanh_cr(cn));
            if (!isfinite(hv)) hv = 0.0f;
            const int t = d ? L - 1 - s : s;
            const int unit = kLstmUnits * cr + uu;
            a.hout[(int64_t)(d * kLstmH + unit) * a.R + (int64_t)t * a.B + b] = hv;
            float *dst = hn + unit * Bc + bl;
#pragma unroll
            for (int r = 0; r < kLstmCl; ++r) *cluster.map_shared_rank(dst, r) = hv;
        }
        cluster.sync();
    }
}

template <int RPT, int SPT>
static cudaError_t launch_rec(const LstmRecArgs &a, int n_clusters, cudaStream_t st) {
    const size_t smem = lstm_rec_smem(a.Bc);
    cudaError_t e = cudaFuncSetAttribute(k_lstm_rec<RPT, SPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_lstm_rec<RPT, SPT><<<n_clusters * kLstmCl, kLstmThreads, smem, st>>>(a);
    return cudaGetLastError();
}

cudaError_t lstm_recurrence(const LstmRecArgs &a, cudaStream_t st) {
    if (a.B < 1 || a.max_len < 1) return cudaSuccess;
    if (!(a.Bc == 1 || a.Bc == 2 || a.Bc == 4 || a.Bc == 8 || a.Bc == 16 || a.Bc == 32)) return cudaErrorInvalidValue;
    const int groups = (a.B + a.Bc - 1) / a.Bc;
    const int n_clusters = 2 * groups;
    switch (a.Bc) {
        case 1:
        case 2: return launch_rec<1, 1>(a, n_clusters, st);
        case 4: return launch_rec<2, 1>(a, n_clusters, st);
        case 8: return launch_rec<4, 1>(a, n_clusters, st);
        case 16: return launch_rec<4, 2>(a, n_clusters, st);
        default: return launch_rec<4, 4>(a, n_clusters, st);
    }
}

// ---------------------------------------------------------------------------
// packing
// ---------------------------------------------------------------------------

// x: per sequence [len_b][D] feature-fastest, back to back (offsets cum[b]);
// X: [C][R] with row t * B + b. Channels [D, D + Ds) take the sequence's style
// vector (the duration encoder's concat); rows past a sequence stay as they
// are (zero from the caller's memset).
__global__ void k_lstm_pack(const float *__restrict__ x, int D, const float *__restrict__ style, int Ds,
                            float *__restrict__ X, int64_t R, const int32_t *__restrict__ len,
                            const int64_t *__restrict__ cum, int B) {
    const int b = blockIdx.y;
    const int L = len[b];
    const int C = D + Ds;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)L * C;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(idx / C), c = (int)(idx % C);
        const float v = c < D ? x[(cum[b] + t) * D + c] : style[(int64_t)b * Ds + (c - D)];
        X[(int64_t)c * R + (int64_t)t * B + b] = v;
    }
}

// inverse: out[cum[b] + t][c] = X[c][t * B + b], c < C
__global__ void k_lstm_unpack(const float *__restrict__ X, int64_t R, int C, float *__restrict__ out,
                              const int32_t *__restrict__ len, const int64_t *__restrict__ cum, int B) {
    const int b = blockIdx.y;
    const int L = len[b];
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)L * C;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(idx / C), c = (int)(idx % C);
        out[(cum[b] + t) * C + c] = X[(int64_t)c * R + (int64_t)t * B + b];
    }
}

// X [C][R] in the LSTM layout (row t * B + b) -> dst [C][R_dst] at rows
// m * offT[b] + t of a packed ragged level (t < len[b]); other rows untouched.
__global__ void k_lstm_to_level(const float *__restrict__ X, int64_t R, int B, const int32_t *__restrict__ len,
                                float *__restrict__ dst, int64_t R_dst, const int64_t *__restrict__ offT, int m) {
    const int b = blockIdx.y, c = blockIdx.z;
    const int L = len[b];
    const int64_t o = (int64_t)m * offT[b];
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < L; t += gridDim.x * blockDim.x)
        dst[(int64_t)c * R_dst + o + t] = X[(int64_t)c * R + (int64_t)t * B + b];
}

void lstm_to_level(const float *X, int64_t R, int C, int B, const int32_t *len, int max_len, float *dst,
                   int64_t R_dst, const int64_t *offT, int m, cudaStream_t st) {
    int bx = (max_len + 255) / 256;
    if (bx > 64) bx = 64;
    if (bx < 1) bx = 1;
    k_lstm_to_level<<<dim3(bx, B, C), 256, 0, st>>>(X, R, B, len, dst, R_dst, offT, m);
}

void lstm_pack(const float *x, int D, const float *style, int Ds, float *X, int64_t R, const int32_t *len,
               const int64_t *cum, int B, int max_len, cudaStream_t st) {
    int bx = (int)(((int64_t)max_len * (D + Ds) + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_lstm_pack<<<dim3(bx, B), 256, 0, st>>>(x, D, style, Ds, X, R, len, cum, B);
}

void lstm_unpack(const float *X, int64_t R, int C, float *out, const int32_t *len, const int64_t *cum, int B,
                 int max_len, cudaStream_t st) {
    int bx = (int)(((int64_t)max_len * C + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_lstm_unpack<<<dim3(bx, B), 256, 0, st>>>(X, R, C, out, len, cum, B);
}

// ---------------------------------------------------------------------------
// AdaLayerNorm (ada_layer_norm, src/arch/kokoro/graph_ops.cpp:865-886)
// ---------------------------------------------------------------------------

// gamma / beta of one AdaLayerNorm per sequence: linear (graph_ops.cpp:636-654)
// with the sequential F32 sum, the style rounded to half for an F16 weight.
// w: [C][Ds] values; out: [B][C].
__global__ void k_style_linear(const float *__restrict__ w, const float *__restrict__ bias, int f16,
                               const float *__restrict__ style, int Ds, int C, float *__restrict__ out) {
    const int b = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float *s = style + (int64_t)b * Ds;
    const float *wr = w + (int64_t)c * Ds;
    float acc = 0.0f;
    for (int i = 0; i < Ds; ++i) {
        const float x = f16 ? round_f16(s[i]) : s[i];
        acc = __fadd_rn(acc, __fmul_rn(wr[i], x));
    }
    out[(int64_t)b * C + c] = __fadd_rn(acc, bias[c]);
}

void style_linear(const float *w, const float *bias, int f16, const float *style, int Ds, int C, int B, float *out,
                  cudaStream_t st) {
    k_style_linear<<<dim3((C + 127) / 128, B), 128, 0, st>>>(w, bias, f16, style, Ds, C, out);
}

// ggml_norm over the D features of each row (mean, then the variance of
// x - mean, sums in double), then (y + y * gamma) + beta; result into X rows
// (channels [0, D)). One block of 256 threads handles 32 rows: lane = row,
// warp = channel slice.
__global__ void __launch_bounds__(256) k_ada_layer_norm(const float *__restrict__ h, int64_t R, int D,
                                                        const float *__restrict__ gamma,
                                                        const float *__restrict__ beta, float *__restrict__ X,
                                                        const int32_t *__restrict__ len, int B, float eps) {
    __shared__ double part[8][33];
    __shared__ float stat[2][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t row = (int64_t)blockIdx.x * 32 + lane;
    const int b = (int)(row % B);
    const int64_t t = row / B;
    const bool live = row < R && t < len[b];
    // pass 1: mean
    double s = 0.0;
    if (live)
        for (int c = w; c < D; c += 8) s += (double)h[(int64_t)c * R + row];
    part[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        double tot = 0.0;
        for (int i = 0; i < 8; ++i) tot += part[i][lane];
        stat[0][lane] = __fdiv_rn((float)tot, (float)D);
    }
    __syncthreads();
    const float mean = stat[0][lane];
    // pass 2: variance of x - mean
    s = 0.0;
    if (live)
        for (int c = w; c < D; c += 8) {
            const float v = __fsub_rn(h[(int64_t)c * R + row], mean);
            s += (double)__fmul_rn(v, v);
        }
    __syncthreads();
    part[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        double tot = 0.0;
        for (int i = 0; i < 8; ++i) tot += part[i][lane];
        const float var = (float)(tot / (double)D);
        stat[1][lane] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const float scale = stat[1][lane];
    if (row >= R) return;
    for (int c = w; c < D; c += 8) {
        float v = 0.0f;
        if (live) {
            const float y = __fmul_rn(__fsub_rn(h[(int64_t)c * R + row], mean), scale);
            v = __fadd_rn(__fadd_rn(y, __fmul_rn(y, gamma[(int64_t)b * D + c])), beta[(int64_t)b * D + c]);
        }
        X[(int64_t)c * R + row] = v;
    }
}

void ada_layer_norm(const float *h, int64_t R, int D, const float *gamma, const float *beta, float *X,
                    const int32_t *len, int B, cudaStream_t st) {
    k_ada_layer_norm<<<(unsigned)((R + 31) / 32), 256, 0, st>>>(h, R, D, gamma, beta, X, len, B, 1e-5f);
}

// ---------------------------------------------------------------------------
// R11: durations -> frames, alignment (src/arch/kokoro/kokoro.cpp:115-193,
// :669-674)
// ---------------------------------------------------------------------------

// frames[i] = clamp(int(lrint(d[i] / speed)), 1, 50); non-finite -> 1. The
// speed was sanitised on the host (non-finite or <= 0 -> 1).
__global__ void k_duration_frames(const float *__restrict__ d, int64_t n, float speed, int32_t *__restrict__ frames) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = __fdiv_rn(d[i], speed);
        int r = 1;
        if (isfinite(v)) {
            // lrint rounds to nearest-even into a 64-bit long; the reference
            // then narrows it to int (two's-complement truncation)
            const long long l = __float2ll_rn(v);
            const int n32 = (int)(unsigned int)(unsigned long long)l;
            r = n32 < 1 ? 1 : (n32 > 50 ? 50 : n32);
        }
        frames[i] = r;
    }
}

// exclusive prefix sum of frames (one block; n up to a few thousand tokens)
// and the frame -> token map; start[n] = total.
__global__ void k_duration_scan(const int32_t *__restrict__ frames, int64_t n, int64_t *__restrict__ start) {
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += blockDim.x) {
        __shared__ int64_t buf[1024];
        const int64_t i = base + threadIdx.x;
        buf[threadIdx.x] = i < n ? frames[i] : 0;
        __syncthreads();
        for (int off = 1; off < (int)blockDim.x; off <<= 1) {
            const int64_t v = threadIdx.x >= (unsigned)off ? buf[threadIdx.x - off] : 0;
            __syncthreads();
            buf[threadIdx.x] += v;
            __syncthreads();
        }
        const int64_t incl = buf[threadIdx.x];
        const int64_t excl = incl - (i < n ? frames[i] : 0);
        if (i < n) start[i] = carry + excl;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) start[n] = carry;
}

// en[f][:] = hidden[token(f)][:]: the one-hot alignment matmul d . mask is
// a copy of the frame's token row.
__global__ void k_align_gather(const float *__restrict__ hidden, int64_t D, const int32_t *__restrict__ frames,
                               const int64_t *__restrict__ start, int64_t n, float *__restrict__ en) {
    const int64_t i = blockIdx.y;  // token
    if (i >= n) return;
    const int64_t f0 = start[i];
    const int nf = frames[i];
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < (int64_t)nf * D;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / D, c = idx % D;
        en[(f0 + r) * D + c] = hidden[i * D + c];
    }
}

void duration_frames(const float *d, int64_t n, float speed, int32_t *frames, int64_t *start, cudaStream_t st) {
    int bx = (int)((n + 255) / 256);
    if (bx > 1024) bx = 1024;
    if (bx < 1) bx = 1;
    k_duration_frames<<<bx, 256, 0, st>>>(d, n, speed, frames);
    k_duration_scan<<<1, 1024, 0, st>>>(frames, n, start);
}

void align_gather(const float *hidden, int64_t D, const int32_t *frames, const int64_t *start, int64_t n, float *en,
                  cudaStream_t st) {
    if (n < 1) return;
    int bx = (int)((50 * D + 255) / 256);
    if (bx > 64) bx = 64;
    k_align_gather<<<dim3(bx, (unsigned)n), 256, 0, st>>>(hidden, D, frames, start, n, en);
}

}  // namespace kk
