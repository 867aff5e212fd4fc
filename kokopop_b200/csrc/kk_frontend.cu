// Kernels of the Kokoro-82M front end (sm_100a): the embedding lookups and
// the per-token LayerNorm (the text encoder's CNN, text_encoder,
// src/arch/kokoro/graph_ops.cpp:1578-1624; ALBERT's embeddings and layers,
// src/arch/kokoro/kokoro.cpp:279-337), ALBERT's self-attention and GELU, the
// token-major output gather, and the duration projection with the bucket
// sum that the reference runs on the host in double (kokoro.cpp:469-516).
// The convolutions and linears run on the conv kernels of kk_conv_tc.cu /
// kk_conv_simt.cu, the biLSTMs on kk_lstm.cu.
#include "kk_common.cuh"
#include "kk_kernels.h"

#include <atomic>

namespace kk {

// ggml_get_rows of the embedding [C, vocab] into the packed level-1 layout:
// X[c][q] = emb[id * C + c] on the token rows of each utterance (id =
// ids[cum[u] + t]), zero on the gap rows; with pos (ALBERT) the row is
// (emb + pos[t * C + c]) + type[c], as ggml_add twice. An id outside
// [0, vocab) gives a zero row and sets *err to kErrTokenId.
__global__ void k_embed(const float *__restrict__ emb, int C, int vocab, const int32_t *__restrict__ ids,
                        const int64_t *__restrict__ cum, Batch b, float *__restrict__ X, int64_t R, int *err,
                        const float *__restrict__ pos, const float *__restrict__ type) {
    const int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (q >= R) return;
    const int u = utt_of_row(b, 1, q);
    const int64_t t = q - b.offT[u];
    int id = -1;
    if (t >= 0 && t < b.T[u]) {
        id = ids[cum[u] + t];
        if (id < 0 || id >= vocab) {
            atomicCAS(err, 0, kErrTokenId);
            id = -1;
        }
    }
    for (int c = blockIdx.y; c < C; c += gridDim.y) {
        float v = 0.0f;
        if (id >= 0) {
            v = emb[(int64_t)id * C + c];
            if (pos) v = __fadd_rn(__fadd_rn(v, pos[t * C + c]), type[c]);
        }
        X[(int64_t)c * R + q] = v;
    }
}

void embed(const float *emb, int C, int vocab, const int32_t *ids, const int64_t *cum, const Batch &b, float *X,
           int64_t R, int *err, cudaStream_t st, const float *pos, const float *type) {
    const unsigned gx = (unsigned)((R + 255) / 256);
    k_embed<<<dim3(gx, C < 64 ? C : 64), 256, 0, st>>>(emb, C, vocab, ids, cum, b, X, R, err, pos, type);
}

// ggml_norm over the C channels of each token row, as the reference's CPU op
// (kko_norm_time on one row): the sum in double in channel order, mean =
// (float)sum / C, the sum of the float squares (x - mean)^2 in double,
// variance = (float)(s2 / C), scale = 1 / sqrtf(variance + eps); then
// y * scale, * gamma[c], + beta[c] and (leaky_on) LeakyReLU(slope), each
// rounded once. A block of 128 threads takes 32 rows: the [C][32] tile is
// staged in shared memory with coalesced loads, warp 0 (lane = row) runs the
// two sequential double sums from there (the reference's order), and all
// threads write the result; the tile is read whole before anything is
// written, so y may be x. Gap rows are written as zero. lstm_B > 0: row t of
// utterance u goes to row t * lstm_B + u of y (the LSTM layout, rows beyond
// the utterances untouched). yh (level layout only): the result also as the
// half chunk-major operand of the next linear (chunk stride Ryh, with the lo
// halves lo_off further when lo_off > 0), valid rows only.
constexpr int kLnMaxC = 1024;

__global__ void __launch_bounds__(128) k_layer_norm_ch(const float *x, int64_t R, int C,
                                                       const float *__restrict__ gamma,
                                                       const float *__restrict__ beta, int leaky_on, float slope,
                                                       Batch b, float *y, int64_t R_out, int lstm_B, float eps,
                                                       __half *yh, int64_t Ryh, int64_t lo_off) {
    extern __shared__ float tile[];  // [C][32]
    __shared__ float stat[2][32];
    __shared__ int64_t orow_s[32];
    __shared__ int live_s[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t q0 = (int64_t)blockIdx.x * 32;
    if (warp == 0) {
        const int64_t q = q0 + lane;
        int live = 0;
        int64_t orow = q;
        if (q < R) {
            const int u = utt_of_row(b, 1, q);
            const int64_t t = q - b.offT[u];
            live = t >= 0 && t < b.T[u];
            if (lstm_B > 0) orow = t * lstm_B + u;
        }
        live_s[lane] = live;
        orow_s[lane] = orow;
    }
    for (int i = tid; i < C * 32; i += 128) {
        const int c = i >> 5, r = i & 31;
        tile[i] = q0 + r < R ? x[(int64_t)c * R + q0 + r] : 0.0f;
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
    // thread = (chunk of 8 channels, row): the F32 values, and with yh the
    // chunk's 8 halves of the row as one 16-byte store
    const int nch = (C + 7) / 8;
    for (int i = tid; i < nch * 32; i += 128) {
        const int ck = i >> 5, r = i & 31;
        if (q0 + r >= R) continue;
        const bool lv = live_s[r] != 0;
        if (!lv && lstm_B > 0) continue;
        __align__(16) __half hh[8], ll[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int c = ck * 8 + e;
            float v = 0.0f;
            if (c < C && lv) {
                v = __fmul_rn(__fsub_rn(tile[c * 32 + r], stat[0][r]), stat[1][r]);
                v = __fadd_rn(__fmul_rn(v, gamma[c]), beta[c]);
                if (leaky_on) v = leaky(v, slope);
            }
            if (c < C) y[(int64_t)c * R_out + (lv ? orow_s[r] : q0 + r)] = v;
            hh[e] = __float2half_rn(v);
            ll[e] = split_lo(v, hh[e]);
        }
        if (yh && lv) {
            __half *dst = yh + ((int64_t)ck * Ryh + q0 + r) * 8;
            *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(hh);
            if (lo_off > 0) *reinterpret_cast<uint4 *>(dst + lo_off) = *reinterpret_cast<const uint4 *>(ll);
        }
    }
}

cudaError_t layer_norm_ch(const float *x, int64_t R, int C, const float *gamma, const float *beta, int leaky_on,
                          float slope, float eps, const Batch &b, float *y, int64_t R_out, int lstm_B,
                          cudaStream_t st, __half *yh, int64_t Ryh, int64_t lo_off) {
    if (yh && lstm_B > 0) return cudaErrorInvalidValue;
    static std::atomic<bool> attr[64];
    int dev = 0;
    if (C < 1 || C > kLnMaxC) return cudaErrorInvalidValue;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(k_layer_norm_ch, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kLnMaxC * 32 * sizeof(float)));
        if (e != cudaSuccess) return e;
        attr[dev].store(true, std::memory_order_release);
    }
    const size_t smem = (size_t)C * 32 * sizeof(float);
    k_layer_norm_ch<<<(unsigned)((R + 31) / 32), 128, smem, st>>>(x, R, C, gamma, beta, leaky_on, slope, b, y, R_out,
                                                                  lstm_B, eps, yh, Ryh, lo_off);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// ALBERT attention (kokoro.cpp:303-321): per sequence, head and tile of 32
// queries, scores[q][k] = sum over d of K[d][k] Q[d][q] (F32, d ascending),
// the softmax of ggml_soft_max_ext (w = s * scale, exp(w - max) with the sum
// in double in key order, times (float)(1 / sum)), then out[d][q] = sum over
// keys ascending of p[q][k] V[d][k]. exp is evaluated in double and rounded
// once, the correctly rounded expf. qkv: [3 H][R] (Q, K, V channel blocks);
// out: [H][R].
// ---------------------------------------------------------------------------
constexpr int kAttQ = 32;      // queries per block
constexpr int kAttKC = 128;    // keys per staged chunk
constexpr int kAttMaxN = 512;  // tokens per sequence
constexpr int kAttHS = 64;     // head size
constexpr int kAttS = kAttMaxN + 1;
constexpr size_t kAttSmem = (size_t)(kAttQ * kAttS + kAttHS * kAttQ + kAttHS * kAttKC) * sizeof(float);

__global__ void __launch_bounds__(256) k_attention(const float *__restrict__ qkv, int64_t R, int H, Batch b,
                                                   float scale, float *__restrict__ out) {
    extern __shared__ float sm[];
    float *S = sm;                        // [kAttQ][kAttS]
    float *Qs = S + kAttQ * kAttS;        // [kAttHS][kAttQ]
    float *KV = Qs + kAttHS * kAttQ;      // [kAttHS][kAttKC]
    const int u = blockIdx.z, h = blockIdx.y;
    const int n = b.T[u];
    const int q0 = blockIdx.x * kAttQ;
    if (q0 >= n) return;  // the whole block
    const int64_t off = b.offT[u];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *Q = qkv + (int64_t)(h * kAttHS) * R + off;
    const float *K = qkv + (int64_t)(H + h * kAttHS) * R + off;
    const float *V = qkv + (int64_t)(2 * H + h * kAttHS) * R + off;
    for (int i = tid; i < kAttHS * kAttQ; i += 256) {
        const int d = i / kAttQ, qi = i % kAttQ;
        Qs[i] = q0 + qi < n ? Q[(int64_t)d * R + q0 + qi] : 0.0f;
    }
    // scores: thread (qi = lane, key j = warp + 8 m of the chunk)
    for (int k0 = 0; k0 < n; k0 += kAttKC) {
        const int kn = n - k0 < kAttKC ? n - k0 : kAttKC;
        __syncthreads();
        for (int i = tid; i < kAttHS * kAttKC; i += 256) {
            const int d = i / kAttKC, j = i % kAttKC;
            KV[i] = j < kn ? K[(int64_t)d * R + k0 + j] : 0.0f;
        }
        __syncthreads();
        for (int j = warp; j < kn; j += 8) {
            float acc = 0.0f;
            for (int d = 0; d < kAttHS; ++d) acc = __fadd_rn(acc, __fmul_rn(KV[d * kAttKC + j], Qs[d * kAttQ + lane]));
            S[lane * kAttS + k0 + j] = acc;
        }
    }
    __syncthreads();
    // softmax: warp per query row
    for (int qi = warp; qi < kAttQ; qi += 8) {
        float *row = S + qi * kAttS;
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) {
            const float w = __fmul_rn(row[j], scale);
            row[j] = w;
            mx = fmaxf(mx, w);
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (int j = lane; j < n; j += 32) row[j] = __double2float_rn(exp((double)__fsub_rn(row[j], mx)));
        __syncwarp();
        float inv = 0.0f;
        if (lane == 0) {
            double sum = 0.0;
            for (int j = 0; j < n; ++j) sum = __dadd_rn(sum, (double)row[j]);
            inv = __double2float_rn(__ddiv_rn(1.0, sum));
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int j = lane; j < n; j += 32) row[j] = __fmul_rn(row[j], inv);
    }
    // weighted sum of V: thread (qi = lane, d = warp + 8 m)
    float acc[kAttHS / 8];
#pragma unroll
    for (int m = 0; m < kAttHS / 8; ++m) acc[m] = 0.0f;
    for (int k0 = 0; k0 < n; k0 += kAttKC) {
        const int kn = n - k0 < kAttKC ? n - k0 : kAttKC;
        __syncthreads();
        for (int i = tid; i < kAttHS * kAttKC; i += 256) {
            const int d = i / kAttKC, j = i % kAttKC;
            KV[i] = j < kn ? V[(int64_t)d * R + k0 + j] : 0.0f;
        }
        __syncthreads();
        const float *prow = S + lane * kAttS + k0;
        for (int j = 0; j < kn; ++j) {
            const float p = prow[j];
#pragma unroll
            for (int m = 0; m < kAttHS / 8; ++m) acc[m] = __fadd_rn(acc[m], __fmul_rn(p, KV[(warp + 8 * m) * kAttKC + j]));
        }
    }
    if (q0 + lane < n) {
#pragma unroll
        for (int m = 0; m < kAttHS / 8; ++m)
            out[(int64_t)(h * kAttHS + warp + 8 * m) * R + off + q0 + lane] = acc[m];
    }
}

cudaError_t attention(const float *qkv, int64_t R, int H, int n_heads, int max_len, const Batch &b, float scale,
                      float *out, cudaStream_t st) {
    if (H != n_heads * kAttHS || max_len < 1 || max_len > kAttMaxN) return cudaErrorInvalidValue;
    static std::atomic<bool> attr[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttSmem);
        if (e != cudaSuccess) return e;
        attr[dev].store(true, std::memory_order_release);
    }
    const dim3 grid((unsigned)((max_len + kAttQ - 1) / kAttQ), (unsigned)n_heads, (unsigned)b.n);
    k_attention<<<grid, 256, kAttSmem, st>>>(qkv, R, H, b, scale, out);
    return cudaGetLastError();
}

// ggml_gelu on F32 as ggml's CPU op with its F16 table (GGML_GELU_FP16): 0
// for x <= -10, x for x >= 10, else half(gelu(half(x))) with the tanh
// approximation 0.5 h (1 + tanh(sqrt(2/pi) h (1 + 0.044715 h^2))); tanh in
// double, rounded once. In place over n values.
__global__ void k_gelu(float *__restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        float g;
        if (v <= -10.0f) {
            g = 0.0f;
        } else if (v >= 10.0f) {
            g = v;
        } else {
            const float hv = round_f16(v);
            const float a = __fmul_rn(0.79788456080286535587989211986876f, hv);
            const float inner = __fmul_rn(a, __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, hv), hv)));
            const float th = __double2float_rn(tanh((double)inner));
            g = round_f16(__fmul_rn(__fmul_rn(0.5f, hv), __fadd_rn(1.0f, th)));
        }
        x[i] = g;
    }
}

void gelu(float *x, int64_t n, cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    k_gelu<<<(unsigned)blocks, 256, 0, st>>>(x, n);
}

// Packed level-1 [C][R] -> token-major out[(cum[u] + t) * C + c].
__global__ void k_rows_out(const float *__restrict__ x, int64_t R, int C, Batch b, const int64_t *__restrict__ cum,
                           float *__restrict__ out) {
    const int u = blockIdx.y;
    const int64_t n = b.T[u];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * C;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / C;
        const int c = (int)(i % C);
        out[(cum[u] + t) * C + c] = x[(int64_t)c * R + b.offT[u] + t];
    }
}

void rows_out(const float *x, int64_t R, int C, const Batch &b, const int64_t *cum, int max_len, float *out,
              cudaStream_t st) {
    int64_t bx = ((int64_t)max_len * C + 255) / 256;
    if (bx > 1024) bx = 1024;
    k_rows_out<<<dim3((unsigned)bx, (unsigned)b.n), 256, 0, st>>>(x, R, C, b, cum, out);
}

// The duration projection and bucket sum. Token j of a block (kDurTok tokens
// per block, row r = t * B + s of the LSTM layout, h(r, k) = h[r * s_row + k *
// s_k]) is staged in shared memory; thread (j, n) forms bucket n: acc =
// bias[n] + sum over k ascending of w[n][k] * h[k] with separately rounded
// double products and sums, x = (float)acc, then the logistic function in
// double by the branch that cannot overflow. Thread n = 0 adds the bucket
// terms in order and writes (float)sum to out[cum[s] + t].
constexpr int kDurTok = 4;
constexpr int kDurMaxBuckets = 64;
constexpr int kDurMaxIn = 1024;

__global__ void __launch_bounds__(kDurTok * kDurMaxBuckets) k_duration_proj(
    const float *__restrict__ h, int64_t s_row, int64_t s_k, int P, const float *__restrict__ w,
    const float *__restrict__ bias, int NB, const int32_t *__restrict__ len, const int64_t *__restrict__ cum, int B,
    int64_t n_rows, float *__restrict__ out) {
    __shared__ float hs[kDurTok][kDurMaxIn];
    __shared__ double term[kDurTok][kDurMaxBuckets];
    const int j = threadIdx.x / kDurMaxBuckets, n = threadIdx.x % kDurMaxBuckets;
    const int64_t r = (int64_t)blockIdx.x * kDurTok + j;
    const int s = (int)(r % B);
    const int64_t t = r / B;
    const bool live = r < n_rows && t < len[s];
    if (live)
        for (int k = n; k < P; k += kDurMaxBuckets) hs[j][k] = h[r * s_row + (int64_t)k * s_k];
    __syncthreads();
    if (live && n < NB) {
        const float *wr = w + (int64_t)n * P;
        double acc = (double)bias[n];
        for (int k = 0; k < P; ++k) acc = __dadd_rn(acc, __dmul_rn((double)wr[k], (double)hs[j][k]));
        const double x = (double)__double2float_rn(acc);
        double v;
        if (x >= 0.0) {
            v = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-x)));
        } else {
            const double e = exp(x);
            v = __ddiv_rn(e, __dadd_rn(1.0, e));
        }
        term[j][n] = v;
    }
    __syncthreads();
    if (live && n == 0) {
        double sum = 0.0;
        for (int i = 0; i < NB; ++i) sum = __dadd_rn(sum, term[j][i]);
        out[cum[s] + t] = __double2float_rn(sum);
    }
}

cudaError_t duration_proj(const float *h, int64_t s_row, int64_t s_k, int P, const float *w, const float *bias,
                          int NB, const int32_t *len, const int64_t *cum, int B, int64_t n_rows, float *out,
                          cudaStream_t st) {
    if (P < 1 || P > kDurMaxIn || NB < 1 || NB > kDurMaxBuckets || B < 1 || n_rows < 1) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)((n_rows + kDurTok - 1) / kDurTok);
    k_duration_proj<<<grid, kDurTok * kDurMaxBuckets, 0, st>>>(h, s_row, s_k, P, w, bias, NB, len, cum, B, n_rows,
                                                                out);
    return cudaGetLastError();
}

}  // namespace kk
