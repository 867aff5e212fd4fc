// Text encoder and duration head of the Kokoro-82M front end (sm_100a):
// the embedding lookup and the per-token LayerNorm of the text encoder's CNN
// (text_encoder, src/arch/kokoro/graph_ops.cpp:1578-1624; its k = 5 convs
// run on the conv kernels of kk_conv_tc.cu / kk_conv_simt.cu and its biLSTM
// on kk_lstm.cu), and the duration projection with the bucket sum that the
// reference runs on the host in double (src/arch/kokoro/kokoro.cpp:469-516).
#include "kk_common.cuh"
#include "kk_kernels.h"

namespace kk {

// ggml_get_rows of the embedding [C, vocab] into the packed level-1 layout:
// X[c][q] = emb[id * C + c] on the token rows of each utterance (id =
// ids[cum[u] + t]), zero on the gap rows. An id outside [0, vocab) gives a
// zero row and sets *err to kErrTokenId.
__global__ void k_embed(const float *__restrict__ emb, int C, int vocab, const int32_t *__restrict__ ids,
                        const int64_t *__restrict__ cum, Batch b, float *__restrict__ X, int64_t R, int *err) {
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
    for (int c = blockIdx.y; c < C; c += gridDim.y)
        X[(int64_t)c * R + q] = id >= 0 ? emb[(int64_t)id * C + c] : 0.0f;
}

void embed(const float *emb, int C, int vocab, const int32_t *ids, const int64_t *cum, const Batch &b, float *X,
           int64_t R, int *err, cudaStream_t st) {
    const unsigned gx = (unsigned)((R + 255) / 256);
    k_embed<<<dim3(gx, C < 64 ? C : 64), 256, 0, st>>>(emb, C, vocab, ids, cum, b, X, R, err);
}

// ggml_norm over the C channels of each token row, as the reference's CPU op
// (kko_norm_time on one row): the sum in double in channel order, mean =
// (float)sum / C, the sum of the float squares (x - mean)^2 in double,
// variance = (float)(s2 / C), scale = 1 / sqrtf(variance + eps); then
// y * scale, * gamma[c], + beta[c], LeakyReLU(slope), each rounded once.
// One thread per row (coalesced across the warp's rows), so the double sums
// run in the reference's order. Gap rows are written as zero. lstm_B > 0:
// row t of utterance u goes to row t * lstm_B + u of y (the LSTM layout,
// rows beyond the utterances untouched).
__global__ void __launch_bounds__(128) k_layer_norm_ch(const float *__restrict__ x, int64_t R, int C,
                                                       const float *__restrict__ gamma,
                                                       const float *__restrict__ beta, float slope, Batch b,
                                                       float *__restrict__ y, int64_t R_out, int lstm_B,
                                                       float eps) {
    const int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (q >= R) return;
    const int u = utt_of_row(b, 1, q);
    const int64_t t = q - b.offT[u];
    const bool live = t >= 0 && t < b.T[u];
    if (lstm_B > 0) {
        if (!live) return;
    } else if (!live) {
        for (int c = 0; c < C; ++c) y[(int64_t)c * R_out + q] = 0.0f;
        return;
    }
    const int64_t orow = lstm_B > 0 ? t * lstm_B + u : q;
    double s = 0.0;
    for (int c = 0; c < C; ++c) s = __dadd_rn(s, (double)x[(int64_t)c * R + q]);
    const float mean = __fdiv_rn((float)s, (float)C);
    double s2 = 0.0;
    for (int c = 0; c < C; ++c) {
        const float v = __fsub_rn(x[(int64_t)c * R + q], mean);
        s2 = __dadd_rn(s2, (double)__fmul_rn(v, v));
    }
    const float var = (float)__ddiv_rn(s2, (double)C);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int c = 0; c < C; ++c) {
        float v = __fmul_rn(__fsub_rn(x[(int64_t)c * R + q], mean), scale);
        v = __fadd_rn(__fmul_rn(v, gamma[c]), beta[c]);
        y[(int64_t)c * R_out + orow] = leaky(v, slope);
    }
}

void layer_norm_ch(const float *x, int64_t R, int C, const float *gamma, const float *beta, float slope,
                   const Batch &b, float *y, int64_t R_out, int lstm_B, cudaStream_t st) {
    k_layer_norm_ch<<<(unsigned)((R + 127) / 128), 128, 0, st>>>(x, R, C, gamma, beta, slope, b, y, R_out, lstm_B,
                                                                1e-5f);
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
