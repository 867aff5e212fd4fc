// Kernel launch interface of the Kokoro-82M hot path (host side of the .cu
// files). All launches are asynchronous on the given stream.
#pragma once

#include "kk_common.cuh"

namespace kk {

enum { ACT_NONE = 0, ACT_LEAKY = 1, ACT_SNAKE = 2, ACT_GELU = 3 };

// One AdaIN site (adain_1d / ada_layer_norm): fc weights transposed to
// [128, C] (F32 values), and per-utterance outputs gamma/beta [n_utts, C].
struct AdainSite {
    const float *gw, *gb, *bw, *bb;
    float *gamma, *beta;
    int C;
    int f16;  // weight stored as F16: ggml rounds the style to half
};

struct PrologueArgs {
    int norm;                 // apply the AdaIN normalisation
    const float2 *ms;         // [n, C] (mean, scale)
    const float *norm_w, *norm_b;
    const float *gamma, *beta;  // [n, C]
    int act;                  // ACT_*
    float slope;              // LeakyReLU slope
    const float *alpha;       // Snake alpha [C]
    int round16;              // round the result to half (F16 conv operand)
    // x2, x3 non-null (without norm): the input is ((x + x2) + x3) * sum_scale,
    // the average of the three residual-block branches (graph_ops.cpp:1300-1320)
    const float *x2, *x3;
    float sum_scale;
    // > 0 (half operands): also write lo = half(v - half(v)) lo_off halves
    // after each hi value, the split-F32 operand [hi chunks | lo chunks]
    int64_t lo_off;
};

// Dense convolution over a packed [IC, R_in] operand (zero gaps):
//   y[oc, orow(q)] = epi( sum_{ic,k} W[oc, ic, k] * x[ic, q*s - p + k*d] )
// for q in [0, n_pos), orow(q) = q * omul + oadd (rows outside [0, R_out)
// are skipped). Epilogue, with each step rounded as the reference's
// separate ggml ops:
//   v = acc (+ bias[oc]); if resid: v = resid[oc, rrow] + v;
//   v *= scale1; if accum: v = y_old + v; v *= scale2; y = v
// rrow = orow, or orow / 2 when resid_half (nearest x2 upsample of the
// shortcut, maybe_upsample_nearest at graph_ops.cpp:925-933).
struct ConvArgs {
    const float *in;
    int64_t R_in;
    int IC;
    const float *w;  // [OC, IC, K] F32 values
    int OC, K, s, p, d;
    float *out;
    int64_t R_out;
    int64_t n_pos;
    int64_t omul, oadd;
    const float *bias;
    const float *resid;
    int64_t R_resid;
    int resid_half;
    float scale1;
    int accum;
    float scale2;
    int round16;  // round the operand to half on load (F16 weights)
};

struct ConvTRow0Args {
    const float *in;      // F32 [C][R] operand, or
    const __half *in_h;   // half chunk-major operand (when non-null)
    int64_t lo_off;       // > 0: in_h is split F32, value = hi + the half lo_off further
    int64_t R_in;         // row stride of `in`, or the chunk stride of `in_h`
    int IC, m_in;
    const float *w;  // ggml [K, OC, IC]
    int OC, K, crop, m_out;
    const float *bias;
    const float *add;
    float *out;
    int64_t R_out;
    int round16;
};

struct SineArgs {
    float mw_scaled[kHarmonics];  // merge weights * 0.1
    float mb;                     // merge bias
    float unvoiced;               // tanhf(mb), host C library
};

struct StftTables {
    float c[kStftN][kBins], s[kStftN][kBins];
    float window[kStftN];
};

struct IstftTables {
    float c[kBins][kStftN], s[kBins][kStftN];
    float window[kStftN], window_sq[kStftN];
};

void scatter(const float *src, float *dst, int64_t R, int C, int m, int extra, const Batch &b,
             const int64_t *cumT, int max_len, cudaStream_t st);
// gather: the inverse of scatter (packed [C, R] -> per-utterance tensors)
void gather(const float *src, float *dst, int64_t R, int C, int m, int extra, const Batch &b,
            const int64_t *cumT, int max_len, cudaStream_t st);
void adain_affine(const AdainSite *sites_dev, int n_sites, const float *style, int n_utts,
                  cudaStream_t st);
void stats(const float *x, int64_t R, int C, int m, int extra, const Batch &b, float2 *ms,
           cudaStream_t st);
// stats_blocks: the same terms from the 32-row block partials of a tensor
// (part[c * NB + row / 32] = (sum, sum of squares about the block mean))
// whose utterances all start on a 32-row boundary
void stats_blocks(const float2 *part, int64_t NB, int C, int m, int extra, const Batch &b, float2 *ms,
                  cudaStream_t st);
void prologue(const float *x, float *y, int64_t R, int C, int m, int extra, const Batch &b,
              int max_len, const PrologueArgs &a, cudaStream_t st);
void convt_row0(const ConvTRow0Args &a, const Batch &b, cudaStream_t st);
void pool_up(const float *x, float *y, int64_t R_in, int64_t R_out, int C, const float *w,
             const float *bias, const Batch &b, int max_T, int round16, cudaStream_t st);
void f0n_conv(const float *in, int64_t R_in, float *out0, float *out1, int64_t R_out, const float *w,
              const float *bias, const Batch &b, int max_T, cudaStream_t st);
// Packed per-utterance lengths are multiples of the base unit b.T: the F0
// curve has mf * T frames (mf = 2 for asr-frame units, 1 for decoder-frame
// units), the source 300 mf T samples, the STFT 60 mf T + 1 frames.
void sinegen(const float *f0, int mf, float *source, const Batch &b, const int64_t *cumT,
             const SineArgs &a, cudaStream_t st);
// Thread blocks (one SM each at most) the harmonic source of n utterances
// occupies while it runs.
int sinegen_blocks(int n_utts);
void stft(const float *source, float *har, int64_t R, int mf, const Batch &b, const int64_t *cumT,
          const StftTables *tab, int max_T, cudaStream_t st);
// post has a_nf * T + 1 frames per utterance at rows a_nf * offT; audio is
// 5 a_nf T samples per utterance, back to back.
void istft(const float *post, int64_t R, int a_nf, float *audio, const Batch &b, const int64_t *cumT,
           const IstftTables *tab, int max_T, cudaStream_t st);

// kk_conv_simt.cu
void conv_simt(const ConvArgs &a, cudaStream_t st);
cudaError_t conv_simt_init();

// Half chunk-major operands of the tensor-core path. Channel chunk j (8
// channels) holds rows [-kHalfLo, R + kHalfHi) at a stride of
// Ry = R + kHalfLo + kHalfHi rows of 16 bytes; the pointer handed around
// addresses row 0 of chunk 0, so row r of chunk j is y[(j * Ry + r) * 8 ...].
// The margins (and all gap rows) read as zero: they are the convolution's
// zero padding, fetched with plain bulk copies instead of a clipped tensor
// map.
constexpr int64_t kHalfLo = 64;
constexpr int64_t kHalfHi = 256;
__host__ __device__ constexpr int64_t half_stride(int64_t R) { return R + kHalfLo + kHalfHi; }

// kk_conv_tc.cu: tensor-core convolution, stride 1, half operands.
// in: half operand (row 0 of chunk 0), chunk stride R_in = half_stride(R)
// for an operand of R rows; n_pos <= R. w: packed half
// [K][IC_pad/64][n_tiles][8][128][8]; epilogue as ConvArgs.
struct ConvTcArgs {
    const __half *in;
    int64_t R_in;
    int IC_pad;
    // > 0: the K blocks of 64 channels past a_wrap read operand block
    // b - a_wrap again (the split-F32 GEMM's third term reuses the hi part)
    int a_wrap;
    // non-zero and not 1: the accumulator is multiplied by this power of two
    // before the epilogue (split weights packed scaled by its inverse)
    float acc_scale;
    const __half *w;
    int n_tiles;
    int OC, K, p, d;
    float *out;
    int64_t R_out;
    int64_t n_pos;
    int64_t omul, oadd;
    const float *bias;
    const float *resid;
    int64_t R_resid;
    int resid_half;
    // non-null: per output channel, multiplies the value after the bias and
    // the residual, before scale1 (the Vocos layer scale)
    const float *chscale;
    float scale1;
    int accum;
    float scale2;
    int *err;
    // > 0: the weights are phase-packed (OC = phases x phase_oc, phase-major);
    // channel n writes channel n % phase_oc at rows q * omul + oadd + n / phase_oc
    int phase_oc;
    // > 0: a transposed convolution with stride omul on k_convt_tc. The
    // weights are packed in tiles of omul * phase_nc rows (phase r, channel c
    // at row r * phase_nc + c; OC real channels per phase), and channel c of
    // phase r at input position q writes output row q * omul + oadd + r.
    // Epilogue: bias and residual only.
    int phase_nc;
    // non-null (DevStatus::sched, zero at launch): the channels x positions
    // kernel hands out its tiles past each CTA's first in the order CTAs ask
    // for them, so that CTAs which start late (their SMs held by another
    // stream's kernel) take fewer tiles instead of holding the launch's end
    int *sched;
    // non-null: the instance-norm terms (mean, scale) of the output over each
    // utterance's valid rows at level (sm, sextra) of batch sb, into
    // stats[u * OC + c]. With stats_aligned (every utterance of the level
    // starts on a 32-row boundary) and part (scratch of OC * R_out / 32
    // float2) the convolution keeps block partials as it writes and a small
    // pass reduces them; otherwise a separate pass reads the output.
    float2 *stats;
    Batch sb;
    int sm, sextra;
    int stats_aligned;
    float2 *part;
    // x non-null: the operand is formed inside the conv from the F32 tensor
    // x [IC_pad][R_out] (the output's level) as half(snake(adain(x))) on the
    // valid rows of level (sm, sextra), zero elsewhere: the k_prologue_h
    // arithmetic with (mean, scale) x_ms [n][IC], norm weight/bias [IC],
    // gamma/beta [n][IC] and Snake alpha [IC]; in / R_in are unused. Only
    // where conv_tc_fusable holds.
    const float *x;
    const float2 *x_ms;
    const float *x_nw, *x_nb, *x_gamma, *x_beta, *x_alpha;
};
cudaError_t conv_tc_init();
cudaError_t conv_tc(const ConvTcArgs &a, cudaStream_t st);
bool conv_tc_fusable(const ConvTcArgs &a);
int conv_tc_max_halo();
// Channels per phase of k_convt_tc's tiles for stride S and OC channels per
// phase (0: no instance of the kernel serves this shape).
int convt_phase_nc(int S, int OC);

// prologue_h: y[c/8][row][c%8] = half(act(adain(x[c][row]))) on valid rows
// (x is F32 [C][R]; y a half operand of chunk stride Ry).
void prologue_h(const float *x, __half *y, int64_t R, int64_t Ry, int C, int m, int extra, const Batch &b,
                int mean_len, const PrologueArgs &a, cudaStream_t st);
// har_s2d: space-to-depth half operand [192/8][R][8] (chunk stride Ry) of the
// stride-6 noise convolution (132 real channels), all R rows of the stage-0
// level.
void har_s2d(const float *har, int64_t R_har, __half *y, int64_t R, int64_t Ry, int64_t lo_off, cudaStream_t st);
// pool_up_h: the depthwise x2 pool written as a half operand of chunk stride
// Ry_out. lo_off > 0 on har_s2d and pool_up_h: the split-F32 operand, as
// PrologueArgs::lo_off.
void pool_up_h(const float *x, __half *y, int64_t R_in, int64_t Ry_out, int C, const float *w, const float *bias,
               const Batch &b, int max_T, int64_t lo_off, cudaStream_t st);
// pool_up_h of LeakyReLU(AdaIN(x)) (norm terms, gamma / beta and slope of a,
// the arithmetic of prologue), without the F32 intermediate
void pool_up_adain_h(const float *x, __half *y, int64_t R_in, int64_t Ry_out, int C, const float *w,
                     const float *bias, const Batch &b, int max_T, int64_t lo_off, const PrologueArgs &a,
                     cudaStream_t st);

// kk_frontend.cu: the text encoder's embedding and LayerNorm, the duration
// projection.
constexpr int kErrTokenId = 31;  // device error word: a token id out of range

// The device status block of a context: the error word (0 = none; the first
// error wins) and, per checked tensor, the smallest index of a non-finite
// value (all bits set = none).
enum { kFiniteF0 = 0, kFiniteNoise, kFiniteAsr, kFiniteDecoder, kFiniteStyle, kFiniteLabels };
constexpr int kErrNonFinite = 60;  // + label
struct DevStatus {
    int code;
    int pad;
    // the dynamic tile order of the channels x positions convolution: the
    // next tile past the static first ones, and the CTAs done (both zero
    // between launches: the last CTA of a launch resets them)
    int sched[2];
    unsigned long long first[kFiniteLabels];
};
// Records a non-finite value of x[0, n) (label's smallest index, and the
// error word kErrNonFinite + label if it is still 0).
void check_finite(const float *x, int64_t n, int label, DevStatus *status, cudaStream_t st);
// A bounded wait on an mbarrier that nothing arrives at: after limit_ns the
// waiting thread sets *err to kErrWaitSelftest (if 0) and the kernel returns.
constexpr int kErrWaitSelftest = 77;
// The LSTM recurrence's wait for a step's hidden state ran out (1 s).
constexpr int kErrLstmWait = 45;
cudaError_t wait_selftest(int *err, unsigned long long limit_ns, cudaStream_t st);
// pos / type non-null (ALBERT): + the position row t and the token type row 0
void embed(const float *emb, int C, int vocab, const int32_t *ids, const int64_t *cum, const Batch &b, float *X,
           int64_t R, int *err, cudaStream_t st, const float *pos = nullptr, const float *type = nullptr);
// LayerNorm (eps) over C channels per token row + gamma / beta, then
// LeakyReLU(slope) when leaky_on; lstm_B > 0 writes row t * lstm_B + u (the
// LSTM layout) instead of row q. y may be x.
// (C <= 1024)
// yh non-null: also the half operand of the next linear (see kk_frontend.cu)
cudaError_t layer_norm_ch(const float *x, int64_t R, int C, const float *gamma, const float *beta, int leaky_on,
                          float slope, float eps, const Batch &b, float *y, int64_t R_out, int lstm_B,
                          cudaStream_t st, __half *yh = nullptr, int64_t Ryh = 0, int64_t lo_off = 0);
// ---- sanoTTS Vocos (kk_vocos.cu) ----
// The tables of istft()'s RealRadix2 plan (src/audio/istft.cpp:96-168) for
// one n_fft, each computed in double and rounded once: the periodic Hann
// window and its squares [n], the stage twiddles [half - 1] (entry h - 1 + k
// for stage h), the split factors [half], and the bit-reversal map [half].
struct R2Tables {
    const float *window, *window_sq;
    const float *stage_cos, *stage_sin;
    const float *split_cos, *split_sin;
    const int *rev;
};
// depthwise conv (K taps, zero padding per utterance) + bias, then
// LayerNorm over the C channels (eps) * gamma + beta, into the half operand
// yh (chunk stride Ryh, lo halves at lo_off when > 0) on the valid rows of
// level 1 (C <= 1024)
cudaError_t dw_layer_norm(const float *x, int64_t R, int C, int K, const float *dw_w, const float *dw_b,
                          const float *gamma, const float *beta, float eps, const Batch &b, __half *yh, int64_t Ryh,
                          int64_t lo_off, cudaStream_t st);
// the head output h [2 (n/2 + 1)][R] -> windowed inverse-FFT frames
// fr [R][n] on the valid rows (n a power of two, 64 .. 2048)
cudaError_t vocos_spectrum(const float *h, int64_t R, int n, float mag_clip, const Batch &b, const R2Tables &tab,
                           float *fr, cudaStream_t st);
// overlap-add of fr into audio + cum[u]: hop (T_u - 1) samples per utterance
void vocos_ola(const float *fr, int n, int hop, const Batch &b, const int64_t *cum, const float *window_sq,
               int64_t max_len, float *audio, cudaStream_t st);
// DC blocker in place over audio + cum[u], len[u] samples each
void dc_block(float *audio, const int64_t *cum, const int64_t *len, int n_utts, float pole, cudaStream_t st);

// ALBERT self-attention: qkv [3 H][R] -> out [H][R], heads of 64, at most
// 512 tokens per sequence
cudaError_t attention(const float *qkv, int64_t R, int H, int n_heads, int max_len, const Batch &b, float scale,
                      float *out, cudaStream_t st);
void gelu(float *x, int64_t n, cudaStream_t st);
// packed level-1 [C][R] -> token-major [sum T][C]
void rows_out(const float *x, int64_t R, int C, const Batch &b, const int64_t *cum, int max_len, float *out,
              cudaStream_t st);
// durations[cum[s] + t] from h(r, k) = h[r * s_row + k * s_k], r = t * B + s
// (P <= 1024 inputs, NB <= 64 buckets)
cudaError_t duration_proj(const float *h, int64_t s_row, int64_t s_k, int P, const float *w, const float *bias,
                          int NB, const int32_t *len, const int64_t *cum, int B, int64_t n_rows, float *out,
                          cudaStream_t st);

// kk_lstm.cu: bidirectional LSTM stack and the duration alignment.
// Sequences are packed time-major: row = t * B + b of a [C][R] activation.
struct LstmRecArgs {
    const float *pre;      // [2 * 4H][R]: W_ih x + b_ih, forward rows then backward rows
    int64_t R;
    const float *whh[2];   // per direction, rowwise [4H][H] F32 (gate order i, f, g, o)
    const float *bhh[2];   // per direction, [4H]
    float *hout;           // [2H][R]: forward units then backward units
    const int32_t *len;    // [B] steps of each sequence (device)
    int B;                 // sequences
    int Bc;                // sequences per cluster: 1, 2, 4, 8, 16 or 32
    int max_len;           // max over len
    int *err;              // device error word: set when a bounded wait runs out
};
size_t lstm_rec_smem(int Bc);
// Clusters of the recurrence kernel for group size Bc that the current device
// runs at once (cudaOccupancyMaxActiveClusters; cached per device), 0 if unknown.
int lstm_max_clusters(int Bc);
cudaError_t lstm_recurrence(const LstmRecArgs &a, cudaStream_t st);  // H = 256
void lstm_pack(const float *x, int D, const float *style, int Ds, float *X, int64_t R, const int32_t *len,
               const int64_t *cum, int B, int max_len, cudaStream_t st);
// X [C][R] in the LSTM layout -> rows m * offT[b] + t of a packed level
void lstm_to_level(const float *X, int64_t R, int C, int B, const int32_t *len, int max_len, float *dst,
                   int64_t R_dst, const int64_t *offT, int m, cudaStream_t st);
void lstm_unpack(const float *X, int64_t R, int C, float *out, const int32_t *len, const int64_t *cum, int B,
                 int max_len, cudaStream_t st);
void style_linear(const float *w, const float *bias, int f16, const float *style, int Ds, int C, int B, float *out,
                  cudaStream_t st);
void ada_layer_norm(const float *h, int64_t R, int D, const float *gamma, const float *beta, float *X,
                    const int32_t *len, int B, cudaStream_t st);
// frames[i] and start[0..n] (start[n] = total frames)
void duration_frames(const float *d, int64_t n, float speed, int32_t *frames, int64_t *start, cudaStream_t st);
void align_gather(const float *hidden, int64_t D, const int32_t *frames, const int64_t *start, int64_t n, float *en,
                  cudaStream_t st);

}  // namespace kk
