/*
 * The oracle — CPU restatement of the Kokoro-82M synthesis hot path.
 *
 * TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py as the checker. The product library never
 * links or loads it.
 *
 * Build: see oracle/Makefile (-O3 -ffp-contract=off, no -march, like the
 * reference's own translation units, CMakeLists.txt:38-40). OpenMP splits
 * work across output channels / utterances only; every output element is
 * computed by one thread in a fixed order, so results do not depend on the
 * thread count.
 */
#define _GNU_SOURCE
#include "kk_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

/* Constants of src/core/constants.h. */
#define KO_STFT_N 20
#define KO_STFT_HOP 5
#define KO_BINS (KO_STFT_N / 2 + 1)
#define KO_SAMPLE_RATE 24000
#define KO_HARMONICS 9
#define KO_UPSAMPLE 300
#define KO_SINE_AMP 0.1f
#define KO_INV_SQRT2 0.7071067811865476f
static const int KO_DIL[3] = {1, 3, 5};
static const int KO_KS[3] = {3, 7, 11};

/* ------------------------------------------------------------------------ */
/* errors                                                                   */
/* ------------------------------------------------------------------------ */

static __thread char g_err[512];

const char *kko_last_error(void) { return g_err; }

static int fail(const char *fmt, const char *arg) {
    snprintf(g_err, sizeof g_err, fmt, arg ? arg : "");
    return -1;
}

/* ------------------------------------------------------------------------ */
/* IEEE half conversion (round to nearest even), as GGML_FP32_TO_FP16       */
/* ------------------------------------------------------------------------ */

static float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            exp = 127 - 15 + 1;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                exp--;
            }
            man &= 0x3ffu;
            bits = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below the smallest normal half: subnormal or 0 */
        if (ax < 0x33000000u) { /* < 2^-25: rounds to 0 (2^-25 ties to even 0) */
            return (uint16_t)sign;
        }
        const uint32_t e = ax >> 23;
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e; /* in [14, 24] */
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float kko_round_f16(float x) { return h2f(f2h(x)); }

static void round_f16_array(float *dst, const float *src, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = h2f(f2h(src[i]));
}

/* ------------------------------------------------------------------------ */
/* model: named tensors                                                     */
/* ------------------------------------------------------------------------ */

typedef struct {
    char *name;
    int f16;        /* stored as F16 in the GGUF: selects ggml's F16 arithmetic */
    int64_t ne[4];
    int64_t n;
    float *data;    /* dequantised values */
} ko_tensor;

struct kko_model {
    ko_tensor *t;
    size_t n;
    kko_tap_fn tap;
    void *tap_user;
    int source_libm;  /* 1: harmonic source uses the C library's float tanhf/sinf/cosf */
};

kko_model *kko_model_create(const kk_tensor_desc *descs, size_t n) {
    kko_model *m = (kko_model *)calloc(1, sizeof *m);
    if (!m) return NULL;
    m->t = (ko_tensor *)calloc(n ? n : 1, sizeof(ko_tensor));
    m->n = n;
    for (size_t i = 0; i < n; ++i) {
        ko_tensor *t = &m->t[i];
        t->name = strdup(descs[i].name);
        t->f16 = descs[i].dtype == KK_DTYPE_F16;
        int64_t cnt = 1;
        for (int d = 0; d < 4; ++d) {
            t->ne[d] = d < descs[i].n_dims ? descs[i].ne[d] : 1;
            cnt *= t->ne[d];
        }
        t->n = cnt;
        t->data = (float *)malloc((size_t)cnt * sizeof(float));
        if (t->f16) {
            const uint16_t *src = (const uint16_t *)descs[i].data;
            for (int64_t j = 0; j < cnt; ++j) t->data[j] = h2f(src[j]);
        } else {
            memcpy(t->data, descs[i].data, (size_t)cnt * sizeof(float));
        }
    }
    return m;
}

void kko_model_free(kko_model *m) {
    if (!m) return;
    for (size_t i = 0; i < m->n; ++i) {
        free(m->t[i].name);
        free(m->t[i].data);
    }
    free(m->t);
    free(m);
}

void kko_set_source_libm(kko_model *m, int use_libm) { m->source_libm = use_libm; }

/* Correctly rounded float tanh / sin / cos: evaluated in double, rounded
 * once. The reference calls the C library's float functions here
 * (audio_utils.cpp:182-183, :329, :352); their last bit varies between C
 * libraries (glibc 2.39 tanhf differs from the correctly rounded value for
 * about a third of inputs in [-0.1, 0.1]) and the generator amplifies that
 * last bit through the phases of near-silent STFT bins, so the source is
 * pinned to the correctly rounded values instead. */
static float cr_tanhf(float x) { return (float)tanh((double)x); }
static float cr_sinf(float x) { return (float)sin((double)x); }
static float cr_cosf(float x) { return (float)cos((double)x); }

void kko_set_tap(kko_model *m, kko_tap_fn fn, void *user) {
    m->tap = fn;
    m->tap_user = user;
}

static void tap(kko_model *m, const char *name, const float *d, int64_t ne0, int64_t ne1) {
    if (m->tap) m->tap(name, d, ne0, ne1, m->tap_user);
}

/* require_tensor (src/arch/kokoro/kokoro.cpp:19-25). */
static const ko_tensor *req(kko_model *m, const char *name) {
    for (size_t i = 0; i < m->n; ++i) {
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    }
    fail("missing tensor: %s", name);
    return NULL;
}

static const ko_tensor *opt(kko_model *m, const char *name) {
    for (size_t i = 0; i < m->n; ++i) {
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    }
    return NULL;
}

static float *fbuf(size_t n) { return (float *)calloc(n ? n : 1, sizeof(float)); }

/* ------------------------------------------------------------------------ */
/* elementwise ops                                                          */
/* ------------------------------------------------------------------------ */

/* ggml_leaky_relu: (x > 0 ? x : 0) + slope * (x < 0 ? x : 0). */
static void leaky_relu(float *y, const float *x, size_t n, float slope) {
    for (size_t i = 0; i < n; ++i) {
        const float v = x[i];
        y[i] = (v > 0.f ? v : 0.f) + slope * (v < 0.f ? v : 0.f);
    }
}

/* snake1d_fused_callback scalar path (src/arch/kokoro/graph_ops.cpp:392-497):
 * y = v + sinf(v * alpha)^2 * (1 / alpha). */
static void snake(float *x, int64_t C, int64_t L, const float *alpha) {
    for (int64_t c = 0; c < C; ++c) {
        const float a = alpha[c];
        const float inv_a = 1.0f / a;
        float *xc = x + c * L;
        for (int64_t t = 0; t < L; ++t) {
            const float v = xc[t];
            const float s = sinf(v * a);
            xc[t] = v + s * s * inv_a;
        }
    }
}

/* ggml semantics, ggml_norm over ne[0] (time) per channel, eps 1e-5:
 * mean = (float)sum_double / n; var = sum_double((x-mean)^2) / n;
 * y = (x - mean) * (1 / sqrtf(var + eps)). */
void kko_norm_time(const float *x, int64_t C, int64_t L, float eps, float *y) {
    for (int64_t c = 0; c < C; ++c) {
        const float *xc = x + c * L;
        float *yc = y + c * L;
        double sum = 0.0;
        for (int64_t t = 0; t < L; ++t) sum += (double)xc[t];
        const float fsum = (float)sum;
        const float mean = fsum / (float)L;
        double s2 = 0.0;
        for (int64_t t = 0; t < L; ++t) {
            const float v = xc[t] - mean;
            yc[t] = v;
            s2 += (double)(v * v);
        }
        const float var = (float)(s2 / (double)L);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int64_t t = 0; t < L; ++t) yc[t] *= scale;
    }
}

/* linear (graph_ops.cpp:636-654): y[o] = sum_i W[o][i] x[i] + b[o];
 * ggml mul_mat converts x to F16 when W is F16. Sequential F32 sum. */
static void linear_vec(const ko_tensor *w, const ko_tensor *b, const float *x, float *y) {
    const int64_t in = w->ne[0], out = w->ne[1];
    float *xr = fbuf((size_t)in);
    if (w->f16) round_f16_array(xr, x, (size_t)in);
    else memcpy(xr, x, (size_t)in * sizeof(float));
    for (int64_t o = 0; o < out; ++o) {
        float acc = 0.f;
        const float *wr = w->data + o * in;
        for (int64_t i = 0; i < in; ++i) acc += wr[i] * xr[i];
        y[o] = acc + b->data[o];
    }
    free(xr);
}

/* adain_1d (graph_ops.cpp:888-907): norm -> *norm_w + norm_b ->
 * cur + cur * gamma -> + beta; gamma/beta = linear(fc.{gamma,beta}, style). */
static int adain(kko_model *m, const char *prefix, const float *x, int64_t C, int64_t L,
                 const float *style, float *y) {
    char k[256];
    const ko_tensor *nw, *nb, *gw, *gb, *bw, *bb;
    snprintf(k, sizeof k, "%s.norm.weight", prefix); nw = req(m, k);
    snprintf(k, sizeof k, "%s.norm.bias", prefix); nb = req(m, k);
    snprintf(k, sizeof k, "%s.fc.gamma.weight", prefix); gw = req(m, k);
    snprintf(k, sizeof k, "%s.fc.gamma.bias", prefix); gb = req(m, k);
    snprintf(k, sizeof k, "%s.fc.beta.weight", prefix); bw = req(m, k);
    snprintf(k, sizeof k, "%s.fc.beta.bias", prefix); bb = req(m, k);
    if (!nw || !nb || !gw || !gb || !bw || !bb) return -1;
    if (nw->n != C || gw->ne[1] != C) return fail("adain shape mismatch: %s", prefix);
    float *gamma = fbuf((size_t)C), *beta = fbuf((size_t)C);
    linear_vec(gw, gb, style, gamma);
    linear_vec(bw, bb, style, beta);
    kko_norm_time(x, C, L, 1e-5f, y);
    for (int64_t c = 0; c < C; ++c) {
        const float w = nw->data[c], b = nb->data[c], g = gamma[c], be = beta[c];
        float *yc = y + c * L;
        for (int64_t t = 0; t < L; ++t) {
            float cur = yc[t] * w;
            cur = cur + b;
            cur = cur + cur * g;
            yc[t] = cur + be;
        }
    }
    free(gamma);
    free(beta);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* convolutions                                                             */
/* ------------------------------------------------------------------------ */

/* conv1d (graph_ops.cpp:728-767): y[oc][t] = sum_{ic,k} W[oc][ic*K+k] *
 * x[ic][t*s - p + k*d] with zero padding, then + bias.
 * ggml semantics: a 2D F32 weight takes im2col(F32) + mul_mat F32; an F16
 * weight, or one whose ne[0] == K (F0_conv / N_conv), takes ggml_conv_1d,
 * whose im2col is F16: the input and the weights are rounded to half and the
 * exact products are summed in F32. Sum order here: (ic, k) ascending. */
static int conv1d(const ko_tensor *w, const ko_tensor *b, const float *x, int64_t IC, int64_t L,
                  int s, int p, int d, int K, float *y, int64_t *OL_out) {
    /* 2D weights are ggml [IC*K, OC]; 3D ones [K, IC, OC] */
    const int64_t OC = w->ne[2] > 1 ? w->ne[2] : w->ne[1];
    if (w->n != OC * IC * K) {
        return fail("conv1d weight size mismatch: %s", w->name);
    }
    const int f16 = w->f16 || w->ne[0] == K;
    const int64_t OL = (L + 2 * p - (int64_t)d * (K - 1) - 1) / s + 1;
    *OL_out = OL;
    const float *xs = x;
    float *xr = NULL, *wr = NULL;
    const float *ws = w->data;
    if (f16) {
        xr = fbuf((size_t)(IC * L));
        round_f16_array(xr, x, (size_t)(IC * L));
        xs = xr;
        wr = fbuf((size_t)w->n);
        round_f16_array(wr, w->data, (size_t)w->n);
        ws = wr;
    }
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t oc = 0; oc < OC; ++oc) {
        float *yo = y + oc * OL;
        for (int64_t t = 0; t < OL; ++t) yo[t] = 0.f;
        for (int64_t ic = 0; ic < IC; ++ic) {
            const float *xi = xs + ic * L;
            for (int k = 0; k < K; ++k) {
                const float wv = ws[(oc * IC + ic) * K + k];
                const int64_t off = (int64_t)k * d - p;
                /* valid t: 0 <= t*s + off < L */
                int64_t t0 = 0;
                if (off < 0) t0 = (-off + s - 1) / s;
                int64_t t1 = OL;
                const int64_t lim = (L - 1 - off);
                if (lim < 0) continue;
                if (lim / s + 1 < t1) t1 = lim / s + 1;
                if (s == 1) {
                    const float *xp = xi + off;
                    for (int64_t t = t0; t < t1; ++t) yo[t] += wv * xp[t];
                } else {
                    for (int64_t t = t0; t < t1; ++t) yo[t] += wv * xi[t * s + off];
                }
            }
        }
        if (b) {
            const float bv = b->data[oc];
            for (int64_t t = 0; t < OL; ++t) yo[t] += bv;
        }
    }
    free(xr);
    free(wr);
    return 0;
}

/* conv_transpose1d_crop_bias (graph_ops.cpp:779-855) with ggml semantics of
 * ggml_conv_transpose_1d(W[K, OC, IC], x[L, IC], s, p0 = 0, d = 1): for each
 * output channel, t_in ascending, k ascending: full[t_in*s + k] +=
 * dot_ic(x[:, t_in], W[:, oc, k]). F16 kernels round the input to half.
 * Then the crop [crop_left, crop_left + out_len) and + bias. */
static int conv_transpose1d(const ko_tensor *w, const ko_tensor *b, const float *x, int64_t IC,
                            int64_t L, int s, int crop_left, int64_t out_len, float *y) {
    const int64_t K = w->ne[0], OC = w->ne[1];
    if (w->ne[2] != IC) return fail("conv_transpose1d IC mismatch: %s", w->name);
    const int64_t full_len = (L - 1) * s + K;
    if (crop_left + out_len > full_len) return fail("conv_transpose1d crop too long: %s", w->name);
    /* xT[t][ic] and wT[oc][k][ic] for contiguous dots */
    float *xT = fbuf((size_t)(L * IC));
    for (int64_t ic = 0; ic < IC; ++ic)
        for (int64_t t = 0; t < L; ++t) {
            const float v = x[ic * L + t];
            xT[t * IC + ic] = w->f16 ? kko_round_f16(v) : v;
        }
    float *wT = fbuf((size_t)(OC * K * IC));
    for (int64_t ic = 0; ic < IC; ++ic)
        for (int64_t oc = 0; oc < OC; ++oc)
            for (int64_t k = 0; k < K; ++k)
                wT[(oc * K + k) * IC + ic] = w->data[(ic * OC + oc) * K + k];
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t oc = 0; oc < OC; ++oc) {
        float *full = fbuf((size_t)full_len);
        for (int64_t t = 0; t < L; ++t) {
            const float *xt = xT + t * IC;
            for (int64_t k = 0; k < K; ++k) {
                const float *wk = wT + (oc * K + k) * IC;
                float v = 0.f;
                for (int64_t ic = 0; ic < IC; ++ic) v += xt[ic] * wk[ic];
                full[t * s + k] += v;
            }
        }
        const float bv = b->data[oc];
        for (int64_t t = 0; t < out_len; ++t) y[oc * out_len + t] = full[crop_left + t] + bv;
        free(full);
    }
    free(xT);
    free(wT);
    return 0;
}

/* depthwise_pool_upsample (audio_utils.cpp:73-114): the dense [3, C, C]
 * expansion of the depthwise kernel through the F32 conv_transpose path,
 * s = 2, crop 1, out 2L, + bias. Only the diagonal is non-zero, so each dot
 * is the single product w[c][k] * x[c][t_in]; contributions are added in
 * t_in order as in ggml. */
static int pool_upsample(kko_model *m, const char *prefix, const float *x, int64_t C, int64_t L,
                         float *y) {
    char k[256];
    snprintf(k, sizeof k, "%s.pool.weight", prefix);
    const ko_tensor *pw = req(m, k);
    snprintf(k, sizeof k, "%s.pool.bias", prefix);
    const ko_tensor *pb = req(m, k);
    if (!pw || !pb) return -1;
    const int64_t K = pw->ne[0];
    if (pw->ne[1] != 1 || pw->ne[2] != C || pb->ne[0] != C)
        return fail("invalid depthwise upsample pool shape: %s", prefix);
    const int64_t full_len = (L - 1) * 2 + K;
    const int64_t out_len = 2 * L;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t c = 0; c < C; ++c) {
        float *full = fbuf((size_t)full_len);
        for (int64_t t = 0; t < L; ++t)
            for (int64_t kk = 0; kk < K; ++kk) full[t * 2 + kk] += pw->data[c * K + kk] * x[c * L + t];
        for (int64_t t = 0; t < out_len; ++t) y[c * out_len + t] = full[1 + t] + pb->data[c];
        free(full);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* blocks                                                                   */
/* ------------------------------------------------------------------------ */

/* graph_generator_resblock (graph_ops.cpp:1071-1111, :1113-1208): three
 * iterations of AdaIN -> Snake -> conv(k, dilation d) -> AdaIN -> Snake ->
 * conv(k, d = 1) with a residual add. x is updated in place. */
static int generator_resblock(kko_model *m, const char *prefix, float *x, int64_t C, int64_t L,
                              const float *style, int K) {
    char key[256], pfx[256];
    float *cur = fbuf((size_t)(C * L)), *cur2 = fbuf((size_t)(C * L));
    int rc = 0;
    for (int i = 0; i < 3 && rc == 0; ++i) {
        const int d = KO_DIL[i];
        snprintf(pfx, sizeof pfx, "%s.adain1.%d", prefix, i);
        if ((rc = adain(m, pfx, x, C, L, style, cur)) != 0) break;
        snprintf(key, sizeof key, "%s.alpha1.%d", prefix, i);
        const ko_tensor *a1 = req(m, key);
        if (!a1) { rc = -1; break; }
        snake(cur, C, L, a1->data);
        snprintf(key, sizeof key, "%s.convs1.%d.weight", prefix, i);
        const ko_tensor *w1 = req(m, key);
        snprintf(key, sizeof key, "%s.convs1.%d.bias", prefix, i);
        const ko_tensor *b1 = req(m, key);
        if (!w1 || !b1) { rc = -1; break; }
        int64_t ol;
        if ((rc = conv1d(w1, b1, cur, C, L, 1, (K * d - d) / 2, d, K, cur2, &ol)) != 0) break;
        snprintf(pfx, sizeof pfx, "%s.adain2.%d", prefix, i);
        if ((rc = adain(m, pfx, cur2, C, L, style, cur)) != 0) break;
        snprintf(key, sizeof key, "%s.alpha2.%d", prefix, i);
        const ko_tensor *a2 = req(m, key);
        if (!a2) { rc = -1; break; }
        snake(cur, C, L, a2->data);
        snprintf(key, sizeof key, "%s.convs2.%d.weight", prefix, i);
        const ko_tensor *w2 = req(m, key);
        snprintf(key, sizeof key, "%s.convs2.%d.bias", prefix, i);
        const ko_tensor *b2 = req(m, key);
        if (!w2 || !b2) { rc = -1; break; }
        if ((rc = conv1d(w2, b2, cur, C, L, 1, K / 2, 1, K, cur2, &ol)) != 0) break;
        for (int64_t j = 0; j < C * L; ++j) x[j] = x[j] + cur2[j];
    }
    free(cur);
    free(cur2);
    return rc;
}

/* adain_resblk1d (graph_ops.cpp:996-1065). x [L, Cin] -> y [L', Cout],
 * L' = 2L when upsampling. */
static int adain_resblk(kko_model *m, const char *prefix, const float *x, int64_t Cin, int64_t L,
                        const float *style, int upsample, float *y, int64_t *Cout_out) {
    char key[256];
    snprintf(key, sizeof key, "%s.conv1.weight", prefix);
    const ko_tensor *c1w = req(m, key);
    snprintf(key, sizeof key, "%s.conv1.bias", prefix);
    const ko_tensor *c1b = req(m, key);
    snprintf(key, sizeof key, "%s.conv2.weight", prefix);
    const ko_tensor *c2w = req(m, key);
    snprintf(key, sizeof key, "%s.conv2.bias", prefix);
    const ko_tensor *c2b = req(m, key);
    if (!c1w || !c1b || !c2w || !c2b) return -1;
    snprintf(key, sizeof key, "%s.conv1x1.weight", prefix);
    const ko_tensor *sc = opt(m, key);
    const int64_t Cout = c1w->ne[1];
    const int64_t L2 = upsample ? 2 * L : L;
    *Cout_out = Cout;
    int rc;
    float *cur = fbuf((size_t)(Cin * L));
    snprintf(key, sizeof key, "%s.norm1", prefix);
    if ((rc = adain(m, key, x, Cin, L, style, cur)) != 0) goto out1;
    leaky_relu(cur, cur, (size_t)(Cin * L), 0.2f);
    float *up = cur;
    if (upsample) {
        up = fbuf((size_t)(Cin * L2));
        if ((rc = pool_upsample(m, prefix, cur, Cin, L, up)) != 0) { free(up); goto out1; }
    }
    float *h1 = fbuf((size_t)(Cout * L2)), *h2 = fbuf((size_t)(Cout * L2));
    int64_t ol;
    if ((rc = conv1d(c1w, c1b, up, Cin, L2, 1, 1, 1, 3, h1, &ol)) != 0) goto out2;
    snprintf(key, sizeof key, "%s.norm2", prefix);
    if ((rc = adain(m, key, h1, Cout, L2, style, h2)) != 0) goto out2;
    leaky_relu(h2, h2, (size_t)(Cout * L2), 0.2f);
    if ((rc = conv1d(c2w, c2b, h2, Cout, L2, 1, 1, 1, 3, h1, &ol)) != 0) goto out2;
    /* shortcut: nearest x2 upsample, then the bias-free 1x1 conv */
    {
        float *res = (float *)x;
        float *resbuf = NULL;
        if (upsample) {
            resbuf = fbuf((size_t)(Cin * L2));
            for (int64_t c = 0; c < Cin; ++c)
                for (int64_t t = 0; t < L2; ++t) resbuf[c * L2 + t] = x[c * L + t / 2];
            res = resbuf;
        }
        if (sc) {
            if ((rc = conv1d(sc, NULL, res, Cin, L2, 1, 0, 1, 1, y, &ol)) != 0) { free(resbuf); goto out2; }
        } else {
            if (Cin != Cout) { free(resbuf); rc = fail("missing conv1x1 for %s", prefix); goto out2; }
            memcpy(y, res, (size_t)(Cin * L2) * sizeof(float));
        }
        for (int64_t j = 0; j < Cout * L2; ++j) y[j] = (h1[j] + y[j]) * KO_INV_SQRT2;
        free(resbuf);
    }
out2:
    free(h1);
    free(h2);
    if (up != cur) free(up);
out1:
    free(cur);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* R1: harmonic source + forward STFT                                       */
/* ------------------------------------------------------------------------ */

/* hann_window_20 (audio_utils.cpp:36-45): the double expression rounded. */
static void hann20(float *w) {
    for (int n = 0; n < KO_STFT_N; ++n)
        w[n] = (float)(0.5 - 0.5 * cos(2.0 * M_PI * (double)n / (double)KO_STFT_N));
}

/* StftTwiddles (audio_utils.cpp:47-64): float angle from a double
 * expression, then float cos / sin. */
static void stft_twiddles(float c[KO_STFT_N][KO_BINS], float s[KO_STFT_N][KO_BINS]) {
    for (int n = 0; n < KO_STFT_N; ++n)
        for (int k = 0; k < KO_BINS; ++k) {
            const float a = (float)(2.0 * M_PI * (double)(float)(k * n) / (double)(float)KO_STFT_N);
            c[n][k] = cosf(a);
            s[n][k] = sinf(a);
        }
}

int kko_harmonic_stft(kko_model *m, const float *f0, int64_t n_f0, int64_t target_frames,
                      float *har, float *source_out) {
    const ko_tensor *mw_t = req(m, "kokopop.decoder.generator.m_source.l_linear.weight");
    const ko_tensor *mb_t = req(m, "kokopop.decoder.generator.m_source.l_linear.bias");
    if (!mw_t || !mb_t) return -1;
    if (mw_t->n < KO_HARMONICS) return fail("invalid harmonic source merge weight size%s", "");
    const float mb = mb_t->data[0];
    const float *mw = mw_t->data;
    const int64_t n_samples = n_f0 * KO_UPSAMPLE;
    float (*f_tanh)(float) = m->source_libm ? tanhf : cr_tanhf;
    float (*f_sin)(float) = m->source_libm ? sinf : cr_sinf;
    float (*f_cos)(float) = m->source_libm ? cosf : cr_cosf;
    float *source = fbuf((size_t)n_samples);

    /* scalar path of audio_utils.cpp:318-353 */
    float phase_sin[KO_HARMONICS], phase_cos[KO_HARMONICS];
    for (int h = 0; h < KO_HARMONICS; ++h) {
        phase_sin[h] = 0.f;
        phase_cos[h] = 1.f;
    }
    for (int64_t seg = 0; seg < n_f0; ++seg) {
        const int64_t seg_start = seg * KO_UPSAMPLE;
        const float base_f0 = f0[seg];
        if (base_f0 > 10.0f) {
            float sin_delta[KO_HARMONICS], cos_delta[KO_HARMONICS], mw_scaled[KO_HARMONICS];
            for (int h = 0; h < KO_HARMONICS; ++h) {
                const float delta = (float)(2.0 * M_PI * (double)base_f0 * (double)(float)(h + 1) /
                                            (double)(float)KO_SAMPLE_RATE);
                sin_delta[h] = f_sin(delta);
                cos_delta[h] = f_cos(delta);
                mw_scaled[h] = mw[h] * KO_SINE_AMP;
            }
            for (int64_t j = 0; j < KO_UPSAMPLE; ++j) {
                float merged = mb;
                for (int h = 0; h < KO_HARMONICS; ++h) {
                    const float sv = phase_sin[h], cv = phase_cos[h];
                    const float ns = sv * cos_delta[h] + cv * sin_delta[h];
                    const float nc = cv * cos_delta[h] - sv * sin_delta[h];
                    phase_sin[h] = ns;
                    phase_cos[h] = nc;
                    merged += mw_scaled[h] * ns;
                }
                source[seg_start + j] = f_tanh(merged);
            }
            if ((seg + 1) % 16 == 0) {
                for (int h = 0; h < KO_HARMONICS; ++h) {
                    const float norm = sqrtf(phase_sin[h] * phase_sin[h] + phase_cos[h] * phase_cos[h]);
                    if (norm > 0.0f) {
                        phase_sin[h] /= norm;
                        phase_cos[h] /= norm;
                    }
                }
            }
        } else {
            const float unvoiced = f_tanh(mb);
            for (int64_t j = 0; j < KO_UPSAMPLE; ++j) source[seg_start + j] = unvoiced;
        }
    }
    if (source_out) memcpy(source_out, source, (size_t)n_samples * sizeof(float));

    /* forward DFT, audio_utils.cpp:381-419 */
    float win[KO_STFT_N];
    hann20(win);
    float tc[KO_STFT_N][KO_BINS], ts[KO_STFT_N][KO_BINS];
    stft_twiddles(tc, ts);
    const int64_t center_pad = KO_STFT_N / 2;
#pragma omp parallel for schedule(static)
    for (int64_t frame = 0; frame < target_frames; ++frame) {
        float ws[KO_STFT_N];
        for (int n = 0; n < KO_STFT_N; ++n) ws[n] = 0.f;
        const int64_t first = frame * KO_STFT_HOP - center_pad;
        if (first >= 0 && first + KO_STFT_N <= n_samples) {
            for (int n = 0; n < KO_STFT_N; ++n) ws[n] = source[first + n] * win[n];
        } else {
            for (int n = 0; n < KO_STFT_N; ++n) {
                int64_t src_i = first + n;
                if (src_i < 0) src_i = -src_i - 1;
                else if (src_i >= n_samples) src_i = 2 * n_samples - src_i - 1;
                if (src_i >= 0 && src_i < n_samples) ws[n] = source[src_i] * win[n];
            }
        }
        float re[KO_BINS], im[KO_BINS];
        for (int k = 0; k < KO_BINS; ++k) re[k] = im[k] = 0.f;
        for (int n = 0; n < KO_STFT_N; ++n) {
            const float w = ws[n];
            for (int k = 0; k < KO_BINS; ++k) {
                re[k] += w * tc[n][k];
                im[k] -= w * ts[n][k];
            }
        }
        for (int k = 0; k < KO_BINS; ++k) {
            har[k * target_frames + frame] = sqrtf(re[k] * re[k] + im[k] * im[k]);
            har[(k + KO_STFT_N / 2 + 1) * target_frames + frame] = atan2f(im[k], re[k]);
        }
    }
    free(source);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* R9: iSTFT                                                                */
/* ------------------------------------------------------------------------ */

/* cpu_istft_data (audio_utils.cpp:462-532) + istft DirectDft path
 * (src/audio/istft.cpp:192-313 plan, :334-523 transform, istft_kernels.h
 * scalar kernels). */
int kko_istft(const float *post, int64_t n_frames, float *audio, int64_t *n_out) {
    const int n = KO_STFT_N, hop = KO_STFT_HOP, bins = KO_BINS, half = KO_STFT_N / 2;
    if (n_frames <= 1) {
        if (n_out) *n_out = 0;
        return 0;
    }
    const int64_t padded = (int64_t)hop * (n_frames - 1) + n;
    const int64_t out_len = padded - n;
    float window[KO_STFT_N], window_sq[KO_STFT_N];
    for (int i = 0; i < n; ++i) {
        window[i] = (float)(0.5 - 0.5 * cos(2.0 * M_PI * (double)i / (double)n));
        window_sq[i] = window[i] * window[i];
    }
    float dft_cos[KO_BINS][KO_STFT_N], dft_sin[KO_BINS][KO_STFT_N];
    for (int k = 0; k < bins; ++k)
        for (int i = 0; i < n; ++i) {
            const float a = (float)(2.0 * M_PI * (double)(k * i) / (double)n);
            dft_cos[k][i] = cosf(a);
            dft_sin[k][i] = sinf(a);
        }
    float *ola = fbuf((size_t)padded), *env = fbuf((size_t)padded);
    const float inv_n = 1.0f / (float)n;
    for (int64_t f = 0; f < n_frames; ++f) {
        float re[KO_BINS], im[KO_BINS];
        for (int k = 0; k < bins; ++k) {
            float v = post[k * n_frames + f];
            v = v < -20.0f ? -20.0f : (v > 8.0f ? 8.0f : v);
            const float mag = expf(v);
            const float phase = sinf(post[(k + half + 1) * n_frames + f]);
            re[k] = mag * cosf(phase);
            im[k] = mag * sinf(phase);
        }
        float frame[KO_STFT_N];
        const float dc = re[0], nyq = re[bins - 1];
        for (int i = 0; i < n; i += 2) {
            frame[i] = dc + nyq;
            frame[i + 1] = dc - nyq;
        }
        for (int k = 1; k < half; ++k) {
            const float cr = 2.0f * re[k], ci = 2.0f * im[k];
            for (int i = 0; i < n; ++i) frame[i] += cr * dft_cos[k][i] - ci * dft_sin[k][i];
        }
        for (int i = 0; i < n; ++i) frame[i] = (frame[i] * inv_n) * window[i];
        const int64_t base = (int64_t)hop * f;
        for (int i = 0; i < n; ++i) {
            ola[base + i] += frame[i];
            env[base + i] += window_sq[i];
        }
    }
    const int64_t trim = n / 2;
    for (int64_t j = 0; j < out_len; ++j) {
        const float e = env[trim + j];
        float v = e > 1e-8f ? ola[trim + j] / e : 0.0f;
        v = v < -1.0f ? -1.0f : (v > 1.0f ? 1.0f : v);
        audio[j] = v;
    }
    free(ola);
    free(env);
    if (n_out) *n_out = out_len;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* R10: generator                                                           */
/* ------------------------------------------------------------------------ */

int kko_generator(kko_model *m, int64_t L, const float *decoder, const float *f0,
                  const float *style, float *audio, float *post_out) {
    g_err[0] = 0;
    const int64_t har_len = L * 60 + 1;
    float *har = fbuf((size_t)(22 * har_len));
    if (kko_harmonic_stft(m, f0, L, har_len, har, NULL) != 0) {
        free(har);
        return -1;
    }
    tap(m, "har", har, har_len, 22);

    /* stage table of audio_utils.cpp:651-664 */
    static const struct {
        int kernel, up_stride, up_padding, noise_stride, noise_padding, noise_kernel;
    } sp[2] = {{7, 10, 5, 6, 3, 12}, {11, 6, 3, 1, 0, 1}};

    int64_t C = 512, T = L;
    float *x = fbuf((size_t)(C * T));
    memcpy(x, decoder, (size_t)(C * T) * sizeof(float));
    int rc = 0;
    char key[256], name[64];
    for (int st = 0; st < 2 && rc == 0; ++st) {
        leaky_relu(x, x, (size_t)(C * T), 0.1f);
        /* noise branch */
        snprintf(key, sizeof key, "kokopop.decoder.generator.noise_convs.%d.weight", st);
        const ko_tensor *ncw = req(m, key);
        snprintf(key, sizeof key, "kokopop.decoder.generator.noise_convs.%d.bias", st);
        const ko_tensor *ncb = req(m, key);
        snprintf(key, sizeof key, "kokopop.decoder.generator.ups.%d.weight", st);
        const ko_tensor *uw = req(m, key);
        snprintf(key, sizeof key, "kokopop.decoder.generator.ups.%d.bias", st);
        const ko_tensor *ub = req(m, key);
        if (!ncw || !ncb || !uw || !ub) { rc = -1; break; }
        const int64_t Cn = ncw->ne[1];
        const int64_t nl = (har_len + 2 * sp[st].noise_padding - sp[st].noise_kernel) / sp[st].noise_stride + 1;
        float *xs = fbuf((size_t)(Cn * nl));
        int64_t ol;
        if ((rc = conv1d(ncw, ncb, har, 22, har_len, sp[st].noise_stride, sp[st].noise_padding, 1,
                         sp[st].noise_kernel, xs, &ol)) != 0) { free(xs); break; }
        snprintf(name, sizeof name, "noise_conv%d", st);
        tap(m, name, xs, nl, Cn);
        snprintf(key, sizeof key, "kokopop.decoder.generator.noise_res.%d", st);
        if ((rc = generator_resblock(m, key, xs, Cn, nl, style, sp[st].kernel)) != 0) { free(xs); break; }
        snprintf(name, sizeof name, "noise_res%d", st);
        tap(m, name, xs, nl, Cn);
        /* upsample */
        const int64_t Cu = uw->ne[1];
        const int64_t out_len = (T - 1) * sp[st].up_stride - 2 * sp[st].up_padding + uw->ne[0];
        const int64_t T2 = out_len + (st == 1 ? 1 : 0);
        float *u = fbuf((size_t)(Cu * T2));
        float *ut = st == 1 ? fbuf((size_t)(Cu * out_len)) : u;
        if ((rc = conv_transpose1d(uw, ub, x, C, T, sp[st].up_stride, sp[st].up_padding, out_len, ut)) != 0) {
            free(xs); free(u); if (ut != u) free(ut); break;
        }
        snprintf(name, sizeof name, "ups%d", st);
        tap(m, name, ut, out_len, Cu);
        if (st == 1) { /* ggml_pad_reflect_1d(x, 1, 0) */
            for (int64_t c = 0; c < Cu; ++c) {
                memcpy(u + c * T2 + 1, ut + c * out_len, (size_t)out_len * sizeof(float));
                u[c * T2] = ut[c * out_len + 1];
            }
            free(ut);
        }
        if (T2 != nl || Cu != Cn) { free(xs); free(u); rc = fail("stage length mismatch%s", ""); break; }
        for (int64_t j = 0; j < Cu * T2; ++j) u[j] = u[j] + xs[j];
        free(xs);
        snprintf(name, sizeof name, "pre_rb%d", st);
        tap(m, name, u, T2, Cu);
        /* graph_3branch_main_sum (graph_ops.cpp:1300-1320) */
        float *acc = fbuf((size_t)(Cu * T2)), *br = fbuf((size_t)(Cu * T2));
        for (int k = 0; k < 3 && rc == 0; ++k) {
            memcpy(br, u, (size_t)(Cu * T2) * sizeof(float));
            snprintf(key, sizeof key, "kokopop.decoder.generator.resblocks.%d", st * 3 + k);
            rc = generator_resblock(m, key, br, Cu, T2, style, KO_KS[k]);
            if (k == 0) memcpy(acc, br, (size_t)(Cu * T2) * sizeof(float));
            else for (int64_t j = 0; j < Cu * T2; ++j) acc[j] = acc[j] + br[j];
        }
        const float third = 1.0f / 3.0f;
        for (int64_t j = 0; j < Cu * T2; ++j) acc[j] *= third;
        free(br);
        free(u);
        free(x);
        x = acc;
        C = Cu;
        T = T2;
        snprintf(name, sizeof name, "stage%d", st);
        tap(m, name, x, T, C);
    }
    if (rc == 0) {
        leaky_relu(x, x, (size_t)(C * T), 0.01f);
        const ko_tensor *pw = req(m, "kokopop.decoder.generator.conv_post.weight");
        const ko_tensor *pb = req(m, "kokopop.decoder.generator.conv_post.bias");
        if (!pw || !pb) rc = -1;
        else {
            float *post = fbuf((size_t)(22 * T));
            int64_t ol;
            rc = conv1d(pw, pb, x, C, T, 1, 3, 1, 7, post, &ol);
            if (rc == 0) {
                tap(m, "post", post, T, 22);
                if (post_out) memcpy(post_out, post, (size_t)(22 * T) * sizeof(float));
                int64_t n_out = 0;
                rc = kko_istft(post, T, audio, &n_out);
            }
            free(post);
        }
    }
    free(x);
    free(har);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* R6: decoder                                                              */
/* ------------------------------------------------------------------------ */

int kko_decoder(kko_model *m, int64_t T, const float *asr, const float *f0, const float *noise,
                const float *style, float *decoder_out) {
    g_err[0] = 0;
    const ko_tensor *f0w = req(m, "kokopop.decoder.F0_conv.weight");
    const ko_tensor *f0b = req(m, "kokopop.decoder.F0_conv.bias");
    const ko_tensor *nw = req(m, "kokopop.decoder.N_conv.weight");
    const ko_tensor *nb = req(m, "kokopop.decoder.N_conv.bias");
    const ko_tensor *arw = req(m, "kokopop.decoder.asr_res.0.weight");
    const ko_tensor *arb = req(m, "kokopop.decoder.asr_res.0.bias");
    if (!f0w || !f0b || !nw || !nb || !arw || !arb) return -1;
    int64_t ol;
    float *f0d = fbuf((size_t)T), *nd = fbuf((size_t)T);
    /* conv1d(w, x, stride 2, pad 1, dil 1, k 3): 2T -> T */
    int rc = conv1d(f0w, f0b, f0, 1, 2 * T, 2, 1, 1, 3, f0d, &ol);
    if (rc == 0 && ol != T) rc = fail("F0_conv length mismatch%s", "");
    if (rc == 0) rc = conv1d(nw, nb, noise, 1, 2 * T, 2, 1, 1, 3, nd, &ol);
    float *asr_res = fbuf((size_t)(64 * T));
    if (rc == 0) rc = conv1d(arw, arb, asr, 512, T, 1, 0, 1, 1, asr_res, &ol);
    /* concat [asr, f0, n] -> 514 channels */
    float *x = fbuf((size_t)(1090 * 2 * T));
    float *y = fbuf((size_t)(1024 * 2 * T));
    int64_t C = 514, L = T;
    if (rc == 0) {
        memcpy(x, asr, (size_t)(512 * T) * sizeof(float));
        memcpy(x + 512 * T, f0d, (size_t)T * sizeof(float));
        memcpy(x + 513 * T, nd, (size_t)T * sizeof(float));
        tap(m, "f0_dec", f0d, T, 1);
        tap(m, "asr_res", asr_res, T, 64);
        rc = adain_resblk(m, "kokopop.decoder.encode", x, C, L, style, 0, y, &C);
        if (rc == 0) tap(m, "encode", y, L, C);
    }
    for (int i = 0; i < 4 && rc == 0; ++i) {
        /* concat [x, asr_res, f0, n] -> 1090 channels */
        memcpy(x, y, (size_t)(C * L) * sizeof(float));
        memcpy(x + C * L, asr_res, (size_t)(64 * L) * sizeof(float));
        memcpy(x + (C + 64) * L, f0d, (size_t)L * sizeof(float));
        memcpy(x + (C + 65) * L, nd, (size_t)L * sizeof(float));
        char pfx[64];
        snprintf(pfx, sizeof pfx, "kokopop.decoder.decode.%d", i);
        const int up = i == 3;
        rc = adain_resblk(m, pfx, x, C + 66, L, style, up, y, &C);
        if (up) L *= 2;
        char name[32];
        snprintf(name, sizeof name, "decode%d", i);
        if (rc == 0) tap(m, name, y, L, C);
    }
    if (rc == 0) memcpy(decoder_out, y, (size_t)(C * L) * sizeof(float));
    free(f0d);
    free(nd);
    free(asr_res);
    free(x);
    free(y);
    return rc;
}

int kko_decoder_forward(kko_model *m, int64_t T, const float *asr, const float *f0,
                        const float *noise, const float *style, float *audio) {
    float *dec = fbuf((size_t)(512 * 2 * T));
    int rc = kko_decoder(m, T, asr, f0, noise, style, dec);
    if (rc == 0) rc = kko_generator(m, 2 * T, dec, f0, style, audio, NULL);
    free(dec);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* R7 / R8: LSTM                                                            */
/* ------------------------------------------------------------------------ */

static float sigmoidf_stable(float x) {
    if (x >= 0.0f) {
        const float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    const float z = expf(x);
    return z / (1.0f + z);
}

static float sanitize_gate(float x) {
    if (!isfinite(x)) return 0.0f;
    if (x > 80.0f) return 80.0f;
    if (x < -80.0f) return -80.0f;
    return x;
}

static float clamp_cell(float x) {
    if (!isfinite(x)) return 0.0f;
    if (x > 50.0f) return 50.0f;
    if (x < -50.0f) return -50.0f;
    return x;
}

/* cpu_lstm_contiguous (lstm_fused.cpp:200-247) with the scalar dot
 * (lstm_fused.cpp:165-175). */
void kko_lstm_direction(const float *pre, const float *w, const float *b_hh, int64_t H, int64_t N,
                        int reverse, float *out) {
    const int64_t H4 = 4 * H;
    float *h = fbuf((size_t)H), *c = fbuf((size_t)H), *g = fbuf((size_t)H4);
    for (int64_t step = 0; step < N; ++step) {
        const int64_t t = reverse ? (N - 1 - step) : step;
        const float *pg = pre + H4 * t;
        for (int64_t j = 0; j < H4; ++j) {
            float dot = 0.0f;
            const float *wr = w + j * H;
            for (int64_t k = 0; k < H; ++k) dot += wr[k] * h[k];
            g[j] = b_hh[j] + pg[j] + dot;
        }
        float *ot = out + H * t;
        for (int64_t i = 0; i < H; ++i) {
            const float xi = sanitize_gate(g[i]);
            const float xf = sanitize_gate(g[H + i]);
            const float xg = sanitize_gate(g[2 * H + i]);
            const float xo = sanitize_gate(g[3 * H + i]);
            const float ig = sigmoidf_stable(xi);
            const float fg = sigmoidf_stable(xf);
            const float gg = tanhf(xg);
            const float og = sigmoidf_stable(xo);
            const float cn = clamp_cell(fg * c[i] + ig * gg);
            c[i] = cn;
            const float hn = og * tanhf(cn);
            h[i] = isfinite(hn) ? hn : 0.0f;
            ot[i] = h[i];
        }
    }
    free(h);
    free(c);
    free(g);
}

/* lstm_direction (graph_ops.cpp:1439-1512): pre = W_ih x + b_ih via ggml
 * mul_mat (x rounded to half for an F16 W_ih), then the recurrence. */
static int lstm_dir(kko_model *m, const char *prefix, int reverse, int64_t N, int64_t in_dim,
                    const float *x, float *out) {
    char k[256];
    const char *sfx = reverse ? "_reverse" : "";
    snprintf(k, sizeof k, "%s.weight_ih_l0%s", prefix, sfx);
    const ko_tensor *wih = req(m, k);
    snprintf(k, sizeof k, "%s.weight_hh_l0%s", prefix, sfx);
    const ko_tensor *whh = req(m, k);
    snprintf(k, sizeof k, "%s.bias_ih_l0%s", prefix, sfx);
    const ko_tensor *bih = req(m, k);
    snprintf(k, sizeof k, "%s.bias_hh_l0%s", prefix, sfx);
    const ko_tensor *bhh = req(m, k);
    if (!wih || !whh || !bih || !bhh) return -1;
    const int64_t H = whh->ne[0], H4 = whh->ne[1];
    if (H4 != 4 * H || wih->ne[0] != in_dim || wih->ne[1] != H4)
        return fail("invalid packed LSTM shapes: %s", prefix);
    float *xr = fbuf((size_t)(N * in_dim));
    if (wih->f16) round_f16_array(xr, x, (size_t)(N * in_dim));
    else memcpy(xr, x, (size_t)(N * in_dim) * sizeof(float));
    float *pre = fbuf((size_t)(N * H4));
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < N; ++t) {
        const float *xt = xr + t * in_dim;
        for (int64_t j = 0; j < H4; ++j) {
            const float *wr = wih->data + j * in_dim;
            float acc = 0.f;
            for (int64_t i = 0; i < in_dim; ++i) acc += wr[i] * xt[i];
            pre[t * H4 + j] = acc + bih->data[j];
        }
    }
    /* w_hh is ggml [H, 4H]: w[k + H * j] is already the rowwise layout */
    kko_lstm_direction(pre, whh->data, bhh->data, H, N, reverse, out);
    free(xr);
    free(pre);
    return 0;
}

int kko_bilstm(kko_model *m, const char *prefix, int64_t N, int64_t in_dim, const float *x,
               float *out) {
    g_err[0] = 0;
    char k[256];
    snprintf(k, sizeof k, "%s.weight_hh_l0", prefix);
    const ko_tensor *whh = req(m, k);
    if (!whh) return -1;
    const int64_t H = whh->ne[0];
    float *fw = fbuf((size_t)(N * H)), *bw = fbuf((size_t)(N * H));
    int rc = lstm_dir(m, prefix, 0, N, in_dim, x, fw);
    if (rc == 0) rc = lstm_dir(m, prefix, 1, N, in_dim, x, bw);
    if (rc == 0) {
        for (int64_t t = 0; t < N; ++t) {
            memcpy(out + t * 2 * H, fw + t * H, (size_t)H * sizeof(float));
            memcpy(out + t * 2 * H + H, bw + t * H, (size_t)H * sizeof(float));
        }
    }
    free(fw);
    free(bw);
    return rc;
}

/* The prosody predictor's F0 / N chain (kokoro.cpp:669-708): the biLSTM
 * kokopop.predictor.shared over the frames (cur = [2H, T] after the
 * transpose), then per branch three adain_resblk1d
 * kokopop.predictor.{F0,N}.{0,1,2} (the second with the x2 upsample), the
 * 1x1 conv {F0,N}_proj and its channel bias (add_channel_bias), viewed as a
 * 1-D curve of 2T values. */
int kko_prosody_f0n(kko_model *m, int64_t T, const float *en, const float *style, float *f0,
                    float *nout) {
    g_err[0] = 0;
    const ko_tensor *whh = req(m, "kokopop.predictor.shared.weight_hh_l0");
    if (!whh) return -1;
    const int64_t H2 = 2 * whh->ne[0];
    float *h = fbuf((size_t)(T * H2));
    int rc = kko_bilstm(m, "kokopop.predictor.shared", T, 640, en, h);
    if (rc != 0) {
        free(h);
        return rc;
    }
    float *x = fbuf((size_t)(H2 * T));
    for (int64_t t = 0; t < T; ++t)
        for (int64_t c = 0; c < H2; ++c) x[c * T + t] = h[t * H2 + c];
    free(h);
    for (int br = 0; br < 2 && rc == 0; ++br) {
        const char *name = br ? "N" : "F0";
        const float *cur = x;
        int64_t C = H2, L = T;
        float *bufs[3] = {NULL, NULL, NULL};
        char key[256];
        for (int i = 0; i < 3 && rc == 0; ++i) {
            char pfx[128];
            snprintf(pfx, sizeof pfx, "kokopop.predictor.%s.%d", name, i);
            snprintf(key, sizeof key, "%s.conv1.weight", pfx);
            const ko_tensor *c1w = req(m, key);
            if (!c1w) {
                rc = -1;
                break;
            }
            const int64_t L2 = i == 1 ? 2 * L : L;
            bufs[i] = fbuf((size_t)(c1w->ne[1] * L2));
            rc = adain_resblk(m, pfx, cur, C, L, style, i == 1, bufs[i], &C);
            L = L2;
            cur = bufs[i];
        }
        if (rc == 0) {
            snprintf(key, sizeof key, "kokopop.predictor.%s_proj.weight", name);
            const ko_tensor *pw = req(m, key);
            snprintf(key, sizeof key, "kokopop.predictor.%s_proj.bias", name);
            const ko_tensor *pb = req(m, key);
            int64_t ol;
            rc = (pw && pb) ? conv1d(pw, pb, cur, C, L, 1, 0, 1, 1, br ? nout : f0, &ol) : -1;
        }
        for (int i = 0; i < 3; ++i) free(bufs[i]);
    }
    free(x);
    return rc;
}

/* ada_layer_norm (graph_ops.cpp:865-886): ggml_norm over features per step,
 * then (normed + normed * gamma) + beta. */
static int ada_layer_norm(kko_model *m, const char *prefix, float *x, int64_t D, int64_t N,
                          const float *style) {
    char k[256];
    const ko_tensor *gw, *gb, *bw, *bb;
    snprintf(k, sizeof k, "%s.fc.gamma.weight", prefix); gw = req(m, k);
    snprintf(k, sizeof k, "%s.fc.gamma.bias", prefix); gb = req(m, k);
    snprintf(k, sizeof k, "%s.fc.beta.weight", prefix); bw = req(m, k);
    snprintf(k, sizeof k, "%s.fc.beta.bias", prefix); bb = req(m, k);
    if (!gw || !gb || !bw || !bb) return -1;
    float *gamma = fbuf((size_t)D), *beta = fbuf((size_t)D);
    linear_vec(gw, gb, style, gamma);
    linear_vec(bw, bb, style, beta);
    float *y = fbuf((size_t)D);
    for (int64_t t = 0; t < N; ++t) {
        kko_norm_time(x + t * D, 1, D, 1e-5f, y);
        for (int64_t j = 0; j < D; ++j) {
            const float v = y[j];
            x[t * D + j] = (v + v * gamma[j]) + beta[j];
        }
    }
    free(y);
    free(gamma);
    free(beta);
    return 0;
}

int kko_duration_encoder(kko_model *m, int64_t N, const float *x, const float *style, float *out) {
    g_err[0] = 0;
    const int64_t D = 640;
    float *cur = fbuf((size_t)(N * D)), *h = fbuf((size_t)(N * 512));
    for (int64_t t = 0; t < N; ++t) {
        memcpy(cur + t * D, x + t * 512, 512 * sizeof(float));
        memcpy(cur + t * D + 512, style, 128 * sizeof(float));
    }
    int rc = 0;
    for (int blk = 0; blk < 3 && rc == 0; ++blk) {
        char pfx[128];
        snprintf(pfx, sizeof pfx, "kokopop.predictor.text_encoder.lstms.%d", blk * 2);
        rc = kko_bilstm(m, pfx, N, D, cur, h);
        if (rc) break;
        snprintf(pfx, sizeof pfx, "kokopop.predictor.text_encoder.lstms.%d", blk * 2 + 1);
        rc = ada_layer_norm(m, pfx, h, 512, N, style);
        if (rc) break;
        for (int64_t t = 0; t < N; ++t) {
            memcpy(cur + t * D, h + t * 512, 512 * sizeof(float));
            memcpy(cur + t * D + 512, style, 128 * sizeof(float));
        }
    }
    if (rc == 0) memcpy(out, cur, (size_t)(N * D) * sizeof(float));
    free(cur);
    free(h);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* R11: durations -> frames and the alignment                               */
/* ------------------------------------------------------------------------ */

/* duration_to_frames (kokoro.cpp:181-193). */
/* text_encoder (graph_ops.cpp:1578-1624): ggml_get_rows of the embedding
 * [C, vocab] (ne[0] = C) -> [C, N]; three times: the transpose to [N, C]
 * time-fastest, conv1d_chfirst k = 5, pad 2 (the conv1d arithmetic: F16
 * weights round the input to half) + the channel bias, then per token
 * ggml_norm over the C channels (eps 1e-5), * gamma, + beta, LeakyReLU 0.2;
 * then the biLSTM over the N tokens. */
int kko_text_encoder(kko_model *m, int64_t N, const int32_t *ids, float *out) {
    g_err[0] = 0;
    const ko_tensor *emb = req(m, "kokopop.text_encoder.embedding.weight");
    if (!emb) return -1;
    const int64_t C = emb->ne[0], V = emb->ne[1];
    if (N < 1) return fail("text encoder needs at least one token%s", "");
    for (int64_t t = 0; t < N; ++t)
        if (ids[t] < 0 || ids[t] >= V) return fail("token id out of range%s", "");
    float *x = fbuf((size_t)(C * N)), *y = fbuf((size_t)(C * N));
    float *tok = fbuf((size_t)C), *nrm = fbuf((size_t)C);
    int rc = 0;
    /* x [N, C] time-fastest: x[c * N + t] */
    for (int64_t t = 0; t < N; ++t)
        for (int64_t c = 0; c < C; ++c) x[c * N + t] = emb->data[(int64_t)ids[t] * C + c];
    for (int i = 0; i < 3 && rc == 0; ++i) {
        char k[256];
        const ko_tensor *w, *b, *g, *be;
        snprintf(k, sizeof k, "kokopop.text_encoder.cnn.%d.0.weight", i);
        w = req(m, k);
        snprintf(k, sizeof k, "kokopop.text_encoder.cnn.%d.0.bias", i);
        b = req(m, k);
        snprintf(k, sizeof k, "kokopop.text_encoder.cnn.%d.1.gamma", i);
        g = req(m, k);
        snprintf(k, sizeof k, "kokopop.text_encoder.cnn.%d.1.beta", i);
        be = req(m, k);
        if (!w || !b || !g || !be) {
            rc = -1;
            break;
        }
        int64_t OL = 0;
        rc = conv1d(w, b, x, C, N, 1, 2, 1, 5, y, &OL);
        if (rc == 0 && (OL != N || (w->ne[2] > 1 ? w->ne[2] : w->ne[1]) != C))
            rc = fail("text encoder conv shape mismatch: %s", w->name);
        if (rc != 0) break;
        for (int64_t t = 0; t < N; ++t) {
            for (int64_t c = 0; c < C; ++c) tok[c] = y[c * N + t];
            kko_norm_time(tok, 1, C, 1e-5f, nrm);
            for (int64_t c = 0; c < C; ++c) {
                float v = nrm[c] * g->data[c];
                v = v + be->data[c];
                tok[c] = v;
            }
            leaky_relu(tok, tok, (size_t)C, 0.2f);
            for (int64_t c = 0; c < C; ++c) x[c * N + t] = tok[c];
        }
    }
    if (rc == 0) {
        /* the biLSTM reads [N, C] feature-fastest */
        for (int64_t t = 0; t < N; ++t)
            for (int64_t c = 0; c < C; ++c) y[t * C + c] = x[c * N + t];
        rc = kko_bilstm(m, "kokopop.text_encoder.lstm", N, C, y, out);
    }
    free(x);
    free(y);
    free(tok);
    free(nrm);
    return rc;
}

/* The duration projection and bucket sum (kokoro.cpp:469-516), on the host in
 * double: per token and bucket n, acc = b[n] + sum over k ascending of
 * w[n][k] * h[k] (separate double multiply and add), x = (float)acc, then the
 * logistic function in double by the branch that avoids overflow, summed over
 * n ascending; the duration is (float)sum. */
int kko_duration_proj(kko_model *m, int64_t N, const float *h, float *durations) {
    g_err[0] = 0;
    const ko_tensor *w = req(m, "kokopop.predictor.duration_proj.linear_layer.weight");
    const ko_tensor *b = req(m, "kokopop.predictor.duration_proj.linear_layer.bias");
    if (!w || !b) return -1;
    const int64_t P = w->ne[0], NB = w->ne[1];
    for (int64_t t = 0; t < N; ++t) {
        const float *ht = h + t * P;
        double sum = 0.0;
        for (int64_t n = 0; n < NB; ++n) {
            const float *wr = w->data + n * P;
            double acc = (double)b->data[n];
            for (int64_t k = 0; k < P; ++k) acc += (double)wr[k] * (double)ht[k];
            const double x = (double)(float)acc;
            sum += x >= 0.0 ? 1.0 / (1.0 + exp(-x)) : exp(x) / (1.0 + exp(x));
        }
        durations[t] = (float)sum;
    }
    return 0;
}

/* predictor.lstm over the duration encoder output, then the projection. */
int kko_duration_head(kko_model *m, int64_t N, const float *d, float *durations) {
    g_err[0] = 0;
    const ko_tensor *w = req(m, "kokopop.predictor.duration_proj.linear_layer.weight");
    if (!w) return -1;
    float *h = fbuf((size_t)(N * w->ne[0]));
    int rc = kko_bilstm(m, "kokopop.predictor.lstm", N, 640, d, h);
    if (rc == 0) rc = kko_duration_proj(m, N, h, durations);
    free(h);
    return rc;
}

/* ---- ALBERT (kokoro.cpp:279-337) ---- */

/* layer_norm (graph_ops.cpp:622-634): ggml_norm over the D features of each
 * of the N rows of x [N, D] (feature-fastest), * w, + b, in place. */
static void layer_norm_rows(float *x, int64_t N, int64_t D, const ko_tensor *w, const ko_tensor *b, float eps) {
    float *y = fbuf((size_t)D);
    for (int64_t t = 0; t < N; ++t) {
        float *r = x + t * D;
        kko_norm_time(r, 1, D, eps, y);
        for (int64_t c = 0; c < D; ++c) {
            float v = y[c] * w->data[c];
            r[c] = v + b->data[c];
        }
    }
    free(y);
}

/* ggml semantics, ggml_gelu on F32 (ggml-cpu, GGML_GELU_FP16): 0 for
 * x <= -10, x for x >= 10, else the F16 table entry of half(x): the tanh
 * approximation 0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x^2))) of the
 * half value, rounded to half. tanh is taken correctly rounded here (ggml's
 * table holds the build machine's tanhf; the two differ at most in the
 * table's last bit for a few entries). */
static float gelu_ggml(float x) {
    if (x <= -10.0f) return 0.0f;
    if (x >= 10.0f) return x;
    const float h = kko_round_f16(x);
    const float a = 0.79788456080286535587989211986876f * h;
    const float inner = a * (1.0f + (0.044715f * h) * h);
    const float g = (0.5f * h) * (1.0f + cr_tanhf(inner));
    return kko_round_f16(g);
}

/* ggml semantics, ggml_soft_max_ext(x, NULL, scale, 0) on one row of n:
 * w = x * scale, m = max w, e = exp(w - m) with the sum in double, then
 * e * (float)(1 / sum). exp is taken correctly rounded (ggml's CPU path uses
 * its own vectorised exp approximation). */
static void softmax_row(float *x, int64_t n, float scale) {
    float mx = -INFINITY;
    for (int64_t i = 0; i < n; ++i) {
        x[i] = x[i] * scale;
        if (x[i] > mx) mx = x[i];
    }
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        x[i] = (float)exp((double)(x[i] - mx));
        sum += (double)x[i];
    }
    const float inv = (float)(1.0 / sum);
    for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

static const ko_tensor *albert_req(kko_model *m, const char *suffix) {
    char k[256];
    snprintf(k, sizeof k, "kokopop.albert.encoder.albert_layer_groups.0.albert_layers.0.%s", suffix);
    return req(m, k);
}

/* Embeddings (word + position, + token type 0), LayerNorm (eps 1e-12), the
 * 128 -> 768 mapping, twelve passes of the shared layer (12 heads of 64,
 * scores k . q in F32 scaled by 1/8, softmax over the keys, the weighted sum
 * of v, dense + residual -> LayerNorm, ffn -> GELU -> ffn_output + residual
 * -> LayerNorm), then bert_encoder 768 -> 512. Every linear rounds its input
 * to half for an F16 weight (linear_vec); the attention products are F32. */
int kko_albert(kko_model *m, int64_t N, const int32_t *ids, float *out) {
    g_err[0] = 0;
    const ko_tensor *word = req(m, "kokopop.albert.embeddings.word_embeddings.weight");
    const ko_tensor *pos = req(m, "kokopop.albert.embeddings.position_embeddings.weight");
    const ko_tensor *type = req(m, "kokopop.albert.embeddings.token_type_embeddings.weight");
    const ko_tensor *enw = req(m, "kokopop.albert.embeddings.LayerNorm.weight");
    const ko_tensor *enb = req(m, "kokopop.albert.embeddings.LayerNorm.bias");
    const ko_tensor *mapw = req(m, "kokopop.albert.encoder.embedding_hidden_mapping_in.weight");
    const ko_tensor *mapb = req(m, "kokopop.albert.encoder.embedding_hidden_mapping_in.bias");
    const ko_tensor *encw = req(m, "kokopop.bert_encoder.weight");
    const ko_tensor *encb = req(m, "kokopop.bert_encoder.bias");
    const ko_tensor *qw = albert_req(m, "attention.query.weight"), *qb = albert_req(m, "attention.query.bias");
    const ko_tensor *kw = albert_req(m, "attention.key.weight"), *kb = albert_req(m, "attention.key.bias");
    const ko_tensor *vw = albert_req(m, "attention.value.weight"), *vb = albert_req(m, "attention.value.bias");
    const ko_tensor *ow = albert_req(m, "attention.dense.weight"), *ob = albert_req(m, "attention.dense.bias");
    const ko_tensor *anw = albert_req(m, "attention.LayerNorm.weight");
    const ko_tensor *anb = albert_req(m, "attention.LayerNorm.bias");
    const ko_tensor *fw = albert_req(m, "ffn.weight"), *fb = albert_req(m, "ffn.bias");
    const ko_tensor *f2w = albert_req(m, "ffn_output.weight"), *f2b = albert_req(m, "ffn_output.bias");
    const ko_tensor *onw = albert_req(m, "full_layer_layer_norm.weight");
    const ko_tensor *onb = albert_req(m, "full_layer_layer_norm.bias");
    if (!word || !pos || !type || !enw || !enb || !mapw || !mapb || !encw || !encb || !qw || !qb || !kw || !kb ||
        !vw || !vb || !ow || !ob || !anw || !anb || !fw || !fb || !f2w || !f2b || !onw || !onb)
        return -1;
    const int64_t E = word->ne[0], V = word->ne[1], H = mapw->ne[1], F = fw->ne[1], D = encw->ne[1];
    const int64_t NH = 12, HS = H / NH;
    if (N < 1 || N > pos->ne[1]) return fail("ALBERT sequence length out of range%s", "");
    for (int64_t t = 0; t < N; ++t)
        if (ids[t] < 0 || ids[t] >= V) return fail("token id out of range%s", "");
    float *e = fbuf((size_t)(N * E)), *cur = fbuf((size_t)(N * H)), *q = fbuf((size_t)(N * H));
    float *k = fbuf((size_t)(N * H)), *v = fbuf((size_t)(N * H)), *att = fbuf((size_t)(N * H));
    float *o = fbuf((size_t)(N * H)), *ff = fbuf((size_t)(N * F)), *sc = fbuf((size_t)N);
    for (int64_t t = 0; t < N; ++t)
        for (int64_t c = 0; c < E; ++c) {
            const float a = word->data[(int64_t)ids[t] * E + c] + pos->data[t * E + c];
            e[t * E + c] = a + type->data[c];
        }
    layer_norm_rows(e, N, E, enw, enb, 1e-12f);
    for (int64_t t = 0; t < N; ++t) linear_vec(mapw, mapb, e + t * E, cur + t * H);
    for (int r = 0; r < 12; ++r) {
        for (int64_t t = 0; t < N; ++t) {
            linear_vec(qw, qb, cur + t * H, q + t * H);
            linear_vec(kw, kb, cur + t * H, k + t * H);
            linear_vec(vw, vb, cur + t * H, v + t * H);
        }
        for (int64_t h = 0; h < NH; ++h)
            for (int64_t qi = 0; qi < N; ++qi) {
                for (int64_t ki = 0; ki < N; ++ki) {
                    float acc = 0.f;
                    for (int64_t d = 0; d < HS; ++d) acc += k[ki * H + h * HS + d] * q[qi * H + h * HS + d];
                    sc[ki] = acc;
                }
                softmax_row(sc, N, 0.125f);
                for (int64_t d = 0; d < HS; ++d) {
                    float acc = 0.f;
                    for (int64_t ki = 0; ki < N; ++ki) acc += sc[ki] * v[ki * H + h * HS + d];
                    att[qi * H + h * HS + d] = acc;
                }
            }
        for (int64_t t = 0; t < N; ++t) {
            linear_vec(ow, ob, att + t * H, o + t * H);
            for (int64_t c = 0; c < H; ++c) cur[t * H + c] = o[t * H + c] + cur[t * H + c];
        }
        layer_norm_rows(cur, N, H, anw, anb, 1e-12f);
        for (int64_t t = 0; t < N; ++t) {
            linear_vec(fw, fb, cur + t * H, ff + t * F);
            for (int64_t c = 0; c < F; ++c) ff[t * F + c] = gelu_ggml(ff[t * F + c]);
            linear_vec(f2w, f2b, ff + t * F, o + t * H);
            for (int64_t c = 0; c < H; ++c) cur[t * H + c] = o[t * H + c] + cur[t * H + c];
        }
        layer_norm_rows(cur, N, H, onw, onb, 1e-12f);
    }
    for (int64_t t = 0; t < N; ++t) linear_vec(encw, encb, cur + t * H, out + t * D);
    free(e);
    free(cur);
    free(q);
    free(k);
    free(v);
    free(att);
    free(o);
    free(ff);
    free(sc);
    return 0;
}

static int duration_to_frames(float value, float speed) {
    if (!isfinite(speed) || speed <= 0.0f) speed = 1.0f;
    const float v = value / speed;
    if (!isfinite(v)) return 1;
    /* static_cast<int>(std::lrint(v)) then std::clamp(.., 1, 50) */
    const int r = (int)lrintf(v);
    return r < 1 ? 1 : (r > 50 ? 50 : r);
}

int kko_align_durations(const float *durations, int64_t n_tokens, float speed, int32_t *frames,
                        int64_t *total, const float *hidden, int64_t hidden_dim, float *en,
                        int64_t en_capacity) {
    int64_t tot = 0;
    for (int64_t i = 0; i < n_tokens; ++i) {
        frames[i] = duration_to_frames(durations[i], speed);
        tot += frames[i];
    }
    *total = tot;
    if (hidden && en) {
        if (tot > en_capacity) return fail("alignment output too small%s", "");
        /* build_duration_mask (kokoro.cpp:115-152) + en = d . mask (:669-674):
         * each frame's column is the one-hot of its token, so the matmul is a
         * copy of that token's hidden vector. */
        int64_t f = 0;
        for (int64_t i = 0; i < n_tokens; ++i)
            for (int32_t r = 0; r < frames[i]; ++r, ++f)
                memcpy(en + f * hidden_dim, hidden + i * hidden_dim, (size_t)hidden_dim * sizeof(float));
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* sanoTTS Vocos decoder (src/arch/sanotts/sano_vocos.cpp:94-230)           */
/* ------------------------------------------------------------------------ */

/* The RealRadix2 path of istft (src/audio/istft.cpp:96-168 plan,
 * :186-375 transform; scalar kernels of src/audio/istft_kernels.h:45-151)
 * for a power-of-two n_fft >= 64 with center = true. The spectrum is
 * frame-major (re[f * bins + k], the view sano_run_vocos hands over);
 * audio gets hop * (frames - 1) samples; no clamp. */
int kko_istft_r2(const float *re, const float *im, int64_t frames, int n_fft, int hop, float *audio,
                 int64_t *n_out) {
    const int n = n_fft, half = n_fft / 2, bins = n_fft / 2 + 1;
    if (n < 64 || (n & (n - 1)) || hop <= 0 || hop > n) return fail("istft_r2: bad n_fft / hop%s", "");
    if (n_out) *n_out = 0;
    if (frames <= 0) return 0;
    const int64_t padded = (int64_t)hop * (frames - 1) + n;
    const int64_t out_len = padded - n;
    float *window = fbuf((size_t)n), *window_sq = fbuf((size_t)n);
    for (int i = 0; i < n; ++i) {
        window[i] = (float)(0.5 - 0.5 * cos(2.0 * M_PI * (double)i / (double)n));
        window_sq[i] = window[i] * window[i];
    }
    int log2_half = 0;
    while ((1 << log2_half) < half) ++log2_half;
    int *rev = (int *)calloc((size_t)half, sizeof(int));
    for (int i = 0; i < half; ++i) {
        int r = 0;
        for (int b = 0; b < log2_half; ++b) r = (r << 1) | ((i >> b) & 1);
        rev[i] = r;
    }
    float *twc = fbuf((size_t)half), *tws = fbuf((size_t)half);
    for (int h = 1; h < half; h <<= 1) {
        const int step = half / (2 * h);
        for (int k = 0; k < h; ++k) {
            const double a = 2.0 * M_PI * (double)(k * step) / (double)half;
            twc[h - 1 + k] = (float)cos(a);
            tws[h - 1 + k] = (float)sin(a);
        }
    }
    float *scos = fbuf((size_t)half), *ssin = fbuf((size_t)half);
    for (int k = 0; k < half; ++k) {
        const double a = 2.0 * M_PI * (double)k / (double)n;
        scos[k] = (float)cos(a);
        ssin[k] = (float)sin(a);
    }
    float *zr = fbuf((size_t)half), *zi = fbuf((size_t)half), *frame = fbuf((size_t)n);
    float *ola = fbuf((size_t)padded), *env = fbuf((size_t)padded);
    const float scale = 0.5f / (float)half;
    for (int64_t f = 0; f < frames; ++f) {
        const float *xr = re + f * bins, *xi = im + f * bins;
        /* hermitian_split */
        for (int k = 0; k < half; ++k) {
            const float ar = xr[k], ai = xi[k], mr = xr[half - k], mi = xi[half - k];
            const float er = scale * (ar + mr), ei = scale * (ai - mi);
            const float dr = scale * (ar - mr), di = scale * (ai + mi);
            const float sc = scos[k], ss = ssin[k];
            zr[k] = er - (dr * ss + di * sc);
            zi[k] = ei + (dr * sc - di * ss);
        }
        /* bit-reversal swaps (each pair once) */
        for (int i = 0; i < half; ++i)
            if (rev[i] > i) {
                const int j = rev[i];
                float t = zr[i]; zr[i] = zr[j]; zr[j] = t;
                t = zi[i]; zi[i] = zi[j]; zi[j] = t;
            }
        /* fft_stage_pairs then fft_stage for h = 2, 4, ..., half / 2 */
        for (int i = 0; i < half; i += 2) {
            const float ar = zr[i], ai = zi[i], br = zr[i + 1], bi = zi[i + 1];
            zr[i] = ar + br;
            zi[i] = ai + bi;
            zr[i + 1] = ar - br;
            zi[i + 1] = ai - bi;
        }
        for (int h = 2; h < half; h <<= 1) {
            const float *wc = twc + (h - 1), *ws = tws + (h - 1);
            for (int base = 0; base < half; base += 2 * h)
                for (int k = 0; k < h; ++k) {
                    const int a = base + k, b = a + h;
                    const float brr = zr[b] * wc[k] - zi[b] * ws[k];
                    const float bii = zr[b] * ws[k] + zi[b] * wc[k];
                    zr[b] = zr[a] - brr;
                    zi[b] = zi[a] - bii;
                    zr[a] = zr[a] + brr;
                    zi[a] = zi[a] + bii;
                }
        }
        /* interleave_windowed */
        for (int mm = 0; mm < half; ++mm) {
            frame[2 * mm] = zr[mm] * window[2 * mm];
            frame[2 * mm + 1] = zi[mm] * window[2 * mm + 1];
        }
        const int64_t base = (int64_t)hop * f;
        for (int i = 0; i < n; ++i) {
            ola[base + i] += frame[i];
            env[base + i] += window_sq[i];
        }
    }
    const int64_t trim = n / 2;
    for (int64_t j = 0; j < out_len; ++j) {
        const float e = env[trim + j];
        audio[j] = e > 1e-8f ? ola[trim + j] / e : 0.0f;
    }
    if (n_out) *n_out = out_len;
    free(window); free(window_sq); free(rev); free(twc); free(tws); free(scos); free(ssin);
    free(zr); free(zi); free(frame); free(ola); free(env);
    return 0;
}

/* ggml semantics, ggml_gelu_erf on F32 (ggml-cpu vec.h):
 * y = 0.5f * x * (1.0f + erff(x * SQRT_2_INV)), evaluated left to right;
 * erf taken correctly rounded (the C library's erff differs in the last bit
 * for some arguments). */
static float gelu_erf(float x) {
    const float t = x * 0.70710678118654752440f;
    const float e = (float)erf((double)t);
    return (0.5f * x) * (1.0f + e);
}

/* sano_run_vocos (src/arch/sanotts/sano_vocos.cpp:94-230) for one chunk of
 * `frames` frames: mel [mels][frames] and noise [noise_ch][frames] (ggml
 * [frames, C], time-fastest) -> audio [hop * (frames - 1)]. Weight names
 * under `prefix` ("...dec.embed.weight" etc., sano_arch.cpp:1138-1177).
 * The trunk runs frame-major [frames][dim] as the reference's [C, T]:
 *   stem   x = conv_k(mel) + b + conv_k(noise) + b (F32 im2col + mul_mat,
 *          sano_graph.cpp:35-56), LayerNorm over channels (eps 1e-6)
 *   block  r = depthwise conv_k(x) + dw_b (:58-71), LayerNorm,
 *          h = gelu_erf(pw0 r + b0), x = x + (pw1 h + b1) * gamma
 *   head   LayerNorm, head x + b -> [2 bins]; magnitude
 *          min(exp(clamp(lm, +-60)), mag_clip) with the DC and Nyquist bins
 *          zeroed, real = mag cos(phase), imag = mag sin(phase)
 *   iSTFT  (kko_istft_r2), then the DC blocker (sano_vocos.cpp:81-92).
 * Dot products are summed in ascending index order; exp / cos / sin are
 * correctly rounded. */
int kko_vocos(kko_model *m, const char *prefix, const kko_vocos_dims *d, int64_t frames, const float *mel,
              const float *noise, float *audio, int64_t *n_out) {
    g_err[0] = 0;
    if (frames < 2) return fail("vocos: a chunk needs at least two frames%s", "");
    const int64_t T = frames, D = d->dim, Hd = d->pw_hidden, bins = d->n_fft / 2 + 1;
    char k[320];
#define VREQ(var, suffix)                                   \
    snprintf(k, sizeof k, "%s%s", prefix, suffix);         \
    const ko_tensor *var = req(m, k);                       \
    if (!var) return -1;
    VREQ(ew, "dec.embed.weight") VREQ(eb, "dec.embed.bias") VREQ(nw, "dec.noise.weight")
    VREQ(nb, "dec.noise.bias") VREQ(n0w, "dec.norm.weight") VREQ(n0b, "dec.norm.bias")
    VREQ(fnw, "dec.final_norm.weight") VREQ(fnb, "dec.final_norm.bias") VREQ(hw, "dec.head.weight")
    VREQ(hb, "dec.head.bias")
    if (ew->n != D * d->mels * d->embed_kernel || nw->n != D * d->noise_ch * d->embed_kernel ||
        hw->n != D * 2 * bins)
        return fail("vocos: weight shapes disagree with the dimensions (%s)", prefix);
    /* stem: conv outputs are [D][T] (channel-major) */
    float *s1 = fbuf((size_t)(D * T)), *s2 = fbuf((size_t)(D * T));
    int64_t ol = 0;
    if (conv1d(ew, eb, mel, d->mels, T, 1, d->embed_kernel / 2, 1, d->embed_kernel, s1, &ol) != 0 ||
        conv1d(nw, nb, noise, d->noise_ch, T, 1, d->embed_kernel / 2, 1, d->embed_kernel, s2, &ol) != 0) {
        free(s1); free(s2);
        return -1;
    }
    float *x = fbuf((size_t)(T * D));
    for (int64_t c = 0; c < D; ++c)
        for (int64_t t = 0; t < T; ++t) x[t * D + c] = s1[c * T + t] + s2[c * T + t];
    free(s1); free(s2);
    layer_norm_rows(x, T, D, n0w, n0b, 1e-6f);
    float *r = fbuf((size_t)(T * D)), *h = fbuf((size_t)(T * Hd));
    const int K = d->dw_kernel, pad = K / 2;
    for (int bi = 0; bi < d->blocks; ++bi) {
        char base[200];
        snprintf(base, sizeof base, "dec.blocks.%d.", bi);
        char nm[260];
#define BREQ(var, suffix)                                           \
        snprintf(nm, sizeof nm, "%s%s", base, suffix);             \
        snprintf(k, sizeof k, "%s%s", prefix, nm);                 \
        const ko_tensor *var = req(m, k);                           \
        if (!var) { free(x); free(r); free(h); return -1; }
        BREQ(dww, "dw.weight") BREQ(dwb, "dw.bias") BREQ(lnw, "norm.weight") BREQ(lnb, "norm.bias")
        BREQ(p0w, "pw0.weight") BREQ(p0b, "pw0.bias") BREQ(p1w, "pw1.weight") BREQ(p1b, "pw1.bias")
        BREQ(gam, "gamma")
        /* depthwise conv over time, zero padded, + bias */
        for (int64_t t = 0; t < T; ++t)
            for (int64_t c = 0; c < D; ++c) {
                float acc = 0.f;
                for (int kk = 0; kk < K; ++kk) {
                    const int64_t tt = t - pad + kk;
                    if (tt >= 0 && tt < T) acc += x[tt * D + c] * dww->data[c * K + kk];
                }
                r[t * D + c] = acc + dwb->data[c];
            }
        layer_norm_rows(r, T, D, lnw, lnb, 1e-6f);
#pragma omp parallel for schedule(static)
        for (int64_t t = 0; t < T; ++t) {
            const float *rt = r + t * D;
            float *ht = h + t * Hd;
            for (int64_t j = 0; j < Hd; ++j) {
                const float *wj = p0w->data + j * D;
                float acc = 0.f;
                for (int64_t c = 0; c < D; ++c) acc += wj[c] * rt[c];
                ht[j] = gelu_erf(acc + p0b->data[j]);
            }
            float *xt = x + t * D;
            for (int64_t c = 0; c < D; ++c) {
                const float *wc = p1w->data + c * Hd;
                float acc = 0.f;
                for (int64_t j = 0; j < Hd; ++j) acc += wc[j] * ht[j];
                const float o = acc + p1b->data[c];
                xt[c] = xt[c] + o * gam->data[c];
            }
        }
#undef BREQ
    }
    free(r);
    free(h);
    layer_norm_rows(x, T, D, fnw, fnb, 1e-6f);
    float *re = fbuf((size_t)(T * bins)), *im = fbuf((size_t)(T * bins));
    const float clip = d->mag_clip;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        const float *xt = x + t * D;
        for (int64_t kb = 0; kb < bins; ++kb) {
            float lm = 0.f, ph = 0.f;
            for (int pass = 0; pass < 2; ++pass) {
                const int64_t o = pass * bins + kb;
                const float *wo = hw->data + o * D;
                float acc = 0.f;
                for (int64_t c = 0; c < D; ++c) acc += wo[c] * xt[c];
                if (pass == 0) lm = acc + hb->data[o];
                else ph = acc + hb->data[o];
            }
            float v = lm < -60.0f ? -60.0f : (lm > 60.0f ? 60.0f : lm);
            float mag = (float)exp((double)v);
            mag = mag < 0.0f ? 0.0f : (mag > clip ? clip : mag);
            if (kb == 0 || kb == bins - 1) mag = mag * 0.0f;
            re[t * bins + kb] = mag * (float)cos((double)ph);
            im[t * bins + kb] = mag * (float)sin((double)ph);
        }
    }
    free(x);
    int64_t n = 0;
    const int rc = kko_istft_r2(re, im, T, d->n_fft, d->hop, audio, &n);
    free(re);
    free(im);
    if (rc != 0) return rc;
    kko_dc_block(audio, n, d->dc_pole);
    if (n_out) *n_out = n;
    return 0;
#undef VREQ
}

/* The first-order DC blocker of sano_vocos.cpp:81-92, in sample order:
 * y[n] = x[n] - x[n - 1] + pole * y[n - 1], from zero state. */
void kko_dc_block(float *audio, int64_t n, float pole) {
    float prev_in = 0.0f, prev_out = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        const float input = audio[i];
        const float output = input - prev_in + pole * prev_out;
        prev_in = input;
        prev_out = output;
        audio[i] = output;
    }
}
