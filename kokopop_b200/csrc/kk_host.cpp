// Host side of the B200 Kokoro-82M hot path: the context, the weight
// registry, the packed ragged-batch plan, the decoder / generator
// orchestration and the C ABI of include/kokopop_b200.h.
//
// The orchestration follows the reference's graph builders op for op:
//   decoder   run_kokoro_generation_probe, src/arch/kokoro/kokoro.cpp:716-763
//   block     adain_resblk1d,              src/arch/kokoro/graph_ops.cpp:996-1065
//   generator ggml_generator,              src/arch/kokoro/audio_utils.cpp:594-1051
//   resblock  graph_generator_resblock,    src/arch/kokoro/graph_ops.cpp:1071-1111
//   3 branches graph_3branch_main_sum,     src/arch/kokoro/graph_ops.cpp:1300-1320
// Errors follow src/kokopop.cpp:38-59: no exception leaves this file, every
// failure becomes a status code plus a thread-local message.
#include "../../include/kokopop_b200.h"
#include "kk_kernels.h"
#include "kk_host.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstddef>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_last_error;

constexpr float kInvSqrt2 = 0.7071067811865476f;  // KOKOPOP_INV_SQRT2
constexpr int kDil[3] = {1, 3, 5};                // KOKOPOP_RESBLOCK_DILATIONS
constexpr int kKs[3] = {3, 7, 11};                // KOKOPOP_RESBLOCK_KERNELS
constexpr float kThird = 1.0f / 3.0f;             // the branch average

}  // namespace

namespace kk {

KKError::KKError(int c, const std::string &m) : std::runtime_error(m), code(c) {}

void check_cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess)
        throw KKError(KK_ERROR_INFERENCE, std::string(what) + ": " + cudaGetErrorString(e));
}

static std::atomic<uint64_t> g_allocations{0};
static std::atomic<int32_t> g_fail_next{0};  // allocations still to fail (kk_inject_allocation_failures)

static bool injected_failure() {
    int32_t n = g_fail_next.load(std::memory_order_relaxed);
    while (n > 0)
        if (g_fail_next.compare_exchange_weak(n, n - 1, std::memory_order_relaxed)) return true;
    return false;
}

cudaError_t device_malloc(void **p, size_t bytes) {
    g_allocations.fetch_add(1, std::memory_order_relaxed);
    if (injected_failure()) return cudaErrorMemoryAllocation;
    return cudaMalloc(p, bytes);
}

cudaError_t pinned_malloc(void **p, size_t bytes) {
    g_allocations.fetch_add(1, std::memory_order_relaxed);
    if (injected_failure()) return cudaErrorMemoryAllocation;
    return cudaMallocHost(p, bytes);
}

void DevBuf::ensure(size_t b) {
    if (b <= bytes) return;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    check_cuda(device_malloc(&p, b), "cudaMalloc workspace");
    bytes = b;
}

void DevBuf::release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
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
    std::memcpy(&f, &bits, 4);
    return f;
}

}  // namespace kk

using namespace kk;

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------

kk_ctx::~kk_ctx() {
    for (auto &t : timed) {
        cudaEventDestroy(t.a);
        cudaEventDestroy(t.b);
    }
    for (auto e : event_pool) cudaEventDestroy(e);
    for (auto &kv : w) cudaFree(kv.second.d);
    for (auto &kv : ws) kv.second.release();
    for (auto &b : convt_phase) b.release();
    for (auto &kv : packed) kv.second.buf.release();
    for (auto &kv : adain_t) kv.second.release();
    for (auto &kv : lstm) {
        kv.second.wih.release();
        kv.second.wih_tc.buf.release();
        kv.second.bih_buf.release();
    }
    d_err.release();
    d_sites.release();
    d_tables.release();
    d_batch.release();
    for (auto &s : stage) {
        if (s.ev) cudaEventDestroy(s.ev);
        if (s.p) cudaFreeHost(s.p);
        for (char *r : s.retired) cudaFreeHost(r);
    }
    if (ev_done) cudaEventDestroy(ev_done);
    if (ev_inputs) cudaEventDestroy(ev_inputs);
    if (ev_src) cudaEventDestroy(ev_src);
    if (st2) cudaStreamDestroy(st2);
    if (st) cudaStreamDestroy(st);
}

const DevTensor &kk_ctx::W(const std::string &name) const {
    auto it = w.find(name);
    if (it == w.end()) throw KKError(KK_ERROR_MODEL, "missing tensor: " + name);
    return it->second;
}

const DevTensor *kk_ctx::Wopt(const std::string &name) const {
    auto it = w.find(name);
    return it == w.end() ? nullptr : &it->second;
}

cudaEvent_t kk_ctx::take_event() {
    if (!event_pool.empty()) {
        cudaEvent_t e = event_pool.back();
        event_pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    check_cuda(cudaEventCreate(&e), "cudaEventCreate");
    return e;
}

float *kk_ctx::buf(const char *name, size_t floats) {
    DevBuf &b = ws[name];
    b.ensure(floats * sizeof(float));
    return (float *)b.p;
}

// The device status block: error word 0, no non-finite index recorded.
void kk_ctx::reset_status() {
    d_err.ensure(sizeof(DevStatus));
    check_cuda(cudaMemset(d_err.p, 0, offsetof(DevStatus, first)), "clear status");
    check_cuda(cudaMemset((char *)d_err.p + offsetof(DevStatus, first), 0xff, sizeof(DevStatus::first)),
               "clear status");
}

// Waits for the timed launches' end events and turns them into records (and
// the convolution counters of kk_profile).
void kk_ctx::resolve_timed() {
    for (auto &t : timed) {
        check_cuda(cudaEventSynchronize(t.b), "profile sync");
        float ms = 0.f;
        check_cuda(cudaEventElapsedTime(&ms, t.a, t.b), "profile elapsed");
        if (t.kind == KK_PROF_CONV) {
            conv_ms += ms;
            conv_flop += t.flop;
            conv_launches += 1;
        }
        records.push_back(kk_profile_record{t.kind, t.taps, (double)ms, t.flop, t.bytes});
        event_pool.push_back(t.a);
        event_pool.push_back(t.b);
    }
    timed.clear();
}

void kk_ctx::stage_begin() {
    stage_k ^= 1;
    StageSlot &s = stage[stage_k];
    if (s.pending) {
        check_cuda(cudaEventSynchronize(s.ev), "staging slot reuse");
        s.pending = false;
    }
    for (char *r : s.retired) cudaFreeHost(r);
    s.retired.clear();
    s.used = 0;
}

void kk_ctx::upload(void *dst, const void *src, size_t bytes, cudaStream_t st, const char *what) {
    if (!bytes) return;
    StageSlot &s = stage[stage_k];
    size_t at = (s.used + 63) / 64 * 64;
    if (at + bytes > s.cap) {
        // earlier uploads of this call may still read the old buffer: keep it
        // until the slot's event has passed
        if (s.p) s.retired.push_back(s.p);
        s.p = nullptr;
        s.cap = 0;
        const size_t cap = std::max<size_t>(bytes, 64 * 1024) * 2;
        check_cuda(pinned_malloc((void **)&s.p, cap), "cudaMallocHost staging");
        s.cap = cap;
        at = 0;
    }
    std::memcpy(s.p + at, src, bytes);
    s.used = at + bytes;
    check_cuda(cudaMemcpyAsync(dst, s.p + at, bytes, cudaMemcpyHostToDevice, st), what);
    // the slot is free again once its last copy has run (early in the call's
    // work on the device), not when the whole call has finished
    s.pending = false;
    if (cudaEventRecord(s.ev, st) == cudaSuccess)
        s.pending = true;
    else
        cudaStreamSynchronize(st);  // no event: make sure no copy still reads the slot
}

// Host tables, computed with the C library exactly as the reference does.
static void make_tables(StftTables &st, IstftTables &is) {
    for (int n = 0; n < kStftN; ++n) {
        // hann_window_20 (audio_utils.cpp:36-45) and the iSTFT plan's window
        // (src/audio/istft.cpp:236-242): the double expression, rounded.
        const float wv = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * (double)n / (double)kStftN));
        st.window[n] = wv;
        is.window[n] = wv;
        is.window_sq[n] = wv * wv;
        // StftTwiddles (audio_utils.cpp:47-64)
        for (int k = 0; k < kBins; ++k) {
            const float a = (float)(2.0 * M_PI * (double)(float)(k * n) / (double)(float)kStftN);
            st.c[n][k] = std::cos(a);
            st.s[n][k] = std::sin(a);
        }
    }
    // DirectDft tables (src/audio/istft.cpp:244-254)
    for (int k = 0; k < kBins; ++k)
        for (int i = 0; i < kStftN; ++i) {
            const float a = (float)(2.0 * M_PI * (double)(k * i) / (double)kStftN);
            is.c[k][i] = std::cos(a);
            is.s[k][i] = std::sin(a);
        }
}

namespace kk {
void fill_tables(StftTables &st, IstftTables &is) { make_tables(st, is); }
void set_last_error(const std::string &msg) { g_last_error = msg; }
}  // namespace kk

static std::vector<std::string> adain_site_prefixes() {
    std::vector<std::string> v;
    const std::string d = "kokopop.decoder.";
    v.push_back(d + "encode.norm1");
    v.push_back(d + "encode.norm2");
    for (int i = 0; i < 4; ++i) {
        v.push_back(d + "decode." + std::to_string(i) + ".norm1");
        v.push_back(d + "decode." + std::to_string(i) + ".norm2");
    }
    std::vector<std::string> blocks = {d + "generator.noise_res.0", d + "generator.noise_res.1"};
    for (int b = 0; b < 6; ++b) blocks.push_back(d + "generator.resblocks." + std::to_string(b));
    for (auto &p : blocks)
        for (int i = 0; i < 3; ++i) {
            v.push_back(p + ".adain1." + std::to_string(i));
            v.push_back(p + ".adain2." + std::to_string(i));
        }
    return v;
}

// The prosody predictor's F0 / N chain (kokoro.cpp:669-708): its AdaIN sites
// and convolutions, used when a weight set carries them.
static std::vector<std::string> prosody_site_prefixes() {
    std::vector<std::string> v;
    for (const char *br : {"F0", "N"})
        for (int i = 0; i < 3; ++i) {
            const std::string p = std::string("kokopop.predictor.") + br + "." + std::to_string(i);
            v.push_back(p + ".norm1");
            v.push_back(p + ".norm2");
        }
    return v;
}

static std::vector<std::pair<std::string, int>> prosody_convs() {
    std::vector<std::pair<std::string, int>> v;
    for (const char *br : {"F0", "N"}) {
        for (int i = 0; i < 3; ++i) {
            const std::string p = std::string("kokopop.predictor.") + br + "." + std::to_string(i);
            v.push_back({p + ".conv1.weight", 3});
            v.push_back({p + ".conv2.weight", 3});
            v.push_back({p + ".conv1x1.weight", 1});
        }
        v.push_back({std::string("kokopop.predictor.") + br + "_proj.weight", 1});
    }
    return v;
}

// ALBERT's linear layers (kokoro.cpp:52-81, :297-337) and bert_encoder.
static const char *kAlbertLayer = "kokopop.albert.encoder.albert_layer_groups.0.albert_layers.0.";
static std::vector<std::string> albert_linears() {
    std::vector<std::string> v = {"kokopop.albert.encoder.embedding_hidden_mapping_in.weight",
                                  "kokopop.bert_encoder.weight"};
    for (const char *n : {"attention.query.weight", "attention.key.weight", "attention.value.weight",
                          "attention.dense.weight", "ffn.weight", "ffn_output.weight"})
        v.push_back(std::string(kAlbertLayer) + n);
    return v;
}

// The text encoder's three k = 5 convolutions (graph_ops.cpp:1593-1611).
static std::vector<std::string> text_convs() {
    std::vector<std::string> v;
    for (int i = 0; i < 3; ++i) v.push_back("kokopop.text_encoder.cnn." + std::to_string(i) + ".0.weight");
    return v;
}

// Packs a convolution weight W[oc, ic, k] (via `get`) into the tensor-core
// kernel's shared-memory images: half [K][IC_pad/64][n_tiles][8][tile_n][8]
// (tiles of tile_n output rows, 128 unless a kernel asks otherwise), zero in
// the channel padding. The values are F16 already, so the conversion is
// exact.
template <typename Get>
static void pack_tc(PackedW &pw, int OC, int IC, int K, Get get, int tile_n = 128) {
    pw.IC = IC;
    pw.OC = OC;
    pw.K = K;
    pw.IC_pad = (IC + 63) / 64 * 64;
    pw.n_tiles = (OC + tile_n - 1) / tile_n;
    const int NB = pw.IC_pad / 64;
    std::vector<__half> h((size_t)K * NB * pw.n_tiles * 8 * tile_n * 8, __float2half_rn(0.f));
    for (int k = 0; k < K; ++k)
        for (int oc = 0; oc < OC; ++oc)
            for (int ic = 0; ic < IC; ++ic) {
                const int b = ic / 64, c = (ic % 64) / 8, e = ic % 8, nt = oc / tile_n, n = oc % tile_n;
                const size_t idx =
                    ((((size_t)k * NB + b) * pw.n_tiles + nt) * 8 + c) * ((size_t)tile_n * 8) + (size_t)n * 8 + e;
                h[idx] = __float2half_rn(get(oc, ic, k));
            }
    pw.buf.ensure(h.size() * sizeof(__half));
    check_cuda(cudaMemcpy(pw.buf.p, h.data(), h.size() * sizeof(__half), cudaMemcpyHostToDevice), "upload packed");
}

// Split-F32 packing: the F32 weight as [W_lo | W_hi | W_hi] over 3 blocks of
// IC rounded to 64 virtual channels (hi = half(w), lo = half(w - hi)),
// against the operand [x_hi | x_lo] whose hi blocks the kernel reads again
// for the third (a_wrap), so that one GEMM with F32 accumulation sums
// W_lo x_hi + W_hi x_lo + W_hi x_hi. The two small correction terms come
// first, into a small accumulator: the tensor cores' accumulation error then
// stays near that of the W_hi x_hi GEMM alone.
// The weights are scaled by 2^s, s the largest with max |w| 2^s <= 2^14,
// before the split (a lo half then sits in the half subnormal range, with
// its coarser absolute spacing, only for |w| below 2^-3 of the largest),
// and the conv takes acc_scale = 2^-s back, exactly.
template <typename Get>
static void pack_tc_split(PackedW &pw, int OC, int IC, int K, Get get, int tile_n = 128) {
    const int ICp = (IC + 63) / 64 * 64;
    float amax = 0.f;
    for (int k = 0; k < K; ++k)
        for (int oc = 0; oc < OC; ++oc)
            for (int ic = 0; ic < IC; ++ic) amax = std::fmax(amax, std::fabs(get(oc, ic, k)));
    int s = 0;
    if (amax > 0.f && std::isfinite(amax)) {
        int e = 0;
        std::frexp(amax, &e);  // amax < 2^e
        s = std::min(std::max(14 - e, -100), 100);
    }
    const float up = std::ldexp(1.0f, s);
    pack_tc(pw, OC, 3 * ICp, K, [&](int oc, int v, int k) {
        const int part = v / ICp, ic = v % ICp;
        if (ic >= IC) return 0.f;
        const float w = get(oc, ic, k) * up;
        const float hi = __half2float(__float2half_rn(w));
        return part > 0 ? hi : __half2float(__float2half_rn(w - hi));
    }, tile_n);
    pw.IC = IC;
    pw.a_wrap = 2 * ICp / 64;
    pw.acc_scale = std::ldexp(1.0f, -s);
}

// The convolutions that run on the tensor cores, with their tap counts.
static std::vector<std::pair<std::string, int>> tc_convs() {
    std::vector<std::pair<std::string, int>> v;
    const std::string d = "kokopop.decoder.", g = d + "generator.";
    v.push_back({d + "asr_res.0.weight", 1});
    for (const std::string &b : {d + "encode", d + "decode.0", d + "decode.1", d + "decode.2", d + "decode.3"}) {
        v.push_back({b + ".conv1.weight", 3});
        v.push_back({b + ".conv2.weight", 3});
        v.push_back({b + ".conv1x1.weight", 1});
    }
    const std::pair<std::string, int> blocks[8] = {{"noise_res.0", 7}, {"noise_res.1", 11}, {"resblocks.0", 3},
                                                   {"resblocks.1", 7},  {"resblocks.2", 11}, {"resblocks.3", 3},
                                                   {"resblocks.4", 7},  {"resblocks.5", 11}};
    for (const auto &bk : blocks)
        for (int i = 0; i < 3; ++i) {
            v.push_back({g + bk.first + ".convs1." + std::to_string(i) + ".weight", bk.second});
            v.push_back({g + bk.first + ".convs2." + std::to_string(i) + ".weight", bk.second});
        }
    v.push_back({g + "conv_post.weight", 7});
    return v;
}

// Builds everything derived from the raw weights: ConvTranspose phase
// weights, the AdaIN site table, the harmonic-source constants and tables.
void kk_ctx::derive() {
    generator_ready = decoder_ready = false;
    missing.clear();
    auto need = [&](const std::string &n) {
        if (!Wopt(n) && missing.empty()) missing = n;
        return Wopt(n) != nullptr;
    };
    // ConvTranspose ups.s as s phase convolutions with 2 taps each:
    // phase r, tap 0 reads t_in = q - 1 with W[r + s], tap 1 reads q with W[r].
    static const int strides[2] = {10, 6};
    bool ok = true;
    std::vector<float> phase_host[2];
    for (int s = 0; s < 2; ++s) {
        const std::string nm = "kokopop.decoder.generator.ups." + std::to_string(s) + ".weight";
        if (!need(nm)) {
            ok = false;
            continue;
        }
        const DevTensor &t = W(nm);
        const int K = (int)t.ne[0], OC = (int)t.ne[1], IC = (int)t.ne[2], S = strides[s];
        if (K > 2 * S) throw KKError(KK_ERROR_MODEL, "ConvTranspose kernel longer than 2 strides: " + nm);
        std::vector<float> h((size_t)t.n), ph((size_t)S * OC * IC * 2, 0.f);
        check_cuda(cudaMemcpy(h.data(), t.d, h.size() * 4, cudaMemcpyDeviceToHost), "read ups weight");
        for (int r = 0; r < S; ++r)
            for (int oc = 0; oc < OC; ++oc)
                for (int ic = 0; ic < IC; ++ic) {
                    const size_t o = (((size_t)r * OC + oc) * IC + ic) * 2;
                    const size_t src = ((size_t)ic * OC + oc) * K;
                    ph[o + 0] = (r + S < K) ? h[src + r + S] : 0.f;
                    ph[o + 1] = (r < K) ? h[src + r] : 0.f;
                }
        convt_phase[s].ensure(ph.size() * 4);
        check_cuda(cudaMemcpy(convt_phase[s].p, ph.data(), ph.size() * 4, cudaMemcpyHostToDevice),
                   "upload phase weights");
        convt_f16[s] = t.f16;
        phase_host[s] = std::move(ph);
    }
    // tensor-core path: taken when every convolution weight is stored as F16
    // (the converter's policy); F32 weight sets keep the F32 CUDA-core path.
    for (auto &kv : packed) kv.second.buf.release();
    packed.clear();
    for (auto &kv : lstm) {
        kv.second.wih.release();
        kv.second.wih_tc.buf.release();
        kv.second.bih_buf.release();
    }
    lstm.clear();
    for (auto &kv : vocos) {
        VocosNet &v = kv.second;
        v.embed.buf.release();
        v.noise.buf.release();
        v.head.buf.release();
        for (auto &p : v.pw0) p.buf.release();
        for (auto &p : v.pw1) p.buf.release();
        v.tables.release();
    }
    vocos.clear();
    bool all16 = ok && convt_f16[0] && convt_f16[1], all32 = ok && !convt_f16[0] && !convt_f16[1];
    {
        std::vector<std::pair<std::string, int>> convs = tc_convs();
        convs.push_back({"kokopop.decoder.generator.noise_convs.0.weight", 12});
        convs.push_back({"kokopop.decoder.generator.noise_convs.1.weight", 1});
        for (const auto &cv : convs) {
            const DevTensor *t = Wopt(cv.first);
            if (t) {
                all16 = all16 && t->f16;
                all32 = all32 && !t->f16;
            } else if (cv.first.find("conv1x1") == std::string::npos) {
                all16 = all32 = false;
            }
        }
        const char *f = std::getenv("KOKOPOP_B200_F32_SPLIT");
        f32_split = !(f && f[0] == '0');
        all32 = all32 && f32_split;
    }
    tc_mode = all16 || all32;
    split_mode = all32;
    {
        // the operand formed inside the conv (k_conv_tcf) for the residual
        // blocks' convs with at least this many taps: "1" all of them, "7"
        // the k = 7 and k = 11 ones; unset or "0": none
        const char *f = std::getenv("KOKOPOP_B200_FUSED_OPERAND");
        fuse_min_taps = f ? std::atoi(f) : 0;
        fuse_operand = fuse_min_taps > 0;
        // the ConvTranspose as phase-major 128-channel tiles on k_conv_tc
        // (every S-th output row per store) instead of k_convt_tc
        const char *g = std::getenv("KOKOPOP_B200_CONVT_PHASES");
        convt_phases = g && g[0] == '1';
    }
    // the prosody chain's convolutions on the tensor cores when they are all
    // F16, whatever the rest of the weight set
    prosody_tc = true;
    for (const auto &cv : prosody_convs()) {
        const DevTensor *t = Wopt(cv.first);
        if (t ? !t->f16 : cv.first.find("conv1x1") == std::string::npos) prosody_tc = false;
    }
    if (prosody_tc && (!tc_mode || split_mode)) {
        check_cuda(conv_tc_init(), "tensor-core conv init");
        std::vector<float> h;
        for (const auto &cv : prosody_convs()) {
            const DevTensor *t = Wopt(cv.first);
            if (!t) continue;
            const int K = cv.second, OC = (int)t->ne[1], IC = (int)(t->ne[0] / K);
            h.resize((size_t)t->n);
            check_cuda(cudaMemcpy(h.data(), t->d, h.size() * 4, cudaMemcpyDeviceToHost), "read conv weight");
            pack_tc(packed[cv.first], OC, IC, K,
                    [&](int oc, int ic, int k) { return h[((size_t)oc * IC + ic) * K + k]; });
        }
    }
    // the text encoder's convs: tensor cores when all F16, split when all F32
    {
        bool t16 = true, t32 = true, any = false;
        for (const auto &n : text_convs()) {
            const DevTensor *t = Wopt(n);
            if (!t) {
                t16 = t32 = false;
                continue;
            }
            any = true;
            t16 = t16 && t->f16;
            t32 = t32 && !t->f16;
        }
        text_mode = !any ? 0 : t16 ? 1 : (t32 && f32_split) ? 2 : 0;
        if (text_mode) {
            check_cuda(conv_tc_init(), "tensor-core conv init");
            std::vector<float> h;
            for (const auto &n : text_convs()) {
                const DevTensor *t = Wopt(n);
                const int K = 5, OC = (int)t->ne[1], IC = (int)(t->ne[0] / K);
                h.resize((size_t)t->n);
                check_cuda(cudaMemcpy(h.data(), t->d, h.size() * 4, cudaMemcpyDeviceToHost), "read conv weight");
                auto get = [&](int oc, int ic, int k) { return h[((size_t)oc * IC + ic) * K + k]; };
                if (text_mode == 1)
                    pack_tc(packed[n], OC, IC, K, get);
                else
                    pack_tc_split(packed[n], OC, IC, K, get);
            }
        }
    }
    // ALBERT's linears: the same rule as the text encoder's convs
    {
        bool t16 = true, t32 = true, all = true;
        for (const auto &n : albert_linears()) {
            const DevTensor *t = Wopt(n);
            if (!t) {
                all = false;
                continue;
            }
            t16 = t16 && t->f16;
            t32 = t32 && !t->f16;
        }
        albert_mode = !all ? 0 : t16 ? 1 : (t32 && f32_split) ? 2 : 0;
        if (albert_mode) {
            check_cuda(conv_tc_init(), "tensor-core conv init");
            std::vector<float> h;
            for (const auto &n : albert_linears()) {
                const DevTensor *t = Wopt(n);
                const int OC = (int)t->ne[1], IC = (int)t->ne[0];
                h.resize((size_t)t->n);
                check_cuda(cudaMemcpy(h.data(), t->d, h.size() * 4, cudaMemcpyDeviceToHost), "read linear weight");
                auto get = [&](int oc, int ic, int) { return h[(size_t)oc * IC + ic]; };
                if (albert_mode == 1)
                    pack_tc(packed[n], OC, IC, 1, get);
                else
                    pack_tc_split(packed[n], OC, IC, 1, get);
            }
            // query | key | value along the output channels
            const std::string L = kAlbertLayer;
            const DevTensor *qkv[3] = {Wopt(L + "attention.query.weight"), Wopt(L + "attention.key.weight"),
                                       Wopt(L + "attention.value.weight")};
            const DevTensor *qkvb[3] = {Wopt(L + "attention.query.bias"), Wopt(L + "attention.key.bias"),
                                        Wopt(L + "attention.value.bias")};
            const int H = (int)qkv[0]->ne[1], IC = (int)qkv[0]->ne[0];
            bool same = true;
            for (int i = 0; i < 3; ++i)
                same = same && qkv[i]->ne[0] == IC && qkv[i]->ne[1] == H && qkvb[i] && qkvb[i]->n == H;
            if (same) {
                std::vector<float> hw((size_t)3 * H * IC), hb((size_t)3 * H);
                for (int i = 0; i < 3; ++i) {
                    check_cuda(cudaMemcpy(hw.data() + (size_t)i * H * IC, qkv[i]->d, (size_t)H * IC * 4,
                                          cudaMemcpyDeviceToHost),
                               "read qkv weight");
                    check_cuda(cudaMemcpy(hb.data() + (size_t)i * H, qkvb[i]->d, (size_t)H * 4, cudaMemcpyDeviceToHost),
                               "read qkv bias");
                }
                auto get = [&](int oc, int ic, int) { return hw[(size_t)oc * IC + ic]; };
                if (albert_mode == 1)
                    pack_tc(packed["albert.qkv"], 3 * H, IC, 1, get);
                else
                    pack_tc_split(packed["albert.qkv"], 3 * H, IC, 1, get);
                albert_qkv_bbuf.ensure(hb.size() * 4);
                check_cuda(cudaMemcpy(albert_qkv_bbuf.p, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice),
                           "upload qkv bias");
                albert_qkv_b.d = (float *)albert_qkv_bbuf.p;
                albert_qkv_b.ne[0] = 3 * H;
                albert_qkv_b.n = 3 * H;
            }
        }
    }
    reset_status();
    if (tc_mode) {
        check_cuda(conv_tc_init(), "tensor-core conv init");
        // F16 weights pack as they are; F32 ones split (split_mode)
        auto pack = [&](PackedW &pw, int OC, int IC, int K, const std::function<float(int, int, int)> &get,
                        int tile_n = 128) {
            if (split_mode)
                pack_tc_split(pw, OC, IC, K, get, tile_n);
            else
                pack_tc(pw, OC, IC, K, get, tile_n);
        };
        std::vector<float> h;
        std::vector<std::pair<std::string, int>> convs = tc_convs();
        for (const auto &cv : prosody_convs()) {
            const DevTensor *t = Wopt(cv.first);
            if (t && t->f16 && !split_mode) convs.push_back(cv);
        }
        for (const auto &cv : convs) {
            const DevTensor *t = Wopt(cv.first);
            if (!t) continue;
            const int K = cv.second, OC = (int)t->ne[1], IC = (int)(t->ne[0] / K);
            h.resize((size_t)t->n);
            check_cuda(cudaMemcpy(h.data(), t->d, h.size() * 4, cudaMemcpyDeviceToHost), "read conv weight");
            pack(packed[cv.first], OC, IC, K,
                 [&](int oc, int ic, int k) { return h[((size_t)oc * IC + ic) * K + k]; });
        }
        // noise_convs.1: 1x1 over the 22 har channels
        {
            const DevTensor &t = W("kokopop.decoder.generator.noise_convs.1.weight");
            const int OC = (int)t.ne[1], IC = (int)t.ne[0];
            h.resize((size_t)t.n);
            check_cuda(cudaMemcpy(h.data(), t.d, h.size() * 4, cudaMemcpyDeviceToHost), "read noise conv");
            pack(packed["noise_convs.1"], OC, IC, 1, [&](int oc, int ic, int) { return h[(size_t)oc * IC + ic]; });
        }
        // noise_convs.0 (k=12, stride 6, pad 3) as 2 taps over the
        // space-to-depth operand: channel r*22+ic, tap j <- W[oc][ic][6j + r]
        {
            const DevTensor &t = W("kokopop.decoder.generator.noise_convs.0.weight");
            const int OC = (int)t.ne[1], K = 12, IC = (int)(t.ne[0] / K);
            if (IC * K != (int)t.ne[0] || IC != 22) throw KKError(KK_ERROR_MODEL, "noise_convs.0 shape mismatch");
            h.resize((size_t)t.n);
            check_cuda(cudaMemcpy(h.data(), t.d, h.size() * 4, cudaMemcpyDeviceToHost), "read noise conv");
            pack(packed["noise_convs.0.s2d"], OC, 6 * IC, 2, [&](int oc, int c6, int j) {
                const int r = c6 / IC, ic = c6 % IC;
                return h[((size_t)oc * IC + ic) * K + 6 * j + r];
            });
        }
        for (int s = 0; s < 2; ++s) {
            const DevTensor &t = W("kokopop.decoder.generator.ups." + std::to_string(s) + ".weight");
            const int OC = (int)t.ne[1], IC = (int)t.ne[2], S = strides[s];
            const std::vector<float> &ph = phase_host[s];
            const int NC = convt_phase_nc(S, OC);
            if (NC > 0 && !convt_phases) {
                // k_convt_tc: tile nt holds the S phases of channels
                // [nt NC, nt NC + NC), row n = r NC + c (phase r, channel c)
                const int N = S * NC;
                pack(
                    packed["ups." + std::to_string(s) + ".inter"], OC / NC * N, IC, 2,
                    [&](int v, int ic, int k) {
                        const int nt = v / N, r = (v % N) / NC, oc = nt * NC + (v % N) % NC;
                        return ph[(((size_t)r * OC + oc) * IC + ic) * 2 + k];
                    },
                    N);
            } else if (OC % 128 == 0) {
                // all phases as one convolution, phase-major output channels
                // n = r * OC + oc, so the CTAs writing the interleaved rows of
                // one position tile run together
                pack(packed["ups." + std::to_string(s) + ".phases"], S * OC, IC, 2,
                     [&](int n, int ic, int k) { return ph[((size_t)n * IC + ic) * 2 + k]; });
            } else {
                for (int r = 0; r < S; ++r)
                    pack(packed["ups." + std::to_string(s) + ".phase." + std::to_string(r)], OC, IC, 2,
                         [&](int oc, int ic, int k) { return ph[(((size_t)r * OC + oc) * IC + ic) * 2 + k]; });
            }
        }
    }
    // AdaIN sites
    sites.clear();
    site_total_C = 0;
    std::vector<std::string> site_list = adain_site_prefixes();
    const size_t n_required_sites = site_list.size();
    for (const auto &p : prosody_site_prefixes()) site_list.push_back(p);
    for (size_t si_i = 0; si_i < site_list.size(); ++si_i) {
        const std::string &p = site_list[si_i];
        const DevTensor *gw = Wopt(p + ".fc.gamma.weight"), *gb = Wopt(p + ".fc.gamma.bias");
        const DevTensor *bw = Wopt(p + ".fc.beta.weight"), *bb = Wopt(p + ".fc.beta.bias");
        if (!gw || !gb || !bw || !bb || !Wopt(p + ".norm.weight") || !Wopt(p + ".norm.bias")) {
            if (si_i < n_required_sites) {
                if (missing.empty()) missing = p + ".fc/norm";
                ok = false;
            }
            continue;
        }
        SiteInfo si;
        si.prefix = p;
        si.C = (int)gw->ne[1];
        si.f16 = gw->f16;
        // transpose [C][128] -> [128][C] for coalesced reads in adain_affine
        {
            const int C = si.C;
            std::vector<float> h((size_t)C * kStyle), t2((size_t)2 * C * kStyle);
            for (int which = 0; which < 2; ++which) {
                check_cuda(cudaMemcpy(h.data(), (which ? bw : gw)->d, h.size() * 4, cudaMemcpyDeviceToHost),
                           "read adain fc");
                for (int c = 0; c < C; ++c)
                    for (int i = 0; i < kStyle; ++i) t2[(size_t)which * C * kStyle + (size_t)i * C + c] = h[(size_t)c * kStyle + i];
            }
            DevBuf &db = adain_t[p];
            db.ensure(t2.size() * 4);
            check_cuda(cudaMemcpy(db.p, t2.data(), t2.size() * 4, cudaMemcpyHostToDevice), "upload adain fc");
            si.gw = (const float *)db.p;
            si.bw = (const float *)db.p + (size_t)C * kStyle;
        }
        si.gb = gb->d;
        si.bb = bb->d;
        si.off = site_total_C;
        site_total_C += si.C;
        site_index[p] = (int)sites.size();
        sites.push_back(si);
    }
    // harmonic source constants (audio_utils.cpp:145-176)
    const std::string mw_n = "kokopop.decoder.generator.m_source.l_linear.weight";
    const std::string mb_n = "kokopop.decoder.generator.m_source.l_linear.bias";
    if (need(mw_n) && need(mb_n)) {
        const DevTensor &mw = W(mw_n), &mb = W(mb_n);
        if (mw.host.size() < (size_t)kHarmonics || mb.host.empty())
            throw KKError(KK_ERROR_MODEL, "invalid harmonic source merge weight size");
        for (int h = 0; h < kHarmonics; ++h) sine.mw_scaled[h] = mw.host[h] * 0.1f;
        sine.mb = mb.host[0];
        sine.unvoiced = (float)std::tanh((double)sine.mb);  // correctly rounded, as in the kernel
    } else {
        ok = false;
    }
    // remaining generator / decoder tensors
    for (const char *n : {"kokopop.decoder.generator.conv_post.weight", "kokopop.decoder.generator.conv_post.bias",
                          "kokopop.decoder.generator.noise_convs.0.weight", "kokopop.decoder.generator.noise_convs.1.weight"})
        ok = need(n) && ok;
    generator_ready = ok;
    bool dok = ok;
    for (const char *n : {"kokopop.decoder.F0_conv.weight", "kokopop.decoder.N_conv.weight",
                          "kokopop.decoder.asr_res.0.weight", "kokopop.decoder.encode.conv1.weight",
                          "kokopop.decoder.decode.3.pool.weight"})
        dok = need(n) && dok;
    decoder_ready = dok;
    // prosody predictor F0 / N chain (optional)
    {
        bool pok = true;
        missing_prosody.clear();
        auto needp = [&](const std::string &n) {
            if (!Wopt(n)) {
                if (missing_prosody.empty()) missing_prosody = n;
                pok = false;
            }
        };
        for (const char *sfx : {"", "_reverse"})
            for (const char *w : {"weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0"})
                needp(std::string("kokopop.predictor.shared.") + w + sfx);
        for (const char *br : {"F0", "N"}) {
            for (int i = 0; i < 3; ++i) {
                const std::string p = std::string("kokopop.predictor.") + br + "." + std::to_string(i);
                for (const char *w : {".conv1.weight", ".conv1.bias", ".conv2.weight", ".conv2.bias"}) needp(p + w);
                for (const char *nm : {".norm1", ".norm2"})
                    if (site_index.find(p + nm) == site_index.end()) needp(p + nm + ".fc.gamma.weight");
            }
            needp(std::string("kokopop.predictor.") + br + ".1.pool.weight");
            needp(std::string("kokopop.predictor.") + br + "_proj.weight");
            needp(std::string("kokopop.predictor.") + br + "_proj.bias");
        }
        prosody_ready = pok;
    }
    // text encoder (optional)
    {
        missing_text.clear();
        auto needt = [&](const std::string &n) {
            if (!Wopt(n) && missing_text.empty()) missing_text = n;
        };
        needt("kokopop.text_encoder.embedding.weight");
        for (int i = 0; i < 3; ++i) {
            const std::string p = "kokopop.text_encoder.cnn." + std::to_string(i);
            for (const char *w : {".0.weight", ".0.bias", ".1.gamma", ".1.beta"}) needt(p + w);
        }
        for (const char *sfx : {"", "_reverse"})
            for (const char *w : {"weight_ih_l0", "weight_hh_l0", "bias_ih_l0", "bias_hh_l0"})
                needt(std::string("kokopop.text_encoder.lstm.") + w + sfx);
        text_ready = missing_text.empty();
    }
    // ALBERT + bert_encoder (optional)
    {
        missing_albert.clear();
        auto needa = [&](const std::string &n) {
            if (!Wopt(n) && missing_albert.empty()) missing_albert = n;
        };
        for (const char *n : {"word_embeddings.weight", "position_embeddings.weight", "token_type_embeddings.weight",
                              "LayerNorm.weight", "LayerNorm.bias"})
            needa(std::string("kokopop.albert.embeddings.") + n);
        for (const auto &n : albert_linears()) {
            needa(n);
            needa(n.substr(0, n.size() - 6) + "bias");
        }
        for (const char *n : {"attention.LayerNorm.weight", "attention.LayerNorm.bias",
                              "full_layer_layer_norm.weight", "full_layer_layer_norm.bias"})
            needa(std::string(kAlbertLayer) + n);
        albert_ready = missing_albert.empty();
    }
    // tables
    StftTables stt;
    IstftTables ist;
    make_tables(stt, ist);
    d_tables.ensure(sizeof(StftTables) + sizeof(IstftTables));
    check_cuda(cudaMemcpy(d_tables.p, &stt, sizeof stt, cudaMemcpyHostToDevice), "upload tables");
    check_cuda(cudaMemcpy((char *)d_tables.p + sizeof(StftTables), &ist, sizeof ist, cudaMemcpyHostToDevice),
               "upload tables");
}

// ---------------------------------------------------------------------------
// packed ragged-batch plan
// ---------------------------------------------------------------------------

Plan kk::make_plan(const int32_t *lens, int n) {
    Plan P;
    P.n = n;
    P.T.assign(lens, lens + n);
    P.off.resize(n);
    P.cum.resize(n);
    int64_t off = 8, cum = 0;
    P.maxT = 0;
    for (int u = 0; u < n; ++u) {
        if (lens[u] < 1 || lens[u] > kMaxFrames)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "utterance length out of range [1, 8192]");
        P.off[u] = off;
        P.cum[u] = cum;
        off += ((int64_t)lens[u] + 4 + 7) / 8 * 8;
        cum += lens[u];
        if (lens[u] > P.maxT) P.maxT = lens[u];
    }
    P.S = off;
    P.total = cum;
    return P;
}

const LstmLayer &kk_ctx::lstm_layer(const std::string &prefix) {
    auto it = lstm.find(prefix);
    if (it != lstm.end()) return it->second;
    const DevTensor &wf = W(prefix + ".weight_ih_l0"), &wb = W(prefix + ".weight_ih_l0_reverse");
    const DevTensor &hf = W(prefix + ".weight_hh_l0"), &hb = W(prefix + ".weight_hh_l0_reverse");
    const DevTensor &bif = W(prefix + ".bias_ih_l0"), &bib = W(prefix + ".bias_ih_l0_reverse");
    const DevTensor &bhf = W(prefix + ".bias_hh_l0"), &bhb = W(prefix + ".bias_hh_l0_reverse");
    // load_lstm_weights (graph_ops.cpp:1439-1450): w_ih ne [in, 4H], w_hh ne [H, 4H]
    const int64_t H = hf.ne[0], H4 = hf.ne[1], in = wf.ne[0];
    if (H != 256 || H4 != 4 * H || hb.ne[0] != H || hb.ne[1] != H4 || wf.ne[1] != H4 || wb.ne[0] != in ||
        wb.ne[1] != H4 || bif.n != H4 || bib.n != H4 || bhf.n != H4 || bhb.n != H4)
        throw KKError(KK_ERROR_MODEL, "unsupported LSTM shapes (hidden must be 256): " + prefix);
    if (wf.f16 != wb.f16) throw KKError(KK_ERROR_MODEL, "mixed W_ih types: " + prefix);
    LstmLayer L;
    L.in_dim = (int)in;
    L.H = (int)H;
    L.f16 = wf.f16;
    const size_t nw = (size_t)H4 * in;
    L.wih.ensure(2 * nw * sizeof(float));
    check_cuda(cudaMemcpy(L.wih.p, wf.d, nw * sizeof(float), cudaMemcpyDeviceToDevice), "stack W_ih");
    check_cuda(cudaMemcpy((float *)L.wih.p + nw, wb.d, nw * sizeof(float), cudaMemcpyDeviceToDevice), "stack W_ih");
    L.bih_buf.ensure(2 * (size_t)H4 * sizeof(float));
    check_cuda(cudaMemcpy(L.bih_buf.p, bif.d, (size_t)H4 * 4, cudaMemcpyDeviceToDevice), "stack b_ih");
    check_cuda(cudaMemcpy((float *)L.bih_buf.p + H4, bib.d, (size_t)H4 * 4, cudaMemcpyDeviceToDevice), "stack b_ih");
    L.bih.d = (float *)L.bih_buf.p;
    L.bih.ne[0] = 2 * H4;
    L.bih.n = 2 * H4;
    if (L.f16 || f32_split) {
        // F16: the weights as they are; F32: split hi + lo (pack_tc_split)
        check_cuda(conv_tc_init(), "tensor-core conv init");
        std::vector<float> h(2 * nw);
        check_cuda(cudaMemcpy(h.data(), L.wih.p, h.size() * 4, cudaMemcpyDeviceToHost), "read W_ih");
        auto get = [&](int oc, int ic, int) { return h[(size_t)oc * in + ic]; };
        if (L.f16)
            pack_tc(L.wih_tc, (int)(2 * H4), (int)in, 1, get);
        else
            pack_tc_split(L.wih_tc, (int)(2 * H4), (int)in, 1, get);
    }
    L.whh[0] = hf.d;
    L.whh[1] = hb.d;
    L.bhh[0] = bhf.d;
    L.bhh[1] = bhb.d;
    return lstm.emplace(prefix, std::move(L)).first->second;
}

// load_vocos (src/arch/sanotts/sano_arch.cpp:1081-1180): the range checks of
// the voice's decoder hyper-parameters, the tensor shapes, then the
// packings and the inverse-FFT tables.
const VocosNet &kk_ctx::vocos_net(const std::string &prefix, const kk_vocos_params &p) {
    auto it = vocos.find(prefix);
    if (it != vocos.end() && std::memcmp(&it->second.p, &p, sizeof p) == 0) return it->second;
    const auto bad = [&](const char *what) { throw KKError(KK_ERROR_INVALID_ARGUMENT, std::string("vocos: ") + what); };
    if (p.dim < 1 || p.dim > 1024 || p.pw_hidden < 1 || p.pw_hidden > 1024) bad("dim and pw_hidden must be in [1, 1024]");
    if (p.blocks < 0 || p.blocks > 64) bad("blocks out of range");
    if (p.dw_kernel < 1 || p.dw_kernel % 2 == 0 || p.embed_kernel < 1 || p.embed_kernel % 2 == 0 || p.dw_kernel > 63 ||
        p.embed_kernel > 63)
        bad("kernels must be odd (at most 63)");
    if (p.mels < 1 || p.mels > 1024 || p.noise_ch < 1 || p.noise_ch > 1024) bad("mels / noise_ch out of range");
    if (p.n_fft < 64 || p.n_fft > 2048 || (p.n_fft & (p.n_fft - 1))) bad("n_fft must be a power of two in [64, 2048]");
    if (p.hop < 1 || p.hop > p.n_fft) bad("hop must lie in (0, n_fft]");
    if (!std::isfinite(p.dc_pole) || std::fabs(p.dc_pole) >= 1.0f) bad("dc_pole must be a stable pole in (-1, 1)");
    if (!std::isfinite(p.mag_clip) || p.mag_clip <= 0.0f) bad("mag_clip must be finite and positive");
    if (it != vocos.end()) {
        VocosNet &v = it->second;
        v.embed.buf.release();
        v.noise.buf.release();
        v.head.buf.release();
        for (auto &q : v.pw0) q.buf.release();
        for (auto &q : v.pw1) q.buf.release();
        v.tables.release();
        vocos.erase(it);
    }
    const int64_t D = p.dim, Hd = p.pw_hidden, bins = p.n_fft / 2 + 1;
    const auto get = [&](const std::string &suffix, int64_t ne0, int64_t ne1) -> const DevTensor & {
        const DevTensor &t = W(prefix + suffix);
        if (t.ne[0] != ne0 || t.ne[1] != ne1 || t.ne[2] != 1 || t.ne[3] != 1)
            throw KKError(KK_ERROR_MODEL, "vocos: tensor " + prefix + suffix + " has the wrong shape");
        return t;
    };
    VocosNet v;
    v.p = p;
    const DevTensor &ew = get("dec.embed.weight", (int64_t)p.mels * p.embed_kernel, D);
    const DevTensor &nw = get("dec.noise.weight", (int64_t)p.noise_ch * p.embed_kernel, D);
    const DevTensor &hw = get("dec.head.weight", D, 2 * bins);
    v.embed_b = &get("dec.embed.bias", D, 1);
    v.noise_b = &get("dec.noise.bias", D, 1);
    v.norm_w = &get("dec.norm.weight", D, 1);
    v.norm_b = &get("dec.norm.bias", D, 1);
    v.final_w = &get("dec.final_norm.weight", D, 1);
    v.final_b = &get("dec.final_norm.bias", D, 1);
    v.head_b = &get("dec.head.bias", 2 * bins, 1);
    std::vector<const DevTensor *> pw0w, pw1w;
    for (int i = 0; i < p.blocks; ++i) {
        const std::string b = "dec.blocks." + std::to_string(i) + ".";
        v.dw_w.push_back(&get(b + "dw.weight", p.dw_kernel, D));
        v.dw_b.push_back(&get(b + "dw.bias", D, 1));
        v.ln_w.push_back(&get(b + "norm.weight", D, 1));
        v.ln_b.push_back(&get(b + "norm.bias", D, 1));
        pw0w.push_back(&get(b + "pw0.weight", D, Hd));
        v.pw0_b.push_back(&get(b + "pw0.bias", Hd, 1));
        pw1w.push_back(&get(b + "pw1.weight", Hd, D));
        v.pw1_b.push_back(&get(b + "pw1.bias", D, 1));
        v.gamma.push_back(&get(b + "gamma", D, 1));
    }
    // one tensor-core packing for all the linears: F16 as stored, F32 split
    std::vector<const DevTensor *> lin = {&ew, &nw, &hw};
    lin.insert(lin.end(), pw0w.begin(), pw0w.end());
    lin.insert(lin.end(), pw1w.begin(), pw1w.end());
    const bool f16 = ew.f16;
    for (const DevTensor *t : lin)
        if (t->f16 != f16) throw KKError(KK_ERROR_MODEL, "vocos: the stem, pointwise and head weights mix F16 and F32");
    if (!f16 && !f32_split)
        throw KKError(KK_ERROR_MODEL, "vocos: F32 weights need the split tensor-core path (KOKOPOP_B200_F32_SPLIT)");
    check_cuda(conv_tc_init(), "tensor-core conv init");
    const auto pack = [&](PackedW &pw, const DevTensor &t, int OC, int IC, int K) {
        std::vector<float> h((size_t)t.n);
        check_cuda(cudaMemcpy(h.data(), t.d, h.size() * 4, cudaMemcpyDeviceToHost), "read vocos weight");
        // ggml [IC * K, OC] (im2col order ic * K + k), or [IC, OC] for K = 1
        auto g = [&](int oc, int ic, int k) { return h[((size_t)oc * IC + ic) * K + k]; };
        if (f16)
            pack_tc(pw, OC, IC, K, g);
        else
            pack_tc_split(pw, OC, IC, K, g);
    };
    pack(v.embed, ew, (int)D, p.mels, p.embed_kernel);
    pack(v.noise, nw, (int)D, p.noise_ch, p.embed_kernel);
    pack(v.head, hw, (int)(2 * bins), (int)D, 1);
    v.pw0.resize(p.blocks);
    v.pw1.resize(p.blocks);
    for (int i = 0; i < p.blocks; ++i) {
        pack(v.pw0[i], *pw0w[i], (int)Hd, (int)D, 1);
        pack(v.pw1[i], *pw1w[i], (int)D, (int)Hd, 1);
    }
    // istft()'s RealRadix2 plan tables (src/audio/istft.cpp:82-162), each
    // value computed in double and rounded once
    const int n = p.n_fft, half = n / 2;
    std::vector<float> fl((size_t)2 * n + 2 * half + 2 * half, 0.f);
    float *win = fl.data(), *wsq = win + n, *stc = wsq + n, *sts = stc + half, *spc = sts + half, *sps = spc + half;
    for (int i = 0; i < n; ++i) {
        win[i] = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * (double)i / (double)n));
        wsq[i] = win[i] * win[i];
    }
    for (int h = 1; h < half; h <<= 1) {
        const int step = half / (2 * h);
        for (int k = 0; k < h; ++k) {
            const double a = 2.0 * M_PI * (double)(k * step) / (double)half;
            stc[h - 1 + k] = (float)std::cos(a);
            sts[h - 1 + k] = (float)std::sin(a);
        }
    }
    for (int k = 0; k < half; ++k) {
        const double a = 2.0 * M_PI * (double)k / (double)n;
        spc[k] = (float)std::cos(a);
        sps[k] = (float)std::sin(a);
    }
    int lg = 0;
    while ((1 << lg) < half) ++lg;
    std::vector<int> rev((size_t)half);
    for (int i = 0; i < half; ++i) {
        int r = 0;
        for (int b = 0; b < lg; ++b) r = (r << 1) | ((i >> b) & 1);
        rev[(size_t)i] = r;
    }
    const size_t fb = fl.size() * sizeof(float);
    v.tables.ensure(fb + rev.size() * sizeof(int));
    check_cuda(cudaMemcpy(v.tables.p, fl.data(), fb, cudaMemcpyHostToDevice), "upload vocos tables");
    check_cuda(cudaMemcpy((char *)v.tables.p + fb, rev.data(), rev.size() * sizeof(int), cudaMemcpyHostToDevice),
               "upload vocos tables");
    const float *d = (const float *)v.tables.p;
    v.tab.window = d;
    v.tab.window_sq = d + n;
    v.tab.stage_cos = d + 2 * n;
    v.tab.stage_sin = d + 2 * n + half;
    v.tab.split_cos = d + 2 * n + 2 * half;
    v.tab.split_sin = d + 2 * n + 3 * half;
    v.tab.rev = (const int *)((const char *)v.tables.p + fb);
    return vocos.emplace(prefix, std::move(v)).first->second;
}

// ---------------------------------------------------------------------------
// the forward pass
// ---------------------------------------------------------------------------

namespace {

// An activation operand of a convolution: F32 channel-major [C][R] for the
// CUDA-core path, or half chunk-major [C/8][Ry][8] with zero margins for the
// tensor-core path (h addresses row 0 of chunk 0, Ry = half_stride(R)).
// Its gap rows, margins and padding channels read as zero.
struct Op {
    float *f = nullptr;
    __half *h = nullptr;
    int64_t R = 0;
    int64_t Ry = 0;
    bool split = false;  // half operand of split F32: lo chunks after the hi ones
    // element offset of the lo half of a C-channel split operand (0: none)
    int64_t lo(int C) const { return split ? (int64_t)((C + 63) / 64 * 64) * Ry : 0; }
};

struct Runner {
    kk_ctx &c;
    const Plan &P;
    cudaStream_t st;
    Batch B{};
    const int64_t *d_cum = nullptr;
    float2 *ms = nullptr;
    float2 *ms2 = nullptr;  // a second set, for the conv that writes the next AdaIN input
    float2 *ms3 = nullptr;  // statistics computed just before a fused-operand conv
    float *gbase = nullptr, *bbase = nullptr;
    const bool tc;
    const bool split;  // F32 weights split over the half tensor cores

    // tc_path: the tensor-core path (default: the context's mode, split F32
    // included); split_path: with tc_path set, its operands split F32
    Runner(kk_ctx &ctx, const Plan &plan, cudaStream_t s, int tc_path = -1, bool split_path = false)
        : c(ctx), P(plan), st(s), tc(tc_path < 0 ? ctx.tc_mode : tc_path != 0),
          split(tc_path < 0 ? ctx.tc_mode && ctx.split_mode : tc_path != 0 && split_path) {}

    int64_t R(int m) const { return P.R(m); }

    void setup_batch() {
        const size_t n = (size_t)P.n;
        c.h_batch.resize(n * 5 + 8);
        int32_t *hT = (int32_t *)c.h_batch.data();
        int64_t *hoff = c.h_batch.data() + (n + 1) / 2 + 1;
        int64_t *hcum = hoff + n;
        for (size_t u = 0; u < n; ++u) {
            hT[u] = P.T[u];
            hoff[u] = P.off[u];
            hcum[u] = P.cum[u];
        }
        const size_t bytes = (size_t)((char *)(hcum + n) - (char *)hT);
        c.d_batch.ensure(bytes);
        c.upload(c.d_batch.p, hT, bytes, st, "upload batch");
        char *base = (char *)c.d_batch.p;
        B.n = P.n;
        B.T = (const int32_t *)base;
        B.offT = (const int64_t *)(base + ((char *)hoff - (char *)hT));
        d_cum = (const int64_t *)(base + ((char *)hcum - (char *)hT));
    }

    void setup_adain(const float *style_dev) {
        const size_t n = (size_t)P.n;
        gbase = c.buf("gamma", n * (size_t)c.site_total_C);
        bbase = c.buf("beta", n * (size_t)c.site_total_C);
        c.h_sites.resize(c.sites.size());
        for (size_t i = 0; i < c.sites.size(); ++i) {
            const SiteInfo &s = c.sites[i];
            AdainSite &a = c.h_sites[i];
            a.gw = s.gw;
            a.gb = s.gb;
            a.bw = s.bw;
            a.bb = s.bb;
            a.C = s.C;
            a.f16 = s.f16;
            a.gamma = gbase + n * (size_t)s.off;
            a.beta = bbase + n * (size_t)s.off;
        }
        c.d_sites.ensure(c.h_sites.size() * sizeof(AdainSite));
        c.upload(c.d_sites.p, c.h_sites.data(), c.h_sites.size() * sizeof(AdainSite), st, "upload adain sites");
        adain_affine((const AdainSite *)c.d_sites.p, (int)c.h_sites.size(), style_dev, P.n, st);
        ++c.n_launches;
        ms = (float2 *)c.buf("stats", n * 1090 * 2);
        ms2 = (float2 *)c.buf("stats2", n * 1090 * 2);
        ms3 = (float2 *)c.buf("stats3", n * 1090 * 2);
    }

    const AdainSite &site(const std::string &prefix) {
        auto it = c.site_index.find(prefix);
        if (it == c.site_index.end()) throw KKError(KK_ERROR_MODEL, "missing AdaIN weights: " + prefix);
        return c.h_sites[it->second];
    }

    // sum over utterances of the length at level m (+ extra per utterance)
    int64_t sum_len(int m, int extra) const { return (int64_t)m * P.total + (int64_t)extra * P.n; }

    // The operand buffer of a level (multiplier m) with room for C channels.
    Op op(const char *name, int m, int C) { return op(name, m, C, tc, split); }

    // half == true: the tensor-core operand whatever the context's mode;
    // split: with room for the lo halves of split F32
    Op op(const char *name, int m, int C, bool half, bool sp = false) {
        Op o;
        o.R = R(m);
        o.Ry = o.R;
        if (half) {
            const int cpad = (C + 63) / 64 * 64 * (sp ? 2 : 1);
            o.Ry = half_stride(o.R);
            o.h = (__half *)c.buf(name, ((size_t)cpad * o.Ry + 1) / 2) + kHalfLo * 8;
            o.split = sp;
        } else {
            o.f = c.buf(name, (size_t)C * o.R);
        }
        return o;
    }

    void zero(const Op &o, int C) {
        if (o.h)
            check_cuda(cudaMemsetAsync(o.h - kHalfLo * 8, 0,
                                       (size_t)((C + 63) / 64 * 64) * (o.split ? 2 : 1) * o.Ry * sizeof(__half), st),
                       "memset");
        else
            check_cuda(cudaMemsetAsync(o.f, 0, (size_t)C * o.R * sizeof(float), st), "memset");
    }

    struct Epi {
        const DevTensor *bias = nullptr;
        const float *resid = nullptr;
        int64_t R_resid = 0;
        int resid_half = 0;
        float scale1 = 1.f;
        int accum = 0;
        float scale2 = 1.f;
        int64_t omul = 1, oadd = 0;
        int64_t valid = 0;  // valid output positions (algorithmic FLOP count)
        const float *chscale = nullptr;  // per output channel, after bias and residual (tensor-core path)
        // non-null: the instance-norm terms (mean, scale) of the output over
        // the utterances of level (sm, sextra), for the AdaIN that reads it next
        float2 *stats = nullptr;
        int sm = 1, sextra = 0;
    };

    void timed_begin(cudaEvent_t &e0, cudaEvent_t &e1, cudaStream_t s = nullptr) {
        if (!c.profiling) return;
        e0 = c.take_event();
        e1 = c.take_event();
        check_cuda(cudaEventRecord(e0, s ? s : st), "event");
    }

    void timed_end(cudaEvent_t e0, cudaEvent_t e1, int kind, int taps, double flop, double bytes,
                   cudaStream_t s = nullptr) {
        ++c.n_launches;
        if (!c.profiling) return;
        check_cuda(cudaEventRecord(e1, s ? s : st), "event");
        c.timed.push_back({e0, e1, kind, taps, flop, bytes});
    }

    // One launch of `kind` (f enqueues it on s, default the runner's
    // stream), timed when profiling, with its algorithmic work.
    template <class F>
    void launch(int kind, double flop, double bytes, F &&f, cudaStream_t s = nullptr) {
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        timed_begin(e0, e1, s);
        f();
        timed_end(e0, e1, kind, 0, flop, bytes, s);
    }

    // algorithmic DRAM bytes of a convolution over `valid` output rows:
    // the operand read once (ebytes per input element), the output written
    // once, the residual and an accumulated output read once
    static double conv_bytes(int IC, int OC, double ebytes, int64_t valid, const Epi &e) {
        return (double)valid * ((double)IC * ebytes + 4.0 * OC * (1 + (e.resid ? 1 : 0) + (e.accum ? 1 : 0)));
    }

    // CUDA-core convolution on an F32 operand.
    void conv_f32(const float *w, bool f16, int OC, const float *in, int64_t R_in, int IC, int K, int s, int p,
                  int d, float *out, int64_t R_out, int64_t n_pos, const Epi &e) {
        ConvArgs a{};
        a.in = in;
        a.R_in = R_in;
        a.IC = IC;
        a.w = w;
        a.OC = OC;
        a.K = K;
        a.s = s;
        a.p = p;
        a.d = d;
        a.out = out;
        a.R_out = R_out;
        a.n_pos = n_pos;
        a.omul = e.omul;
        a.oadd = e.oadd;
        a.bias = e.bias ? e.bias->d : nullptr;
        a.resid = e.resid;
        a.R_resid = e.R_resid;
        a.resid_half = e.resid_half;
        a.scale1 = e.scale1;
        a.accum = e.accum;
        a.scale2 = e.scale2;
        a.round16 = f16 ? 1 : 0;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        timed_begin(e0, e1);
        conv_simt(a, st);
        timed_end(e0, e1, KK_PROF_CONV, K, 2.0 * OC * (double)IC * K * (double)e.valid,
                  conv_bytes(IC, OC, 4.0, e.valid, e));
    }

    // Tensor-core convolution on a half chunk-major operand.
    void conv_h(const PackedW &pw, const Op &in, int K, int p, int d, float *out, int64_t R_out, int64_t n_pos,
                const Epi &e, int phase_oc = 0, int phase_nc = 0) {
        if (in.split != (pw.a_wrap > 0))
            throw KKError(KK_ERROR_INFERENCE, "operand and weight packing disagree on the F32 split");
        ConvTcArgs a{};
        a.phase_oc = phase_oc;
        a.phase_nc = phase_nc;
        a.sched = (int *)((char *)c.d_err.p + offsetof(DevStatus, sched));
        a.in = in.h;
        a.R_in = in.Ry;
        a.IC_pad = pw.IC_pad;
        a.a_wrap = pw.a_wrap;
        a.acc_scale = pw.acc_scale;
        a.w = (const __half *)pw.buf.p;
        a.n_tiles = pw.n_tiles;
        // phase-interleaved packing: pw.OC counts the rows of all phases
        a.OC = phase_nc > 0 ? pw.OC / (int)e.omul : pw.OC;
        a.K = K;
        a.p = p;
        a.d = d;
        a.out = out;
        a.R_out = R_out;
        a.n_pos = n_pos;
        a.omul = e.omul;
        a.oadd = e.oadd;
        a.bias = e.bias ? e.bias->d : nullptr;
        a.resid = e.resid;
        a.R_resid = e.R_resid;
        a.resid_half = e.resid_half;
        a.chscale = e.chscale;
        a.scale1 = e.scale1;
        a.accum = e.accum;
        a.scale2 = e.scale2;
        a.err = (int *)c.d_err.p;
        a.stats = e.stats;
        a.sb = B;
        a.sm = e.sm;
        a.sextra = e.sextra;
        if (e.stats) {
            a.stats_aligned = aligned32(e.sm) ? 1 : 0;
            a.part = (float2 *)c.buf("stats_part", (size_t)pw.OC * (size_t)(R_out / 32) * 2);
        }
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        timed_begin(e0, e1);
        check_cuda(conv_tc(a, st), "tensor-core conv launch");
        // split F32 operands carry hi and lo halves: 4 bytes per input element
        timed_end(e0, e1, KK_PROF_CONV, K, 2.0 * pw.OC * (double)pw.IC * K * (double)e.valid,
                  conv_bytes(pw.IC, pw.OC, in.split ? 4.0 : 2.0, e.valid, e));
        if (e.stats) ++c.n_launches;  // the statistics pass
    }

    // Convolution by weight name on an operand of the current path (stride 1).
    void conv_w(const std::string &wname, const std::string &bname, const Op &in, int IC, int K, int p, int d,
                float *out, int64_t R_out, int64_t n_pos, Epi e, int64_t valid) {
        e.valid = valid;
        if (!bname.empty()) e.bias = &c.W(bname);
        const DevTensor &w = c.W(wname);
        const int OC = (int)(w.ne[2] > 1 ? w.ne[2] : w.ne[1]);
        if (w.n != (int64_t)OC * IC * K) throw KKError(KK_ERROR_MODEL, "conv weight shape mismatch: " + wname);
        if (tc) {
            auto it = c.packed.find(wname);
            if (it == c.packed.end()) throw KKError(KK_ERROR_MODEL, "no packed weight for " + wname);
            conv_h(it->second, in, K, p, d, out, R_out, n_pos, e);
        } else {
            conv_f32(w.d, w.f16, OC, in.f, in.R, IC, K, 1, p, d, out, R_out, n_pos, e);
            if (e.stats) stats_pass(out, R_out, OC, e.sm, e.sextra, e.stats);
        }
    }

    // every utterance of level m starts on a 32-row boundary
    bool aligned32(int m) const {
        for (int u = 0; u < P.n; ++u)
            if (((int64_t)m * P.off[u]) % 32 != 0) return false;
        return true;
    }

    // stats + AdaIN + activation into an operand (or an F32 buffer)
    // pre: the statistics of x when already known
    void adain_act(const std::string &prefix, const float *x, const Op &y, int64_t Rm, int C, int m, int extra,
                   int act, float slope, const std::string &alpha, const float2 *pre = nullptr) {
        const AdainSite &s = site(prefix);
        if (s.C != C) throw KKError(KK_ERROR_MODEL, "AdaIN channel mismatch: " + prefix);
        if (!pre) stats_pass(x, Rm, C, m, extra, ms);
        PrologueArgs a{};
        a.norm = 1;
        a.ms = pre ? pre : ms;
        a.norm_w = c.W(prefix + ".norm.weight").d;
        a.norm_b = c.W(prefix + ".norm.bias").d;
        a.gamma = s.gamma;
        a.beta = s.beta;
        a.act = act;
        a.slope = slope;
        a.alpha = alpha.empty() ? nullptr : c.W(alpha).d;
        a.round16 = 0;
        a.lo_off = y.lo(C);
        operand_pass(x, y, Rm, C, m, extra, a);
    }

    // x2 / x3: two more branches averaged in first, ((x + x2) + x3) * sum_scale
    void act_only(const float *x, const Op &y, int64_t Rm, int C, int m, int extra, int act, float slope,
                  const float *x2 = nullptr, const float *x3 = nullptr, float sum_scale = 1.f) {
        PrologueArgs a{};
        a.norm = 0;
        a.act = act;
        a.slope = slope;
        a.x2 = x2;
        a.x3 = x3;
        a.sum_scale = sum_scale;
        a.lo_off = y.lo(C);
        operand_pass(x, y, Rm, C, m, extra, a);
    }

    // The operand pass of one activation: F32 reads of x (and of the other
    // branches averaged in), the operand written once (half, hi + lo halves
    // for split F32, or F32 on the CUDA-core path).
    void operand_pass(const float *x, const Op &y, int64_t Rm, int C, int m, int extra, const PrologueArgs &a) {
        const double elems = (double)C * (double)sum_len(m, extra);
        const double in_b = 4.0 * (1 + (a.x2 ? 1 : 0) + (a.x3 ? 1 : 0));
        const double out_b = y.h ? (y.split ? 4.0 : 2.0) : 4.0;
        launch(KK_PROF_OPERAND, 0.0, elems * (in_b + out_b), [&] {
            if (y.h)
                prologue_h(x, y.h, Rm, y.Ry, C, m, extra, B, (int)(sum_len(m, extra) / P.n), a, st);
            else
                prologue(x, y.f, Rm, C, m, extra, B, m * P.maxT + extra, a, st);
        });
    }

    // Instance-norm statistics of x over the utterances of level (m, extra).
    void stats_pass(const float *x, int64_t Rm, int C, int m, int extra, float2 *out) {
        launch(KK_PROF_STATS, 0.0, 4.0 * C * (double)sum_len(m, extra),
               [&] { stats(x, Rm, C, m, extra, B, out, st); });
    }

    // adain_resblk1d (graph_ops.cpp:996-1065) with its input on level mi (1 or
    // 2; upsampling blocks take level 1 to level 2).
    void adain_resblk(const std::string &pf, const float *x, int Cin, bool up, float *out, int mi = 1) {
        if (mi != 1 && (mi != 2 || up)) throw KKError(KK_ERROR_INFERENCE, "unsupported resblock level");
        const int64_t Ri = R(mi);
        const DevTensor &c1 = c.W(pf + ".conv1.weight");
        const int Cout = (int)c1.ne[1];
        const int m = up ? 2 : mi;
        const int64_t Rc = R(m);
        Op opI = mi == 1 ? op("opT", 1, 1152) : op("op2", 2, 1152);
        Op opL = up ? op("op2", 2, 1152) : opI;
        float *tmp = m == 2 ? c.buf("tmp2", 512 * (size_t)R(2)) : c.buf("tmpT", 1024 * (size_t)R(1));
        if (Cout > (m == 2 ? 512 : 1024)) throw KKError(KK_ERROR_MODEL, "resblock too wide: " + pf);
        // shortcut: nearest x2 upsample (folded into the epilogue's row map)
        // then the bias-free 1x1 conv, on the raw input
        Epi e2;
        e2.scale1 = kInvSqrt2;
        e2.resid_half = up ? 1 : 0;
        e2.R_resid = Ri;
        if (c.Wopt(pf + ".conv1x1.weight")) {
            float *sc = c.buf("scT", 1024 * (size_t)Ri);
            Op xin;
            if (tc) {
                act_only(x, opI, Ri, Cin, mi, 0, ACT_NONE, 0.f);
                xin = opI;
            } else {
                xin.f = const_cast<float *>(x);
                xin.R = Ri;
            }
            conv_w(pf + ".conv1x1.weight", "", xin, Cin, 1, 0, 1, sc, Ri, Ri, Epi{}, sum_len(mi, 0));
            e2.resid = sc;
        } else {
            if (Cin != Cout) throw KKError(KK_ERROR_MODEL, "missing conv1x1 for " + pf);
            e2.resid = x;
        }
        // residual: AdaIN(norm1) -> LeakyReLU(0.2) -> [pool x2] -> conv1
        if (up) {
            const DevTensor &pw = c.W(pf + ".pool.weight"), &pb = c.W(pf + ".pool.bias");
            if (pw.ne[0] != 3 || pw.ne[1] != 1 || pw.ne[2] != Cin)
                throw KKError(KK_ERROR_MODEL, "invalid depthwise upsample pool shape: " + pf);
            // the pool reads F32 activations (the reference's dense F32 kernel)
            const int64_t R1 = R(1), R2 = R(2);
            const double el = (double)Cin * (double)sum_len(1, 0);
            if (tc) {
                // AdaIN + LeakyReLU applied by the pool as it reads x: reads
                // the frame level once, writes the doubled level
                const AdainSite &s = site(pf + ".norm1");
                if (s.C != Cin) throw KKError(KK_ERROR_MODEL, "AdaIN channel mismatch: " + pf + ".norm1");
                stats_pass(x, R1, Cin, 1, 0, ms);
                PrologueArgs a{};
                a.norm = 1;
                a.ms = ms;
                a.norm_w = c.W(pf + ".norm1.norm.weight").d;
                a.norm_b = c.W(pf + ".norm1.norm.bias").d;
                a.gamma = s.gamma;
                a.beta = s.beta;
                a.act = ACT_LEAKY;
                a.slope = 0.2f;
                launch(KK_PROF_OPERAND, 0.0, el * (4.0 + 2.0 * (opL.split ? 4.0 : 2.0)), [&] {
                    pool_up_adain_h(x, opL.h, R1, opL.Ry, Cin, pw.d, pb.d, B, P.maxT, opL.lo(Cin), a, st);
                });
            } else {
                Op pf32;
                pf32.f = c.buf("pfT", 1090 * (size_t)R1);
                pf32.R = R1;
                adain_act(pf + ".norm1", x, pf32, R1, Cin, 1, 0, ACT_LEAKY, 0.2f, "");
                launch(KK_PROF_OTHER, 0.0, el * (4.0 + 2.0 * 4.0),
                       [&] { pool_up(pf32.f, opL.f, R1, R2, Cin, pw.d, pb.d, B, P.maxT, 0, st); });
            }
        } else {
            adain_act(pf + ".norm1", x, opI, Ri, Cin, mi, 0, ACT_LEAKY, 0.2f, "");
        }
        conv_w(pf + ".conv1.weight", pf + ".conv1.bias", opL, Cin, 3, 1, 1, tmp, Rc, Rc, Epi{}, sum_len(m, 0));
        // AdaIN(norm2) -> LeakyReLU(0.2) -> conv2, + shortcut, * 1/sqrt(2)
        adain_act(pf + ".norm2", tmp, opL, Rc, Cout, m, 0, ACT_LEAKY, 0.2f, "");
        conv_w(pf + ".conv2.weight", pf + ".conv2.bias", opL, Cout, 3, 1, 1, out, Rc, Rc, e2, sum_len(m, 0));
    }

    // The prosody predictor's F0 and N chains after the shared biLSTM
    // (kokoro.cpp:682-708): x [512][R(1)] on the frame level -> three
    // adain_resblk1d kokopop.predictor.{F0,N}.{0,1,2} (the second upsamples
    // x2) -> the 1x1 projection {F0,N}_proj with bias -> f0p / np [1][R(2)].
    void prosody_chains(const float *x, int Cx, float *f0p, float *np) {
        const int64_t R1 = R(1), R2 = R(2);
        // operand gaps must read as zero (half operands on the tensor-core
        // path, F32 ones on the CUDA-core path)
        zero(op("opT", 1, 1152), 1152);
        zero(op("op2", 2, 1152), 1152);
        float *y0 = c.buf("pr_y0", 1024 * (size_t)R1);
        float *y1 = c.buf("pr_y1", 512 * (size_t)R2);
        float *y2 = c.buf("pr_y2", 512 * (size_t)R2);
        for (int br = 0; br < 2; ++br) {
            const std::string p = std::string("kokopop.predictor.") + (br ? "N" : "F0");
            const int C0 = (int)c.W(p + ".0.conv1.weight").ne[1];
            const int C1 = (int)c.W(p + ".1.conv1.weight").ne[1];
            const int C2 = (int)c.W(p + ".2.conv1.weight").ne[1];
            if (C0 > 1024 || C1 > 512 || C2 > 512) throw KKError(KK_ERROR_MODEL, "prosody block too wide: " + p);
            adain_resblk(p + ".0", x, Cx, false, y0);
            adain_resblk(p + ".1", y0, C0, true, y1);
            adain_resblk(p + ".2", y1, C1, false, y2, 2);
            Op in;
            if (tc) {
                in = op("op2", 2, 1152);
                act_only(y2, in, R2, C2, 2, 0, ACT_NONE, 0.f);
            } else {
                in.f = y2;
                in.R = R2;
            }
            conv_w(p + "_proj.weight", p + "_proj.bias", in, C2, 1, 0, 1, br ? np : f0p, R2, R2, Epi{},
                   sum_len(2, 0));
        }
    }

    // graph_generator_resblock: x_in -> (3 iterations) -> wb, the last
    // iteration writing final_out (accumulating / scaling) when given.
    // AdaIN + Snake of x (statistics x_stats, or computed here when null),
    // then the conv by weight name into out: inside the conv (k_conv_tcf)
    // where it applies, else the operand prologue into o and the conv.
    void adain_snake_conv(const std::string &adain, const std::string &alpha, const float *x, const float2 *x_stats,
                          const Op &o, int C, int m, int extra, const std::string &wname, const std::string &bname,
                          int K, int p, int d, float *out, Epi e) {
        const int64_t Rm = R(m);
        if (tc && !split && c.fuse_operand && K >= c.fuse_min_taps) {
            const AdainSite &s = site(adain);
            if (s.C != C) throw KKError(KK_ERROR_MODEL, "AdaIN channel mismatch: " + adain);
            auto it = c.packed.find(wname);
            if (it == c.packed.end()) throw KKError(KK_ERROR_MODEL, "no packed weight for " + wname);
            const PackedW &pw = it->second;
            ConvTcArgs a{};
            a.IC_pad = pw.IC_pad;
            a.w = (const __half *)pw.buf.p;
            a.n_tiles = pw.n_tiles;
            a.OC = pw.OC;
            a.K = K;
            a.p = p;
            a.d = d;
            a.out = out;
            a.R_out = Rm;
            a.n_pos = Rm;
            a.omul = 1;
            a.oadd = 0;
            a.bias = bname.empty() ? nullptr : c.W(bname).d;
            a.resid = e.resid;
            a.R_resid = e.R_resid;
            a.resid_half = e.resid_half;
            a.scale1 = e.scale1;
            a.accum = e.accum;
            a.scale2 = e.scale2;
            a.err = (int *)c.d_err.p;
            a.stats = e.stats;
            a.sb = B;
            a.sm = m;
            a.sextra = extra;
            if (e.stats) {
                a.stats_aligned = aligned32(m) ? 1 : 0;
                a.part = (float2 *)c.buf("stats_part", (size_t)pw.OC * (size_t)(Rm / 32) * 2);
            }
            a.x = x;
            a.x_ms = x_stats ? x_stats : ms3;
            a.x_nw = c.W(adain + ".norm.weight").d;
            a.x_nb = c.W(adain + ".norm.bias").d;
            a.x_gamma = s.gamma;
            a.x_beta = s.beta;
            a.x_alpha = c.W(alpha).d;
            if (pw.IC_pad == C && conv_tc_fusable(a)) {
                if (!x_stats) stats_pass(x, Rm, C, m, extra, ms3);
                cudaEvent_t e0 = nullptr, e1 = nullptr;
                timed_begin(e0, e1);
                check_cuda(conv_tc(a, st), "tensor-core conv launch (fused operand)");
                // the operand is read as F32 activations
                timed_end(e0, e1, KK_PROF_CONV, K, 2.0 * pw.OC * (double)pw.IC * K * (double)sum_len(m, extra),
                          conv_bytes(pw.IC, pw.OC, 4.0, sum_len(m, extra), e));
                if (e.stats) ++c.n_launches;
                return;
            }
        }
        adain_act(adain, x, o, Rm, C, m, extra, ACT_SNAKE, 0.f, alpha, x_stats);
        conv_w(wname, bname, o, C, K, p, d, out, Rm, Rm, e, sum_len(m, extra));
    }

    // x_in_stats: the statistics of x_in. A conv whose output feeds an AdaIN
    // leaves that output's statistics behind (ms after conv1, ms2 after conv2).
    void gen_resblock(const std::string &pf, int K, const float *x_in, float *wb, float *final_out, int accum,
                      float scale2, int C, int m, int extra, const Op &o, float *tmp, const float2 *x_in_stats) {
        const int64_t Rm = R(m);
        const float *cur = x_in;
        const float2 *cur_stats = x_in_stats;
        for (int i = 0; i < 3; ++i) {
            const std::string is = std::to_string(i);
            const int d = kDil[i];
            Epi e1;
            e1.stats = ms;
            e1.sm = m;
            e1.sextra = extra;
            adain_snake_conv(pf + ".adain1." + is, pf + ".alpha1." + is, cur, cur_stats, o, C, m, extra,
                             pf + ".convs1." + is + ".weight", pf + ".convs1." + is + ".bias", K, (K * d - d) / 2, d,
                             tmp, e1);
            Epi e;
            e.resid = cur;
            e.R_resid = Rm;
            float *out = wb;
            if (i == 2 && final_out) {
                out = final_out;
                e.accum = accum;
                e.scale2 = scale2;
            }
            if (i < 2) {
                e.stats = ms2;
                e.sm = m;
                e.sextra = extra;
            }
            adain_snake_conv(pf + ".adain2." + is, pf + ".alpha2." + is, tmp, ms, o, C, m, extra,
                             pf + ".convs2." + is + ".weight", pf + ".convs2." + is + ".bias", K, K / 2, 1, out, e);
            cur = wb;
            cur_stats = e.stats;
        }
    }

    // ggml_generator (audio_utils.cpp:594-1051) with the input at level gm.
    void generator(int gm, const float *x_in, float *har, float *audio) {
        static const struct {
            int kernel, up_stride, up_padding, noise_stride, noise_padding, noise_kernel;
        } sp[2] = {{7, 10, 5, 6, 3, 12}, {11, 6, 3, 1, 0, 1}};
        const int mlev[2] = {10 * gm, 60 * gm};
        const int extra[2] = {0, 1};
        const int64_t R_har = R(60 * gm);
        const float *x = x_in;
        const float *x2 = nullptr, *x3 = nullptr;  // further branches of x (averaged)
        int C = 512, m_prev = gm;
        Op op_prev = op("op2", gm, 1152);
        const std::string g = "kokopop.decoder.generator.";
        for (int s = 0; s < 2; ++s) {
            const int m = mlev[s];
            const int64_t Rm = R(m);
            const std::string ss = std::to_string(s);
            const DevTensor &ncw = c.W(g + "noise_convs." + ss + ".weight");
            const int Cs = (int)ncw.ne[1];
            float *xs = c.buf(("xs" + ss).c_str(), (size_t)Cs * Rm);
            float *xst = c.buf(("xst" + ss).c_str(), (size_t)Cs * Rm);
            // the three residual blocks' outputs, averaged by the consumer
            float *br[3] = {c.buf(("acc" + ss).c_str(), (size_t)Cs * Rm), c.buf(("xb" + ss).c_str(), (size_t)Cs * Rm),
                            c.buf(("xc" + ss).c_str(), (size_t)Cs * Rm)};
            float *tmp = c.buf(("tmp" + ss).c_str(), (size_t)Cs * Rm);
            Op o = op(s == 0 ? "op0" : "op1", m, Cs);
            // noise branch: noise_convs + noise_res (audio_utils.cpp:714-731)
            {
                Epi e;
                e.bias = &c.W(g + "noise_convs." + ss + ".bias");
                e.valid = sum_len(m, extra[s]);
                e.stats = ms2;
                e.sm = m;
                e.sextra = extra[s];
                const int K = sp[s].noise_kernel;
                if (ncw.n != (int64_t)Cs * 22 * K) throw KKError(KK_ERROR_MODEL, "noise_convs shape mismatch");
                if (tc && s == 0) {
                    // stride 6 as 2 taps over the space-to-depth operand
                    Op sd = op("s2d", m, 192);
                    launch(KK_PROF_OTHER, 0.0, (double)sum_len(60 * gm, 1) * 22 * (4.0 + (sd.split ? 4.0 : 2.0)),
                           [&] { har_s2d(har, R_har, sd.h, Rm, sd.Ry, sd.lo(192), st); });
                    e.valid = sum_len(m, extra[s]);
                    conv_h(c.packed.at("noise_convs.0.s2d"), sd, 2, 0, 1, xs, Rm, Rm, e);
                } else if (tc) {
                    Op hh = op("op1", m, Cs);
                    act_only(har, hh, R_har, 22, m, extra[s], ACT_NONE, 0.f);
                    conv_h(c.packed.at("noise_convs.1"), hh, 1, 0, 1, xs, Rm, Rm, e);
                } else {
                    conv_f32(ncw.d, ncw.f16, Cs, har, R_har, 22, K, sp[s].noise_stride, sp[s].noise_padding, 1, xs,
                             Rm, Rm, e);
                    stats_pass(xs, Rm, Cs, m, extra[s], ms2);
                }
            }
            gen_resblock(g + "noise_res." + ss, sp[s].kernel, xs, xs, nullptr, 0, 1.f, Cs, m, extra[s], o, tmp,
                         ms2);
            // LeakyReLU(0.1) then ConvTranspose as phase convolutions,
            // + bias, [reflect pad], + noise branch (audio_utils.cpp:687-760)
            const int64_t Rp = R(m_prev);
            act_only(x, op_prev, Rp, C, m_prev, 0, ACT_LEAKY, 0.1f, x2, x3, kThird);
            const DevTensor &uw = c.W(g + "ups." + ss + ".weight");
            const DevTensor &ub = c.W(g + "ups." + ss + ".bias");
            if ((int)uw.ne[1] != Cs || (int)uw.ne[2] != C) throw KKError(KK_ERROR_MODEL, "ups shape mismatch");
            const int S = sp[s].up_stride, crop = sp[s].up_padding, pad = s == 1 ? 1 : 0;
            auto inter = c.packed.find("ups." + ss + ".inter");
            auto all_phases = inter != c.packed.end() ? inter : c.packed.find("ups." + ss + ".phases");
            if (tc && all_phases != c.packed.end()) {
                Epi e;
                e.bias = &ub;
                e.resid = xs;
                e.R_resid = Rm;
                e.omul = S;
                e.oadd = -crop + pad;
                e.valid = sum_len(m_prev, 0);
                if (inter != c.packed.end())
                    conv_h(inter->second, op_prev, 2, 1, 1, xst, Rm, Rp, e, 0, convt_phase_nc(S, Cs));
                else
                    conv_h(all_phases->second, op_prev, 2, 1, 1, xst, Rm, Rp, e, Cs);
            }
            for (int r = 0; r < S && !(tc && all_phases != c.packed.end()); ++r) {
                Epi e;
                e.bias = &ub;
                e.resid = xs;
                e.R_resid = Rm;
                e.omul = S;
                e.oadd = r - crop + pad;
                e.valid = sum_len(m_prev, 0);
                if (tc) {
                    const PackedW &pw = c.packed.at("ups." + ss + ".phase." + std::to_string(r));
                    conv_h(pw, op_prev, 2, 1, 1, xst, Rm, Rp, e);
                } else {
                    conv_f32((const float *)c.convt_phase[s].p + (size_t)r * Cs * C * 2, c.convt_f16[s], Cs,
                             op_prev.f, Rp, C, 2, 1, 1, 1, xst, Rm, Rp, e);
                }
            }
            if (pad) {
                ConvTRow0Args a{};
                a.in = op_prev.f;
                a.in_h = op_prev.h;
                a.lo_off = op_prev.lo(C);
                a.R_in = op_prev.h ? op_prev.Ry : Rp;
                a.IC = C;
                a.m_in = m_prev;
                a.w = uw.d;
                a.OC = Cs;
                a.K = (int)uw.ne[0];
                a.crop = crop;
                a.m_out = m;
                a.bias = ub.d;
                a.add = xs;
                a.out = xst;
                a.R_out = Rm;
                a.round16 = uw.f16 ? 1 : 0;
                launch(KK_PROF_OTHER, 0.0, 8.0 * Cs * P.n, [&] { convt_row0(a, B, st); });
            }
            // three main resblocks, averaged (graph_ops.cpp:1300-1320); they
            // share the input, so its statistics are computed once
            float2 *ms_stage = (float2 *)c.buf("stats_stage", (size_t)P.n * 1090 * 2);
            stats_pass(xst, Rm, Cs, m, extra[s], ms_stage);
            for (int k = 0; k < 3; ++k) {
                const std::string pf = g + "resblocks." + std::to_string(s * 3 + k);
                gen_resblock(pf, kKs[k], xst, br[k], nullptr, 0, 1.f, Cs, m, extra[s], o, tmp, ms_stage);
            }
            // the stage output ((r0 + r1) + r2) / 3 is formed by the next
            // operand prologue (graph_ops.cpp:1300-1320)
            x = br[0];
            x2 = br[1];
            x3 = br[2];
            C = Cs;
            m_prev = m;
            op_prev = o;
        }
        // LeakyReLU(0.01) -> conv_post -> iSTFT (audio_utils.cpp:814-831, :1043)
        const int m = mlev[1];
        const int64_t Rm = R(m);
        act_only(x, op_prev, Rm, C, m, 1, ACT_LEAKY, 0.01f, x2, x3, kThird);
        float *post = c.buf("post", (size_t)22 * Rm);
        conv_w(g + "conv_post.weight", g + "conv_post.bias", op_prev, C, 7, 3, 1, post, Rm, Rm, Epi{},
               sum_len(m, 1));
        const IstftTables *it = (const IstftTables *)((char *)c.d_tables.p + sizeof(StftTables));
        // 22 post values read per frame, 5 samples written per frame
        const double frames = (double)sum_len(m, 1);
        launch(KK_PROF_ISTFT, 0.0, 88.0 * frames + 20.0 * (frames - P.n),
               [&] { istft(post, Rm, 60 * gm, audio, B, d_cum, it, P.maxT, st); });
    }

    // ---- LSTM stack: the plan is one "utterance" of R rows (rows t * B + b) ----

    // Sequences of a bidirectional layer: device lengths and output offsets.
    struct Seqs {
        int B = 0, max_len = 0;
        int64_t rows = 0;  // sum of lengths
        const int32_t *d_len = nullptr;
        const int64_t *d_cum = nullptr;
    };

    // bidirectional_lstm (graph_ops.cpp:1514-1529) over X [in_dim][R]:
    // hout [2H][R] (forward units first, the ggml_concat order).
    void bilstm(const LstmLayer &L, const float *X, float *hout, const Seqs &q) {
        const int64_t Rr = R(1);
        const int OC = 8 * L.H;
        float *pre = c.buf("lstm_pre", (size_t)OC * Rr);
        Epi e;
        e.bias = &L.bih;
        e.valid = q.rows;
        if (L.wih_tc.buf.p) {
            Op xh = op("lstm_xh", 1, L.in_dim, true, L.wih_tc.a_wrap > 0);
            zero(xh, L.in_dim);
            act_only(X, xh, Rr, L.in_dim, 1, 0, ACT_NONE, 0.f);
            conv_h(L.wih_tc, xh, 1, 0, 1, pre, Rr, Rr, e);
        } else {
            conv_f32((const float *)L.wih.p, L.f16, OC, X, Rr, L.in_dim, 1, 1, 0, 1, pre, Rr, Rr, e);
        }
        LstmRecArgs a{};
        a.pre = pre;
        a.R = Rr;
        a.whh[0] = L.whh[0];
        a.whh[1] = L.whh[1];
        a.bhh[0] = L.bhh[0];
        a.bhh[1] = L.bhh[1];
        a.hout = hout;
        a.len = q.d_len;
        a.B = q.B;
        a.max_len = q.max_len;
        a.err = (int *)c.d_err.p;
        // smallest group that keeps the clusters (2 per group) within one
        // wave of the device's co-resident clusters (16 when unknown)
        a.Bc = 32;
        for (int bc : {1, 2, 4, 8, 16, 32}) {
            const int fit = lstm_max_clusters(bc);
            if (2 * ((q.B + bc - 1) / bc) <= (fit > 0 ? fit : 16)) {
                a.Bc = bc;
                break;
            }
        }
        // per row and direction: the 4H pre-gates read, H outputs written,
        // 4H x H multiply-adds with W_hh (read from shared memory)
        const double rows = (double)q.rows, H = L.H;
        launch(KK_PROF_LSTM, 2.0 * 2.0 * 4.0 * H * H * rows, 2.0 * rows * (16.0 * H + 4.0 * H),
               [&] { check_cuda(lstm_recurrence(a, st), "LSTM recurrence launch"); });
    }

    // zero every operand buffer whose gaps must read as zero
    void zero_operands(int gm, bool decoder) {
        if (decoder) zero(op("opT", 1, 1152), 1152);
        zero(op("op2", gm, 1152), 1152);
        zero(op("op0", 10 * gm, 256), 256);
        zero(op("op1", 60 * gm, 128), 128);
        if (tc) zero(op("s2d", 10 * gm, 192), 192);
    }

    // harmonic source + STFT on the side stream, from the packed F0 (level mf)
    float *source_and_har(const float *f0p, int mf) {
        const int64_t Rh = R(60 * mf);
        float *har = c.buf("har", (size_t)22 * Rh);
        float *src = c.buf("source", (size_t)kUpsample * mf * (size_t)P.total + 1);
        check_cuda(cudaEventRecord(c.ev_inputs, st), "event");
        check_cuda(cudaStreamWaitEvent(c.st2, c.ev_inputs, 0), "wait");
        check_cuda(cudaMemsetAsync(har, 0, (size_t)22 * Rh * sizeof(float), c.st2), "memset har");
        // the source writes 300 mf samples per base frame; the STFT reads
        // them and writes 22 values per frame of 5 samples (+1 per utterance)
        const double samples = (double)kUpsample * mf * (double)P.total;
        launch(KK_PROF_SOURCE, 0.0, 4.0 * samples, [&] { sinegen(f0p, mf, src, B, d_cum, c.sine, c.st2); }, c.st2);
        const StftTables *tab = (const StftTables *)c.d_tables.p;
        launch(KK_PROF_SOURCE, 0.0, 4.0 * samples + 88.0 * (samples / 5.0 + P.n),
               [&] { stft(src, har, Rh, mf, B, d_cum, tab, P.maxT, c.st2); }, c.st2);
        check_cuda(cudaEventRecord(c.ev_src, c.st2), "event");
        return har;
    }

    // decoder encode / decode (kokoro.cpp:716-763) then the generator.
    void decoder_forward(const float *asr, const float *f0, const float *noise, const float *style, float *audio) {
        setup_batch();
        const int64_t R1 = R(1), R2 = R(2);
        // all_finite on the inputs, in the reference's order (kokoro.cpp:933-940);
        // indices are into the caller's arrays
        DevStatus *status = (DevStatus *)c.d_err.p;
        launch(KK_PROF_OTHER, 0.0, 4.0 * (516.0 * P.total), [&] {
            check_finite(f0, 2 * P.total, kFiniteF0, status, st);
            check_finite(noise, 2 * P.total, kFiniteNoise, status, st);
            check_finite(asr, 512 * P.total, kFiniteAsr, status, st);
        });
        c.n_launches += 2;
        float *Xenc = c.buf("Xenc", 514 * (size_t)R1);
        float *Xdec = c.buf("Xdec", 1090 * (size_t)R1);
        float *f0p = c.buf("f0p", (size_t)R2);
        float *np = c.buf("np", (size_t)R2);
        check_cuda(cudaMemsetAsync(f0p, 0, (size_t)R2 * 4, st), "memset");
        check_cuda(cudaMemsetAsync(np, 0, (size_t)R2 * 4, st), "memset");
        zero_operands(2, true);
        scatter(asr, Xenc, R1, 512, 1, 0, B, d_cum, P.maxT, st);
        scatter(f0, f0p, R2, 1, 2, 0, B, d_cum, 2 * P.maxT, st);
        scatter(noise, np, R2, 1, 2, 0, B, d_cum, 2 * P.maxT, st);
        c.n_launches += 3;
        float *har = source_and_har(f0p, 2);
        setup_adain(style);
        const std::string d = "kokopop.decoder.";
        const DevTensor &f0w = c.W(d + "F0_conv.weight"), &f0b = c.W(d + "F0_conv.bias");
        const DevTensor &nw = c.W(d + "N_conv.weight"), &nb = c.W(d + "N_conv.bias");
        f0n_conv(f0p, R2, Xenc + 512 * R1, Xdec + 1088 * R1, R1, f0w.d, f0b.d, B, P.maxT, st);
        f0n_conv(np, R2, Xenc + 513 * R1, Xdec + 1089 * R1, R1, nw.d, nb.d, B, P.maxT, st);
        c.n_launches += 2;
        // asr_res: 1x1 conv 512 -> 64 on the raw asr features
        Op a_in;
        if (tc) {
            a_in = op("opT", 1, 1152);
            act_only(Xenc, a_in, R1, 512, 1, 0, ACT_NONE, 0.f);
        } else {
            a_in.f = Xenc;
            a_in.R = R1;
        }
        conv_w(d + "asr_res.0.weight", d + "asr_res.0.bias", a_in, 512, 1, 0, 1, Xdec + 1024 * R1, R1, R1, Epi{},
               sum_len(1, 0));
        adain_resblk(d + "encode", Xenc, 514, false, Xdec);
        for (int i = 0; i < 3; ++i) adain_resblk(d + "decode." + std::to_string(i), Xdec, 1090, false, Xdec);
        float *dec = c.buf("dec_out", 512 * (size_t)R2);
        adain_resblk(d + "decode.3", Xdec, 1090, true, dec);
        // the decoder output (packed rows; gap rows are zero) and the style
        launch(KK_PROF_OTHER, 0.0, 4.0 * (512.0 * R2 + 128.0 * P.n), [&] {
            check_finite(dec, 512 * R2, kFiniteDecoder, status, st);
            check_finite(style, (int64_t)kStyle * P.n, kFiniteStyle, status, st);
        });
        ++c.n_launches;
        check_cuda(cudaStreamWaitEvent(st, c.ev_src, 0), "wait source");
        generator(2, dec, har, audio);
    }

    // sano_run_vocos (sano_vocos.cpp:94-230) over the chunks of the plan
    // (level 1 = frames): mel / noise per chunk [C][F_u] back to back ->
    // audio per chunk [hop (F_u - 1)] back to back. The residual stream x
    // [dim][R] stays F32; every linear reads a half operand (hi + lo halves
    // with F32 weights) written by the pass before it.
    void vocos_forward(const VocosNet &v, const float *mel, const float *noise, float *audio) {
        const kk_vocos_params &p = v.p;
        setup_batch();
        const int64_t R1 = R(1);
        const int D = p.dim, Hd = p.pw_hidden, n = p.n_fft, bins = n / 2 + 1;
        float *xm = c.buf("vo_xm", (size_t)p.mels * R1);
        float *xn = c.buf("vo_xn", (size_t)p.noise_ch * R1);
        float *x = c.buf("vo_x", (size_t)D * R1);
        float *hid = c.buf("vo_hid", (size_t)Hd * R1);
        float *hd = c.buf("vo_head", (size_t)2 * bins * R1);
        float *fr = c.buf("vo_frames", (size_t)n * R1);
        check_cuda(cudaMemsetAsync(xm, 0, (size_t)p.mels * R1 * 4, st), "memset");
        check_cuda(cudaMemsetAsync(xn, 0, (size_t)p.noise_ch * R1 * 4, st), "memset");
        Op om = op("vo_om", 1, p.mels), on = op("vo_on", 1, p.noise_ch), od = op("vo_od", 1, D),
           oh = op("vo_oh", 1, Hd);
        zero(om, p.mels);
        zero(on, p.noise_ch);
        zero(od, D);
        zero(oh, Hd);
        launch(KK_PROF_OTHER, 0.0, 8.0 * (p.mels + p.noise_ch) * (double)P.total, [&] {
            scatter(mel, xm, R1, p.mels, 1, 0, B, d_cum, P.maxT, st);
            scatter(noise, xn, R1, p.noise_ch, 1, 0, B, d_cum, P.maxT, st);
        });
        ++c.n_launches;
        act_only(xm, om, R1, p.mels, 1, 0, ACT_NONE, 0.f);
        act_only(xn, on, R1, p.noise_ch, 1, 0, ACT_NONE, 0.f);
        const int64_t valid = sum_len(1, 0);
        // stem: x = (conv(mel) + b) + (conv(noise) + b), then LayerNorm
        Epi e;
        e.bias = v.embed_b;
        e.valid = valid;
        conv_h(v.embed, om, p.embed_kernel, p.embed_kernel / 2, 1, x, R1, R1, e);
        Epi e2;
        e2.bias = v.noise_b;
        e2.accum = 1;
        e2.valid = valid;
        conv_h(v.noise, on, p.embed_kernel, p.embed_kernel / 2, 1, x, R1, R1, e2);
        const double el = (double)D * (double)valid;
        launch(KK_PROF_OTHER, 0.0, 8.0 * el, [&] {
            check_cuda(layer_norm_ch(x, R1, D, v.norm_w->d, v.norm_b->d, 0, 0.f, 1e-6f, B, x, R1, 0, st),
                       "layer norm launch");
        });
        for (int i = 0; i < p.blocks; ++i) {
            launch(KK_PROF_OPERAND, 0.0, el * (4.0 + (od.split ? 4.0 : 2.0)), [&] {
                check_cuda(dw_layer_norm(x, R1, D, p.dw_kernel, v.dw_w[i]->d, v.dw_b[i]->d, v.ln_w[i]->d,
                                         v.ln_b[i]->d, 1e-6f, B, od.h, od.Ry, od.lo(D), st),
                           "depthwise conv + layer norm launch");
            });
            Epi e0;
            e0.bias = v.pw0_b[i];
            e0.valid = valid;
            conv_h(v.pw0[i], od, 1, 0, 1, hid, R1, R1, e0);
            act_only(hid, oh, R1, Hd, 1, 0, ACT_GELU, 0.f);
            Epi e1;
            e1.bias = v.pw1_b[i];
            e1.chscale = v.gamma[i]->d;
            e1.accum = 1;
            e1.valid = valid;
            conv_h(v.pw1[i], oh, 1, 0, 1, x, R1, R1, e1);
        }
        launch(KK_PROF_OPERAND, 0.0, el * (8.0 + (od.split ? 4.0 : 2.0)), [&] {
            check_cuda(layer_norm_ch(x, R1, D, v.final_w->d, v.final_b->d, 0, 0.f, 1e-6f, B, x, R1, 0, st, od.h,
                                     od.Ry, od.lo(D)),
                       "layer norm launch");
        });
        Epi eh;
        eh.bias = v.head_b;
        eh.valid = valid;
        conv_h(v.head, od, 1, 0, 1, hd, R1, R1, eh);
        // per chunk: audio offsets and lengths (hop (F_u - 1) samples)
        std::vector<int64_t> ol((size_t)2 * P.n);
        int64_t acc = 0, max_len = 0;
        for (int u = 0; u < P.n; ++u) {
            const int64_t len = (int64_t)p.hop * (P.T[u] - 1);
            ol[(size_t)u] = acc;
            ol[(size_t)P.n + u] = len;
            acc += len;
            max_len = std::max(max_len, len);
        }
        int64_t *d_ol = (int64_t *)c.buf("vo_ol", (size_t)4 * P.n);
        c.upload(d_ol, ol.data(), ol.size() * sizeof(int64_t), st, "upload audio offsets");
        launch(KK_PROF_ISTFT, 0.0, 4.0 * (2.0 * bins + n) * (double)valid, [&] {
            check_cuda(vocos_spectrum(hd, R1, n, p.mag_clip, B, v.tab, fr, st), "vocos spectrum launch");
        });
        launch(KK_PROF_ISTFT, 0.0, 4.0 * (double)n * valid + 4.0 * (double)acc,
               [&] { vocos_ola(fr, n, p.hop, B, d_ol, v.tab.window_sq, max_len, audio, st); });
        launch(KK_PROF_OTHER, 0.0, 8.0 * (double)acc,
               [&] { dc_block(audio, d_ol, d_ol + P.n, P.n, p.dc_pole, st); });
    }

    // ggml_generator seam: decoder output given per utterance.
    void generator_forward(const float *decoder, const float *f0, const float *style, float *audio) {
        setup_batch();
        const int64_t R1 = R(1);
        float *dec = c.buf("dec_in", 512 * (size_t)R1);
        float *f0p = c.buf("f0p1", (size_t)R1);
        check_cuda(cudaMemsetAsync(f0p, 0, (size_t)R1 * 4, st), "memset");
        zero_operands(1, false);
        scatter(decoder, dec, R1, 512, 1, 0, B, d_cum, P.maxT, st);
        scatter(f0, f0p, R1, 1, 1, 0, B, d_cum, P.maxT, st);
        c.n_launches += 2;
        float *har = source_and_har(f0p, 1);
        setup_adain(style);
        check_cuda(cudaStreamWaitEvent(st, c.ev_src, 0), "wait source");
        generator(1, dec, har, audio);
    }
};

template <typename F>
int guarded(F &&f) noexcept {
    try {
        return f();
    } catch (const KKError &e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::exception &e) {
        g_last_error = e.what();
        return KK_ERROR_INFERENCE;
    } catch (...) {
        g_last_error = "unknown C++ exception";
        return KK_ERROR_INFERENCE;
    }
}

void use_device(kk_ctx *ctx) { check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice"); }

// Brackets one entry point's work on `st`: orders it after the context's
// previous call, which may have run on another stream and whose workspaces
// this call reuses, and opens a pinned staging slot for its small uploads.
struct CallScope {
    kk_ctx &c;
    cudaStream_t st;
    CallScope(kk_ctx &ctx, cudaStream_t s) : c(ctx), st(s) {
        if (c.done_recorded) check_cuda(cudaStreamWaitEvent(st, c.ev_done, 0), "order after the previous call");
        c.stage_begin();
    }
    ~CallScope() {
        c.done_recorded = cudaEventRecord(c.ev_done, st) == cudaSuccess;
        if (!c.done_recorded) cudaStreamSynchronize(st);  // nothing to wait for next time
    }
    CallScope(const CallScope &) = delete;
    CallScope &operator=(const CallScope &) = delete;
};

// After a synchronising call: surfaces what the device status block
// recorded since the last check (and clears it): a non-finite input or
// intermediate (the reference's all_finite, kokoro.cpp:91-99, :933-940), a
// token id out of range, or a bounded wait that ran out.
void check_device_error(kk_ctx *ctx) {
    if (!ctx->d_err.p) return;
    DevStatus s;
    check_cuda(cudaMemcpy(&s, ctx->d_err.p, sizeof s, cudaMemcpyDeviceToHost), "read device status");
    if (s.code == 0) return;
    ctx->reset_status();
    const int e = s.code;
    if (e >= kErrNonFinite && e < kErrNonFinite + kFiniteLabels) {
        static const char *labels[kFiniteLabels] = {"f0", "noise", "asr", "decoder", "decoder style"};
        const int l = e - kErrNonFinite;
        throw KKError(KK_ERROR_INFERENCE, std::string("non-finite Kokoro ") + labels[l] + " value at index " +
                                              std::to_string(s.first[l]));
    }
    if (e == kErrTokenId) throw KKError(KK_ERROR_INVALID_ARGUMENT, "token id out of range (device input)");
    if (e == kErrWaitSelftest)
        throw KKError(KK_ERROR_INFERENCE, "bounded wait ran out (self-test, code " + std::to_string(e) + ")");
    if (e == kErrLstmWait)
        throw KKError(KK_ERROR_INFERENCE, "LSTM recurrence timed out waiting for a step's hidden state (code " +
                                              std::to_string(e) + ")");
    throw KKError(KK_ERROR_INFERENCE, "tensor-core convolution timed out waiting (code " + std::to_string(e) + ")");
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

extern "C" {

const char *kk_last_error(void) { return g_last_error.c_str(); }

int kk_ctx_create(int device, kk_ctx **out) {
    return guarded([&] {
        if (!out) throw KKError(KK_ERROR_INVALID_ARGUMENT, "out is null");
        *out = nullptr;
        int n = 0;
        check_cuda(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) throw KKError(KK_ERROR_INVALID_ARGUMENT, "CUDA device out of range");
        cudaDeviceProp prop;
        check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major != 10)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, std::string("device is not sm_100 (B200): ") + prop.name);
        std::unique_ptr<kk_ctx> c(new kk_ctx());
        c->device = device;
        check_cuda(cudaSetDevice(device), "cudaSetDevice");
        check_cuda(cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking), "stream");
        check_cuda(cudaStreamCreateWithFlags(&c->st2, cudaStreamNonBlocking), "stream");
        check_cuda(cudaEventCreateWithFlags(&c->ev_inputs, cudaEventDisableTiming), "event");
        check_cuda(cudaEventCreateWithFlags(&c->ev_src, cudaEventDisableTiming), "event");
        check_cuda(cudaEventCreateWithFlags(&c->ev_done, cudaEventDisableTiming), "event");
        for (auto &s : c->stage) check_cuda(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming), "event");
        check_cuda(conv_simt_init(), "conv init");
        c->reset_status();
        *out = c.release();
        return KK_OK;
    });
}

void kk_ctx_destroy(kk_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->done_recorded) cudaEventSynchronize(ctx->ev_done);  // a call on the caller's stream
    cudaStreamSynchronize(ctx->st);
    cudaStreamSynchronize(ctx->st2);
    delete ctx;
}

int kk_weights_upload(kk_ctx *ctx, const kk_tensor_desc *descs, size_t n) {
    return guarded([&] {
        if (!ctx || (!descs && n)) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        // the packed weights may be rewritten below: let every earlier call finish
        if (ctx->done_recorded) check_cuda(cudaEventSynchronize(ctx->ev_done), "sync");
        check_cuda(cudaStreamSynchronize(ctx->st), "sync");
        std::vector<float> tmp;
        for (size_t i = 0; i < n; ++i) {
            const kk_tensor_desc &d = descs[i];
            if (!d.name || !d.data) throw KKError(KK_ERROR_INVALID_ARGUMENT, "tensor without name or data");
            if (d.dtype != KK_DTYPE_F32 && d.dtype != KK_DTYPE_F16)
                throw KKError(KK_ERROR_MODEL, std::string("unsupported tensor type for ") + d.name);
            if (d.n_dims < 1 || d.n_dims > 4) throw KKError(KK_ERROR_MODEL, std::string("bad rank: ") + d.name);
            DevTensor t;
            int64_t cnt = 1;
            for (int k = 0; k < 4; ++k) {
                t.ne[k] = k < d.n_dims ? d.ne[k] : 1;
                if (t.ne[k] < 1) throw KKError(KK_ERROR_MODEL, std::string("bad shape: ") + d.name);
                cnt *= t.ne[k];
            }
            t.n = cnt;
            t.f16 = d.dtype == KK_DTYPE_F16;
            tmp.resize((size_t)cnt);
            if (t.f16) {
                const uint16_t *s = (const uint16_t *)d.data;
                for (int64_t j = 0; j < cnt; ++j) tmp[j] = half_to_float(s[j]);
            } else {
                std::memcpy(tmp.data(), d.data, (size_t)cnt * 4);
            }
            if (cnt <= 4096) t.host = tmp;
            auto it = ctx->w.find(d.name);
            if (it != ctx->w.end()) {
                cudaFree(it->second.d);
                ctx->w.erase(it);
            }
            check_cuda(device_malloc((void **)&t.d, (size_t)cnt * 4), "cudaMalloc weight");
            check_cuda(cudaMemcpy(t.d, tmp.data(), (size_t)cnt * 4, cudaMemcpyHostToDevice), "upload weight");
            ctx->w.emplace(d.name, std::move(t));
        }
        ctx->derive();
        return KK_OK;
    });
}

static void check_ready(kk_ctx *ctx, bool decoder) {
    if (decoder ? !ctx->decoder_ready : !ctx->generator_ready)
        throw KKError(KK_ERROR_MODEL, "weights incomplete, first missing: " + ctx->missing);
}

int kk_decoder_forward_device(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *asr,
                              const float *f0, const float *noise, const float *style, float *audio,
                              void *stream) {
    return guarded([&] {
        if (!ctx || n_utts < 0 || (n_utts && (!n_frames || !asr || !f0 || !noise || !style || !audio)))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        if (n_utts == 0) return KK_OK;
        use_device(ctx);
        check_ready(ctx, true);
        const Plan P = make_plan(n_frames, n_utts);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        Runner r(*ctx, P, st);
        r.decoder_forward(asr, f0, noise, style, audio);
        check_cuda(cudaGetLastError(), "kernel launch");
        return KK_OK;
    });
}

int kk_decoder_forward(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *asr, const float *f0,
                       const float *noise, const float *style, float *audio) {
    return guarded([&] {
        if (!ctx || n_utts < 0 || (n_utts && (!n_frames || !asr || !f0 || !noise || !style || !audio)))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        if (n_utts == 0) return KK_OK;
        use_device(ctx);
        check_ready(ctx, true);
        const Plan P = make_plan(n_frames, n_utts);
        const size_t tot = (size_t)P.total;
        float *d_asr = ctx->buf("in_asr", 512 * tot);
        float *d_f0 = ctx->buf("in_f0", 2 * tot);
        float *d_n = ctx->buf("in_n", 2 * tot);
        float *d_style = ctx->buf("in_style", (size_t)kStyle * n_utts);
        float *d_audio = ctx->buf("out_audio", 600 * tot);
        cudaStream_t st = ctx->st;
        CallScope call_scope(*ctx, st);
        check_cuda(cudaMemcpyAsync(d_asr, asr, 512 * tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_f0, f0, 2 * tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_n, noise, 2 * tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_style, style, (size_t)kStyle * n_utts * 4, cudaMemcpyHostToDevice, st), "H2D");
        Runner r(*ctx, P, st);
        r.decoder_forward(d_asr, d_f0, d_n, d_style, d_audio);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(audio, d_audio, 600 * tot * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "decoder forward");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_generator_forward(kk_ctx *ctx, int32_t n_utts, const int32_t *n_decoder_frames, const float *decoder,
                         const float *f0, const float *style, float *audio) {
    return guarded([&] {
        if (!ctx || n_utts < 0 || (n_utts && (!n_decoder_frames || !decoder || !f0 || !style || !audio)))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        if (n_utts == 0) return KK_OK;
        use_device(ctx);
        check_ready(ctx, false);
        const Plan P = make_plan(n_decoder_frames, n_utts);
        const size_t tot = (size_t)P.total;
        float *d_dec = ctx->buf("in_dec", 512 * tot);
        float *d_f0 = ctx->buf("in_f0", tot);
        float *d_style = ctx->buf("in_style", (size_t)kStyle * n_utts);
        float *d_audio = ctx->buf("out_audio", 300 * tot);
        cudaStream_t st = ctx->st;
        CallScope call_scope(*ctx, st);
        check_cuda(cudaMemcpyAsync(d_dec, decoder, 512 * tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_f0, f0, tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_style, style, (size_t)kStyle * n_utts * 4, cudaMemcpyHostToDevice, st), "H2D");
        Runner r(*ctx, P, st);
        r.generator_forward(d_dec, d_f0, d_style, d_audio);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(audio, d_audio, 300 * tot * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "generator forward");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_istft(kk_ctx *ctx, int64_t n_frames, const float *post, float *audio) {
    return guarded([&] {
        if (!ctx || n_frames < 0 || (n_frames > 1 && (!post || !audio)))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        if (n_frames <= 1) return KK_OK;  // (frames - 1) * hop = 0 samples
        if (n_frames - 1 > (int64_t)INT32_MAX) throw KKError(KK_ERROR_INVALID_ARGUMENT, "too many frames");
        use_device(ctx);
        if (!ctx->d_tables.p) {
            StftTables stt;
            IstftTables ist;
            make_tables(stt, ist);
            ctx->d_tables.ensure(sizeof stt + sizeof ist);
            check_cuda(cudaMemcpy(ctx->d_tables.p, &stt, sizeof stt, cudaMemcpyHostToDevice), "tables");
            check_cuda(cudaMemcpy((char *)ctx->d_tables.p + sizeof stt, &ist, sizeof ist, cudaMemcpyHostToDevice),
                       "tables");
        }
        cudaStream_t st = ctx->st;
        CallScope call_scope(*ctx, st);
        // one utterance with base length n_frames - 1 and a_nf = 1:
        // frames = T + 1, samples = 5 T, offsets 0
        const int32_t T = (int32_t)(n_frames - 1);
        Plan P;
        P.n = 1;
        P.T = {T};
        P.off = {0};
        P.cum = {0};
        P.S = n_frames;
        P.total = T;
        P.maxT = T;
        float *d_post = ctx->buf("istft_post", 22 * (size_t)n_frames);
        float *d_audio = ctx->buf("istft_audio", 5 * (size_t)T);
        check_cuda(cudaMemcpyAsync(d_post, post, 22 * (size_t)n_frames * 4, cudaMemcpyHostToDevice, st), "H2D");
        Runner r(*ctx, P, st);
        r.setup_batch();
        const IstftTables *it = (const IstftTables *)((char *)ctx->d_tables.p + sizeof(StftTables));
        istft(d_post, n_frames, 1, d_audio, r.B, r.d_cum, it, T, st);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(audio, d_audio, 5 * (size_t)T * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "istft");
        return KK_OK;
    });
}

// ---------------------------------------------------------------------------
// sanoTTS Vocos decoder
// ---------------------------------------------------------------------------

static void vocos_args(kk_ctx *ctx, const char *prefix, const kk_vocos_params *params, int32_t n_chunks,
                       const int32_t *n_frames, const void *mel, const void *noise, const void *audio) {
    if (!ctx || !prefix || !params || n_chunks < 0 || (n_chunks && (!n_frames || !mel || !noise || !audio)))
        throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
    for (int32_t u = 0; u < n_chunks; ++u)
        if (n_frames[u] < 2 || n_frames[u] > kMaxFrames)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "vocos: a chunk needs 2 to 8192 frames");
}

int kk_vocos_forward_device(kk_ctx *ctx, const char *prefix, const kk_vocos_params *params, int32_t n_chunks,
                            const int32_t *n_frames, const float *mel, const float *noise, float *audio,
                            void *stream) {
    return guarded([&] {
        vocos_args(ctx, prefix, params, n_chunks, n_frames, mel, noise, audio);
        if (n_chunks == 0) return KK_OK;
        use_device(ctx);
        const VocosNet &v = ctx->vocos_net(prefix, *params);
        const Plan P = make_plan(n_frames, n_chunks);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        Runner r(*ctx, P, st, 1, v.embed.a_wrap > 0);
        r.vocos_forward(v, mel, noise, audio);
        check_cuda(cudaGetLastError(), "kernel launch");
        return KK_OK;
    });
}

int kk_vocos_forward(kk_ctx *ctx, const char *prefix, const kk_vocos_params *params, int32_t n_chunks,
                     const int32_t *n_frames, const float *mel, const float *noise, float *audio) {
    return guarded([&] {
        vocos_args(ctx, prefix, params, n_chunks, n_frames, mel, noise, audio);
        if (n_chunks == 0) return KK_OK;
        use_device(ctx);
        const VocosNet &v = ctx->vocos_net(prefix, *params);
        const Plan P = make_plan(n_frames, n_chunks);
        int64_t samples = 0;
        for (int32_t u = 0; u < n_chunks; ++u) samples += (int64_t)params->hop * (n_frames[u] - 1);
        const size_t tot = (size_t)P.total;
        float *d_mel = ctx->buf("vo_in_mel", (size_t)params->mels * tot);
        float *d_noise = ctx->buf("vo_in_noise", (size_t)params->noise_ch * tot);
        float *d_audio = ctx->buf("vo_out_audio", (size_t)samples);
        cudaStream_t st = ctx->st;
        CallScope call_scope(*ctx, st);
        check_cuda(cudaMemcpyAsync(d_mel, mel, (size_t)params->mels * tot * 4, cudaMemcpyHostToDevice, st), "H2D");
        check_cuda(cudaMemcpyAsync(d_noise, noise, (size_t)params->noise_ch * tot * 4, cudaMemcpyHostToDevice, st),
                   "H2D");
        Runner r(*ctx, P, st, 1, v.embed.a_wrap > 0);
        r.vocos_forward(v, d_mel, d_noise, d_audio);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(audio, d_audio, (size_t)samples * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "vocos forward");
        check_device_error(ctx);
        return KK_OK;
    });
}

// ---------------------------------------------------------------------------
// LSTM stack and duration alignment
// ---------------------------------------------------------------------------

namespace {

constexpr int32_t kMaxSteps = 65536;

// One plan "utterance" covering the R rows of a time-major packed batch.
Plan lstm_plan(int B, int max_len) {
    Plan P;
    P.n = 1;
    const int64_t rows = (int64_t)max_len * B;
    P.T = {(int32_t)rows};
    P.off = {0};
    P.cum = {0};
    P.S = rows;
    P.total = rows;
    P.maxT = (int32_t)rows;
    return P;
}

// Validates lengths and uploads them (int32) with the output offsets (int64).
Runner::Seqs lstm_seqs(kk_ctx &c, int32_t n_seqs, const int32_t *n_steps, cudaStream_t st) {
    if (n_seqs < 1 || !n_steps) throw KKError(KK_ERROR_INVALID_ARGUMENT, "need at least one sequence");
    Runner::Seqs q;
    q.B = n_seqs;
    std::vector<int64_t> h((size_t)n_seqs * 2);
    int32_t *hl = (int32_t *)h.data();
    int64_t *hc = h.data() + ((size_t)n_seqs + 1) / 2;
    for (int b = 0; b < n_seqs; ++b) {
        if (n_steps[b] < 1 || n_steps[b] > kMaxSteps)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "sequence length out of range [1, 65536]");
        hl[b] = n_steps[b];
        hc[b] = q.rows;
        q.rows += n_steps[b];
        if (n_steps[b] > q.max_len) q.max_len = n_steps[b];
    }
    if ((int64_t)q.max_len * n_seqs > INT32_MAX) throw KKError(KK_ERROR_INVALID_ARGUMENT, "batch too large");
    const size_t bytes = (size_t)((char *)(hc + n_seqs) - (char *)h.data());
    float *d = c.buf("lstm_seq", (bytes + 3) / 4);
    c.upload(d, h.data(), bytes, st, "upload lengths");
    q.d_len = (const int32_t *)d;
    q.d_cum = (const int64_t *)((char *)d + ((char *)hc - (char *)h.data()));
    return q;
}

}  // namespace

int kk_bilstm_forward(kk_ctx *ctx, const char *prefix, int32_t n_seqs, const int32_t *n_steps, int64_t in_dim,
                      const float *x, float *out) {
    return guarded([&] {
        if (!ctx || !prefix || !x || !out) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        const LstmLayer &L = c.lstm_layer(prefix);
        if (in_dim != L.in_dim) throw KKError(KK_ERROR_INVALID_ARGUMENT, "in_dim does not match the weights");
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        Runner::Seqs q = lstm_seqs(c, n_seqs, n_steps, st);
        Plan P = lstm_plan(n_seqs, q.max_len);
        Runner r(c, P, st);
        r.setup_batch();
        const int64_t Rr = P.R(1);
        float *xin = c.buf("lstm_xin", (size_t)q.rows * in_dim);
        check_cuda(cudaMemcpyAsync(xin, x, (size_t)q.rows * in_dim * 4, cudaMemcpyHostToDevice, st), "upload x");
        float *X = c.buf("lstm_X", (size_t)in_dim * Rr);
        check_cuda(cudaMemsetAsync(X, 0, (size_t)in_dim * Rr * 4, st), "memset");
        lstm_pack(xin, (int)in_dim, nullptr, 0, X, Rr, q.d_len, q.d_cum, n_seqs, q.max_len, st);
        float *hout = c.buf("lstm_h", (size_t)2 * L.H * Rr);
        r.bilstm(L, X, hout, q);
        float *od = c.buf("lstm_out", (size_t)q.rows * 2 * L.H);
        lstm_unpack(hout, Rr, 2 * L.H, od, q.d_len, q.d_cum, n_seqs, q.max_len, st);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(out, od, (size_t)q.rows * 2 * L.H * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "bilstm");
        check_device_error(ctx);
        return KK_OK;
    });
}

namespace {

// The duration encoder on device-resident x [rows][512], style [B][128] and
// out [rows][640], asynchronous on st.
void duration_encoder_device(kk_ctx &c, int32_t n_seqs, const int32_t *n_steps, const float *xin, const float *sd,
                             float *od, cudaStream_t st) {
    const std::string p = "kokopop.predictor.text_encoder.lstms.";
    const LstmLayer *Ls[3];
    for (int blk = 0; blk < 3; ++blk) {
        Ls[blk] = &c.lstm_layer(p + std::to_string(2 * blk));
        if (Ls[blk]->in_dim != 640) throw KKError(KK_ERROR_MODEL, "duration encoder LSTM input must be 640");
    }
    Runner::Seqs q = lstm_seqs(c, n_seqs, n_steps, st);
    Plan P = lstm_plan(n_seqs, q.max_len);
    Runner r(c, P, st);
    r.setup_batch();
    const int64_t Rr = P.R(1);
    const int B = n_seqs;
    // AdaLayerNorm gamma / beta per sequence
    float *gam = c.buf("lstm_gamma", (size_t)3 * B * 512), *bet = c.buf("lstm_beta", (size_t)3 * B * 512);
    for (int blk = 0; blk < 3; ++blk) {
        const std::string ln = p + std::to_string(2 * blk + 1) + ".fc.";
        const DevTensor &gw = c.W(ln + "gamma.weight"), &gb = c.W(ln + "gamma.bias");
        const DevTensor &bw = c.W(ln + "beta.weight"), &bb = c.W(ln + "beta.bias");
        if (gw.ne[0] != 128 || gw.ne[1] != 512 || bw.ne[0] != 128 || bw.ne[1] != 512 || gb.n != 512 || bb.n != 512)
            throw KKError(KK_ERROR_MODEL, "AdaLayerNorm fc shape mismatch: " + ln);
        style_linear(gw.d, gb.d, gw.f16, sd, 128, 512, B, gam + (size_t)blk * B * 512, st);
        style_linear(bw.d, bb.d, bw.f16, sd, 128, 512, B, bet + (size_t)blk * B * 512, st);
    }
    float *X = c.buf("lstm_X", (size_t)640 * Rr);
    check_cuda(cudaMemsetAsync(X, 0, (size_t)640 * Rr * 4, st), "memset");
    lstm_pack(xin, 512, sd, 128, X, Rr, q.d_len, q.d_cum, B, q.max_len, st);
    float *hout = c.buf("lstm_h", (size_t)512 * Rr);
    for (int blk = 0; blk < 3; ++blk) {
        r.bilstm(*Ls[blk], X, hout, q);
        ada_layer_norm(hout, Rr, 512, gam + (size_t)blk * B * 512, bet + (size_t)blk * B * 512, X, q.d_len, B, st);
    }
    lstm_unpack(X, Rr, 640, od, q.d_len, q.d_cum, B, q.max_len, st);
    c.n_launches += 3 + 6 + 3 + 2;
    check_cuda(cudaGetLastError(), "kernel launch");
}

// The prosody predictor's F0 / N chain (kokoro.cpp:669-708) from the aligned
// duration-encoder output: the biLSTM kokopop.predictor.shared over the
// frames, then the F0 and N chains on the packed frame level.
void prosody_device(kk_ctx &c, int32_t n_utts, const int32_t *n_frames, const float *en, const float *style,
                    float *f0, float *nn, cudaStream_t st) {
    if (!c.prosody_ready) throw KKError(KK_ERROR_MODEL, "prosody weights incomplete, first missing: " + c.missing_prosody);
    const LstmLayer &L = c.lstm_layer("kokopop.predictor.shared");
    if (L.in_dim != 640 || L.H != 256) throw KKError(KK_ERROR_MODEL, "predictor.shared must be a biLSTM 640 -> 2 x 256");
    Runner::Seqs q = lstm_seqs(c, n_utts, n_frames, st);
    Plan Pl = lstm_plan(n_utts, q.max_len);
    Runner rl(c, Pl, st);
    rl.setup_batch();
    const int64_t Rr = Pl.R(1);
    float *X = c.buf("lstm_X", (size_t)640 * Rr);
    check_cuda(cudaMemsetAsync(X, 0, (size_t)640 * Rr * 4, st), "memset");
    lstm_pack(en, 640, nullptr, 0, X, Rr, q.d_len, q.d_cum, n_utts, q.max_len, st);
    float *hout = c.buf("lstm_h", (size_t)512 * Rr);
    rl.bilstm(L, X, hout, q);
    // the frame level of a ragged plan (kMaxFrames per utterance)
    Plan P = make_plan(n_frames, n_utts);
    Runner r(c, P, st, c.prosody_tc ? 1 : 0);
    r.setup_batch();
    r.setup_adain(style);
    const int64_t R1 = P.R(1), R2 = P.R(2);
    float *x = c.buf("pr_x", (size_t)512 * R1);
    lstm_to_level(hout, Rr, 512, n_utts, q.d_len, q.max_len, x, R1, r.B.offT, 1, st);
    float *f0p = c.buf("pr_f0", (size_t)R2), *np = c.buf("pr_n", (size_t)R2);
    r.prosody_chains(x, 512, f0p, np);
    gather(f0p, f0, R2, 1, 2, 0, r.B, r.d_cum, 2 * P.maxT, st);
    gather(np, nn, R2, 1, 2, 0, r.B, r.d_cum, 2 * P.maxT, st);
    c.n_launches += 3 + 1 + 2;
    check_cuda(cudaGetLastError(), "kernel launch");
}

// text_encoder (graph_ops.cpp:1578-1624) up to its biLSTM, for n sequences
// of token ids (device, concatenated) -> out [sum n_tokens][512] (device).
// The CNN runs on a ragged plan (tokens as level 1); the last LayerNorm
// writes the LSTM layout (rows t * n + s) directly.
void text_encoder_device(kk_ctx &c, int32_t n, const int32_t *n_tokens, const int32_t *ids, float *out,
                         cudaStream_t st) {
    if (!c.text_ready) throw KKError(KK_ERROR_MODEL, "text encoder weights incomplete, first missing: " + c.missing_text);
    const DevTensor &emb = c.W("kokopop.text_encoder.embedding.weight");
    const int C = (int)emb.ne[0], vocab = (int)emb.ne[1];
    const LstmLayer &L = c.lstm_layer("kokopop.text_encoder.lstm");
    if (C != 512 || L.in_dim != C || L.H != 256)
        throw KKError(KK_ERROR_MODEL, "text encoder must be 512 channels into a biLSTM 512 -> 2 x 256");
    Plan P = make_plan(n_tokens, n);
    Runner r(c, P, st, c.text_mode != 0 ? 1 : 0, c.text_mode == 2);
    r.setup_batch();
    const int64_t R1 = P.R(1);
    float *X = c.buf("te_x", (size_t)C * R1);
    float *Y = c.buf("te_y", (size_t)C * R1);
    embed(emb.d, C, vocab, ids, r.d_cum, r.B, X, R1, (int *)c.d_err.p, st);
    ++c.n_launches;
    // the biLSTM's input in its own layout
    Runner::Seqs q = lstm_seqs(c, n, n_tokens, st);
    Plan Pl = lstm_plan(n, q.max_len);
    const int64_t Rr = Pl.R(1);
    float *Xl = c.buf("lstm_X", (size_t)C * Rr);
    check_cuda(cudaMemsetAsync(Xl, 0, (size_t)C * Rr * 4, st), "memset");
    Op in;
    if (r.tc) {
        in = r.op("opT", 1, C);
        r.zero(in, C);
    } else {
        in.f = X;
        in.R = R1;
    }
    for (int i = 0; i < 3; ++i) {
        const std::string p = "kokopop.text_encoder.cnn." + std::to_string(i);
        // the first conv's operand from the embeddings; the others' from
        // the LayerNorm before them
        if (r.tc && i == 0) r.act_only(X, in, R1, C, 1, 0, ACT_NONE, 0.f);
        r.conv_w(p + ".0.weight", p + ".0.bias", in, C, 5, 2, 1, Y, R1, R1, Runner::Epi{}, r.sum_len(1, 0));
        const bool last = i == 2;
        const bool to_op = r.tc && !last;
        check_cuda(layer_norm_ch(Y, R1, C, c.W(p + ".1.gamma").d, c.W(p + ".1.beta").d, 1, 0.2f, 1e-5f, r.B,
                                 last ? Xl : X, last ? Rr : R1, last ? n : 0, st, to_op ? in.h : nullptr, in.Ry,
                                 to_op ? in.lo(C) : 0),
                   "layer norm launch");
        ++c.n_launches;
    }
    Runner rl(c, Pl, st);
    rl.setup_batch();
    float *hout = c.buf("lstm_h", (size_t)512 * Rr);
    rl.bilstm(L, Xl, hout, q);
    lstm_unpack(hout, Rr, 512, out, q.d_len, q.d_cum, n, q.max_len, st);
    ++c.n_launches;
    check_cuda(cudaGetLastError(), "kernel launch");
}

// ALBERT + bert_encoder (kokoro.cpp:279-337) for n sequences of token ids
// (device, concatenated; positions 0..N-1, token type 0) -> out [sum
// n_tokens][512] (device), the duration encoder's input. Tokens are level 1
// of a ragged plan; every linear is a K = 1 conv on the operand path of the
// weights' type; the attention, GELU and LayerNorms are kk_frontend.cu.
void albert_device(kk_ctx &c, int32_t n, const int32_t *n_tokens, const int32_t *ids, float *out,
                   cudaStream_t st) {
    if (!c.albert_ready) throw KKError(KK_ERROR_MODEL, "ALBERT weights incomplete, first missing: " + c.missing_albert);
    const std::string e = "kokopop.albert.embeddings.", L = kAlbertLayer;
    const DevTensor &word = c.W(e + "word_embeddings.weight"), &pos = c.W(e + "position_embeddings.weight");
    const DevTensor &type = c.W(e + "token_type_embeddings.weight");
    const int E = (int)word.ne[0], vocab = (int)word.ne[1];
    const DevTensor &mapw = c.W("kokopop.albert.encoder.embedding_hidden_mapping_in.weight");
    const DevTensor &ffw = c.W(L + "ffn.weight"), &encw = c.W("kokopop.bert_encoder.weight");
    const int H = (int)mapw.ne[1], F = (int)ffw.ne[1], D = (int)encw.ne[1];
    if (pos.ne[0] != E || type.ne[0] != E || mapw.ne[0] != E || H != 768 || ffw.ne[0] != H || encw.ne[0] != H)
        throw KKError(KK_ERROR_MODEL, "ALBERT shapes: embeddings E, hidden 768 (12 heads of 64)");
    int max_len = 0;
    for (int b = 0; b < n; ++b) {
        if (n_tokens[b] > pos.ne[1] || n_tokens[b] > 512)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "sequence longer than the position table");
        max_len = std::max(max_len, (int)n_tokens[b]);
    }
    Plan P = make_plan(n_tokens, n);
    Runner r(c, P, st, c.albert_mode != 0 ? 1 : 0, c.albert_mode == 2);
    r.setup_batch();
    const int64_t R1 = P.R(1);
    float *x = c.buf("al_x", (size_t)E * R1);
    float *cur = c.buf("al_cur", (size_t)H * R1);
    float *qkv = c.buf("al_qkv", (size_t)3 * H * R1);
    float *att = c.buf("al_att", (size_t)H * R1);
    float *tmp = c.buf("al_tmp", (size_t)H * R1);
    float *ff = c.buf("al_ff", (size_t)F * R1);
    embed(word.d, E, vocab, ids, r.d_cum, r.B, x, R1, (int *)c.d_err.p, st, pos.d, type.d);
    c.n_launches += 2;
    const int Cmax = std::max(std::max(E, H), F);
    Op op;
    if (r.tc) {
        op = r.op("opA", 1, Cmax);
        r.zero(op, Cmax);
    }
    // LayerNorm (eps 1e-12) of x into y, and on the tensor-core path the
    // operand of the next linear
    auto norm = [&](const float *xin, int C, const std::string &wn, float *yout) {
        check_cuda(layer_norm_ch(xin, R1, C, c.W(wn + ".weight").d, c.W(wn + ".bias").d, 0, 0.f, 1e-12f, r.B, yout,
                                 R1, 0, st, r.tc ? op.h : nullptr, op.Ry, r.tc ? op.lo(C) : 0),
                   "layer norm launch");
    };
    norm(x, E, e + "LayerNorm", x);
    // linear(w, b, in [C][R1]) -> o [OC][R1] (+ resid); ready: the operand of
    // `in` is in `op` already (written by the LayerNorm that produced it)
    auto linear = [&](const std::string &w, const float *in, int C, float *o, const float *resid,
                      bool ready = false) {
        Op src;
        if (r.tc) {
            if (!ready) r.act_only(in, op, R1, C, 1, 0, ACT_NONE, 0.f);
            src = op;
        } else {
            src.f = const_cast<float *>(in);
            src.R = R1;
        }
        Runner::Epi ep;
        if (resid) {
            ep.resid = resid;
            ep.R_resid = R1;
        }
        r.conv_w(w, w.substr(0, w.size() - 6) + "bias", src, C, 1, 0, 1, o, R1, R1, ep, r.sum_len(1, 0));
    };
    linear("kokopop.albert.encoder.embedding_hidden_mapping_in.weight", x, E, cur, nullptr, true);
    for (int layer = 0; layer < 12; ++layer) {
        auto fused = c.packed.find("albert.qkv");
        if (r.tc && fused != c.packed.end()) {
            // one GEMM for query | key | value (each channel's sum as in the
            // separate ones); from layer 1 on its operand is the LayerNorm's
            if (layer == 0) r.act_only(cur, op, R1, H, 1, 0, ACT_NONE, 0.f);
            Runner::Epi ep;
            ep.bias = &c.albert_qkv_b;
            ep.valid = r.sum_len(1, 0);
            r.conv_h(fused->second, op, 1, 0, 1, qkv, R1, R1, ep);
        } else {
            linear(L + "attention.query.weight", cur, H, qkv, nullptr);
            linear(L + "attention.key.weight", cur, H, qkv + (size_t)H * R1, nullptr);
            linear(L + "attention.value.weight", cur, H, qkv + (size_t)2 * H * R1, nullptr);
        }
        check_cuda(attention(qkv, R1, H, 12, max_len, r.B, 0.125f, att, st), "attention launch");
        linear(L + "attention.dense.weight", att, H, tmp, cur);
        norm(tmp, H, L + "attention.LayerNorm", cur);
        linear(L + "ffn.weight", cur, H, ff, nullptr, true);
        gelu(ff, (int64_t)F * R1, st);
        linear(L + "ffn_output.weight", ff, F, tmp, cur);
        norm(tmp, H, L + "full_layer_layer_norm", cur);
        c.n_launches += 4;
    }
    float *y = c.buf("al_y", (size_t)D * R1);
    linear("kokopop.bert_encoder.weight", cur, H, y, nullptr, true);
    rows_out(y, R1, D, r.B, r.d_cum, max_len, out, st);
    ++c.n_launches;
    check_cuda(cudaGetLastError(), "kernel launch");
}

// The duration projection's weights, checked against the predictor biLSTM.
static void duration_proj_weights(kk_ctx &c, const DevTensor *&w, const DevTensor *&b) {
    const std::string p = "kokopop.predictor.duration_proj.linear_layer.";
    if (!c.Wopt(p + "weight") || !c.Wopt(p + "bias")) throw KKError(KK_ERROR_MODEL, "missing " + p + "weight / bias");
    w = &c.W(p + "weight");
    b = &c.W(p + "bias");
    if (w->ne[0] != 512 || w->ne[1] < 1 || w->ne[1] > 64 || b->n != w->ne[1])
        throw KKError(KK_ERROR_MODEL, "duration_proj must be 512 -> 1..64 buckets");
}

// predictor.lstm over the duration encoder output d [sum n][640] (device),
// then the projection and bucket sum (kokoro.cpp:343-355, :469-516) into
// durations [sum n] (device).
void duration_head_device(kk_ctx &c, int32_t n, const int32_t *n_tokens, const float *d, float *durations,
                          cudaStream_t st) {
    const DevTensor *w = nullptr, *b = nullptr;
    duration_proj_weights(c, w, b);
    const LstmLayer &L = c.lstm_layer("kokopop.predictor.lstm");
    if (L.in_dim != 640 || L.H != 256) throw KKError(KK_ERROR_MODEL, "predictor.lstm must be a biLSTM 640 -> 2 x 256");
    Runner::Seqs q = lstm_seqs(c, n, n_tokens, st);
    Plan Pl = lstm_plan(n, q.max_len);
    Runner rl(c, Pl, st);
    rl.setup_batch();
    const int64_t Rr = Pl.R(1);
    float *X = c.buf("lstm_X", (size_t)640 * Rr);
    check_cuda(cudaMemsetAsync(X, 0, (size_t)640 * Rr * 4, st), "memset");
    lstm_pack(d, 640, nullptr, 0, X, Rr, q.d_len, q.d_cum, n, q.max_len, st);
    float *hout = c.buf("lstm_h", (size_t)512 * Rr);
    rl.bilstm(L, X, hout, q);
    check_cuda(duration_proj(hout, 1, Rr, 512, w->d, b->d, (int)w->ne[1], q.d_len, q.d_cum, n,
                             (int64_t)q.max_len * n, durations, st),
               "duration projection launch");
    c.n_launches += 2;
}

int64_t total_steps(int32_t n_seqs, const int32_t *n_steps) {
    int64_t rows = 0;
    for (int b = 0; b < n_seqs; ++b) rows += n_steps[b];
    return rows;
}

}  // namespace

int kk_duration_encoder_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_steps, const float *x,
                                const float *style, float *out) {
    return guarded([&] {
        if (!ctx || !x || !style || !out || !n_steps || n_seqs < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        for (int b = 0; b < n_seqs; ++b)
            if (n_steps[b] < 1 || n_steps[b] > kMaxSteps)
                throw KKError(KK_ERROR_INVALID_ARGUMENT, "sequence length out of range [1, 65536]");
        const int64_t rows = total_steps(n_seqs, n_steps);
        float *xin = c.buf("lstm_xin", (size_t)rows * 512);
        check_cuda(cudaMemcpyAsync(xin, x, (size_t)rows * 512 * 4, cudaMemcpyHostToDevice, st), "upload x");
        float *sd = c.buf("lstm_style", (size_t)n_seqs * 128);
        check_cuda(cudaMemcpyAsync(sd, style, (size_t)n_seqs * 128 * 4, cudaMemcpyHostToDevice, st), "upload style");
        float *od = c.buf("lstm_out", (size_t)rows * 640);
        duration_encoder_device(c, n_seqs, n_steps, xin, sd, od, st);
        check_cuda(cudaMemcpyAsync(out, od, (size_t)rows * 640 * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "duration encoder");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_duration_encoder_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_steps, const float *x,
                                       const float *style, float *out, void *stream) {
    return guarded([&] {
        if (!ctx || !x || !style || !out || !n_steps || n_seqs < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        duration_encoder_device(*ctx, n_seqs, n_steps, x, style, out, st);
        return KK_OK;
    });
}

int kk_prosody_f0n(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *en, const float *style,
                   float *f0, float *n) {
    return guarded([&] {
        if (!ctx || !n_frames || !en || !style || !f0 || !n || n_utts < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        int64_t rows = 0;
        for (int b = 0; b < n_utts; ++b) {
            if (n_frames[b] < 1 || n_frames[b] > kMaxFrames)
                throw KKError(KK_ERROR_INVALID_ARGUMENT, "utterance length out of range [1, 8192]");
            rows += n_frames[b];
        }
        float *d_en = c.buf("pr_en", (size_t)rows * 640);
        float *d_style = c.buf("pr_style", (size_t)n_utts * 128);
        float *d_f0 = c.buf("pr_f0_out", (size_t)rows * 2), *d_n = c.buf("pr_n_out", (size_t)rows * 2);
        check_cuda(cudaMemcpyAsync(d_en, en, (size_t)rows * 640 * 4, cudaMemcpyHostToDevice, st), "upload en");
        check_cuda(cudaMemcpyAsync(d_style, style, (size_t)n_utts * 128 * 4, cudaMemcpyHostToDevice, st),
                   "upload style");
        prosody_device(c, n_utts, n_frames, d_en, d_style, d_f0, d_n, st);
        check_cuda(cudaMemcpyAsync(f0, d_f0, (size_t)rows * 2 * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaMemcpyAsync(n, d_n, (size_t)rows * 2 * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "prosody F0 / N");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_prosody_f0n_device(kk_ctx *ctx, int32_t n_utts, const int32_t *n_frames, const float *en,
                          const float *style, float *f0, float *n, void *stream) {
    return guarded([&] {
        if (!ctx || !n_frames || !en || !style || !f0 || !n || n_utts < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        for (int b = 0; b < n_utts; ++b)
            if (n_frames[b] < 1 || n_frames[b] > kMaxFrames)
                throw KKError(KK_ERROR_INVALID_ARGUMENT, "utterance length out of range [1, 8192]");
        use_device(ctx);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        prosody_device(*ctx, n_utts, n_frames, en, style, f0, n, st);
        return KK_OK;
    });
}

namespace {
// total tokens of a ragged batch of 1..kMaxFrames tokens per sequence
int64_t token_rows(int32_t n_seqs, const int32_t *n_tokens) {
    int64_t rows = 0;
    for (int b = 0; b < n_seqs; ++b) {
        if (n_tokens[b] < 1 || n_tokens[b] > kMaxFrames)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "sequence length out of range [1, 8192]");
        rows += n_tokens[b];
    }
    return rows;
}
}  // namespace

int kk_text_encoder_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out) {
    return guarded([&] {
        if (!ctx || !n_tokens || !ids || !out || n_seqs < 1) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        const int64_t rows = token_rows(n_seqs, n_tokens);
        if (!c.text_ready) throw KKError(KK_ERROR_MODEL, "text encoder weights incomplete, first missing: " + c.missing_text);
        const int64_t vocab = c.W("kokopop.text_encoder.embedding.weight").ne[1];
        for (int64_t i = 0; i < rows; ++i)
            if (ids[i] < 0 || ids[i] >= vocab) throw KKError(KK_ERROR_INVALID_ARGUMENT, "token id out of range");
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        int32_t *d_ids = (int32_t *)c.buf("te_ids", (size_t)rows);
        float *d_out = c.buf("te_out", (size_t)rows * 512);
        check_cuda(cudaMemcpyAsync(d_ids, ids, (size_t)rows * 4, cudaMemcpyHostToDevice, st), "upload ids");
        text_encoder_device(c, n_seqs, n_tokens, d_ids, d_out, st);
        check_cuda(cudaMemcpyAsync(out, d_out, (size_t)rows * 512 * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "text encoder");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_text_encoder_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids,
                                   float *out, void *stream) {
    return guarded([&] {
        if (!ctx || !n_tokens || !ids || !out || n_seqs < 1) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        token_rows(n_seqs, n_tokens);
        use_device(ctx);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        text_encoder_device(*ctx, n_seqs, n_tokens, ids, out, st);
        return KK_OK;
    });
}

int kk_albert_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out) {
    return guarded([&] {
        if (!ctx || !n_tokens || !ids || !out || n_seqs < 1) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        const int64_t rows = token_rows(n_seqs, n_tokens);
        if (!c.albert_ready) throw KKError(KK_ERROR_MODEL, "ALBERT weights incomplete, first missing: " + c.missing_albert);
        const int64_t vocab = c.W("kokopop.albert.embeddings.word_embeddings.weight").ne[1];
        for (int64_t i = 0; i < rows; ++i)
            if (ids[i] < 0 || ids[i] >= vocab) throw KKError(KK_ERROR_INVALID_ARGUMENT, "token id out of range");
        const int D = (int)c.W("kokopop.bert_encoder.weight").ne[1];
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        int32_t *d_ids = (int32_t *)c.buf("al_ids", (size_t)rows);
        float *d_out = c.buf("al_out", (size_t)rows * D);
        check_cuda(cudaMemcpyAsync(d_ids, ids, (size_t)rows * 4, cudaMemcpyHostToDevice, st), "upload ids");
        albert_device(c, n_seqs, n_tokens, d_ids, d_out, st);
        check_cuda(cudaMemcpyAsync(out, d_out, (size_t)rows * D * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "ALBERT");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_albert_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const int32_t *ids, float *out,
                             void *stream) {
    return guarded([&] {
        if (!ctx || !n_tokens || !ids || !out || n_seqs < 1) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        token_rows(n_seqs, n_tokens);
        use_device(ctx);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        albert_device(*ctx, n_seqs, n_tokens, ids, out, st);
        return KK_OK;
    });
}

int kk_duration_head_forward(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const float *d,
                             float *durations) {
    return guarded([&] {
        if (!ctx || !n_tokens || !d || !durations || n_seqs < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        kk_ctx &c = *ctx;
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        for (int b = 0; b < n_seqs; ++b)
            if (n_tokens[b] < 1 || n_tokens[b] > kMaxSteps)
                throw KKError(KK_ERROR_INVALID_ARGUMENT, "sequence length out of range [1, 65536]");
        const int64_t rows = total_steps(n_seqs, n_tokens);
        float *d_in = c.buf("dh_in", (size_t)rows * 640);
        float *d_out = c.buf("dh_out", (size_t)rows);
        check_cuda(cudaMemcpyAsync(d_in, d, (size_t)rows * 640 * 4, cudaMemcpyHostToDevice, st), "upload d");
        duration_head_device(c, n_seqs, n_tokens, d_in, d_out, st);
        check_cuda(cudaMemcpyAsync(durations, d_out, (size_t)rows * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "duration head");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_duration_head_forward_device(kk_ctx *ctx, int32_t n_seqs, const int32_t *n_tokens, const float *d,
                                    float *durations, void *stream) {
    return guarded([&] {
        if (!ctx || !n_tokens || !d || !durations || n_seqs < 1)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        cudaStream_t st = stream ? (cudaStream_t)stream : ctx->st;
        CallScope call_scope(*ctx, st);
        duration_head_device(*ctx, n_seqs, n_tokens, d, durations, st);
        return KK_OK;
    });
}

int kk_duration_proj(kk_ctx *ctx, int64_t n_rows, const float *h, float *durations) {
    return guarded([&] {
        if (!ctx || !h || !durations || n_rows < 1 || n_rows > kMaxSteps)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument or n_rows out of range [1, 65536]");
        use_device(ctx);
        kk_ctx &c = *ctx;
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        const DevTensor *w = nullptr, *b = nullptr;
        duration_proj_weights(c, w, b);
        const int32_t n = (int32_t)n_rows;
        Runner::Seqs q = lstm_seqs(c, 1, &n, st);
        float *d_h = c.buf("dh_h", (size_t)n_rows * 512);
        float *d_out = c.buf("dh_out", (size_t)n_rows);
        check_cuda(cudaMemcpyAsync(d_h, h, (size_t)n_rows * 512 * 4, cudaMemcpyHostToDevice, st), "upload h");
        check_cuda(duration_proj(d_h, 512, 1, 512, w->d, b->d, (int)w->ne[1], q.d_len, q.d_cum, 1, n_rows, d_out, st),
                   "duration projection launch");
        ++c.n_launches;
        check_cuda(cudaMemcpyAsync(durations, d_out, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "duration projection");
        return KK_OK;
    });
}

int kk_align_durations(kk_ctx *ctx, int64_t n_tokens, const float *durations, float speed, int32_t *frames,
                       int64_t *total, const float *hidden, int64_t hidden_dim, float *en, int64_t en_capacity) {
    return guarded([&] {
        if (!ctx || !total || n_tokens < 0 || (n_tokens > 0 && (!durations || !frames)) || (!hidden != !en) ||
            (hidden && hidden_dim < 1))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "null or invalid argument");
        if (n_tokens > 65535) throw KKError(KK_ERROR_INVALID_ARGUMENT, "too many tokens (at most 65535)");
        *total = 0;
        if (n_tokens == 0) return KK_OK;
        use_device(ctx);
        kk_ctx &c = *ctx;
        cudaStream_t st = c.st;
        CallScope call_scope(*ctx, st);
        // duration_to_frames (kokoro.cpp:181-193): a non-finite or
        // non-positive speed counts as 1
        if (!std::isfinite(speed) || speed <= 0.0f) speed = 1.0f;
        float *dd = c.buf("align_dur", (size_t)n_tokens);
        check_cuda(cudaMemcpyAsync(dd, durations, (size_t)n_tokens * 4, cudaMemcpyHostToDevice, st), "upload");
        float *idx = c.buf("align_idx", (size_t)n_tokens * 3 + 4);
        int64_t *dstart = (int64_t *)idx;
        int32_t *dframes = (int32_t *)(dstart + n_tokens + 1);
        duration_frames(dd, n_tokens, speed, dframes, dstart, st);
        check_cuda(cudaGetLastError(), "kernel launch");
        int64_t tot = 0;
        check_cuda(cudaMemcpyAsync(frames, dframes, (size_t)n_tokens * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaMemcpyAsync(&tot, dstart + n_tokens, sizeof tot, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "durations");
        *total = tot;
        if (!hidden) return KK_OK;
        if (tot > en_capacity) throw KKError(KK_ERROR_INVALID_ARGUMENT, "alignment output too small");
        float *hd = c.buf("align_hidden", (size_t)n_tokens * hidden_dim);
        float *ed = c.buf("align_en", (size_t)tot * hidden_dim);
        check_cuda(cudaMemcpyAsync(hd, hidden, (size_t)n_tokens * hidden_dim * 4, cudaMemcpyHostToDevice, st), "H2D");
        align_gather(hd, hidden_dim, dframes, dstart, n_tokens, ed, st);
        check_cuda(cudaGetLastError(), "kernel launch");
        check_cuda(cudaMemcpyAsync(en, ed, (size_t)tot * hidden_dim * 4, cudaMemcpyDeviceToHost, st), "D2H");
        check_cuda(cudaStreamSynchronize(st), "alignment");
        return KK_OK;
    });
}

int kk_profile_enable(kk_ctx *ctx, int enable) {
    return guarded([&] {
        if (!ctx) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null context");
        ctx->profiling = enable != 0;
        return KK_OK;
    });
}

int kk_profile_read(kk_ctx *ctx, kk_profile *out, int reset) {
    return guarded([&] {
        if (!ctx || !out) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        ctx->resolve_timed();
        out->launches = ctx->n_launches;
        out->conv_launches = ctx->conv_launches;
        out->conv_ms = ctx->conv_ms;
        out->conv_flop = ctx->conv_flop;
        if (reset) {
            ctx->n_launches = 0;
            ctx->conv_launches = 0;
            ctx->conv_ms = 0.0;
            ctx->conv_flop = 0.0;
            ctx->records.clear();
        }
        return KK_OK;
    });
}

int kk_profile_records(kk_ctx *ctx, kk_profile_record *out, size_t cap, size_t *n) {
    return guarded([&] {
        if (!ctx || !n || (cap && !out)) throw KKError(KK_ERROR_INVALID_ARGUMENT, "null argument");
        use_device(ctx);
        ctx->resolve_timed();
        *n = ctx->records.size();
        std::copy(ctx->records.begin(), ctx->records.begin() + std::min(cap, ctx->records.size()), out);
        return KK_OK;
    });
}

int kk_inject_allocation_failures(int32_t n) {
    if (n < 0) {
        g_last_error = "kk_inject_allocation_failures: negative count";
        return KK_ERROR_INVALID_ARGUMENT;
    }
    g_fail_next.store(n, std::memory_order_relaxed);
    return KK_OK;
}

int kk_wait_selftest(kk_ctx *ctx, int64_t limit_us) {
    return guarded([&] {
        if (!ctx || limit_us < 1 || limit_us > 2000000) throw KKError(KK_ERROR_INVALID_ARGUMENT, "bad argument");
        use_device(ctx);
        CallScope call_scope(*ctx, ctx->st);
        check_cuda(wait_selftest((int *)ctx->d_err.p, (unsigned long long)limit_us * 1000ull, ctx->st),
                   "wait self-test launch");
        check_cuda(cudaStreamSynchronize(ctx->st), "wait self-test");
        check_device_error(ctx);
        return KK_OK;
    });
}

int kk_allocation_count(uint64_t *out) {
    if (!out) {
        g_last_error = "kk_allocation_count: out is null";
        return KK_ERROR_INVALID_ARGUMENT;
    }
    *out = g_allocations.load(std::memory_order_relaxed);
    return KK_OK;
}

}  // extern "C"
