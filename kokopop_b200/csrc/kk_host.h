// Host-side state of a kk_ctx (see kk_host.cpp).
#pragma once

#include "../../include/kokopop_b200.h"
#include "kk_kernels.h"

#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace kk {

constexpr int32_t kMaxFrames = 8192;  // per-utterance asr frames (kokoro.cpp:584-590 warns above this)

struct KKError : std::runtime_error {
    int code;
    KKError(int c, const std::string &m);
};

void check_cuda(cudaError_t e, const char *what);
float half_to_float(uint16_t h);

// Every device and pinned-host allocation of the library goes through these
// two, which count it (kk_allocation_count).
cudaError_t device_malloc(void **p, size_t bytes);
cudaError_t pinned_malloc(void **p, size_t bytes);

// kk_queue.cpp: sets the message of kk_queue_last_error on this thread;
// returns code.
int queue_error(int code, const char *msg);

// A weight as F32 values on the device (F16 tensors are widened exactly);
// `f16` records the stored type because it selects ggml's F16 arithmetic.
struct DevTensor {
    float *d = nullptr;
    int64_t ne[4] = {1, 1, 1, 1};
    int64_t n = 0;
    bool f16 = false;
    std::vector<float> host;  // small tensors only (<= 4096 values)
};

struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
    void ensure(size_t b);
    void release();
};

// A convolution weight packed for the tensor-core kernel: half,
// [K][IC_pad/64][n_tiles][8][128][8] (the shared-memory image of each
// (tap, 64-channel block, 128-channel tile)).
struct PackedW {
    DevBuf buf;
    int IC = 0, IC_pad = 0, OC = 0, K = 0, n_tiles = 0;
    // > 0: split-F32 packing over 3 * (IC rounded to 64) virtual channels
    // [W_lo | W_hi | W_hi]; K blocks from a_wrap on read the operand's hi
    // blocks again (ConvTcArgs::a_wrap)
    int a_wrap = 0;
    // split packing: the weights are packed times 2^s (the hi and lo halves
    // of small weights stay in the normal half range); the conv multiplies
    // its accumulator by acc_scale = 2^-s, exactly
    float acc_scale = 1.f;
};

// One bidirectional LSTM layer (prefix.weight_ih_l0[_reverse], ...), derived
// on first use: W_ih of both directions stacked as one K = 1 convolution
// weight [8H][in_dim] (forward rows first) with its bias, W_hh / b_hh as F32.
struct LstmLayer {
    int in_dim = 0, H = 0;
    bool f16 = false;   // W_ih stored as F16: ggml rounds the input to half
    DevBuf wih;         // F32 values [8H][in_dim]
    PackedW wih_tc;     // tensor-core packing of wih (F16 weights, or split F32)
    DevBuf bih_buf;     // [8H]
    DevTensor bih;      // view of bih_buf
    const float *whh[2] = {nullptr, nullptr};  // rowwise [4H][H] (the uploaded tensors)
    const float *bhh[2] = {nullptr, nullptr};
};

// A sanoTTS Vocos decoder of one voice (its tensor prefix), derived on first
// use from the uploaded weights and the voice's hyper-parameters: the
// tensor-core packings of its two stem convolutions, its pointwise linears
// and its head (F16 weights as they are, F32 weights split hi + lo), the
// F32 vectors it reads, and the tables of its inverse FFT.
struct VocosNet {
    kk_vocos_params p{};
    PackedW embed, noise, head;
    std::vector<PackedW> pw0, pw1;
    const DevTensor *embed_b = nullptr, *noise_b = nullptr, *norm_w = nullptr, *norm_b = nullptr;
    const DevTensor *final_w = nullptr, *final_b = nullptr, *head_b = nullptr;
    std::vector<const DevTensor *> dw_w, dw_b, ln_w, ln_b, pw0_b, pw1_b, gamma;
    DevBuf tables;
    R2Tables tab{};
};

struct SiteInfo {
    std::string prefix;
    int C = 0;
    int f16 = 0;
    const float *gw = nullptr, *gb = nullptr, *bw = nullptr, *bb = nullptr;
    int64_t off = 0;  // channel offset into the per-forward gamma/beta buffers
};

// Ragged batch plan: utterance u occupies base rows [off[u], off[u] + T[u])
// at the start of a slot of round_up(T[u] + 4, 8) rows (at least 4 gap rows
// follow it), the first slot after an 8-row lead gap. A level with multiplier
// m uses rows m * off[u] .. and R(m) rows in total, padded to the 128-row
// tile. Slots on 8-row boundaries put every utterance of the generator's
// levels (m = 20, 60, 120) on a 32-row boundary, where the convolution keeps
// per-block statistics.
struct Plan {
    int n = 0;
    std::vector<int32_t> T;
    std::vector<int64_t> off, cum;
    int64_t S = 0;      // base rows including gaps
    int64_t total = 0;  // sum of T
    int32_t maxT = 0;
    int64_t R(int m) const { return ((int64_t)m * S + 127) / 128 * 128; }
};

Plan make_plan(const int32_t *lens, int n);

// The STFT / iSTFT tables (C library values) and the calling thread's
// kk_last_error() slot, for entry points outside kk_host.cpp.
void fill_tables(StftTables &st, IstftTables &is);
void set_last_error(const std::string &msg);

}  // namespace kk

struct kk_ctx {
    int device = 0;
    cudaStream_t st = nullptr, st2 = nullptr;
    cudaEvent_t ev_inputs = nullptr, ev_src = nullptr;
    std::unordered_map<std::string, kk::DevTensor> w;
    // derived from the weights
    bool decoder_ready = false, generator_ready = false;
    std::string missing;
    bool prosody_ready = false;  // the prosody predictor's F0 / N chain
    bool prosody_tc = false;     // its convolutions all F16: the tensor-core path
    std::string missing_prosody;
    bool text_ready = false;  // the text encoder up to its biLSTM
    std::string missing_text;
    // its k = 5 convs: 0 CUDA cores (mixed types, or F32 without the split),
    // 1 tensor cores on F16 weights, 2 split F32 on the tensor cores
    int text_mode = 0;
    bool albert_ready = false;  // ALBERT + bert_encoder
    std::string missing_albert;
    int albert_mode = 0;  // its linears, as text_mode
    // tensor-core modes: query | key | value as one packed weight
    // ("albert.qkv", 3 x 768 output channels) with its bias
    kk::DevBuf albert_qkv_bbuf;
    kk::DevTensor albert_qkv_b;
    kk::DevBuf convt_phase[2];
    bool convt_f16[2] = {false, false};
    // tensor-core path: every convolution weight is F16, or every one is F32
    // (split_mode) unless KOKOPOP_B200_F32_SPLIT=0 at upload
    bool tc_mode = false;
    // F32 weights on the half tensor cores: weights and operands split as
    // hi + lo halves, one GEMM over 3x the input channels (W_hi x_hi +
    // W_hi x_lo + W_lo x_hi, F32 accumulation); mixed F16 / F32 weight sets
    // keep the CUDA-core path
    bool split_mode = false;
    // KOKOPOP_B200_F32_SPLIT is not 0: F32 weights may take the split path
    // (the decoder when all its convolutions are F32, each F32 LSTM W_ih)
    bool f32_split = true;
    // KOKOPOP_B200_FUSED_OPERAND=1 at upload: the residual-block convs form
    // their AdaIN + Snake operand inside the conv (k_conv_tcf, bit-identical
    // to the separate operand pass, slower than it on B200 so far)
    bool fuse_operand = false;
    int fuse_min_taps = 0;  // fuse_operand: only convs with at least this many taps
    bool convt_phases = false;  // ConvTranspose on k_conv_tc phase tiles instead of k_convt_tc
    std::unordered_map<std::string, kk::PackedW> packed;
    std::unordered_map<std::string, kk::DevBuf> adain_t;  // fc weights transposed to [128][C]
    kk::DevBuf d_err;  // device status block (kk::DevStatus): error word, non-finite indices
    void reset_status();
    kk::SineArgs sine{};
    std::vector<kk::SiteInfo> sites;
    std::unordered_map<std::string, int> site_index;
    int64_t site_total_C = 0;
    kk::DevBuf d_tables;
    // Pinned staging of each call's small host-built tables (batch
    // descriptors, AdaIN site tables, sequence lengths), so that their
    // uploads are asynchronous: a copy from pageable memory would first wait
    // for the stream. Two slots serve alternate calls; a slot is written
    // again only after the copies of the call that last used it have run
    // (its event, recorded after each upload).
    struct StageSlot {
        char *p = nullptr;
        size_t cap = 0, used = 0;
        cudaEvent_t ev = nullptr;
        bool pending = false;
        std::vector<char *> retired;  // outgrown buffers, freed once `ev` has passed
    };
    StageSlot stage[2];
    int stage_k = 0;
    void stage_begin();
    // copies `bytes` of host data into the current slot and queues their
    // upload to `dst` on `st` (the slot's event follows the last upload)
    void upload(void *dst, const void *src, size_t bytes, cudaStream_t st, const char *what);
    // Calls on one context share its workspaces, so each call is ordered
    // after the previous one even when they run on different streams: a call
    // waits (on the device) for the event the previous call recorded.
    cudaEvent_t ev_done = nullptr;
    bool done_recorded = false;
    // per-forward staging
    std::vector<kk::AdainSite> h_sites;
    kk::DevBuf d_sites;
    std::vector<int64_t> h_batch;
    kk::DevBuf d_batch;
    std::unordered_map<std::string, kk::DevBuf> ws;
    std::unordered_map<std::string, kk::LstmLayer> lstm;
    std::unordered_map<std::string, kk::VocosNet> vocos;
    // measurement
    uint64_t n_launches = 0;
    bool profiling = false;
    struct TimedLaunch {
        cudaEvent_t a, b;
        int kind, taps;
        double flop, bytes;
    };
    std::vector<TimedLaunch> timed;         // events not read yet
    std::vector<kk_profile_record> records;  // read, since the last reset
    void resolve_timed();
    std::vector<cudaEvent_t> event_pool;
    uint64_t conv_launches = 0;
    double conv_ms = 0.0, conv_flop = 0.0;
    cudaEvent_t take_event();

    ~kk_ctx();
    const kk::DevTensor &W(const std::string &name) const;
    const kk::DevTensor *Wopt(const std::string &name) const;
    float *buf(const char *name, size_t floats);
    void derive();
    const kk::LstmLayer &lstm_layer(const std::string &prefix);
    const kk::VocosNet &vocos_net(const std::string &prefix, const kk_vocos_params &p);
};
