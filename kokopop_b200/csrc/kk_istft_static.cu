// kk_istft_static: the Kokoro iSTFT of kk_istft for callers that must not
// allocate device memory.
//
// kk_istft stages its input, output, tables and batch descriptor in buffers
// of a kk_ctx, which it allocates on first use and grows with the input.
// Some callers cannot allow that: a real-time audio thread (cudaMalloc and
// cudaFree may synchronise the whole device and stall it), or a serving
// process that fixes its device-memory budget at start-up (an allocation can
// fail later, mid-request). This entry point needs no context and allocates
// nothing: everything it stages lives in one file-scope device array, sized
// for KK_ISTFT_STATIC_MAX_FRAMES frames and reserved when the library's
// device code is loaded. The arithmetic is the same kernel as kk_istft.
//
// Scratch layout (bytes from the start of the array):
//   [0, 4096)                 iSTFT tables (written once per device)
//   [4096, 4352)              batch descriptor of this call (T, row offset,
//                             output offset)
//   [4352, ...)               post, 22 x n_frames F32 (this call's input)
//   [audio_off(n_frames), ...) audio, 5 (n_frames - 1) F32 (this call's output)
// Nothing in it has to start at zero: the tables are written before their
// first use, and every call writes its descriptor, its whole input and every
// output sample before reading them.
#include "kk_host.h"

#include <mutex>
#include <string>

namespace {

using kk::KKError;

constexpr int64_t kMaxFrames = KK_ISTFT_STATIC_MAX_FRAMES;
constexpr size_t kTabOff = 0, kDescOff = 4096, kPostOff = 4352;
constexpr size_t round256(size_t b) { return (b + 255) / 256 * 256; }
constexpr size_t audio_off(int64_t nf) { return round256(kPostOff + 22 * (size_t)nf * sizeof(float)); }
constexpr size_t kScratchBytes = round256(audio_off(kMaxFrames) + 5 * (size_t)(kMaxFrames - 1) * sizeof(float));
static_assert(sizeof(kk::IstftTables) <= kDescOff - kTabOff, "tables do not fit their slot");

// One per process and device (about 3.5 MB). Calls that overlap in time on
// one device share it: see the header.
static __device__ __align__(256) unsigned char g_istft_scratch[kScratchBytes];

struct Desc {
    int32_t T;  // base length = n_frames - 1
    int32_t pad;
    int64_t offT;  // row offset of the utterance (0)
    int64_t cum;   // output offset in base units (0)
};
static_assert(sizeof(Desc) <= kPostOff - kDescOff, "descriptor does not fit its slot");

constexpr int kMaxDevices = 64;
std::mutex g_init_mu;
unsigned char *g_base[kMaxDevices] = {};  // device address of the scratch, per device

// First call on a device (that device current): look up the array's device
// address and upload the tables. Synchronous.
unsigned char *scratch_for(int device) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (!g_base[device]) {
        void *p = nullptr;
        kk::check_cuda(cudaGetSymbolAddress(&p, g_istft_scratch), "cudaGetSymbolAddress (iSTFT scratch)");
        kk::StftTables stt;
        kk::IstftTables ist;
        kk::fill_tables(stt, ist);
        kk::check_cuda(cudaMemcpy((unsigned char *)p + kTabOff, &ist, sizeof ist, cudaMemcpyHostToDevice),
                       "upload iSTFT tables");
        g_base[device] = (unsigned char *)p;
    }
    return g_base[device];
}

// Makes `device` current for the call and restores the caller's device.
struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int device) {
        kk::check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
        kk::check_cuda(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceScope() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" int kk_istft_static(int device, int64_t n_frames, const float *post, float *audio, void *stream) {
    try {
        if (n_frames < 0 || (n_frames > 1 && (!post || !audio)))
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "kk_istft_static: null buffer or negative n_frames");
        if (n_frames > kMaxFrames)
            throw KKError(KK_ERROR_INVALID_ARGUMENT,
                          "kk_istft_static: n_frames = " + std::to_string(n_frames) +
                              " exceeds the static scratch, which holds at most " + std::to_string(kMaxFrames) +
                              " frames (use kk_istft for longer inputs)");
        if (device < 0 || device >= kMaxDevices)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "kk_istft_static: device index out of range");
        if (n_frames <= 1) return KK_OK;  // (frames - 1) * hop = 0 samples
        DeviceScope scope(device);
        unsigned char *base = scratch_for(device);
        cudaStream_t st = (cudaStream_t)stream;
        const int32_t T = (int32_t)(n_frames - 1);
        const Desc h{T, 0, 0, 0};
        Desc *d_desc = (Desc *)(base + kDescOff);
        float *d_post = (float *)(base + kPostOff);
        float *d_audio = (float *)(base + audio_off(n_frames));
        // pageable sources: each copy has read its host bytes when it returns
        kk::check_cuda(cudaMemcpyAsync(d_desc, &h, sizeof h, cudaMemcpyHostToDevice, st), "upload descriptor");
        kk::check_cuda(cudaMemcpyAsync(d_post, post, 22 * (size_t)n_frames * sizeof(float), cudaMemcpyHostToDevice, st),
                       "upload post");
        kk::Batch b;
        b.n = 1;
        b.T = &d_desc->T;
        b.offT = &d_desc->offT;
        kk::istft(d_post, n_frames, 1, d_audio, b, &d_desc->cum, (const kk::IstftTables *)(base + kTabOff), T, st);
        kk::check_cuda(cudaGetLastError(), "iSTFT launch");
        kk::check_cuda(cudaMemcpyAsync(audio, d_audio, 5 * (size_t)T * sizeof(float), cudaMemcpyDeviceToHost, st),
                       "download audio");
        kk::check_cuda(cudaStreamSynchronize(st), "iSTFT");
        return KK_OK;
    } catch (const KKError &e) {
        kk::set_last_error(e.what());
        return e.code;
    } catch (const std::exception &e) {
        kk::set_last_error(e.what());
        return KK_ERROR_INFERENCE;
    } catch (...) {
        kk::set_last_error("unknown C++ exception");
        return KK_ERROR_INFERENCE;
    }
}
