// kk_istft_static: the Kokoro iSTFT of kk_istft for callers that must not
// allocate device memory.
//
// kk_istft stages its input, output, tables and batch descriptor in buffers
// of a kk_ctx, which it allocates on first use and grows with the input.
// Some callers cannot allow that: a real-time audio thread (cudaMalloc and
// cudaFree may synchronise the whole device and stall it), or a serving
// process that fixes its device-memory budget at start-up (an allocation can
// fail later, mid-request). This entry point needs no context and allocates
// nothing itself: everything it stages lives in one file-scope device array,
// sized for KK_ISTFT_STATIC_MAX_FRAMES frames. The arithmetic is the same
// kernel as kk_istft.
//
// When the array's memory is reserved: with CUDA's default lazy module
// loading, the module that holds the array is loaded (and the array's memory
// reserved) the first time host code looks up its address on a device, i.e.
// on the first call of this entry point on that device. A call with
// n_frames = 0 or 1 does that and nothing else, so a caller makes one such
// call per device at start-up (or runs with CUDA_MODULE_LOADING=EAGER, which
// loads every module when the context is created).
//
// Scratch layout (bytes from the start of the array):
//   [0, 4096)                 iSTFT tables (uploaded by every call)
//   [4096, 4352)              batch descriptor of this call (T, row offset,
//                             output offset)
//   [4352, ...)               post, 22 x n_frames F32 (this call's input)
//   [audio_off(n_frames), ...) audio, 5 (n_frames - 1) F32 (this call's output)
// Nothing in it has to start at zero: every call writes the tables, its
// descriptor, its whole input and every output sample before reading them.
#include "kk_host.h"

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

// The iSTFT tables in host memory, computed once per process.
const kk::IstftTables &host_tables() {
    static const kk::IstftTables t = [] {
        kk::StftTables stt;
        kk::IstftTables ist;
        kk::fill_tables(stt, ist);
        return ist;
    }();
    return t;
}

// The array's device address on the current device. Looked up on every call
// (the lookup allocates nothing once the module is loaded), so nothing goes
// stale if the caller resets the device or recreates its primary context.
unsigned char *scratch_base() {
    void *p = nullptr;
    kk::check_cuda(cudaGetSymbolAddress(&p, g_istft_scratch), "cudaGetSymbolAddress (iSTFT scratch)");
    return (unsigned char *)p;
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
        if (device < 0) throw KKError(KK_ERROR_INVALID_ARGUMENT, "kk_istft_static: negative device index");
        int n_dev = 0;
        if (cudaGetDeviceCount(&n_dev) != cudaSuccess) {
            cudaGetLastError();  // leave no error pending on this thread
            n_dev = 0;
        }
        if (device >= n_dev)
            throw KKError(KK_ERROR_INVALID_ARGUMENT, "kk_istft_static: device " + std::to_string(device) +
                                                         " out of range (" + std::to_string(n_dev) +
                                                         " CUDA devices)");
        DeviceScope scope(device);
        cudaGetLastError();  // an error left pending by earlier runtime calls is not this call's
        unsigned char *base = scratch_base();  // the first call on a device loads the module here
        if (n_frames <= 1) return KK_OK;       // (frames - 1) * hop = 0 samples
        cudaStream_t st = (cudaStream_t)stream;
        const int32_t T = (int32_t)(n_frames - 1);
        const Desc h{T, 0, 0, 0};
        Desc *d_desc = (Desc *)(base + kDescOff);
        float *d_post = (float *)(base + kPostOff);
        float *d_audio = (float *)(base + audio_off(n_frames));
        // pageable sources: each copy has read its host bytes when it returns
        kk::check_cuda(cudaMemcpyAsync(base + kTabOff, &host_tables(), sizeof(kk::IstftTables),
                                       cudaMemcpyHostToDevice, st),
                       "upload iSTFT tables");
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
