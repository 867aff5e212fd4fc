// Batching request queue in front of the decoder: the per-GPU counterpart of
// the reference's single-worker SynthesisScheduler
// (src/http/synthesis_scheduler.cpp:15-209), which runs one chunk of one
// request at a time, round-robin over the requests. Here every worker owns
// one executor (a kk_ctx on its GPU, or a caller's function) and runs a
// ragged batch per call: the oldest pending chunk of each request, in
// arrival order, up to max_batch chunks and max_batch_frames frames. A
// request has at most one chunk dispatched at a time, so its chunks finish
// in submission order, as in the reference. A worker that owns a kk_ctx
// overlaps the host work of one batch (packing into pinned memory,
// delivering results) with the GPU work of the previous one.
#include "../../include/kokopop_b200.h"
#include "kk_host.h"

#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

using Clock = std::chrono::steady_clock;

struct QJob {
    uint64_t ticket = 0, request = 0;
    int32_t T = 0;
    const float *asr = nullptr, *f0 = nullptr, *noise = nullptr, *style = nullptr;
    float *audio = nullptr;
    Clock::time_point t0;
};

thread_local std::string q_last_error;

}  // namespace

struct kk_queue {
    std::mutex m;
    std::condition_variable cv_work, cv_done;
    std::deque<QJob> pending;
    std::unordered_set<uint64_t> in_flight;  // requests with a chunk dispatched
    std::unordered_set<uint64_t> live;       // tickets not yet returned by kk_queue_wait
    std::unordered_map<uint64_t, int> done;  // ticket -> result
    uint64_t next_ticket = 1;
    bool stop = false;
    int32_t max_batch = 64;
    int64_t max_frames = 0;
    std::chrono::microseconds max_wait{0};
    kk_queue_exec_fn fn = nullptr;
    std::vector<std::thread> workers;
    uint64_t n_batches = 0, n_jobs = 0, max_seen = 0;

    bool dispatchable() const {
        for (const QJob &j : pending)
            if (!in_flight.count(j.request)) return true;
        return false;
    }

    // The next batch (empty on stop). With `block`, waits for a dispatchable
    // chunk, then up to max_wait past its arrival for the batch to fill.
    std::vector<QJob> take(std::unique_lock<std::mutex> &lk, bool block) {
        if (block) {
            cv_work.wait(lk, [&] { return stop || dispatchable(); });
            while (!stop) {
                int n = 0;
                Clock::time_point oldest = Clock::time_point::max();
                std::unordered_set<uint64_t> seen;
                for (const QJob &j : pending)
                    if (!in_flight.count(j.request) && seen.insert(j.request).second) {
                        ++n;
                        if (j.t0 < oldest) oldest = j.t0;
                    }
                if (n >= max_batch || n == 0 || Clock::now() >= oldest + max_wait) break;
                cv_work.wait_until(lk, oldest + max_wait);
            }
            if (stop) return {};
        }
        std::vector<QJob> b;
        std::unordered_set<uint64_t> blocked;  // requests with an earlier chunk left behind
        int64_t frames = 0;
        for (auto it = pending.begin(); it != pending.end() && (int32_t)b.size() < max_batch;) {
            if (in_flight.count(it->request) || blocked.count(it->request)) {
                ++it;
                continue;
            }
            blocked.insert(it->request);
            if (!b.empty() && frames + it->T > max_frames) {
                ++it;
                continue;
            }
            frames += it->T;
            b.push_back(*it);
            it = pending.erase(it);
        }
        for (const QJob &j : b) in_flight.insert(j.request);
        return b;
    }

    void complete(const std::vector<QJob> &b, int status) {
        std::lock_guard<std::mutex> lk(m);
        for (const QJob &j : b) {
            done[j.ticket] = status;
            in_flight.erase(j.request);
        }
        ++n_batches;
        n_jobs += b.size();
        if (b.size() > max_seen) max_seen = b.size();
        cv_done.notify_all();
        cv_work.notify_all();
    }
};

namespace {

// Host packing of a batch into the concatenated kk_decoder_forward layout.
struct Packed {
    std::vector<int32_t> T;
    int64_t frames = 0;
};

void pack(const std::vector<QJob> &b, Packed &p, float *asr, float *f0, float *noise, float *style) {
    p.T.clear();
    p.frames = 0;
    for (const QJob &j : b) {
        p.T.push_back(j.T);
        std::memcpy(asr + p.frames * 512, j.asr, (size_t)j.T * 512 * sizeof(float));
        std::memcpy(f0 + 2 * p.frames, j.f0, (size_t)j.T * 2 * sizeof(float));
        std::memcpy(noise + 2 * p.frames, j.noise, (size_t)j.T * 2 * sizeof(float));
        std::memcpy(style + (p.T.size() - 1) * 128, j.style, 128 * sizeof(float));
        p.frames += j.T;
    }
}

void deliver(const std::vector<QJob> &b, const float *audio) {
    int64_t off = 0;
    for (const QJob &j : b) {
        std::memcpy(j.audio, audio + 600 * off, (size_t)j.T * 600 * sizeof(float));
        off += j.T;
    }
}

// A caller's executor: pack, call, deliver, one batch at a time.
void worker_fn(kk_queue *q, void *user) {
    std::vector<float> asr, f0, noise, style, audio;
    Packed p;
    for (;;) {
        std::vector<QJob> b;
        {
            std::unique_lock<std::mutex> lk(q->m);
            b = q->take(lk, true);
        }
        if (b.empty()) return;
        int status = KK_OK;
        try {
            int64_t frames = 0;
            for (const QJob &j : b) frames += j.T;
            asr.resize((size_t)frames * 512);
            f0.resize((size_t)frames * 2);
            noise.resize((size_t)frames * 2);
            style.resize(b.size() * 128);
            audio.resize((size_t)frames * 600);
            pack(b, p, asr.data(), f0.data(), noise.data(), style.data());
            status = q->fn(user, (int32_t)b.size(), p.T.data(), asr.data(), f0.data(), noise.data(), style.data(),
                           audio.data());
            if (status == KK_OK) deliver(b, audio.data());
        } catch (...) {
            status = KK_ERROR_INFERENCE;
        }
        q->complete(b, status);
    }
}

// A kk_ctx on its GPU: two pinned staging sets and device buffers, batch k's
// packing and launch while batch k - 1 runs, then k - 1 delivered.
struct Slot {
    float *h_in = nullptr, *h_out = nullptr;  // pinned: asr | f0 | noise | style, audio
    float *d_in = nullptr, *d_out = nullptr;
    cudaEvent_t ev = nullptr;
    std::vector<QJob> jobs;
    Packed p;
    int status = KK_OK;
};

void worker_ctx(kk_queue *q, kk_ctx *ctx) {
    const int64_t F = q->max_frames, NB = q->max_batch;
    const size_t n_in = (size_t)F * 516 + (size_t)NB * 128, n_out = (size_t)F * 600;
    Slot s[2];
    cudaStream_t st = nullptr;
    bool ok = cudaSetDevice(ctx->device) == cudaSuccess && cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) ==
                                                                cudaSuccess;
    for (int i = 0; i < 2 && ok; ++i)
        ok = kk::pinned_malloc((void **)&s[i].h_in, n_in * 4) == cudaSuccess &&
             kk::pinned_malloc((void **)&s[i].h_out, n_out * 4) == cudaSuccess &&
             kk::device_malloc((void **)&s[i].d_in, n_in * 4) == cudaSuccess &&
             kk::device_malloc((void **)&s[i].d_out, n_out * 4) == cudaSuccess &&
             cudaEventCreateWithFlags(&s[i].ev, cudaEventDisableTiming) == cudaSuccess;
    int k = 0;
    bool busy = false;  // slot k ^ 1 holds a batch in flight
    auto launch = [&](Slot &sl) {
        float *asr = sl.h_in, *f0 = asr + F * 512, *noise = f0 + F * 2, *style = noise + F * 2;
        pack(sl.jobs, sl.p, asr, f0, noise, style);
        const int64_t fr = sl.p.frames;
        const int64_t nb = (int64_t)sl.jobs.size();
        float *d_asr = sl.d_in, *d_f0 = d_asr + F * 512, *d_noise = d_f0 + F * 2, *d_style = d_noise + F * 2;
        sl.status = KK_OK;
        if (cudaMemcpyAsync(d_asr, asr, (size_t)fr * 512 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_f0, f0, (size_t)fr * 2 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_noise, noise, (size_t)fr * 2 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaMemcpyAsync(d_style, style, (size_t)nb * 128 * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
            sl.status = KK_ERROR_INFERENCE;
        if (sl.status == KK_OK)
            sl.status = kk_decoder_forward_device(ctx, (int32_t)nb, sl.p.T.data(), d_asr, d_f0, d_noise, d_style,
                                                  sl.d_out, st);
        if (sl.status == KK_OK &&
            cudaMemcpyAsync(sl.h_out, sl.d_out, (size_t)fr * 600 * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
            sl.status = KK_ERROR_INFERENCE;
        if (cudaEventRecord(sl.ev, st) != cudaSuccess) sl.status = KK_ERROR_INFERENCE;
    };
    auto finish = [&](Slot &sl) {
        if (cudaEventSynchronize(sl.ev) != cudaSuccess && sl.status == KK_OK) sl.status = KK_ERROR_INFERENCE;
        if (sl.status == KK_OK) deliver(sl.jobs, sl.h_out);
        q->complete(sl.jobs, sl.status);
        sl.jobs.clear();
    };
    for (;;) {
        std::vector<QJob> b;
        {
            std::unique_lock<std::mutex> lk(q->m);
            b = q->take(lk, !busy);
        }
        if (!ok) {
            if (b.empty()) break;
            q->complete(b, KK_ERROR_INFERENCE);
            continue;
        }
        if (!b.empty()) {
            s[k].jobs = std::move(b);
            try {
                launch(s[k]);
            } catch (...) {
                s[k].status = KK_ERROR_INFERENCE;
            }
        }
        if (busy) finish(s[k ^ 1]);
        busy = !s[k].jobs.empty();
        if (busy) {
            k ^= 1;
        } else {
            std::lock_guard<std::mutex> lk(q->m);
            if (q->stop) break;
        }
    }
    if (busy) finish(s[k ^ 1]);
    for (int i = 0; i < 2; ++i) {
        if (s[i].h_in) cudaFreeHost(s[i].h_in);
        if (s[i].h_out) cudaFreeHost(s[i].h_out);
        if (s[i].d_in) cudaFree(s[i].d_in);
        if (s[i].d_out) cudaFree(s[i].d_out);
        if (s[i].ev) cudaEventDestroy(s[i].ev);
    }
    if (st) cudaStreamDestroy(st);
}

int q_fail(int code, const char *msg) {
    q_last_error = msg;
    return code;
}

// No C++ exception crosses the C ABI: thread creation and allocation
// failures become KK_ERROR_INFERENCE with a message.
template <typename F>
int q_guard(F &&f) noexcept {
    try {
        return f();
    } catch (const std::exception &e) {
        return q_fail(KK_ERROR_INFERENCE, e.what());
    } catch (...) {
        return q_fail(KK_ERROR_INFERENCE, "unknown C++ exception");
    }
}

// Stops and joins the workers started so far (creation failed part way).
void q_abort(kk_queue *q) {
    {
        std::lock_guard<std::mutex> lk(q->m);
        q->stop = true;
        q->cv_work.notify_all();
    }
    for (std::thread &t : q->workers)
        if (t.joinable()) t.join();
    delete q;
}

int q_config(kk_queue *q, int32_t max_batch, int64_t max_batch_frames, int32_t max_wait_us) {
    if (max_batch < 1 || max_batch > 4096 || max_batch_frames < 1 || max_batch_frames > ((int64_t)1 << 24) ||
        max_wait_us < 0)
        return q_fail(KK_ERROR_INVALID_ARGUMENT, "queue limits out of range");
    q->max_batch = max_batch;
    q->max_frames = max_batch_frames;
    q->max_wait = std::chrono::microseconds(max_wait_us);
    return KK_OK;
}

}  // namespace

namespace kk {
// Sets the message kk_queue_last_error returns on this thread (the
// streaming sessions of kk_stream.cpp report through it too); returns code.
int queue_error(int code, const char *msg) { return q_fail(code, msg); }
}  // namespace kk

extern "C" {

int kk_queue_create(kk_ctx *const *ctxs, int32_t n_ctx, int32_t max_batch, int64_t max_batch_frames,
                    int32_t max_wait_us, kk_queue **out) {
    if (!ctxs || n_ctx < 1 || !out) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    for (int i = 0; i < n_ctx; ++i) {
        if (!ctxs[i]) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null context");
        // two workers on one context would share its workspaces without a lock
        for (int j = 0; j < i; ++j)
            if (ctxs[j] == ctxs[i]) return q_fail(KK_ERROR_INVALID_ARGUMENT, "the same context appears twice");
    }
    return q_guard([&] {
        kk_queue *q = new kk_queue();
        const int rc = q_config(q, max_batch, max_batch_frames, max_wait_us);
        if (rc != KK_OK) {
            delete q;
            return rc;
        }
        if (max_batch_frames > kk::kMaxFrames * (int64_t)max_batch)
            q->max_frames = kk::kMaxFrames * (int64_t)max_batch;
        try {
            for (int i = 0; i < n_ctx; ++i) q->workers.emplace_back(worker_ctx, q, ctxs[i]);
        } catch (...) {
            q_abort(q);
            throw;
        }
        *out = q;
        return (int)KK_OK;
    });
}

int kk_queue_create_exec(kk_queue_exec_fn fn, void *const *users, int32_t n_workers, int32_t max_batch,
                         int64_t max_batch_frames, int32_t max_wait_us, kk_queue **out) {
    if (!fn || n_workers < 1 || !out) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    return q_guard([&] {
        kk_queue *q = new kk_queue();
        const int rc = q_config(q, max_batch, max_batch_frames, max_wait_us);
        if (rc != KK_OK) {
            delete q;
            return rc;
        }
        q->fn = fn;
        try {
            for (int i = 0; i < n_workers; ++i) q->workers.emplace_back(worker_fn, q, users ? users[i] : nullptr);
        } catch (...) {
            q_abort(q);
            throw;
        }
        *out = q;
        return (int)KK_OK;
    });
}

int kk_queue_submit(kk_queue *q, uint64_t request, int32_t n_frames, const float *asr, const float *f0,
                    const float *noise, const float *style, float *audio, uint64_t *ticket) {
    if (!q || !asr || !f0 || !noise || !style || !audio || !ticket)
        return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    if (n_frames < 1 || n_frames > kk::kMaxFrames || n_frames > q->max_frames)
        return q_fail(KK_ERROR_INVALID_ARGUMENT, "chunk length out of range");
    return q_guard([&] {
        std::lock_guard<std::mutex> lk(q->m);
        if (q->stop) return q_fail(KK_ERROR_INVALID_ARGUMENT, "queue stopped");
        QJob j;
        j.ticket = q->next_ticket++;
        j.request = request;
        j.T = n_frames;
        j.asr = asr;
        j.f0 = f0;
        j.noise = noise;
        j.style = style;
        j.audio = audio;
        j.t0 = Clock::now();
        q->pending.push_back(j);
        try {
            q->live.insert(j.ticket);
        } catch (...) {
            q->pending.pop_back();
            throw;
        }
        *ticket = j.ticket;
        q->cv_work.notify_all();
        return (int)KK_OK;
    });
}

int kk_queue_wait(kk_queue *q, uint64_t ticket, int32_t timeout_ms) {
    if (!q) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    std::unique_lock<std::mutex> lk(q->m);
    if (!q->live.count(ticket)) return q_fail(KK_ERROR_INVALID_ARGUMENT, "unknown ticket");
    auto ready = [&] { return q->done.count(ticket) != 0; };
    if (timeout_ms < 0)
        q->cv_done.wait(lk, ready);
    else if (!q->cv_done.wait_for(lk, std::chrono::milliseconds(timeout_ms), ready))
        return KK_QUEUE_PENDING;
    const int r = q->done[ticket];
    q->done.erase(ticket);
    q->live.erase(ticket);
    return r;
}

int kk_queue_cancel(kk_queue *q, uint64_t request, int32_t *n_cancelled) {
    if (!q) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lk(q->m);
    int32_t n = 0;
    for (auto it = q->pending.begin(); it != q->pending.end();) {
        if (it->request == request) {
            q->done[it->ticket] = KK_QUEUE_CANCELLED;
            it = q->pending.erase(it);
            ++n;
        } else {
            ++it;
        }
    }
    if (n_cancelled) *n_cancelled = n;
    q->cv_done.notify_all();
    return KK_OK;
}

int kk_queue_stats(kk_queue *q, uint64_t *batches, uint64_t *jobs, uint64_t *max_batch_seen) {
    if (!q) return q_fail(KK_ERROR_INVALID_ARGUMENT, "null argument");
    std::lock_guard<std::mutex> lk(q->m);
    if (batches) *batches = q->n_batches;
    if (jobs) *jobs = q->n_jobs;
    if (max_batch_seen) *max_batch_seen = q->max_seen;
    return KK_OK;
}

const char *kk_queue_last_error(void) { return q_last_error.c_str(); }

void kk_queue_destroy(kk_queue *q) {
    if (!q) return;
    {
        std::lock_guard<std::mutex> lk(q->m);
        q->stop = true;
        for (const QJob &j : q->pending) q->done[j.ticket] = KK_QUEUE_CANCELLED;
        q->pending.clear();
        q->cv_work.notify_all();
        q->cv_done.notify_all();
    }
    for (std::thread &t : q->workers)
        if (t.joinable()) t.join();
    delete q;
}

}  // extern "C"
