// Cross-context batcher (include/vxk.h, vxk_batcher_*): the host runtime that
// turns many contexts' single-token decoder steps into one batched forward
// per GPU.  The reference steps each voxtral_context separately
// (voxtral_ctx_decoder_step, src/voxtral-internal.h:243-251, from
// pump_incremental, src/voxtral-stream-decoder.cpp:92-98, 163-164); here each
// such call enqueues a request and blocks, and one dispatcher thread per
// batcher forms batches and runs them (the decoder's forward by default).
//
// Batch formation: the dispatcher sleeps until a request is queued, then
// waits until max_rows requests are queued, or `expected` of them, or
// max_wait_us has passed since the oldest one was queued.  It then takes the
// queue front to back, skipping a request whose stream already has a row in
// the batch (it stays queued for the next one), runs the batch outside the
// lock, and hands each request its result.  A submitter waits at most
// timeout_ms; a request not yet taken is withdrawn, one already running
// finishes with its batch and its result is dropped.
#include "vxk.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

namespace {

using Clock = std::chrono::steady_clock;

struct Request {
    int32_t stream = 0;
    int32_t token = 0;
    int32_t audio_slot = 0;
    int32_t out_token = -1;
    vxk_status status = VXK_STATUS_OK;
    bool done = false;
    bool abandoned = false;  // the submitter gave up; the dispatcher frees it
    Clock::time_point queued;
};

// The decoder executor's state.
struct DecoderExec {
    vxk_decoder * dec = nullptr;
    vxk_pool * pool = nullptr;
    cudaStream_t stream = nullptr;
    int device = 0;
    int32_t max_rows = 0;
    int32_t * d_argmax = nullptr;
    int32_t * h_argmax = nullptr;
    std::vector<int32_t> ones;
};

vxk_status decoder_exec(void * user, int32_t n, const int32_t * streams, const int32_t * tokens,
                        const int32_t * audio_slots, int32_t * out_tokens) {
    DecoderExec * e = static_cast<DecoderExec *>(user);
    if (n > e->max_rows) return VXK_STATUS_INVALID_ARGUMENT;
    cudaSetDevice(e->device);
    if ((int32_t) e->ones.size() < n) e->ones.assign((size_t) n, 1);
    vxk_status st = vxk_batch_plan(e->pool, streams, e->ones.data(), n, e->stream);
    if (st != VXK_STATUS_OK) return st;
    st = vxk_decoder_forward(e->dec, tokens, audio_slots, e->d_argmax, nullptr, nullptr, e->stream);
    if (st == VXK_STATUS_OK &&
        cudaMemcpyAsync(e->h_argmax, e->d_argmax, (size_t) n * sizeof(int32_t), cudaMemcpyDeviceToHost, e->stream) !=
            cudaSuccess)
        st = VXK_STATUS_BACKEND_ERROR;
    if (st == VXK_STATUS_OK) st = vxk_decoder_sync(e->dec, e->stream, 60000);
    if (st != VXK_STATUS_OK) {
        vxk_batch_abort(e->pool);
        return st;
    }
    st = vxk_batch_commit(e->pool);
    if (st != VXK_STATUS_OK) return st;
    std::memcpy(out_tokens, e->h_argmax, (size_t) n * sizeof(int32_t));
    return VXK_STATUS_OK;
}

}  // namespace

struct vxk_batcher {
    vxk_batcher_config cfg{};
    vxk_batch_fn fn = nullptr;
    void * user = nullptr;
    std::unique_ptr<DecoderExec> exec;  // set by vxk_batcher_create_for_decoder

    mutable std::mutex mu;
    std::condition_variable cv_queue;  // dispatcher: a request arrived or stop
    std::condition_variable cv_done;   // submitters: a batch finished
    std::deque<Request *> queue;
    bool stop = false;
    int32_t active = 0;  // threads inside vxk_batcher_step
    std::thread worker;

    vxk_batcher_stats stats{};
    double wait_sum_us = 0.0;
};

namespace {

void run_dispatcher(vxk_batcher * b) {
    std::vector<Request *> batch;
    std::vector<int32_t> streams, tokens, slots, outs;
    std::unordered_set<int32_t> in_batch;
    std::unique_lock<std::mutex> lock(b->mu);
    while (true) {
        b->cv_queue.wait(lock, [&] { return b->stop || !b->queue.empty(); });
        if (b->stop) break;
        // wait for company: max_rows, `expected`, or the oldest request's deadline
        const Clock::time_point deadline = b->queue.front()->queued + std::chrono::microseconds(b->cfg.max_wait_us);
        b->cv_queue.wait_until(lock, deadline, [&] {
            const int32_t q = (int32_t) b->queue.size();
            return b->stop || q >= b->cfg.max_rows || (b->cfg.expected > 0 && q >= b->cfg.expected);
        });
        if (b->stop) break;
        batch.clear();
        in_batch.clear();
        const Clock::time_point now = Clock::now();
        for (auto it = b->queue.begin(); it != b->queue.end() && (int32_t) batch.size() < b->cfg.max_rows;) {
            Request * r = *it;
            if (in_batch.count(r->stream)) {
                ++it;  // this stream's next step waits for the next batch
                continue;
            }
            in_batch.insert(r->stream);
            batch.push_back(r);
            b->wait_sum_us += std::chrono::duration<double, std::micro>(now - r->queued).count();
            it = b->queue.erase(it);
        }
        const int32_t n = (int32_t) batch.size();
        // every queued request was withdrawn while the batch formed
        if (n == 0) continue;
        streams.resize((size_t) n);
        tokens.resize((size_t) n);
        slots.resize((size_t) n);
        outs.assign((size_t) n, -1);
        for (int32_t i = 0; i < n; ++i) {
            streams[(size_t) i] = batch[(size_t) i]->stream;
            tokens[(size_t) i] = batch[(size_t) i]->token;
            slots[(size_t) i] = batch[(size_t) i]->audio_slot;
        }
        lock.unlock();
        vxk_status st;
        try {
            st = b->fn(b->user, n, streams.data(), tokens.data(), slots.data(), outs.data());
        } catch (...) {
            st = VXK_STATUS_INTERNAL_ERROR;
        }
        lock.lock();
        ++b->stats.batches;
        b->stats.rows += n;
        b->stats.max_rows_seen = std::max<int64_t>(b->stats.max_rows_seen, n);
        if (st != VXK_STATUS_OK) ++b->stats.failed_batches;
        for (int32_t i = 0; i < n; ++i) {
            Request * r = batch[(size_t) i];
            if (r->abandoned) {
                delete r;
                continue;
            }
            r->status = st;
            r->out_token = outs[(size_t) i];
            r->done = true;
        }
        b->cv_done.notify_all();
    }
    // stopped: whatever is still queued fails
    for (Request * r : b->queue) {
        if (r->abandoned) {
            delete r;
            continue;
        }
        r->status = VXK_STATUS_INVALID_STATE;
        r->done = true;
    }
    b->queue.clear();
    b->cv_done.notify_all();
}

vxk_status make(const vxk_batcher_config * config, vxk_batch_fn fn, void * user, vxk_batcher ** out,
                std::unique_ptr<DecoderExec> exec) {
    if (out) *out = nullptr;
    if (!fn || !out) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_batcher_config c = vxk_batcher_default_config();
    if (config) {
        if (config->struct_size < sizeof(uint32_t) * 2) return VXK_STATUS_INVALID_ARGUMENT;
        std::memcpy(&c, config, std::min<size_t>(config->struct_size, sizeof(c)));
    }
    if (c.max_rows < 1 || c.max_rows > 4096 || c.max_wait_us < 0 || c.expected < 0 || c.timeout_ms < 1)
        return VXK_STATUS_INVALID_ARGUMENT;
    vxk_batcher * b = new (std::nothrow) vxk_batcher();
    if (!b) return VXK_STATUS_OUT_OF_MEMORY;
    b->cfg = c;
    b->fn = fn;
    b->user = exec ? exec.get() : user;
    b->exec = std::move(exec);
    try {
        b->worker = std::thread(run_dispatcher, b);
    } catch (...) {
        delete b;
        return VXK_STATUS_INTERNAL_ERROR;
    }
    *out = b;
    return VXK_STATUS_OK;
}

}  // namespace

extern "C" {

vxk_batcher_config vxk_batcher_default_config(void) {
    vxk_batcher_config c{};
    c.struct_size = sizeof(vxk_batcher_config);
    c.api_version = VXK_API_VERSION;
    c.max_rows = 64;
    c.max_wait_us = 2000;
    c.expected = 0;
    c.timeout_ms = 30000;
    return c;
}

vxk_status vxk_batcher_create(const vxk_batcher_config * config, vxk_batch_fn fn, void * user, vxk_batcher ** out) {
    return make(config, fn, user, out, nullptr);
}

vxk_status vxk_batcher_create_for_decoder(const vxk_batcher_config * config, vxk_decoder * d, vxk_pool * pool,
                                          void * cuda_stream, vxk_batcher ** out) {
    if (out) *out = nullptr;
    if (!d || !pool || !out) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_decoder_info info{};
    vxk_status st = vxk_decoder_get_info(d, &info);
    if (st != VXK_STATUS_OK) return st;
    const int32_t max_rows = config ? config->max_rows : vxk_batcher_default_config().max_rows;
    if (max_rows < 1 || max_rows > info.max_rows || max_rows > info.max_streams) return VXK_STATUS_INVALID_ARGUMENT;
    std::unique_ptr<DecoderExec> e(new (std::nothrow) DecoderExec());
    if (!e) return VXK_STATUS_OUT_OF_MEMORY;
    e->dec = d;
    e->pool = pool;
    e->stream = static_cast<cudaStream_t>(cuda_stream);
    e->max_rows = max_rows;
    cudaGetDevice(&e->device);
    if (cudaMalloc(&e->d_argmax, (size_t) max_rows * sizeof(int32_t)) != cudaSuccess) return VXK_STATUS_OUT_OF_MEMORY;
    if (cudaHostAlloc(reinterpret_cast<void **>(&e->h_argmax), (size_t) max_rows * sizeof(int32_t),
                      cudaHostAllocDefault) != cudaSuccess) {
        cudaFree(e->d_argmax);
        return VXK_STATUS_OUT_OF_MEMORY;
    }
    DecoderExec * raw = e.get();
    st = make(config, decoder_exec, nullptr, out, std::move(e));
    if (st != VXK_STATUS_OK) {
        cudaFree(raw->d_argmax);
        cudaFreeHost(raw->h_argmax);
    }
    return st;
}

void vxk_batcher_destroy(vxk_batcher * b) {
    if (!b) return;
    {
        std::lock_guard<std::mutex> lock(b->mu);
        b->stop = true;
    }
    b->cv_queue.notify_all();
    if (b->worker.joinable()) b->worker.join();
    {
        // every submitter has its answer now; wait until the last one has left
        std::unique_lock<std::mutex> lock(b->mu);
        b->cv_done.wait(lock, [&] { return b->active == 0; });
    }
    if (b->exec) {
        cudaSetDevice(b->exec->device);
        cudaFree(b->exec->d_argmax);
        cudaFreeHost(b->exec->h_argmax);
    }
    delete b;
}

vxk_status vxk_batcher_step(vxk_batcher * b, int32_t stream, int32_t token, int32_t audio_slot, int32_t * out_token) {
    if (!b || !out_token || stream < 0) return VXK_STATUS_INVALID_ARGUMENT;
    Request * r = new (std::nothrow) Request();
    if (!r) return VXK_STATUS_OUT_OF_MEMORY;
    r->stream = stream;
    r->token = token;
    r->audio_slot = audio_slot;
    std::unique_lock<std::mutex> lock(b->mu);
    if (b->stop) {
        delete r;
        return VXK_STATUS_INVALID_STATE;
    }
    ++b->active;
    struct Leave {
        vxk_batcher * b;
        ~Leave() {
            if (--b->active == 0) b->cv_done.notify_all();
        }
    } leave{b};  // runs with the lock held (declared after it)
    r->queued = Clock::now();
    b->queue.push_back(r);
    b->cv_queue.notify_one();
    const bool done = b->cv_done.wait_for(lock, std::chrono::milliseconds(b->cfg.timeout_ms), [&] { return r->done; });
    if (!done) {
        ++b->stats.timeouts;
        auto it = std::find(b->queue.begin(), b->queue.end(), r);
        if (it != b->queue.end()) {
            b->queue.erase(it);  // never taken: withdraw it
            delete r;
        } else {
            r->abandoned = true;  // running: the dispatcher frees it
        }
        return VXK_STATUS_TIMEOUT;
    }
    const vxk_status st = r->status;
    *out_token = r->out_token;
    delete r;
    return st;
}

vxk_status vxk_batcher_get_stats(const vxk_batcher * b, vxk_batcher_stats * out) {
    if (!b || !out) return VXK_STATUS_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(b->mu);
    *out = b->stats;
    out->mean_wait_us = b->stats.rows > 0 ? b->wait_sum_us / (double) b->stats.rows : 0.0;
    return VXK_STATUS_OK;
}

}  // extern "C"
