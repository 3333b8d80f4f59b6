// Host runtime of the decoder KV pool (include/vxk.h).
//
// Owns the device page pool, per-stream rings and block tables, the RoPE
// cos/sin table, batch planning (one voxtral_decoder_kv_plan per stream,
// src/voxtral.cpp:5219-5360 / 5161-5213), kernel launches, compaction and
// readback.  No exception crosses the C boundary: every entry point maps
// failures to a vxk_status and records a message, like the reference's C
// adapter (src/voxtral-c-api.cpp:539-544).
#include "vxk.h"
#include "vxk_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <random>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_create_error;

struct StatusError {
    vxk_status status;
    std::string message;
};

[[noreturn]] void fail(vxk_status status, const std::string & message) {
    throw StatusError{status, message};
}

#define VXK_CUDA(expr)                                                                  \
    do {                                                                                \
        const cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                        \
            fail(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY             \
                                                 : VXK_STATUS_BACKEND_ERROR,            \
                 std::string(#expr) + ": " + cudaGetErrorString(e_));                   \
        }                                                                               \
    } while (0)

class DeviceScope {
public:
    explicit DeviceScope(int device) {
        cudaGetDevice(&previous_);
        if (previous_ != device) cudaSetDevice(device);
        device_ = device;
    }
    ~DeviceScope() {
        if (previous_ != device_) cudaSetDevice(previous_);
    }

private:
    int previous_ = 0;
    int device_ = 0;
};

struct StreamState {
    bool open = false;
    vxk_decoder_kv_ring ring{};
    std::vector<int32_t> table;  // ring of page ids, -1 = unallocated
};

struct PlanEntry {
    int32_t stream;
    vxk_decoder_kv_plan plan;
};

struct NewPage {
    int32_t stream;
    int32_t entry;
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Builds the cos/sin table of RoPE mode 0 exactly like ggml's CPU rope cache:
// theta_scale = powf(base, -2/n_dims); theta_0 = pos; theta_{i+1} =
// theta_i * theta_scale; (cosf, sinf) per pair (freq_scale 1, ext_factor 0,
// attn_factor 1 as passed at src/voxtral.cpp:2668-2671).
std::vector<float2> build_rope_table(int32_t rows, int32_t n_dims, float base) {
    std::vector<float2> table((size_t) rows * (size_t) (n_dims / 2));
    const float theta_scale = powf(base, -2.0f / (float) n_dims);
    for (int32_t p = 0; p < rows; ++p) {
        float theta = (float) p;
        float2 * row = table.data() + (size_t) p * (size_t) (n_dims / 2);
        for (int32_t i = 0; i < n_dims / 2; ++i) {
            row[i].x = cosf(theta);
            row[i].y = sinf(theta);
            theta = theta * theta_scale;
        }
    }
    return table;
}

}  // namespace

struct vxk_pool {
    vxk_pool_config cfg{};
    int sm_count = 148;
    int32_t decode_slots = 0;        // resident decode CTAs on the device
    int32_t bt_cap = 0;
    int64_t tile_data_bytes = 0;
    int64_t page_data_bytes = 0;
    int64_t layer_data_bytes = 0;

    uint8_t * k_data = nullptr;
    uint8_t * v_data = nullptr;
    int32_t * d_table = nullptr;
    float2 * d_rope = nullptr;
    float * d_partials = nullptr;
    int32_t * d_counters = nullptr;
    int32_t * d_error = nullptr;
    int32_t max_items = 0;
    int32_t max_updates = 0;

    uint8_t * d_stage = nullptr;
    uint8_t * h_stage[2] = {nullptr, nullptr};
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    int stage_next = 0;
    size_t stage_bytes = 0;
    size_t off_items = 0;
    size_t off_sched = 0;            // [n_ctas + 1] offsets, then the unit list
    size_t off_updates = 0;
    // offsets of the current plan's regions, packed so that one small copy
    // carries exactly the bytes the batch uses (each <= the static offset)
    size_t cur_items = 0;
    size_t cur_sched = 0;
    size_t cur_updates = 0;
    int64_t device_bytes = 0;

    std::vector<StreamState> streams;
    std::vector<int32_t> free_pages;  // stack: back() is handed out next
    std::vector<int32_t> owner_stream;
    std::vector<int32_t> owner_entry;
    int64_t streams_open = 0;
    int64_t compactions = 0;
    int64_t pages_moved = 0;
    int64_t bytes_moved = 0;
    int64_t launches = 0;

    bool planned = false;
    bool single_token = false;
    bool items_ok = false;          // the batch's splits fit the scratch
    int32_t batch_decodes = 0;      // decode launches since the plan
    std::vector<PlanEntry> plan;
    std::vector<vxk::RowDesc> rows;
    std::vector<vxk::WorkItem> items;
    std::vector<int32_t> order;
    std::vector<int32_t> sched;      // offsets (n_ctas + 1) followed by units
    int32_t n_ctas = 0;
    std::vector<vxk::TableUpdate> updates;
    std::vector<NewPage> new_pages;

    // end-to-end host path
    float * d_io = nullptr;
    size_t io_bytes = 0;
    cudaStream_t h2d = nullptr;
    cudaStream_t d2h = nullptr;
    std::vector<cudaEvent_t> ev_in;
    std::vector<cudaEvent_t> ev_out;
    cudaEvent_t ev_begin = nullptr;
    cudaEvent_t ev_done = nullptr;
    cudaEvent_t ev_sync = nullptr;
    int32_t * h_err = nullptr;

    uint8_t * d_read = nullptr;
    size_t read_bytes = 0;
    int2 * d_moves = nullptr;
    int2 * h_moves = nullptr;

    std::string last_error;
};

namespace {

template <typename F>
vxk_status guarded(vxk_pool * pool, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const StatusError & e) {
        if (pool) pool->last_error = e.message;
        return e.status;
    } catch (const std::bad_alloc &) {
        if (pool) pool->last_error = "host allocation failed";
        return VXK_STATUS_OUT_OF_MEMORY;
    } catch (...) {
        if (pool) pool->last_error = "internal error";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

void release_device(vxk_pool * p) {
    cudaFree(p->k_data);
    cudaFree(p->v_data);
    cudaFree(p->d_table);
    cudaFree(p->d_rope);
    cudaFree(p->d_partials);
    cudaFree(p->d_counters);
    cudaFree(p->d_error);
    cudaFree(p->d_stage);
    cudaFree(p->d_io);
    cudaFree(p->d_read);
    cudaFree(p->d_moves);
    for (int i = 0; i < 2; ++i) {
        if (p->h_stage[i]) cudaFreeHost(p->h_stage[i]);
        if (p->stage_ev[i]) cudaEventDestroy(p->stage_ev[i]);
    }
    if (p->h_err) cudaFreeHost(p->h_err);
    if (p->h_moves) cudaFreeHost(p->h_moves);
    for (cudaEvent_t e : p->ev_in) cudaEventDestroy(e);
    for (cudaEvent_t e : p->ev_out) cudaEventDestroy(e);
    if (p->ev_begin) cudaEventDestroy(p->ev_begin);
    if (p->ev_done) cudaEventDestroy(p->ev_done);
    if (p->ev_sync) cudaEventDestroy(p->ev_sync);
    if (p->h2d) cudaStreamDestroy(p->h2d);
    if (p->d2h) cudaStreamDestroy(p->d2h);
}

template <typename T>
T * device_alloc(vxk_pool * p, size_t bytes) {
    void * ptr = nullptr;
    VXK_CUDA(cudaMalloc(&ptr, bytes));
    p->device_bytes += (int64_t) bytes;
    return static_cast<T *>(ptr);
}

// Bytes of one cache value in the pool's tiles (q8_0: the int8 value; its
// block scales are stored apart).
int64_t elem_bytes(vxk_dtype dt) { return dt == VXK_DTYPE_Q8_0 ? 1 : dt == VXK_DTYPE_F32 ? 4 : 2; }

// Reads a caller's config: fields past the caller's struct_size (added in a
// later version of the struct) keep the defaults.
vxk_pool_config read_config(const vxk_pool_config * in) {
    vxk_pool_config c = vxk_pool_default_config();
    if (in->struct_size < offsetof(vxk_pool_config, split_pages))
        fail(VXK_STATUS_INVALID_ARGUMENT, "config struct_size too small");
    std::memcpy(&c, in, std::min<size_t>(in->struct_size, sizeof(c)));
    c.struct_size = sizeof(c);
    return c;
}

void validate_config(const vxk_pool_config & c) {
    if (c.split_pages < 0) fail(VXK_STATUS_INVALID_ARGUMENT, "split_pages must be >= 0");
    if (c.head_dim != vxk::kHeadDim) fail(VXK_STATUS_INVALID_ARGUMENT, "head_dim must be 128");
    if (c.n_kv_heads < 1 || c.n_q_heads != c.n_kv_heads * vxk::kGroup)
        fail(VXK_STATUS_INVALID_ARGUMENT, "n_q_heads must be 4 * n_kv_heads");
    if (c.block_tokens != vxk::kBlockTokens) fail(VXK_STATUS_INVALID_ARGUMENT, "block_tokens must be 16");
    if (c.capacity < c.block_tokens || c.capacity % c.block_tokens != 0)
        fail(VXK_STATUS_INVALID_ARGUMENT, "capacity must be a positive multiple of block_tokens");
    if (c.n_layers < 1 || c.n_blocks < 1 || c.max_streams < 1 || c.max_rows < 1 || c.max_position < 1)
        fail(VXK_STATUS_INVALID_ARGUMENT, "n_layers, n_blocks, max_streams, max_rows, max_position must be >= 1");
    if (c.dtype != VXK_DTYPE_F16 && c.dtype != VXK_DTYPE_Q8_0 && c.dtype != VXK_DTYPE_F32)
        fail(VXK_STATUS_INVALID_ARGUMENT, "decoder pool dtype must be F16, Q8_0 or F32");
    if (!(c.rope_theta > 0.0f)) fail(VXK_STATUS_INVALID_ARGUMENT, "rope_theta must be positive");
}

StreamState & stream_at(vxk_pool * p, int32_t s) {
    if (s < 0 || s >= (int32_t) p->streams.size() || !p->streams[(size_t) s].open)
        fail(VXK_STATUS_INVALID_ARGUMENT, "stream id is not open");
    return p->streams[(size_t) s];
}

void free_stream_pages(vxk_pool * p, int32_t s) {
    StreamState & st = p->streams[(size_t) s];
    for (int32_t e = 0; e < (int32_t) st.table.size(); ++e) {
        const int32_t pg = st.table[(size_t) e];
        if (pg >= 0) {
            p->free_pages.push_back(pg);
            p->owner_stream[(size_t) pg] = -1;
            p->owner_entry[(size_t) pg] = -1;
            st.table[(size_t) e] = -1;
        }
    }
}

void rollback_new_pages(vxk_pool * p) {
    for (const NewPage & np : p->new_pages) {
        StreamState & st = p->streams[(size_t) np.stream];
        const int32_t pg = st.table[(size_t) np.entry];
        if (pg >= 0) {
            p->free_pages.push_back(pg);
            p->owner_stream[(size_t) pg] = -1;
            p->owner_entry[(size_t) pg] = -1;
            st.table[(size_t) np.entry] = -1;
        }
    }
    p->new_pages.clear();
}

void clear_plan(vxk_pool * p) {
    p->planned = false;
    p->single_token = false;
    p->items_ok = false;
    p->batch_decodes = 0;
    p->plan.clear();
    p->rows.clear();
    p->items.clear();
    p->order.clear();
    p->sched.clear();
    p->n_ctas = 0;
    p->updates.clear();
    p->new_pages.clear();
}

int32_t alloc_page(vxk_pool * p, int32_t stream, int32_t entry) {
    if (p->free_pages.empty()) return -1;
    const int32_t pg = p->free_pages.back();
    p->free_pages.pop_back();
    p->owner_stream[(size_t) pg] = stream;
    p->owner_entry[(size_t) pg] = entry;
    p->streams[(size_t) stream].table[(size_t) entry] = pg;
    p->updates.push_back({stream * p->bt_cap + entry, pg});
    p->new_pages.push_back({stream, entry});
    return pg;
}

// Smallest power of two >= x (x >= 1).
int32_t pow2_ceil(int64_t x) {
    int32_t r = 1;
    while ((int64_t) r < x && r < (1 << 30)) r *= 2;
    return r;
}

// Splits every row's window into work items of chunk_pages logical pages.
void build_items(vxk_pool * p) {
    const int32_t bt = p->cfg.block_tokens;
    int64_t total_pages = 0;
    int64_t max_pages = 0;
    std::vector<int32_t> row_pages(p->rows.size());
    for (size_t r = 0; r < p->rows.size(); ++r) {
        const int32_t first = p->rows[r].win_start / bt;
        const int32_t last = p->rows[r].pos / bt;
        row_pages[r] = last - first + 1;
        total_pages += row_pages[r];
        max_pages = std::max<int64_t>(max_pages, row_pages[r]);
    }
    int32_t cp = p->cfg.split_pages > 0 ? pow2_ceil(p->cfg.split_pages) : 0;
    if (cp <= 0) {
        // A split pays a fixed prologue (descriptor, block-table and first-copy
        // latency) and epilogue (partials written, read back and combined by
        // the row's last CTA), so splits are made as large as load balance
        // allows: at most about one wave of the resident decode CTAs' worth
        // of pages each (rounded up to a power of two), launched longest first
        // so the short ones fill the tail.  For 64 streams of <= 4096 tokens
        // this leaves every (stream, kv head) unsplit.
        const int64_t slots = std::max<int64_t>(1, p->decode_slots);
        cp = pow2_ceil(std::max<int64_t>(1, (total_pages * p->cfg.n_kv_heads + slots - 1) / slots));
    }
    cp = std::min(cp, vxk::kMaxSplitPages);
    while (true) {
        int64_t n_items = 0;
        int64_t max_chunks = 0;
        for (int32_t pages : row_pages) {
            const int64_t c = (pages + cp - 1) / cp;
            n_items += c;
            max_chunks = std::max(max_chunks, c);
        }
        if (n_items <= p->max_items && max_chunks <= 256) break;
        if (cp >= vxk::kMaxSplitPages) {
            // Append-only batches (prefill) never attend; an attention call on
            // this batch reports the overflow.
            p->items.clear();
            p->order.clear();
            p->items_ok = false;
            return;
        }
        cp *= 2;
    }
    p->items_ok = true;
    p->items.clear();
    for (size_t r = 0; r < p->rows.size(); ++r) {
        const int32_t first = p->rows[r].win_start / bt;
        const int32_t pages = row_pages[r];
        const int32_t n_chunks = (pages + cp - 1) / cp;
        p->rows[r].item_base = (int32_t) p->items.size();
        p->rows[r].n_chunks = n_chunks;
        for (int32_t c = 0; c < n_chunks; ++c) {
            vxk::WorkItem it{};
            it.row = (int32_t) r;
            it.chunk = c;
            it.page_begin = first + c * cp;
            it.page_end = std::min(first + (c + 1) * cp, first + pages);
            p->items.push_back(it);
        }
    }
    // Longest splits first, then a greedy longest-processing-time assignment
    // of the (split, kv head) units to the resident CTAs of the persistent
    // decode kernel: each unit goes to the CTA with the least pages so far.
    p->order.resize(p->items.size());
    std::iota(p->order.begin(), p->order.end(), 0);
    std::stable_sort(p->order.begin(), p->order.end(), [&](int32_t a, int32_t b) {
        return p->items[(size_t) a].page_end - p->items[(size_t) a].page_begin >
               p->items[(size_t) b].page_end - p->items[(size_t) b].page_begin;
    });
    const int32_t nkv = p->cfg.n_kv_heads;
    const int64_t n_units = (int64_t) p->items.size() * nkv;
    // One CTA per unit, launched longest-first and balanced by the hardware
    // (measured faster than a persistent grid of one CTA per resident slot).
    const int32_t G = (int32_t) std::max<int64_t>(1, n_units);
    std::vector<std::pair<int64_t, int32_t>> heap;  // (pages assigned, cta) min-heap
    heap.reserve((size_t) G);
    for (int32_t b = 0; b < G; ++b) heap.emplace_back(0, b);
    std::vector<int32_t> unit_cta((size_t) n_units);
    std::vector<int32_t> count((size_t) G, 0);
    auto cmp = [](const std::pair<int64_t, int32_t> & x, const std::pair<int64_t, int32_t> & y) {
        return x.first != y.first ? x.first > y.first : x.second > y.second;
    };
    std::vector<int32_t> unit_list;
    unit_list.reserve((size_t) n_units);
    for (int32_t idx : p->order) {
        const vxk::WorkItem & it = p->items[(size_t) idx];
        for (int32_t h = 0; h < nkv; ++h) {
            std::pop_heap(heap.begin(), heap.end(), cmp);
            auto & top = heap.back();
            top.first += it.page_end - it.page_begin;
            const int32_t uid = idx * nkv + h;
            unit_list.push_back(uid);
            unit_cta[(size_t) uid] = top.second;
            ++count[(size_t) top.second];
            std::push_heap(heap.begin(), heap.end(), cmp);
        }
    }
    p->n_ctas = G;
    p->sched.assign((size_t) G + 1 + (size_t) n_units, 0);
    for (int32_t b = 0; b < G; ++b) p->sched[(size_t) b + 1] = p->sched[(size_t) b] + count[(size_t) b];
    std::vector<int32_t> fill(p->sched.begin(), p->sched.begin() + G);
    for (int32_t uid : unit_list) {
        const int32_t b = unit_cta[(size_t) uid];
        p->sched[(size_t) G + 1 + (size_t) fill[(size_t) b]++] = uid;
    }
}

void upload_plan(vxk_pool * p, cudaStream_t stream) {
    const size_t rows_b = p->rows.size() * sizeof(vxk::RowDesc);
    const size_t items_b = p->items.size() * sizeof(vxk::WorkItem);
    const size_t upd_b = p->updates.size() * sizeof(vxk::TableUpdate);
    if (p->updates.size() > (size_t) p->max_updates) fail(VXK_STATUS_INTERNAL_ERROR, "too many table updates");
    const size_t sched_b = p->sched.size() * sizeof(int32_t);
    p->cur_items = align_up(rows_b, 256);
    p->cur_sched = p->cur_items + align_up(items_b, 256);
    p->cur_updates = p->cur_sched + align_up(sched_b, 256);
    const int idx = p->stage_next;
    VXK_CUDA(cudaEventSynchronize(p->stage_ev[idx]));
    uint8_t * h = p->h_stage[idx];
    std::memcpy(h, p->rows.data(), rows_b);
    std::memcpy(h + p->cur_items, p->items.data(), items_b);
    std::memcpy(h + p->cur_sched, p->sched.data(), sched_b);
    if (upd_b) std::memcpy(h + p->cur_updates, p->updates.data(), upd_b);
    const size_t n = p->cur_updates + upd_b;
    VXK_CUDA(cudaMemcpyAsync(p->d_stage, h, n, cudaMemcpyHostToDevice, stream));
    VXK_CUDA(cudaEventRecord(p->stage_ev[idx], stream));
    p->stage_next ^= 1;
    if (!p->updates.empty()) ++p->launches;
    VXK_CUDA(vxk::launch_table_updates(p->d_table,
                                       reinterpret_cast<const vxk::TableUpdate *>(p->d_stage + p->cur_updates),
                                       (int32_t) p->updates.size(), stream));
}

vxk::DecodeParams decode_params(vxk_pool * p, int32_t layer, const float * q, const float * k,
                                const float * v, float * out, int fuse) {
    vxk::DecodeParams d{};
    d.k_data = p->k_data + (int64_t) layer * p->layer_data_bytes;
    d.v_data = p->v_data + (int64_t) layer * p->layer_data_bytes;
    d.n_blocks = p->cfg.n_blocks;
    d.n_kv = p->cfg.n_kv_heads;
    d.n_q = p->cfg.n_q_heads;
    d.bt_cap = p->bt_cap;
    d.block_table = p->d_table;
    d.rows = reinterpret_cast<const vxk::RowDesc *>(p->d_stage);
    d.items = reinterpret_cast<const vxk::WorkItem *>(p->d_stage + p->cur_items);
    d.sched_offsets = reinterpret_cast<const int32_t *>(p->d_stage + p->cur_sched);
    d.sched_units = d.sched_offsets + p->n_ctas + 1;
    d.n_ctas = p->n_ctas;
    d.n_rows = (int32_t) p->rows.size();
    d.n_items = (int32_t) p->items.size();
    d.q = q;
    d.k = k;
    d.v = v;
    d.out = out;
    d.rope = p->d_rope;
    d.rope_rows = p->cfg.max_position;
    d.scale_log2 = (1.0f / sqrtf((float) p->cfg.head_dim)) * 1.4426950408889634f;
    d.partials = p->d_partials;
    d.counters = p->d_counters;
    d.error = p->d_error;
    d.fuse_append = fuse;
    d.dtype = (int32_t) p->cfg.dtype;
    return d;
}

void check_layer(vxk_pool * p, int32_t layer) {
    if (!p->planned) fail(VXK_STATUS_INVALID_STATE, "no batch is planned");
    if (layer < 0 || layer >= p->cfg.n_layers) fail(VXK_STATUS_INVALID_ARGUMENT, "layer out of range");
}

void check_attention(vxk_pool * p) {
    if (!p->items_ok) fail(VXK_STATUS_INVALID_ARGUMENT, "batch windows exceed the split scratch capacity");
}

// Programmatic dependent launch is used only when this pool's previous
// launch was a fused decode of the same batch: that kernel writes nothing the
// next decode prologue reads (descriptors, block table, other layers' pages).
// Any other launch of the pool (plan upload, append, attend, compaction,
// readback) clears the condition.
bool use_pdl(vxk_pool * p) { return p->batch_decodes > 0; }

void do_plan(vxk_pool * p, const int32_t * ids, const int32_t * n_new, int32_t n, cudaStream_t stream) {
    if (p->planned) fail(VXK_STATUS_INVALID_STATE, "a batch is already planned");
    if (!ids || !n_new || n <= 0) fail(VXK_STATUS_INVALID_ARGUMENT, "empty batch");
    clear_plan(p);
    std::vector<char> seen(p->streams.size(), 0);
    int64_t total_rows = 0;
    bool single = true;
    for (int32_t i = 0; i < n; ++i) {
        stream_at(p, ids[i]);
        if (seen[(size_t) ids[i]]) fail(VXK_STATUS_INVALID_ARGUMENT, "stream listed twice in a batch");
        seen[(size_t) ids[i]] = 1;
        if (n_new[i] <= 0) fail(VXK_STATUS_INVALID_ARGUMENT, "n_new must be >= 1");
        total_rows += n_new[i];
        single = single && n_new[i] == 1;
    }
    if (total_rows > p->cfg.max_rows) fail(VXK_STATUS_INVALID_ARGUMENT, "batch rows exceed max_rows");
    const int32_t bt = p->cfg.block_tokens;
    const int64_t cap = p->cfg.capacity;
    try {
        for (int32_t i = 0; i < n; ++i) {
            const int32_t s = ids[i];
            StreamState & st = p->streams[(size_t) s];
            vxk_decoder_kv_plan pl;
            if (vxk_decoder_kv_plan_make(&st.ring, st.ring.next_absolute_position, n_new[i], &pl) != VXK_STATUS_OK)
                fail(VXK_STATUS_INVALID_ARGUMENT, "invalid KV append plan");
            if (n_new[i] > 1 && pl.evicted > 0)
                fail(VXK_STATUS_INVALID_ARGUMENT, "a multi-token append must not evict");
            if (pl.next_after - 1 >= (int64_t) p->cfg.max_position)
                fail(VXK_STATUS_INVALID_ARGUMENT, "position beyond the RoPE table (max_position)");
            const int64_t lp0 = pl.absolute_start / bt;
            const int64_t lp1 = (pl.next_after - 1) / bt;
            for (int64_t lp = lp0; lp <= lp1; ++lp) {
                const int32_t e = (int32_t) (lp % p->bt_cap);
                if (st.table[(size_t) e] < 0 && alloc_page(p, s, e) < 0)
                    fail(VXK_STATUS_OUT_OF_MEMORY, "KV page pool exhausted");
            }
            for (int32_t t = 0; t < n_new[i]; ++t) {
                const int64_t pos = pl.absolute_start + t;
                vxk::RowDesc rd{};
                rd.stream = s;
                rd.pos = (int32_t) pos;
                rd.win_start = (int32_t) std::max<int64_t>(st.ring.oldest_absolute_position, pos - cap + 1);
                rd.flags = single ? vxk::kRowAppend : 0;
                p->rows.push_back(rd);
            }
            p->plan.push_back({s, pl});
        }
        build_items(p);
        upload_plan(p, stream);
    } catch (...) {
        rollback_new_pages(p);
        clear_plan(p);
        throw;
    }
    p->planned = true;
    p->single_token = single;
}

void do_commit(vxk_pool * p) {
    if (!p->planned) fail(VXK_STATUS_INVALID_STATE, "no batch is planned");
    for (const PlanEntry & e : p->plan) {
        vxk_decoder_kv_plan_commit(&p->streams[(size_t) e.stream].ring, &e.plan);
    }
    clear_plan(p);
}

vxk_status bounded_wait(cudaEvent_t ev, int32_t timeout_ms) {
    const auto t0 = std::chrono::steady_clock::now();
    int spins = 0;
    while (true) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return VXK_STATUS_OK;
        if (e != cudaErrorNotReady) return VXK_STATUS_BACKEND_ERROR;
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
            std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) return VXK_STATUS_TIMEOUT;
        // a step of a few milliseconds is waited for by polling (a 50 us sleep
        // per poll cost up to ~0.1 ms of idle GPU per step); longer waits sleep
        if (ms < 20) {
            std::this_thread::yield();
        } else if (++spins > 64) {
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
}

void check_error_word(vxk_pool * p) {
    int32_t err = 0;
    VXK_CUDA(cudaMemcpy(&err, p->d_error, sizeof(err), cudaMemcpyDeviceToHost));
    if (err != 0) {
        // A kernel that gave up may have left split counters half counted.
        VXK_CUDA(cudaMemset(p->d_counters, 0,
                            (size_t) p->cfg.max_rows * (size_t) p->cfg.n_kv_heads * sizeof(int32_t)));
        VXK_CUDA(cudaMemset(p->d_error, 0, sizeof(int32_t)));
        fail(err == 2 ? VXK_STATUS_TIMEOUT : VXK_STATUS_BACKEND_ERROR,
             err == 2 ? "device pipeline wait timed out" : "kernel met an unallocated page");
    }
}

}  // namespace

namespace vxk {

bool pool_batch_view(const vxk_pool * pool, PoolBatchView * out) {
    if (!pool || !out || !pool->planned) return false;
    out->row_stream.resize(pool->rows.size());
    out->row_pos.resize(pool->rows.size());
    for (size_t r = 0; r < pool->rows.size(); ++r) {
        out->row_stream[r] = pool->rows[r].stream;
        out->row_pos[r] = pool->rows[r].pos;
    }
    out->last_rows.clear();
    int32_t end = 0;
    for (const PlanEntry & e : pool->plan) {
        end += e.plan.n_new;
        out->last_rows.push_back(end - 1);
    }
    out->single_token = pool->single_token;
    return true;
}

PoolShape pool_shape(const vxk_pool * pool) {
    const vxk_pool_config & c = pool->cfg;
    return PoolShape{c.device, c.n_layers, c.n_q_heads, c.n_kv_heads, c.head_dim, c.max_streams, c.max_rows,
                     c.rope_theta};
}

bool pool_decode_quant_ok(const vxk_pool * pool) {
    return pool && pool->cfg.dtype == VXK_DTYPE_F16 && pool->cfg.head_dim == kHeadDim &&
           pool->cfg.n_q_heads == pool->cfg.n_kv_heads * kGroup;
}

int32_t pool_decode_layer_quant(vxk_pool * pool, int32_t layer, const float * q, const float * k, const float * v,
                                float * out, const QtcTiles & t, cudaStream_t stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        check_layer(pool, layer);
        if (!pool->single_token) fail(VXK_STATUS_INVALID_STATE, "decode_layer needs a single-token batch");
        if (!q || !k || !v || !t.dx) fail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        if (!pool_decode_quant_ok(pool)) fail(VXK_STATUS_INVALID_ARGUMENT, "quantized output needs an f16 cache");
        check_attention(pool);
        DeviceScope scope(pool->cfg.device);
        ++pool->launches;
        const bool pdl = use_pdl(pool);
        pool->batch_decodes = 0;
        DecodeParams d = decode_params(pool, layer, q, k, v, out, 1);
        d.q_tiles = t.b;
        d.q_bmin = t.bmin;
        d.q_tiles8 = t.b8;
        d.q_dx = t.dx;
        d.q_npad = t.npad;
        d.q_units = pool->cfg.n_q_heads * pool->cfg.head_dim / 256;
        VXK_CUDA(launch_decode_quant(d, stream, pdl));
        pool->batch_decodes = 1;
    });
}

}  // namespace vxk

extern "C" {

vxk_pool_config vxk_pool_default_config(void) {
    vxk_pool_config c{};
    c.struct_size = sizeof(vxk_pool_config);
    c.api_version = VXK_API_VERSION;
    c.device = 0;
    c.n_layers = 26;
    c.n_q_heads = 32;
    c.n_kv_heads = 8;
    c.head_dim = 128;
    c.block_tokens = 16;
    c.capacity = 8192;
    c.n_blocks = 8192 / 16;
    c.max_streams = 1;
    c.max_rows = 64;
    c.max_position = 32768;
    c.dtype = VXK_DTYPE_F16;
    c.rope_theta = 1000000.0f;
    c.alloc_seed = 0;
    c.split_pages = 0;
    return c;
}

vxk_status vxk_pool_create(const vxk_pool_config * config, vxk_pool ** out_pool) {
    if (out_pool) *out_pool = nullptr;
    if (!config || !out_pool) {
        g_create_error = "null argument";
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_pool * p = nullptr;
    try {
        p = new vxk_pool();
    } catch (...) {
        g_create_error = "host allocation failed";
        return VXK_STATUS_OUT_OF_MEMORY;
    }
    const vxk_status st = guarded(p, [&] {
        p->cfg = read_config(config);
        validate_config(p->cfg);
        int n_dev = 0;
        VXK_CUDA(cudaGetDeviceCount(&n_dev));
        if (config->device < 0 || config->device >= n_dev) fail(VXK_STATUS_INVALID_ARGUMENT, "no such CUDA device");
        DeviceScope scope(config->device);
        VXK_CUDA(cudaDeviceGetAttribute(&p->sm_count, cudaDevAttrMultiProcessorCount, config->device));
        const vxk_pool_config & c = p->cfg;
        p->bt_cap = c.capacity / c.block_tokens;
        const bool q8 = c.dtype == VXK_DTYPE_Q8_0;
        // a tile's record: its values, then (q8_0) its f16 block scales, so that
        // one bulk copy brings both
        p->tile_data_bytes = (int64_t) c.block_tokens * c.head_dim * elem_bytes(c.dtype) +
                             (q8 ? (int64_t) c.block_tokens * (c.head_dim / vxk::kQ8Block) * 2 : 0);
        p->page_data_bytes = p->tile_data_bytes * c.n_kv_heads;
        p->layer_data_bytes = p->page_data_bytes * c.n_blocks;
        const size_t data_bytes = (size_t) p->layer_data_bytes * (size_t) c.n_layers;
        p->k_data = device_alloc<uint8_t>(p, data_bytes);
        p->v_data = device_alloc<uint8_t>(p, data_bytes);
        VXK_CUDA(cudaMemset(p->k_data, 0, data_bytes));
        VXK_CUDA(cudaMemset(p->v_data, 0, data_bytes));
        const size_t table_n = (size_t) c.max_streams * (size_t) p->bt_cap;
        p->d_table = device_alloc<int32_t>(p, table_n * sizeof(int32_t));
        VXK_CUDA(cudaMemset(p->d_table, 0xff, table_n * sizeof(int32_t)));
        {
            const std::vector<float2> rope = build_rope_table(c.max_position, c.head_dim, c.rope_theta);
            p->d_rope = device_alloc<float2>(p, rope.size() * sizeof(float2));
            VXK_CUDA(cudaMemcpy(p->d_rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));
        }
        p->max_items = std::max(2048, 8 * c.max_rows);
        p->max_updates = c.max_rows + c.max_streams + 16;
        p->d_partials = device_alloc<float>(
            p, (size_t) p->max_items * (size_t) c.n_q_heads * vxk::kPartialStride * sizeof(float));
        p->d_counters = device_alloc<int32_t>(p, (size_t) c.max_rows * (size_t) c.n_kv_heads * sizeof(int32_t));
        VXK_CUDA(cudaMemset(p->d_counters, 0, (size_t) c.max_rows * (size_t) c.n_kv_heads * sizeof(int32_t)));
        p->d_error = device_alloc<int32_t>(p, sizeof(int32_t));
        VXK_CUDA(cudaMemset(p->d_error, 0, sizeof(int32_t)));
        p->off_items = align_up((size_t) c.max_rows * sizeof(vxk::RowDesc), 256);
        p->decode_slots = p->sm_count * vxk::decode_ctas_per_sm((int) c.dtype);
        if (p->decode_slots <= 0) fail(VXK_STATUS_BACKEND_ERROR, "cannot size the decode kernel grid");
        p->off_sched = p->off_items + align_up((size_t) p->max_items * sizeof(vxk::WorkItem), 256);
        // schedule: (grid + 1) offsets, grid <= units, then the unit list
        p->off_updates = p->off_sched + align_up((2 * (size_t) p->max_items * (size_t) c.n_kv_heads + 1) *
                                                     sizeof(int32_t), 256);
        p->stage_bytes = p->off_updates + align_up((size_t) p->max_updates * sizeof(vxk::TableUpdate), 256);
        p->d_stage = device_alloc<uint8_t>(p, p->stage_bytes);
        for (int i = 0; i < 2; ++i) {
            VXK_CUDA(cudaMallocHost(reinterpret_cast<void **>(&p->h_stage[i]), p->stage_bytes));
            VXK_CUDA(cudaEventCreateWithFlags(&p->stage_ev[i], cudaEventDisableTiming));
        }
        VXK_CUDA(cudaEventCreateWithFlags(&p->ev_sync, cudaEventDisableTiming));
        VXK_CUDA(cudaMallocHost(reinterpret_cast<void **>(&p->h_err), sizeof(int32_t)));
        p->streams.resize((size_t) c.max_streams);
        p->owner_stream.assign((size_t) c.n_blocks, -1);
        p->owner_entry.assign((size_t) c.n_blocks, -1);
        p->free_pages.resize((size_t) c.n_blocks);
        std::iota(p->free_pages.begin(), p->free_pages.end(), 0);
        if (c.alloc_seed != 0) {
            std::mt19937_64 rng(c.alloc_seed);
            std::shuffle(p->free_pages.begin(), p->free_pages.end(), rng);
        }
        std::reverse(p->free_pages.begin(), p->free_pages.end());
        VXK_CUDA(cudaDeviceSynchronize());
    });
    if (st != VXK_STATUS_OK) {
        g_create_error = p->last_error;
        {
            DeviceScope scope(std::max(0, config->device));
            release_device(p);
        }
        delete p;
        return st;
    }
    *out_pool = p;
    return VXK_STATUS_OK;
}

void vxk_pool_destroy(vxk_pool * pool) {
    if (!pool) return;
    {
        DeviceScope scope(pool->cfg.device);
        release_device(pool);
    }
    delete pool;
}

vxk_status vxk_pool_last_error(const vxk_pool * pool, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    const std::string & m = pool ? pool->last_error : g_create_error;
    const size_t n = std::min(capacity - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_pool_get_stats(const vxk_pool * pool, vxk_pool_stats * out) {
    if (!pool || !out) return VXK_STATUS_INVALID_ARGUMENT;
    out->pages_total = pool->cfg.n_blocks;
    out->pages_used = pool->cfg.n_blocks - (int64_t) pool->free_pages.size();
    int64_t hw = 0;
    for (int32_t i = pool->cfg.n_blocks - 1; i >= 0; --i) {
        if (pool->owner_stream[(size_t) i] >= 0) {
            hw = i + 1;
            break;
        }
    }
    out->pages_high_water = hw;
    out->streams_open = pool->streams_open;
    out->compactions = pool->compactions;
    out->pages_moved = pool->pages_moved;
    out->bytes_moved = pool->bytes_moved;
    out->device_bytes = pool->device_bytes;
    out->kernel_launches = pool->launches;
    return VXK_STATUS_OK;
}

int64_t vxk_pool_row_bytes(const vxk_pool * pool) {
    if (!pool) return -1;
    const int64_t n = (int64_t) pool->cfg.n_kv_heads * pool->cfg.head_dim;
    return pool->cfg.dtype == VXK_DTYPE_Q8_0 ? n / 32 * 34 : n * elem_bytes(pool->cfg.dtype);
}

vxk_status vxk_stream_open(vxk_pool * pool, int32_t * out_stream) {
    if (!pool || !out_stream) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        *out_stream = -1;
        for (size_t s = 0; s < pool->streams.size(); ++s) {
            StreamState & st = pool->streams[s];
            if (!st.open) {
                st.open = true;
                st.ring = vxk_decoder_kv_ring{};
                st.ring.capacity = pool->cfg.capacity;
                st.table.assign((size_t) pool->bt_cap, -1);
                ++pool->streams_open;
                *out_stream = (int32_t) s;
                return;
            }
        }
        fail(VXK_STATUS_OUT_OF_MEMORY, "all max_streams stream slots are open");
    });
}

vxk_status vxk_stream_close(vxk_pool * pool, int32_t stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (pool->planned) fail(VXK_STATUS_INVALID_STATE, "cannot close a stream while a batch is planned");
        stream_at(pool, stream);
        free_stream_pages(pool, stream);
        pool->streams[(size_t) stream].open = false;
        --pool->streams_open;
    });
}

vxk_status vxk_stream_reset(vxk_pool * pool, int32_t stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (pool->planned) fail(VXK_STATUS_INVALID_STATE, "cannot reset a stream while a batch is planned");
        StreamState & st = stream_at(pool, stream);
        free_stream_pages(pool, stream);
        st.ring = vxk_decoder_kv_ring{};
        st.ring.capacity = pool->cfg.capacity;
    });
}

vxk_status vxk_stream_get_ring(const vxk_pool * pool, int32_t stream, vxk_decoder_kv_ring * out) {
    if (!pool || !out) return VXK_STATUS_INVALID_ARGUMENT;
    if (stream < 0 || stream >= (int32_t) pool->streams.size() || !pool->streams[(size_t) stream].open)
        return VXK_STATUS_INVALID_ARGUMENT;
    *out = pool->streams[(size_t) stream].ring;
    return VXK_STATUS_OK;
}

vxk_status vxk_stream_evict(vxk_pool * pool, int32_t stream, int64_t new_oldest) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (pool->planned) fail(VXK_STATUS_INVALID_STATE, "cannot evict while a batch is planned");
        StreamState & st = stream_at(pool, stream);
        vxk_decoder_kv_ring & r = st.ring;
        if (new_oldest < r.oldest_absolute_position || new_oldest > r.next_absolute_position)
            fail(VXK_STATUS_INVALID_ARGUMENT, "new_oldest outside [oldest, next]");
        const int64_t dropped = new_oldest - r.oldest_absolute_position;
        if (dropped == 0) return;
        const int32_t bt = pool->cfg.block_tokens;
        // Ring entries still referenced by the surviving window.
        std::vector<char> live((size_t) pool->bt_cap, 0);
        if (new_oldest < r.next_absolute_position) {
            const int64_t lp0 = new_oldest / bt;
            const int64_t lp1 = (r.next_absolute_position - 1) / bt;
            if (lp1 - lp0 + 1 >= pool->bt_cap) {
                std::fill(live.begin(), live.end(), 1);
            } else {
                for (int64_t lp = lp0; lp <= lp1; ++lp) live[(size_t) (lp % pool->bt_cap)] = 1;
            }
        }
        const int64_t d0 = r.oldest_absolute_position / bt;
        const int64_t d1 = (new_oldest - 1) / bt;
        for (int64_t lp = d0; lp <= d1 && lp - d0 < pool->bt_cap; ++lp) {
            const int32_t e = (int32_t) (lp % pool->bt_cap);
            const int32_t pg = st.table[(size_t) e];
            if (!live[(size_t) e] && pg >= 0) {
                pool->free_pages.push_back(pg);
                pool->owner_stream[(size_t) pg] = -1;
                pool->owner_entry[(size_t) pg] = -1;
                st.table[(size_t) e] = -1;
            }
        }
        r.oldest_absolute_position = new_oldest;
        r.used -= dropped;
        r.evictions += dropped;
    });
}

vxk_status vxk_batch_plan(vxk_pool * pool, const int32_t * stream_ids, const int32_t * n_new,
                          int32_t n_streams, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        DeviceScope scope(pool->cfg.device);
        do_plan(pool, stream_ids, n_new, n_streams, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_batch_rows(const vxk_pool * pool, int32_t * out_rows) {
    if (!pool || !out_rows) return VXK_STATUS_INVALID_ARGUMENT;
    if (!pool->planned) return VXK_STATUS_INVALID_STATE;
    *out_rows = (int32_t) pool->rows.size();
    return VXK_STATUS_OK;
}

vxk_status vxk_batch_commit(vxk_pool * pool) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] { do_commit(pool); });
}

vxk_status vxk_batch_abort(vxk_pool * pool) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (!pool->planned) fail(VXK_STATUS_INVALID_STATE, "no batch is planned");
        rollback_new_pages(pool);
        clear_plan(pool);
    });
}

vxk_status vxk_decode_layer(vxk_pool * pool, int32_t layer, const float * q, const float * k,
                            const float * v, float * out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        check_layer(pool, layer);
        if (!pool->single_token) fail(VXK_STATUS_INVALID_STATE, "decode_layer needs a single-token batch");
        if (!q || !k || !v || !out) fail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        check_attention(pool);
        DeviceScope scope(pool->cfg.device);
        ++pool->launches;
        const bool pdl = use_pdl(pool);
        pool->batch_decodes = 0;
        VXK_CUDA(vxk::launch_decode(decode_params(pool, layer, q, k, v, out, 1),
                                    static_cast<cudaStream_t>(cuda_stream), pdl));
        pool->batch_decodes = 1;
    });
}

vxk_status vxk_decode_layer_static_scratch(vxk_pool * pool, int32_t layer, const float * q, const float * k,
                                           const float * v, float * out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        check_layer(pool, layer);
        if (!pool->single_token) fail(VXK_STATUS_INVALID_STATE, "decode_layer needs a single-token batch");
        if (!q || !k || !v || !out) fail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        check_attention(pool);
        const size_t need_partials =
            pool->items.size() * (size_t) pool->cfg.n_q_heads * (size_t) vxk::kPartialStride;
        const size_t need_counters = pool->rows.size() * (size_t) pool->cfg.n_kv_heads;
        if (need_partials > vxk::kStaticScratchPartialFloats || need_counters > vxk::kStaticScratchCounters) {
            fail(VXK_STATUS_INVALID_ARGUMENT,
                 "batch needs " + std::to_string(need_partials) + " partial floats and " +
                     std::to_string(need_counters) + " counters; the static scratch holds " +
                     std::to_string(vxk::kStaticScratchPartialFloats) + " and " +
                     std::to_string(vxk::kStaticScratchCounters));
        }
        DeviceScope scope(pool->cfg.device);
        ++pool->launches;
        pool->batch_decodes = 0;
        VXK_CUDA(vxk::launch_decode_static_scratch(decode_params(pool, layer, q, k, v, out, 1),
                                                   static_cast<cudaStream_t>(cuda_stream)));
    });
}

vxk_status vxk_append_layer(vxk_pool * pool, int32_t layer, const float * k, const float * v,
                            void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        check_layer(pool, layer);
        if (!k || !v) fail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        DeviceScope scope(pool->cfg.device);
        vxk::AppendParams a{};
        a.k_data = pool->k_data + (int64_t) layer * pool->layer_data_bytes;
        a.v_data = pool->v_data + (int64_t) layer * pool->layer_data_bytes;
        a.n_blocks = pool->cfg.n_blocks;
        a.n_kv = pool->cfg.n_kv_heads;
        a.bt_cap = pool->bt_cap;
        a.block_table = pool->d_table;
        a.rows = reinterpret_cast<const vxk::RowDesc *>(pool->d_stage);
        a.n_rows = (int32_t) pool->rows.size();
        a.k = k;
        a.v = v;
        a.rope = pool->d_rope;
        a.rope_rows = pool->cfg.max_position;
        a.error = pool->d_error;
        a.dtype = (int32_t) pool->cfg.dtype;
        ++pool->launches;
        pool->batch_decodes = 0;
        VXK_CUDA(vxk::launch_append(a, static_cast<cudaStream_t>(cuda_stream)));
    });
}

vxk_status vxk_attend_layer(vxk_pool * pool, int32_t layer, const float * q, float * out,
                            void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        check_layer(pool, layer);
        if (!q || !out) fail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        check_attention(pool);
        DeviceScope scope(pool->cfg.device);
        ++pool->launches;
        pool->batch_decodes = 0;
        VXK_CUDA(vxk::launch_decode(decode_params(pool, layer, q, nullptr, nullptr, out, 0),
                                    static_cast<cudaStream_t>(cuda_stream), false));
    });
}

vxk_status vxk_decode_step_host(vxk_pool * pool, const int32_t * stream_ids, int32_t n_streams,
                                const float * h_q, const float * h_k, const float * h_v,
                                float * h_out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (!h_q || !h_k || !h_v || !h_out) fail(VXK_STATUS_INVALID_ARGUMENT, "null host buffer");
        DeviceScope scope(pool->cfg.device);
        const vxk_pool_config & c = pool->cfg;
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        const size_t hd = (size_t) c.head_dim;
        const size_t q_per_row = (size_t) c.n_q_heads * hd;
        const size_t kv_per_row = (size_t) c.n_kv_heads * hd;
        if (n_streams <= 0 || n_streams > c.max_rows) fail(VXK_STATUS_INVALID_ARGUMENT, "bad stream count");
        // Device staging for this call's rows of every layer, grown on demand
        // (not sized by max_rows: a pool planned for long prefills would
        // otherwise hold gigabytes for a step of a few streams).
        const size_t layer_floats = (size_t) n_streams * (q_per_row * 2 + kv_per_row * 2);
        const size_t need = layer_floats * (size_t) c.n_layers * sizeof(float);
        if (pool->io_bytes < need) {
            if (pool->d_io) {
                VXK_CUDA(cudaStreamSynchronize(cs));
                cudaFree(pool->d_io);
                pool->device_bytes -= (int64_t) pool->io_bytes;
                pool->d_io = nullptr;
                pool->io_bytes = 0;
            }
            pool->d_io = device_alloc<float>(pool, need);
            pool->io_bytes = need;
        }
        if (!pool->h2d) {
            VXK_CUDA(cudaStreamCreateWithFlags(&pool->h2d, cudaStreamNonBlocking));
            VXK_CUDA(cudaStreamCreateWithFlags(&pool->d2h, cudaStreamNonBlocking));
            pool->ev_in.resize((size_t) c.n_layers);
            pool->ev_out.resize((size_t) c.n_layers);
            for (int32_t l = 0; l < c.n_layers; ++l) {
                VXK_CUDA(cudaEventCreateWithFlags(&pool->ev_in[(size_t) l], cudaEventDisableTiming));
                VXK_CUDA(cudaEventCreateWithFlags(&pool->ev_out[(size_t) l], cudaEventDisableTiming));
            }
            VXK_CUDA(cudaEventCreateWithFlags(&pool->ev_begin, cudaEventDisableTiming));
            VXK_CUDA(cudaEventCreateWithFlags(&pool->ev_done, cudaEventDisableTiming));
        }
        std::vector<int32_t> ones((size_t) std::max(0, n_streams), 1);
        do_plan(pool, stream_ids, ones.data(), n_streams, cs);
        if (!pool->items_ok) {
            rollback_new_pages(pool);
            clear_plan(pool);
            check_attention(pool);
        }
        const size_t rows = pool->rows.size();
        const int32_t L = c.n_layers;
        VXK_CUDA(cudaEventRecord(pool->ev_begin, cs));
        VXK_CUDA(cudaStreamWaitEvent(pool->h2d, pool->ev_begin, 0));
        VXK_CUDA(cudaStreamWaitEvent(pool->d2h, pool->ev_begin, 0));
        // Staging is blocked like the host buffers: [q of every layer][k][v][out],
        // so a run of layers moves as one copy per tensor.
        const size_t qn = rows * q_per_row, kvn = rows * kv_per_row;
        float * const q0 = pool->d_io;
        float * const k0 = q0 + (size_t) L * qn;
        float * const v0 = k0 + (size_t) L * kvn;
        float * const o0 = v0 + (size_t) L * kvn;
        // Inputs go up in runs of layers [2^g - 1, 2^(g+1) - 1): layer 0 waits for
        // its own rows only, and each later run is copied while the layers before
        // it compute (a run is as long as the layers ahead of it, and a layer's
        // rows copy far faster than it attends).  Outputs come down in runs that
        // end at layers L - 2^g, so the copy left after the last layer is that
        // layer's rows.  The layer kernels wait on an event only at the runs'
        // edges: every other layer boundary keeps the programmatic overlap of
        // one layer's prologue with the previous layer's tail.
        int32_t n_in = 0;
        for (int32_t first = 0; first < L; first = 2 * first + 1) {
            const int32_t end = std::min(L, 2 * first + 1);
            const size_t nl = (size_t) (end - first);
            VXK_CUDA(cudaMemcpyAsync(q0 + first * qn, h_q + first * qn, nl * qn * sizeof(float),
                                     cudaMemcpyHostToDevice, pool->h2d));
            VXK_CUDA(cudaMemcpyAsync(k0 + first * kvn, h_k + first * kvn, nl * kvn * sizeof(float),
                                     cudaMemcpyHostToDevice, pool->h2d));
            VXK_CUDA(cudaMemcpyAsync(v0 + first * kvn, h_v + first * kvn, nl * kvn * sizeof(float),
                                     cudaMemcpyHostToDevice, pool->h2d));
            VXK_CUDA(cudaEventRecord(pool->ev_in[(size_t) n_in++], pool->h2d));
        }
        int32_t in_run = 0, out_run = 0, out_first = 0;
        for (int32_t l = 0; l < L; ++l) {
            if (l == (1 << in_run) - 1) VXK_CUDA(cudaStreamWaitEvent(cs, pool->ev_in[(size_t) in_run++], 0));
            ++pool->launches;
            VXK_CUDA(vxk::launch_decode(decode_params(pool, l, q0 + l * qn, k0 + l * kvn, v0 + l * kvn, o0 + l * qn, 1),
                                        cs, l > 0));
            bool run_end = l == L - 1;
            for (int32_t g = 1; g < 31 && (1 << g) <= L; ++g) run_end = run_end || l == L - (1 << g);
            if (run_end) {
                VXK_CUDA(cudaEventRecord(pool->ev_out[(size_t) out_run], cs));
                VXK_CUDA(cudaStreamWaitEvent(pool->d2h, pool->ev_out[(size_t) out_run++], 0));
                VXK_CUDA(cudaMemcpyAsync(h_out + out_first * qn, o0 + out_first * qn,
                                         (size_t) (l + 1 - out_first) * qn * sizeof(float), cudaMemcpyDeviceToHost,
                                         pool->d2h));
                out_first = l + 1;
            }
        }
        VXK_CUDA(cudaMemcpyAsync(pool->h_err, pool->d_error, sizeof(int32_t), cudaMemcpyDeviceToHost, pool->d2h));
        VXK_CUDA(cudaEventRecord(pool->ev_done, pool->d2h));
        VXK_CUDA(cudaStreamWaitEvent(cs, pool->ev_done, 0));
        const vxk_status ws = bounded_wait(pool->ev_done, 60000);
        if (ws != VXK_STATUS_OK) {
            rollback_new_pages(pool);
            clear_plan(pool);
            fail(ws, "end-to-end step did not complete");
        }
        if (*pool->h_err != 0) {
            rollback_new_pages(pool);
            clear_plan(pool);
            check_error_word(pool);
        }
        do_commit(pool);
    });
}

vxk_status vxk_pool_probe_wait_timeout(vxk_pool * pool, int32_t limit_ms, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (limit_ms < 1 || limit_ms > 1000) fail(VXK_STATUS_INVALID_ARGUMENT, "limit_ms must be in 1..1000");
        DeviceScope scope(pool->cfg.device);
        ++pool->launches;
        VXK_CUDA(vxk::launch_wait_probe(pool->d_error, (uint64_t) limit_ms * 1000000ull,
                                        static_cast<cudaStream_t>(cuda_stream)));
    });
}

vxk_status vxk_sync(vxk_pool * pool, void * cuda_stream, int32_t timeout_ms) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        DeviceScope scope(pool->cfg.device);
        VXK_CUDA(cudaEventRecord(pool->ev_sync, static_cast<cudaStream_t>(cuda_stream)));
        const vxk_status ws = bounded_wait(pool->ev_sync, timeout_ms);
        if (ws != VXK_STATUS_OK) fail(ws, "stream did not drain within the timeout");
        check_error_word(pool);
    });
}

vxk_status vxk_pool_compact(vxk_pool * pool, void * cuda_stream, int64_t * out_pages_moved,
                            int64_t * out_bytes_moved) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (pool->planned) fail(VXK_STATUS_INVALID_STATE, "cannot compact while a batch is planned");
        DeviceScope scope(pool->cfg.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        const vxk_pool_config & c = pool->cfg;
        std::vector<int2> moves;
        // Move the highest used page into the lowest free page until the used
        // pages form a prefix of the pool.
        std::vector<int32_t> free_sorted = pool->free_pages;
        std::sort(free_sorted.begin(), free_sorted.end());
        size_t fi = 0;
        int32_t hi = c.n_blocks - 1;
        while (fi < free_sorted.size()) {
            while (hi >= 0 && pool->owner_stream[(size_t) hi] < 0) --hi;
            const int32_t lo = free_sorted[fi];
            if (hi < 0 || lo >= hi) break;
            const int32_t s = pool->owner_stream[(size_t) hi];
            const int32_t e = pool->owner_entry[(size_t) hi];
            pool->owner_stream[(size_t) lo] = s;
            pool->owner_entry[(size_t) lo] = e;
            pool->owner_stream[(size_t) hi] = -1;
            pool->owner_entry[(size_t) hi] = -1;
            pool->streams[(size_t) s].table[(size_t) e] = lo;
            moves.push_back(make_int2(hi, lo));
            ++fi;
            --hi;
        }
        if (!moves.empty()) {
            // Free pages are now exactly the unowned ones; hand out low ones first.
            pool->free_pages.clear();
            for (int32_t i = c.n_blocks - 1; i >= 0; --i) {
                if (pool->owner_stream[(size_t) i] < 0) pool->free_pages.push_back(i);
            }
        }
        const int64_t per_page = pool->page_data_bytes * 2 * c.n_layers;
        if (!moves.empty()) {
            if (!pool->d_moves) {
                pool->d_moves = device_alloc<int2>(pool, (size_t) c.n_blocks * sizeof(int2));
                VXK_CUDA(cudaMallocHost(reinterpret_cast<void **>(&pool->h_moves), (size_t) c.n_blocks * sizeof(int2)));
            }
            // Any previous use of the staging buffers must be complete.
            VXK_CUDA(cudaStreamSynchronize(cs));
            std::memcpy(pool->h_moves, moves.data(), moves.size() * sizeof(int2));
            VXK_CUDA(cudaMemcpyAsync(pool->d_moves, pool->h_moves, moves.size() * sizeof(int2),
                                     cudaMemcpyHostToDevice, cs));
            vxk::CompactParams cp{};
            cp.k_data = pool->k_data;
            cp.v_data = pool->v_data;
            cp.layer_data_bytes = pool->layer_data_bytes;
            cp.page_data_bytes = pool->page_data_bytes;
            cp.n_layers = c.n_layers;
            cp.moves = pool->d_moves;
            cp.n_moves = (int32_t) moves.size();
            ++pool->launches;
            VXK_CUDA(vxk::launch_compact(cp, cs));
            // Rewrite the moved block-table entries through the plan staging.
            pool->updates.clear();
            for (const int2 & mv : moves) {
                const int32_t s = pool->owner_stream[(size_t) mv.y];
                const int32_t e = pool->owner_entry[(size_t) mv.y];
                pool->updates.push_back({s * pool->bt_cap + e, mv.y});
                pool->streams[(size_t) s].ring.bytes_moved += per_page;
            }
            size_t done = 0;
            while (done < pool->updates.size()) {
                const size_t n = std::min(pool->updates.size() - done, (size_t) pool->max_updates);
                const int idx = pool->stage_next;
                VXK_CUDA(cudaEventSynchronize(pool->stage_ev[idx]));
                std::memcpy(pool->h_stage[idx] + pool->off_updates, pool->updates.data() + done,
                            n * sizeof(vxk::TableUpdate));
                VXK_CUDA(cudaMemcpyAsync(pool->d_stage + pool->off_updates, pool->h_stage[idx] + pool->off_updates,
                                         n * sizeof(vxk::TableUpdate), cudaMemcpyHostToDevice, cs));
                VXK_CUDA(cudaEventRecord(pool->stage_ev[idx], cs));
                pool->stage_next ^= 1;
                ++pool->launches;
                VXK_CUDA(vxk::launch_table_updates(
                    pool->d_table, reinterpret_cast<const vxk::TableUpdate *>(pool->d_stage + pool->off_updates),
                    (int32_t) n, cs));
                VXK_CUDA(cudaStreamSynchronize(cs));
                done += n;
            }
            pool->updates.clear();
        }
        const int64_t moved_bytes = (int64_t) moves.size() * per_page;
        ++pool->compactions;
        pool->pages_moved += (int64_t) moves.size();
        pool->bytes_moved += moved_bytes;
        if (out_pages_moved) *out_pages_moved = (int64_t) moves.size();
        if (out_bytes_moved) *out_bytes_moved = moved_bytes;
    });
}

vxk_status vxk_read_rows(vxk_pool * pool, int32_t layer, int32_t stream, int64_t pos_start, int32_t n,
                         void * k_out, void * v_out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return guarded(pool, [&] {
        if (!k_out || !v_out || n <= 0) fail(VXK_STATUS_INVALID_ARGUMENT, "bad output buffers or count");
        if (layer < 0 || layer >= pool->cfg.n_layers) fail(VXK_STATUS_INVALID_ARGUMENT, "layer out of range");
        const StreamState & st = stream_at(pool, stream);
        const int64_t lo = st.ring.oldest_absolute_position;
        // A planned (uncommitted) batch has already written its new rows.
        int64_t hi = st.ring.next_absolute_position;
        for (const PlanEntry & e : pool->plan) {
            if (e.stream == stream) hi = e.plan.next_after;
        }
        if (pos_start < lo || pos_start + n > hi) fail(VXK_STATUS_INVALID_ARGUMENT, "positions outside the window");
        if (pos_start + n - lo > pool->cfg.capacity) fail(VXK_STATUS_INVALID_ARGUMENT, "span exceeds capacity");
        DeviceScope scope(pool->cfg.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        const bool q8 = pool->cfg.dtype == VXK_DTYPE_Q8_0;
        const int32_t nkv = pool->cfg.n_kv_heads;
        const size_t elems = (size_t) n * (size_t) nkv * vxk::kHeadDim;
        const size_t data_b = elems * (size_t) elem_bytes(pool->cfg.dtype);
        const size_t scale_b = q8 ? (size_t) n * (size_t) nkv * (vxk::kHeadDim / vxk::kQ8Block) * 2 : 0;
        const size_t need = 2 * align_up(data_b, 256) + 2 * align_up(scale_b, 256);
        if (pool->read_bytes < need) {
            cudaFree(pool->d_read);
            pool->device_bytes -= (int64_t) pool->read_bytes;
            pool->d_read = nullptr;
            pool->read_bytes = 0;
            pool->d_read = device_alloc<uint8_t>(pool, need);
            pool->read_bytes = need;
        }
        vxk::GatherParams g{};
        g.k_data = pool->k_data + (int64_t) layer * pool->layer_data_bytes;
        g.v_data = pool->v_data + (int64_t) layer * pool->layer_data_bytes;
        g.n_blocks = pool->cfg.n_blocks;
        g.n_kv = nkv;
        g.bt_cap = pool->bt_cap;
        g.block_table = pool->d_table + (size_t) stream * (size_t) pool->bt_cap;
        g.pos_start = pos_start;
        g.n = n;
        g.k_out = pool->d_read;
        g.v_out = pool->d_read + align_up(data_b, 256);
        g.k_scale_out = pool->d_read + 2 * align_up(data_b, 256);
        g.v_scale_out = g.k_scale_out + align_up(scale_b, 256);
        g.dtype = (int32_t) pool->cfg.dtype;
        ++pool->launches;
        pool->batch_decodes = 0;
        VXK_CUDA(vxk::launch_gather(g, cs));
        std::vector<uint8_t> host(need);
        VXK_CUDA(cudaMemcpyAsync(host.data(), pool->d_read, need, cudaMemcpyDeviceToHost, cs));
        VXK_CUDA(cudaStreamSynchronize(cs));
        const uint8_t * hk = host.data();
        const uint8_t * hv = host.data() + align_up(data_b, 256);
        if (!q8) {
            std::memcpy(k_out, hk, data_b);
            std::memcpy(v_out, hv, data_b);
            return;
        }
        const uint8_t * hks = host.data() + 2 * align_up(data_b, 256);
        const uint8_t * hvs = hks + align_up(scale_b, 256);
        const size_t n_blocks = elems / vxk::kQ8Block;
        uint8_t * ko = static_cast<uint8_t *>(k_out);
        uint8_t * vo = static_cast<uint8_t *>(v_out);
        for (size_t b = 0; b < n_blocks; ++b) {
            std::memcpy(ko + b * 34, hks + b * 2, 2);
            std::memcpy(ko + b * 34 + 2, hk + b * 32, 32);
            std::memcpy(vo + b * 34, hvs + b * 2, 2);
            std::memcpy(vo + b * 34 + 2, hv + b * 32, 32);
        }
    });
}

}  // extern "C"
