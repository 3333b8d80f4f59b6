// Host runtime of the streaming-encoder KV rings (include/vxk.h).
//
// One ring of `capacity` (878) slots per (stream, layer, head), addressed by
// absolute frame % capacity; every batch is planned with the reference's
// encoder ring planner (voxtral_enc_kv_plan, src/voxtral.cpp:3656-3692) and
// the attention mask keeps q - (window - 1) <= kv <= q
// (voxtral_enc_kv_mask_allows, src/voxtral.cpp:3636-3638).
#include "vxk.h"
#include "vxk_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>


namespace {

thread_local std::string g_enc_create_error;

struct EncError {
    vxk_status status;
    std::string message;
};

[[noreturn]] void efail(vxk_status s, const std::string & m) { throw EncError{s, m}; }

#define VXK_ECUDA(expr)                                                                 \
    do {                                                                                \
        const cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                        \
            efail(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY            \
                                                  : VXK_STATUS_BACKEND_ERROR,           \
                  std::string(#expr) + ": " + cudaGetErrorString(e_));                  \
        }                                                                               \
    } while (0)

struct EncStream {
    bool open = false;
    int64_t next = 0;
    int64_t evicted = 0;
};

struct EncPlan {
    int32_t stream;
    vxk_enc_kv_plan plan;
};

// Query rows of one stream attended together (the N extent of the tensor-core
// tiles).
constexpr int kEncRowsPerGroup = 8;

// Stored rows per ring: the capacity rounded up to whole 8-slot groups (the
// pad rows stay zero), so that 128-byte swizzled rows of any 8-aligned run of
// slots form the tensor cores' shared-memory layout after a plain bulk copy.
int32_t ring_slots_of(int32_t capacity) { return (capacity + 7) & ~7; }

// Bytes of one stored ring value: fp32 rows for F32 rings, 16-bit otherwise.
size_t ring_elem_bytes(vxk_dtype dt) { return dt == VXK_DTYPE_F32 ? 4 : 2; }

}  // namespace

struct vxk_enc_pool {
    vxk_enc_config cfg{};
    uint8_t * k_ring = nullptr;
    uint8_t * v_ring = nullptr;
    float2 * d_rope = nullptr;
    int32_t * d_error = nullptr;
    uint8_t * d_stage = nullptr;
    uint8_t * h_stage = nullptr;
    cudaEvent_t stage_ev = nullptr;
    size_t stage_bytes = 0;
    size_t off_groups = 0;   // capacity of the row region
    size_t cur_groups = 0;   // the current batch's group table, right after its rows
    size_t cur_gdesc = 0;    // and its group descriptors, right after the table
    std::vector<EncStream> streams;
    bool planned = false;
    std::vector<EncPlan> plan;
    std::vector<vxk::EncRowDesc> rows;
    std::vector<int32_t> group_first;
    std::vector<int32_t> gdesc;  // 8 ints per group (vxk::EncParams::groups)
    bool one_group_per_stream = false;  // every stream of the batch has <= kEncRowsPerGroup new rows
    int32_t max_group_rows = 0;         // most rows in one group of the batch
    std::vector<uint8_t> h_read;  // readback staging of vxk_enc_read_slots
    std::string last_error;
};

namespace {

template <typename F>
vxk_status eguarded(vxk_enc_pool * pool, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const EncError & e) {
        if (pool) pool->last_error = e.message;
        return e.status;
    } catch (...) {
        if (pool) pool->last_error = "internal error";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

void enc_release(vxk_enc_pool * p) {
    cudaFree(p->k_ring);
    cudaFree(p->v_ring);
    cudaFree(p->d_rope);
    cudaFree(p->d_error);
    cudaFree(p->d_stage);
    if (p->h_stage) cudaFreeHost(p->h_stage);
    if (p->stage_ev) cudaEventDestroy(p->stage_ev);
}

EncStream & enc_stream_at(vxk_enc_pool * p, int32_t s) {
    if (s < 0 || s >= (int32_t) p->streams.size() || !p->streams[(size_t) s].open)
        efail(VXK_STATUS_INVALID_ARGUMENT, "encoder stream id is not open");
    return p->streams[(size_t) s];
}

class EncDevice {
public:
    explicit EncDevice(int d) {
        cudaGetDevice(&prev_);
        dev_ = d;
        if (prev_ != d) cudaSetDevice(d);
    }
    ~EncDevice() {
        if (prev_ != dev_) cudaSetDevice(prev_);
    }

private:
    int prev_ = 0, dev_ = 0;
};

vxk::EncParams enc_params(vxk_enc_pool * p, int32_t layer, const float * q, const float * k,
                          const float * v, float * out) {
    vxk::EncParams e{};
    e.k_ring = p->k_ring;
    e.v_ring = p->v_ring;
    e.n_layers = p->cfg.n_layers;
    e.layer = layer;
    e.n_heads = p->cfg.n_heads;
    e.capacity = p->cfg.capacity;
    e.ring_slots = ring_slots_of(p->cfg.capacity);
    e.window = p->cfg.window;
    e.rows = reinterpret_cast<const vxk::EncRowDesc *>(p->d_stage);
    e.n_rows = (int32_t) p->rows.size();
    e.group_first = reinterpret_cast<const int32_t *>(p->d_stage + p->cur_groups);
    e.n_groups = (int32_t) p->group_first.size() - 1;
    e.groups = reinterpret_cast<const int4 *>(p->d_stage + p->cur_gdesc);
    e.q = q;
    e.k = k;
    e.v = v;
    e.out = out;
    e.rope = p->d_rope;
    e.rope_rows = p->cfg.max_position;
    e.scale_log2 = (1.0f / sqrtf((float) p->cfg.head_dim)) * 1.4426950408889634f;
    e.error = p->d_error;
    e.dtype = (int32_t) p->cfg.dtype;
    e.max_group_rows = p->max_group_rows;
    return e;
}

}  // namespace

namespace vxk {

bool enc_pool_batch_view(const vxk_enc_pool * pool, EncBatchView * out) {
    if (!pool || !out || !pool->planned) return false;
    out->streams.clear();
    out->n_new.clear();
    out->q_start.clear();
    for (const EncPlan & e : pool->plan) {
        out->streams.push_back(e.stream);
        out->n_new.push_back(e.plan.n_new);
        out->q_start.push_back(e.plan.q_start);
    }
    out->rows = (int32_t) pool->rows.size();
    return true;
}

int32_t * enc_pool_error_word(const vxk_enc_pool * pool) { return pool->d_error; }

EncShape enc_pool_shape(const vxk_enc_pool * pool) {
    const vxk_enc_config & c = pool->cfg;
    return EncShape{c.device, c.n_layers, c.n_heads, c.head_dim, c.max_streams, c.max_new, c.rope_theta};
}

}  // namespace vxk

extern "C" {

vxk_enc_config vxk_enc_default_config(void) {
    vxk_enc_config c{};
    c.struct_size = sizeof(vxk_enc_config);
    c.api_version = VXK_API_VERSION;
    c.device = 0;
    c.n_layers = 32;
    c.n_heads = 32;
    c.head_dim = 64;
    c.window = 750;
    c.capacity = 878;
    c.max_streams = 1;
    c.max_new = 128;
    c.max_position = 131072;
    c.dtype = VXK_DTYPE_BF16;
    c.rope_theta = 1000000.0f;
    return c;
}

vxk_status vxk_enc_create(const vxk_enc_config * config, vxk_enc_pool ** out) {
    if (out) *out = nullptr;
    if (!config || !out) {
        g_enc_create_error = "null argument";
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_enc_pool * p = new (std::nothrow) vxk_enc_pool();
    if (!p) return VXK_STATUS_OUT_OF_MEMORY;
    const vxk_status st = eguarded(p, [&] {
        const vxk_enc_config & c = *config;
        if (c.struct_size < sizeof(vxk_enc_config)) efail(VXK_STATUS_INVALID_ARGUMENT, "config struct_size too small");
        if (c.head_dim != 64) efail(VXK_STATUS_INVALID_ARGUMENT, "encoder head_dim must be 64");
        if (c.n_layers < 1 || c.n_heads < 1 || c.max_streams < 1 || c.max_position < 1)
            efail(VXK_STATUS_INVALID_ARGUMENT, "bad encoder shape");
        if (c.window < 1 || c.capacity <= c.window || c.max_new < 1 || c.max_new > c.capacity - c.window)
            efail(VXK_STATUS_INVALID_ARGUMENT, "need 1 <= max_new <= capacity - window");
        {
            // A row group's window (window - 1 + 8 keys), its alignment to
            // 8-slot boxes and the zero pad of the last box must fit the
            // attention kernel's 6 tiles of 128 keys.
            const int pad = ((c.capacity + 7) & ~7) - c.capacity;
            if (7 + (c.window - 1) + (kEncRowsPerGroup - 1) + pad >= 128 * vxk::enc_max_tiles())
                efail(VXK_STATUS_INVALID_ARGUMENT, "window too large for the encoder attention tiles (max 752)");
        }
        if (c.dtype != VXK_DTYPE_BF16 && c.dtype != VXK_DTYPE_F16 && c.dtype != VXK_DTYPE_F32)
            efail(VXK_STATUS_INVALID_ARGUMENT, "encoder dtype must be BF16, F16 or F32");
        p->cfg = c;
        int n_dev = 0;
        VXK_ECUDA(cudaGetDeviceCount(&n_dev));
        if (c.device < 0 || c.device >= n_dev) efail(VXK_STATUS_INVALID_ARGUMENT, "no such CUDA device");
        EncDevice scope(c.device);
        const size_t ring_bytes = (size_t) c.max_streams * c.n_layers * c.n_heads * (size_t) ring_slots_of(c.capacity) *
                                  c.head_dim * ring_elem_bytes(c.dtype);
        VXK_ECUDA(cudaMalloc(&p->k_ring, ring_bytes));
        VXK_ECUDA(cudaMalloc(&p->v_ring, ring_bytes));
        VXK_ECUDA(cudaMemset(p->k_ring, 0, ring_bytes));
        VXK_ECUDA(cudaMemset(p->v_ring, 0, ring_bytes));
        {
            const int32_t half = c.head_dim / 2;
            std::vector<float2> rope((size_t) c.max_position * half);
            const float theta_scale = powf(c.rope_theta, -2.0f / (float) c.head_dim);
            for (int32_t pos = 0; pos < c.max_position; ++pos) {
                float theta = (float) pos;
                for (int32_t i = 0; i < half; ++i) {
                    rope[(size_t) pos * half + i] = make_float2(cosf(theta), sinf(theta));
                    theta = theta * theta_scale;
                }
            }
            VXK_ECUDA(cudaMalloc(&p->d_rope, rope.size() * sizeof(float2)));
            VXK_ECUDA(cudaMemcpy(p->d_rope, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice));
        }
        VXK_ECUDA(cudaMalloc(&p->d_error, sizeof(int32_t)));
        VXK_ECUDA(cudaMemset(p->d_error, 0, sizeof(int32_t)));
        const size_t max_rows = (size_t) c.max_streams * c.max_new;
        const size_t max_groups = max_rows;  // at most one group per row
        p->off_groups = (max_rows * sizeof(vxk::EncRowDesc) + 255) / 256 * 256;
        p->stage_bytes = p->off_groups + ((max_groups + 1) * sizeof(int32_t) + 15) / 16 * 16 +
                         (size_t) max_groups * 8 * sizeof(int32_t);
        VXK_ECUDA(cudaMalloc(&p->d_stage, p->stage_bytes));
        VXK_ECUDA(cudaMallocHost(reinterpret_cast<void **>(&p->h_stage), p->stage_bytes));
        VXK_ECUDA(cudaEventCreateWithFlags(&p->stage_ev, cudaEventDisableTiming));
        p->streams.resize((size_t) c.max_streams);
        VXK_ECUDA(cudaDeviceSynchronize());
    });
    if (st != VXK_STATUS_OK) {
        g_enc_create_error = p->last_error;
        enc_release(p);
        delete p;
        return st;
    }
    *out = p;
    return VXK_STATUS_OK;
}

void vxk_enc_destroy(vxk_enc_pool * pool) {
    if (!pool) return;
    {
        EncDevice scope(pool->cfg.device);
        enc_release(pool);
    }
    delete pool;
}

vxk_status vxk_enc_last_error(const vxk_enc_pool * pool, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    const std::string & m = pool ? pool->last_error : g_enc_create_error;
    const size_t n = std::min(capacity - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_enc_stream_open(vxk_enc_pool * pool, int32_t * out_stream) {
    if (!pool || !out_stream) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        *out_stream = -1;
        for (size_t s = 0; s < pool->streams.size(); ++s) {
            if (!pool->streams[s].open) {
                pool->streams[s] = EncStream{};
                pool->streams[s].open = true;
                *out_stream = (int32_t) s;
                return;
            }
        }
        efail(VXK_STATUS_OUT_OF_MEMORY, "all encoder stream slots are open");
    });
}

vxk_status vxk_enc_stream_close(vxk_enc_pool * pool, int32_t stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        if (pool->planned) efail(VXK_STATUS_INVALID_STATE, "a batch is planned");
        enc_stream_at(pool, stream).open = false;
    });
}

vxk_status vxk_enc_stream_reset(vxk_enc_pool * pool, int32_t stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        if (pool->planned) efail(VXK_STATUS_INVALID_STATE, "a batch is planned");
        EncStream & s = enc_stream_at(pool, stream);
        s.next = 0;
        s.evicted = 0;
    });
}

vxk_status vxk_enc_stream_position(const vxk_enc_pool * pool, int32_t stream, int64_t * out_next,
                                   int64_t * out_evicted) {
    if (!pool || stream < 0 || stream >= (int32_t) pool->streams.size() || !pool->streams[(size_t) stream].open)
        return VXK_STATUS_INVALID_ARGUMENT;
    if (out_next) *out_next = pool->streams[(size_t) stream].next;
    if (out_evicted) *out_evicted = pool->streams[(size_t) stream].evicted;
    return VXK_STATUS_OK;
}

vxk_status vxk_enc_batch_plan(vxk_enc_pool * pool, const int32_t * stream_ids, const int32_t * n_new,
                              int32_t n_streams, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        if (pool->planned) efail(VXK_STATUS_INVALID_STATE, "a batch is already planned");
        if (!stream_ids || !n_new || n_streams <= 0) efail(VXK_STATUS_INVALID_ARGUMENT, "empty batch");
        const vxk_enc_config & c = pool->cfg;
        std::vector<char> seen(pool->streams.size(), 0);
        pool->plan.clear();
        pool->rows.clear();
        pool->group_first.clear();
        for (int32_t i = 0; i < n_streams; ++i) {
            EncStream & st = enc_stream_at(pool, stream_ids[i]);
            if (seen[(size_t) stream_ids[i]]) efail(VXK_STATUS_INVALID_ARGUMENT, "stream listed twice");
            seen[(size_t) stream_ids[i]] = 1;
            if (n_new[i] > c.max_new) efail(VXK_STATUS_INVALID_ARGUMENT, "n_new exceeds max_new");
            vxk_enc_kv_plan pl;
            if (vxk_enc_kv_plan_make(st.next, n_new[i], c.capacity, c.window, &pl) != VXK_STATUS_OK)
                efail(VXK_STATUS_INVALID_ARGUMENT, "invalid encoder ring plan");
            if (pl.win_end - 1 >= (int64_t) c.max_position)
                efail(VXK_STATUS_INVALID_ARGUMENT, "position beyond the RoPE table (max_position)");
            for (int32_t t = 0; t < n_new[i]; ++t) {
                if (t % kEncRowsPerGroup == 0) pool->group_first.push_back((int32_t) pool->rows.size());
                vxk::EncRowDesc rd{};
                const int64_t pos = pl.q_start + t;
                rd.stream = stream_ids[i];
                rd.pos = (int32_t) pos;
                rd.win_start = (int32_t) std::max<int64_t>(0, pos - (c.window - 1));
                rd.slot = (int32_t) (pos % c.capacity);
                pool->rows.push_back(rd);
            }
            pool->plan.push_back({stream_ids[i], pl});
        }
        pool->group_first.push_back((int32_t) pool->rows.size());
        pool->one_group_per_stream = true;
        for (int32_t i = 0; i < n_streams; ++i)
            if (n_new[i] > kEncRowsPerGroup) pool->one_group_per_stream = false;
        pool->max_group_rows = 0;
        for (size_t g = 0; g + 1 < pool->group_first.size(); ++g)
            pool->max_group_rows = std::max(pool->max_group_rows, pool->group_first[g + 1] - pool->group_first[g]);
        EncDevice scope(c.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        VXK_ECUDA(cudaEventSynchronize(pool->stage_ev));
        const size_t rows_b = pool->rows.size() * sizeof(vxk::EncRowDesc);
        const size_t n_groups = pool->group_first.size() - 1;
        pool->gdesc.resize(8 * n_groups);
        const int32_t vslots = ring_slots_of(c.capacity);
        for (size_t g = 0; g < n_groups; ++g) {
            const int32_t r0 = pool->group_first[g], nr = pool->group_first[g + 1] - r0;
            const int32_t ws = pool->rows[(size_t) r0].win_start, we = pool->rows[(size_t) (r0 + nr - 1)].pos;
            const int32_t s0 = (ws % c.capacity) & ~7, wem = we % c.capacity;
            int32_t * d = &pool->gdesc[8 * g];
            d[0] = r0 | (nr << 24);
            d[1] = pool->rows[(size_t) r0].stream;
            d[2] = ws;
            d[3] = we;
            d[4] = s0;                                    // first 8-slot box of the window walk
            d[5] = ((wem - s0 + vslots) % vslots) / 8 + 1;  // boxes walked
            d[6] = wem;                                   // slot of the last row
            d[7] = 0;
        }
        pool->cur_groups = (rows_b + 255) / 256 * 256;  // <= off_groups: one copy of the used bytes
        pool->cur_gdesc = pool->cur_groups + (pool->group_first.size() * sizeof(int32_t) + 15) / 16 * 16;
        std::memcpy(pool->h_stage, pool->rows.data(), rows_b);
        std::memcpy(pool->h_stage + pool->cur_groups, pool->group_first.data(), pool->group_first.size() * sizeof(int32_t));
        std::memcpy(pool->h_stage + pool->cur_gdesc, pool->gdesc.data(), pool->gdesc.size() * sizeof(int32_t));
        VXK_ECUDA(cudaMemcpyAsync(pool->d_stage, pool->h_stage, pool->cur_gdesc + pool->gdesc.size() * sizeof(int32_t),
                                  cudaMemcpyHostToDevice, cs));
        VXK_ECUDA(cudaEventRecord(pool->stage_ev, cs));
        pool->planned = true;
    });
}

vxk_status vxk_enc_batch_rows(const vxk_enc_pool * pool, int32_t * out_rows) {
    if (!pool || !out_rows) return VXK_STATUS_INVALID_ARGUMENT;
    if (!pool->planned) return VXK_STATUS_INVALID_STATE;
    *out_rows = (int32_t) pool->rows.size();
    return VXK_STATUS_OK;
}

vxk_status vxk_enc_batch_commit(vxk_enc_pool * pool) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        if (!pool->planned) efail(VXK_STATUS_INVALID_STATE, "no batch is planned");
        for (const EncPlan & e : pool->plan) {
            EncStream & st = pool->streams[(size_t) e.stream];
            st.next = e.plan.win_end;
            st.evicted += e.plan.evicted;
        }
        pool->plan.clear();
        pool->rows.clear();
        pool->group_first.clear();
        pool->planned = false;
    });
}

vxk_status vxk_enc_layer(vxk_enc_pool * pool, int32_t layer, const float * q, const float * k,
                         const float * v, float * out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        if (!pool->planned) efail(VXK_STATUS_INVALID_STATE, "no batch is planned");
        if (layer < 0 || layer >= pool->cfg.n_layers) efail(VXK_STATUS_INVALID_ARGUMENT, "layer out of range");
        if (!q || !k || !v || !out) efail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        EncDevice scope(pool->cfg.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        vxk::EncParams e = enc_params(pool, layer, q, k, v, out);
        // One group per stream (the steady chunk of <= 8 frames): no other
        // group reads a group's new rows, so the attention kernel stores them
        // itself; otherwise later groups of a stream read the rows of earlier
        // ones, which the separate append kernel writes first.
        e.fuse_append = pool->one_group_per_stream && pool->cfg.dtype != VXK_DTYPE_F32 ? 1 : 0;
        if (!e.fuse_append) VXK_ECUDA(vxk::launch_enc_append(e, cs));
        VXK_ECUDA(vxk::launch_enc_attention(e, cs));
    });
}

vxk_status vxk_enc_read_slots(vxk_enc_pool * pool, int32_t layer, int32_t stream, int32_t slot0, int32_t n,
                              void * k_out, void * v_out, void * cuda_stream) {
    if (!pool) return VXK_STATUS_INVALID_ARGUMENT;
    return eguarded(pool, [&] {
        const vxk_enc_config & c = pool->cfg;
        enc_stream_at(pool, stream);
        if (layer < 0 || layer >= c.n_layers || slot0 < 0 || n <= 0 || slot0 + n > c.capacity || !k_out || !v_out)
            efail(VXK_STATUS_INVALID_ARGUMENT, "bad slot range or buffers");
        EncDevice scope(c.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        VXK_ECUDA(cudaStreamSynchronize(cs));
        const size_t row_b = (size_t) c.head_dim * ring_elem_bytes(c.dtype);
        const int32_t rs = ring_slots_of(c.capacity);
        uint8_t * outs[2] = {static_cast<uint8_t *>(k_out), static_cast<uint8_t *>(v_out)};
        const uint8_t * rings[2] = {pool->k_ring, pool->v_ring};
        pool->h_read.resize((size_t) n * row_b);
        // out layout [n][n_heads][head_dim]; ring rows are stored with the
        // 16-byte chunk c of slot s at chunk c ^ (s & 7)
        for (int kv = 0; kv < 2; ++kv) {
            for (int32_t h = 0; h < c.n_heads; ++h) {
                const size_t base = ((((size_t) stream * c.n_layers + layer) * c.n_heads + h) * (size_t) rs + slot0) * row_b;
                VXK_ECUDA(cudaMemcpy(pool->h_read.data(), rings[kv] + base, (size_t) n * row_b, cudaMemcpyDeviceToHost));
                for (int32_t i = 0; i < n; ++i) {
                    const int32_t slot = slot0 + i;
                    const uint8_t * src = pool->h_read.data() + (size_t) i * row_b;
                    uint8_t * dst = outs[kv] + ((size_t) i * c.n_heads + h) * row_b;
                    for (size_t ch = 0; ch < row_b / 16; ++ch)
                        std::memcpy(dst + ch * 16, src + ((ch ^ (size_t) (slot & 7)) * 16), 16);
                }
            }
        }
    });
}

}  // extern "C"
