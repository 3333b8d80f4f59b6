// Host runtime of the whole decoder step (include/vxk.h, vxk_decoder_*): the
// model's decoder, head and adapter loaded from a GGUF file onto the pool's
// device, the per-stream encoder-output and audio-embedding rings, and the
// launch sequence of one forward over the pool's planned batch.
//
// One forward (the reference builds it per context as the step graph,
// src/voxtral.cpp:3047-3104, or the prefill graph, 2891-2965):
//   embed_norm                       x = emb[token] + audio[slot]; xn = norm(x) * attn_norm[0]
//   per layer l (products in calls of <= 512 rows):
//     q, k, v = W{q,k,v} xn          one activation quantization for the three
//     attention                      vxk_decode_layer (one token per stream) or
//                                    vxk_append_layer + vxk_attend_layer (prefill)
//     proj = Wo att
//     add_norm                       x += proj; xn = norm(x) * ffn_norm[l] * (1 + ada[l])
//     gate, up = W1 xn, W3 xn; proj = W2 (silu(gate) * up), the SwiGLU
//                                    inside W2's activation quantization
//     add_norm                       x += proj; xn = norm(x) * attn_norm[l + 1]
//                                    (after the last layer: dec_norm, each stream's last row only)
//   head                             logits and argmax of those rows
//
// The time conditioning ada[l] = ada2 . gelu_erf(ada0 . time_emb) depends only
// on the model and t (compute_time_embedding, src/voxtral.cpp:730-741), so it is
// computed once here, in fp64 over the weights as ggml's CPU dequantizers give
// them and the activation rounded as ggml's vec_dot_type quantization rounds it.
#include "vxk.h"
#include "vxk_dequant.h"
#include "vxk_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <new>
#include <mutex>
#include <string>
#include <vector>

namespace {

struct DecError {
    vxk_status status;
    std::string message;
};

[[noreturn]] void dfail(vxk_status st, const std::string & m) { throw DecError{st, m}; }

#define VXK_DCUDA(expr)                                                                                     \
    do {                                                                                                    \
        const cudaError_t e_ = (expr);                                                                      \
        if (e_ != cudaSuccess)                                                                              \
            dfail(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY : VXK_STATUS_BACKEND_ERROR,    \
                  std::string(#expr) + ": " + cudaGetErrorString(e_));                                      \
    } while (0)

#define VXK_DCALL(expr, what)                                                                               \
    do {                                                                                                    \
        const vxk_status s_ = (expr);                                                                       \
        if (s_ != VXK_STATUS_OK) dfail(s_, std::string(what) + " failed (" + vxk_status_string(s_) + ")");  \
    } while (0)

std::mutex g_create_mutex;
std::string g_create_error;

struct DevScope {
    int prev = 0;
    explicit DevScope(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~DevScope() { cudaSetDevice(prev); }
};

struct Layer {
    vxk_qweight * q = nullptr;
    vxk_qweight * k = nullptr;
    vxk_qweight * v = nullptr;
    vxk_qweight * o = nullptr;
    vxk_qweight * w1 = nullptr;
    vxk_qweight * w3 = nullptr;
    vxk_qweight * w2 = nullptr;
};

bool is_qtype(int t) { return t == VXK_QTYPE_Q8_0 || t == VXK_QTYPE_Q4_K || t == VXK_QTYPE_Q6_K; }

}  // namespace

struct vxk_decoder {
    vxk_decoder_config cfg{};
    vxk_pool * pool = nullptr;
    vxk::PoolShape ps{};
    int32_t dim = 0, hidden = 0, vocab = 0, ada_dim = 0, n_layers = 0, enc_dim = 0;
    int32_t chunk = 64;  // rows per product call (up to 512)
    float eps = 1e-5f;
    std::vector<Layer> layers;
    std::vector<vxk_qweight *> all_q;
    vxk_qweight * head_q = nullptr;
    vxk_head * head = nullptr;
    uint8_t * emb = nullptr;
    int32_t emb_type = 0;
    int64_t emb_row_bytes = 0;
    const uint8_t * head_w16 = nullptr;  // f16 / bf16 head matrix (may be emb)
    uint8_t * head_w16_own = nullptr;
    int32_t head_type = 0;
    vxk_qweight * ad0 = nullptr;
    vxk_qweight * ad2 = nullptr;
    float * attn_norm = nullptr;  // [L][dim]
    float * ffn_norm = nullptr;   // [L][dim]
    float * dec_norm = nullptr;   // [dim]
    float * ada = nullptr;        // [L][dim] or nullptr
    float * audio = nullptr;      // [max_streams][audio_cap][dim]
    float * enc = nullptr;        // [max_streams][enc_cap][enc_dim]
    float * x = nullptr;
    float * xn = nullptr;
    float * q = nullptr;
    float * k = nullptr;
    float * v = nullptr;
    float * att = nullptr;
    float * proj = nullptr;
    float * gate = nullptr;
    float * up = nullptr;
    float * hn = nullptr;
    float * ad_in = nullptr;
    float * ad_mid = nullptr;
    float * ad_out = nullptr;
    vxk::DecRow * d_rows = nullptr;
    vxk::AdaptRow * d_adapt = nullptr;
    int32_t * d_error = nullptr;
    uint8_t * h_stage[2] = {nullptr, nullptr};
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    int stage_next = 0;
    size_t stage_bytes = 0;
    int64_t device_bytes = 0;
    std::vector<vxk::DecRow> h_rows;
    std::vector<vxk::AdaptRow> h_adapt;
    vxk::PoolBatchView view;
    std::string last_error;
};

namespace {

template <typename F>
vxk_status dguarded(vxk_decoder * d, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const DecError & e) {
        if (d) d->last_error = e.message;
        return e.status;
    } catch (const std::bad_alloc &) {
        if (d) d->last_error = "host allocation failed";
        return VXK_STATUS_OUT_OF_MEMORY;
    } catch (...) {
        if (d) d->last_error = "unexpected exception";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

template <typename T>
T * dalloc(vxk_decoder * d, size_t count) {
    void * p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    VXK_DCUDA(cudaMalloc(&p, bytes));
    d->device_bytes += (int64_t) bytes;
    return static_cast<T *>(p);
}

void destroy(vxk_decoder * d) {
    if (!d) return;
    DevScope scope(d->ps.device);
    for (vxk_qweight * w : d->all_q) {
        vxk::qweight_attach_error(w, nullptr);
        vxk_qweight_destroy(w);
    }
    if (d->head) vxk_head_destroy(d->head);
    for (void * p : {(void *) d->emb, (void *) d->head_w16_own, (void *) d->attn_norm, (void *) d->ffn_norm,
                     (void *) d->dec_norm, (void *) d->ada, (void *) d->audio, (void *) d->enc, (void *) d->x,
                     (void *) d->xn, (void *) d->q, (void *) d->k, (void *) d->v, (void *) d->att, (void *) d->proj,
                     (void *) d->gate, (void *) d->up, (void *) d->hn, (void *) d->ad_in,
                     (void *) d->ad_mid, (void *) d->ad_out, (void *) d->d_rows, (void *) d->d_adapt,
                     (void *) d->d_error})
        if (p) cudaFree(p);
    for (int i = 0; i < 2; ++i) {
        if (d->h_stage[i]) cudaFreeHost(d->h_stage[i]);
        if (d->stage_ev[i]) cudaEventDestroy(d->stage_ev[i]);
    }
    delete d;
}

// ---- GGUF access --------------------------------------------------------

struct TensorRef {
    vxk_gguf_tensor info{};
    const uint8_t * data = nullptr;
};

bool find(const vxk_gguf * g, const std::string & name, TensorRef * out) {
    const int64_t i = vxk_gguf_find_tensor(g, name.c_str());
    if (i < 0) return false;
    if (vxk_gguf_get_tensor(g, i, &out->info) != VXK_STATUS_OK) return false;
    out->data = static_cast<const uint8_t *>(vxk_gguf_tensor_data(g, i));
    return out->data != nullptr;
}

TensorRef need(const vxk_gguf * g, const std::string & name) {
    TensorRef t;
    if (!find(g, name, &t)) dfail(VXK_STATUS_INVALID_ARGUMENT, "tensor " + name + " is missing");
    return t;
}

int64_t key_int(const vxk_gguf * g, const char * key, int64_t def) {
    int64_t v = 0;
    return vxk_gguf_get_int(g, key, &v) == VXK_STATUS_OK ? v : def;
}

double key_float(const vxk_gguf * g, const char * key, double def) {
    double v = 0;
    return vxk_gguf_get_float(g, key, &v) == VXK_STATUS_OK ? v : def;
}

void check_matrix(const TensorRef & t, const std::string & name, int64_t rows, int64_t cols) {
    if (t.info.n_dims != 2 || t.info.ne[0] != cols || t.info.ne[1] != rows)
        dfail(VXK_STATUS_INVALID_ARGUMENT, name + " must be " + std::to_string(rows) + " x " + std::to_string(cols));
}

vxk_qweight * load_q(vxk_decoder * d, const vxk_gguf * g, const std::string & name, int64_t rows, int64_t cols) {
    const TensorRef t = need(g, name);
    check_matrix(t, name, rows, cols);
    if (!is_qtype(t.info.type))
        dfail(VXK_STATUS_INVALID_ARGUMENT, name + ": matrices must be Q8_0, Q4_K or Q6_K (type " +
                                               std::to_string(t.info.type) + ")");
    vxk_qweight * w = nullptr;
    const vxk_status st = vxk_qweight_create_from_gguf(g, name.c_str(), d->ps.device, d->chunk, &w);
    if (st != VXK_STATUS_OK) {
        char buf[512] = {0};
        vxk_qweight_last_error(nullptr, buf, sizeof(buf));
        dfail(st, name + ": " + buf);
    }
    d->all_q.push_back(w);
    vxk::qweight_attach_error(w, d->d_error);
    size_t packed = 0;
    if (vxk_qweight_packed_bytes((vxk_qtype) t.info.type, (int32_t) rows, (int32_t) cols, &packed) == VXK_STATUS_OK)
        d->device_bytes += (int64_t) packed;
    return w;
}

// A norm vector (F32, F16 or BF16) as fp32.
std::vector<float> load_vector(const vxk_gguf * g, const std::string & name, int64_t n) {
    const TensorRef t = need(g, name);
    if (t.info.n_dims != 1 || t.info.ne[0] != n)
        dfail(VXK_STATUS_INVALID_ARGUMENT, name + " must be a vector of " + std::to_string(n));
    if (t.info.type != 0 && t.info.type != 1 && t.info.type != 30)
        dfail(VXK_STATUS_INVALID_ARGUMENT, name + " must be F32, F16 or BF16");
    std::vector<float> out((size_t) n);
    for (int64_t i = 0; i < n; ++i) out[(size_t) i] = vxk::dequant_elem(t.data, t.info.type, i);
    return out;
}

// ---- time conditioning (load time, host) ---------------------------------

// x as ggml's vec_dot_type for weight type wt rounds it before the dot
// product: F16 / BF16 round to 16 bits; Q8_0 weights quantize x to Q8_0
// (quantize_row_q8_0_ref: d = amax / 127 stored as f16, q = roundf(x / d));
// K-quants quantize x to Q8_K (quantize_row_q8_K_ref: the value of largest
// magnitude, first on ties, sets iscale = -127 / max; q = nearest(iscale *
// x) capped at 127; d = 1 / iscale).  Returned as the values the dot sees.
std::vector<float> act_roundtrip(int wt, const std::vector<float> & x) {
    std::vector<float> y(x.size());
    const size_t n = x.size();
    if (wt == 0) return x;
    if (wt == 1) {
        for (size_t i = 0; i < n; ++i) y[i] = (float) (_Float16) x[i];
        return y;
    }
    if (wt == 30) {
        for (size_t i = 0; i < n; ++i) {
            uint32_t b;
            std::memcpy(&b, &x[i], 4);
            b = (b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u;
            std::memcpy(&y[i], &b, 4);
        }
        return y;
    }
    if (wt == VXK_QTYPE_Q8_0) {
        for (size_t b0 = 0; b0 < n; b0 += 32) {
            float amax = 0.0f;
            for (size_t j = b0; j < b0 + 32; ++j) amax = std::max(amax, std::fabs(x[j]));
            const float dd = amax / 127.0f;
            const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
            const float dh = (float) (_Float16) dd;
            for (size_t j = b0; j < b0 + 32; ++j) y[j] = dh * std::roundf(x[j] * id);
        }
        return y;
    }
    for (size_t b0 = 0; b0 < n; b0 += 256) {
        float amax = 0.0f, mx = 0.0f;
        for (size_t j = b0; j < b0 + 256; ++j) {
            const float ax = std::fabs(x[j]);
            if (ax > amax) {
                amax = ax;
                mx = x[j];
            }
        }
        if (amax == 0.0f) {
            for (size_t j = b0; j < b0 + 256; ++j) y[j] = 0.0f;
            continue;
        }
        const float iscale = -127.0f / mx;
        const float dd = 1.0f / iscale;
        for (size_t j = b0; j < b0 + 256; ++j) {
            const float qv = std::min(127.0f, std::nearbyint(iscale * x[j]));
            y[j] = dd * qv;
        }
    }
    return y;
}

// y = W x for a GGUF matrix of any handled type, fp64 sums (exact-math
// target of ggml's product on the rounded activation).
std::vector<float> matvec_host(const TensorRef & w, const std::vector<float> & x) {
    const int64_t cols = w.info.ne[0], rows = w.info.ne[1];
    const int64_t rb = vxk::gguf_row_bytes(w.info.type, cols);
    if (rb == 0) dfail(VXK_STATUS_INVALID_ARGUMENT, std::string(w.info.name) + ": unsupported type");
    if ((int64_t) x.size() != cols) dfail(VXK_STATUS_INVALID_ARGUMENT, "time MLP shape mismatch");
    const std::vector<float> xq = act_roundtrip(w.info.type, x);
    std::vector<float> y((size_t) rows);
    for (int64_t i = 0; i < rows; ++i) {
        double s = 0.0;
        const uint8_t * row = w.data + i * rb;
        for (int64_t j = 0; j < cols; ++j) s += (double) vxk::dequant_elem(row, w.info.type, j) * (double) xq[(size_t) j];
        y[(size_t) i] = (float) s;
    }
    return y;
}

// compute_time_embedding (src/voxtral.cpp:730-741): cos of the first half,
// sin of the second, inv_freq = expf(-logf(10000) * i / half).
std::vector<float> time_embedding(float t, int32_t dim) {
    std::vector<float> out((size_t) dim);
    const int32_t half = dim / 2;
    for (int32_t i = 0; i < half; ++i) {
        const float inv_freq = expf(-logf(10000.0f) * (float) i / (float) half);
        const float angle = t * inv_freq;
        out[(size_t) i] = cosf(angle);
        out[(size_t) (i + half)] = sinf(angle);
    }
    return out;
}

float gelu_erf_host(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

// ---- staging ----------------------------------------------------------------

void upload(vxk_decoder * d, const void * src, size_t bytes, void * dst, cudaStream_t cs) {
    if (bytes > d->stage_bytes) dfail(VXK_STATUS_INVALID_ARGUMENT, "descriptor upload exceeds the staging buffer");
    const int i = d->stage_next;
    d->stage_next ^= 1;
    VXK_DCUDA(cudaEventSynchronize(d->stage_ev[i]));  // the copy that last read this buffer has run
    std::memcpy(d->h_stage[i], src, bytes);
    VXK_DCUDA(cudaMemcpyAsync(dst, d->h_stage[i], bytes, cudaMemcpyHostToDevice, cs));
    VXK_DCUDA(cudaEventRecord(d->stage_ev[i], cs));
}

// ---- create -------------------------------------------------------------------

void create(vxk_decoder * d, const vxk_gguf * g, vxk_pool * pool) {
    d->pool = pool;
    d->ps = vxk::pool_shape(pool);
    const vxk::PoolShape & ps = d->ps;
    if (d->cfg.audio_capacity < 1) dfail(VXK_STATUS_INVALID_ARGUMENT, "audio_capacity must be >= 1");
    if (d->cfg.enc_capacity < 0 || d->cfg.enc_capacity % 4)
        dfail(VXK_STATUS_INVALID_ARGUMENT, "enc_capacity must be a non-negative multiple of 4");
    DevScope scope(ps.device);
    d->chunk = std::min<int32_t>(vxk::kQmmMaxRows, ps.max_rows);

    const TensorRef emb = need(g, "tok_embeddings.weight");
    if (emb.info.n_dims != 2) dfail(VXK_STATUS_INVALID_ARGUMENT, "tok_embeddings.weight must be 2-D");
    d->dim = (int32_t) emb.info.ne[0];
    d->vocab = (int32_t) emb.info.ne[1];
    d->n_layers = (int32_t) key_int(g, "voxtral.decoder.n_layers", ps.n_layers);
    const int64_t heads = key_int(g, "voxtral.decoder.n_heads", ps.n_q);
    const int64_t kv_heads = key_int(g, "voxtral.decoder.n_kv_heads", ps.n_kv);
    const int64_t head_dim = key_int(g, "voxtral.decoder.head_dim", ps.head_dim);
    d->eps = (float) key_float(g, "voxtral.decoder.norm_eps", 1e-5);
    const double theta = key_float(g, "voxtral.decoder.rope_theta", ps.rope_theta);
    if (d->n_layers != ps.n_layers || heads != ps.n_q || kv_heads != ps.n_kv || head_dim != ps.head_dim)
        dfail(VXK_STATUS_INVALID_ARGUMENT, "the pool's layers / heads / head_dim differ from the model's");
    if ((float) theta != ps.rope_theta) dfail(VXK_STATUS_INVALID_ARGUMENT, "the pool's rope_theta differs from the model's");
    if (d->dim % 256 || d->dim > 16384) dfail(VXK_STATUS_INVALID_ARGUMENT, "decoder dim must be a multiple of 256, <= 16384");
    const int32_t qdim = ps.n_q * ps.head_dim, kvdim = ps.n_kv * ps.head_dim;
    {
        const TensorRef w1 = need(g, "dec.blk.0.ffn_w1.weight");
        d->hidden = (int32_t) w1.info.ne[1];
    }

    VXK_DCUDA(cudaMalloc(&d->d_error, sizeof(int32_t)));
    VXK_DCUDA(cudaMemset(d->d_error, 0, sizeof(int32_t)));

    // projections, FFN, norms
    d->layers.resize((size_t) d->n_layers);
    std::vector<float> an((size_t) d->n_layers * d->dim), fn((size_t) d->n_layers * d->dim);
    const bool t_cond = key_int(g, "voxtral.ada_rms_norm_t_cond", 1) != 0;
    TensorRef ada0_0;
    const bool has_ada = t_cond && find(g, "dec.blk.0.ada0.weight", &ada0_0);
    std::vector<float> ada_host;
    std::vector<float> temb;
    if (has_ada) {
        d->ada_dim = (int32_t) ada0_0.info.ne[1];
        ada_host.resize((size_t) d->n_layers * d->dim);
        temb = time_embedding(d->cfg.time_value, d->dim);
    }
    for (int32_t l = 0; l < d->n_layers; ++l) {
        const std::string p = "dec.blk." + std::to_string(l) + ".";
        Layer & L = d->layers[(size_t) l];
        L.q = load_q(d, g, p + "attn_q.weight", qdim, d->dim);
        L.k = load_q(d, g, p + "attn_k.weight", kvdim, d->dim);
        L.v = load_q(d, g, p + "attn_v.weight", kvdim, d->dim);
        L.o = load_q(d, g, p + "attn_o.weight", d->dim, qdim);
        L.w1 = load_q(d, g, p + "ffn_w1.weight", d->hidden, d->dim);
        L.w3 = load_q(d, g, p + "ffn_w3.weight", d->hidden, d->dim);
        L.w2 = load_q(d, g, p + "ffn_w2.weight", d->dim, d->hidden);
        const std::vector<float> a = load_vector(g, p + "attn_norm.weight", d->dim);
        const std::vector<float> f = load_vector(g, p + "ffn_norm.weight", d->dim);
        std::copy(a.begin(), a.end(), an.begin() + (size_t) l * d->dim);
        std::copy(f.begin(), f.end(), fn.begin() + (size_t) l * d->dim);
        if (has_ada) {
            const TensorRef a0 = need(g, p + "ada0.weight");
            const TensorRef a2 = need(g, p + "ada2.weight");
            check_matrix(a0, p + "ada0.weight", d->ada_dim, d->dim);
            check_matrix(a2, p + "ada2.weight", d->dim, d->ada_dim);
            std::vector<float> h = matvec_host(a0, temb);
            for (float & v : h) v = gelu_erf_host(v);
            const std::vector<float> s = matvec_host(a2, h);
            std::copy(s.begin(), s.end(), ada_host.begin() + (size_t) l * d->dim);
        }
    }
    const std::vector<float> dn = load_vector(g, "dec.norm.weight", d->dim);
    d->attn_norm = dalloc<float>(d, an.size());
    d->ffn_norm = dalloc<float>(d, fn.size());
    d->dec_norm = dalloc<float>(d, dn.size());
    VXK_DCUDA(cudaMemcpy(d->attn_norm, an.data(), an.size() * 4, cudaMemcpyHostToDevice));
    VXK_DCUDA(cudaMemcpy(d->ffn_norm, fn.data(), fn.size() * 4, cudaMemcpyHostToDevice));
    VXK_DCUDA(cudaMemcpy(d->dec_norm, dn.data(), dn.size() * 4, cudaMemcpyHostToDevice));
    if (has_ada) {
        d->ada = dalloc<float>(d, ada_host.size());
        VXK_DCUDA(cudaMemcpy(d->ada, ada_host.data(), ada_host.size() * 4, cudaMemcpyHostToDevice));
    }

    // embeddings (gather source) and the head
    d->emb_type = emb.info.type;
    d->emb_row_bytes = vxk::gguf_row_bytes(emb.info.type, d->dim);
    if (d->emb_row_bytes == 0 || (int64_t) emb.info.n_bytes != d->emb_row_bytes * d->vocab)
        dfail(VXK_STATUS_INVALID_ARGUMENT, "tok_embeddings.weight: unsupported type");
    d->emb = dalloc<uint8_t>(d, (size_t) emb.info.n_bytes);
    VXK_DCUDA(cudaMemcpy(d->emb, emb.data, (size_t) emb.info.n_bytes, cudaMemcpyHostToDevice));
    TensorRef out_w;
    const bool untied = find(g, "output.weight", &out_w);
    const TensorRef & hw = untied ? out_w : emb;
    const std::string hname = untied ? "output.weight" : "tok_embeddings.weight";
    check_matrix(hw, hname, d->vocab, d->dim);
    d->head_type = hw.info.type;
    vxk_head_config hc = vxk_head_default_config();
    hc.device = ps.device;
    hc.dim = d->dim;
    hc.vocab = d->vocab;
    if (is_qtype(hw.info.type)) {
        hc.dtype = VXK_DTYPE_F16;
        d->head_q = load_q(d, g, hname, d->vocab, d->dim);
    } else if (hw.info.type == 1 || hw.info.type == 30) {
        hc.dtype = hw.info.type == 1 ? VXK_DTYPE_F16 : VXK_DTYPE_BF16;
        if (untied) {
            d->head_w16_own = dalloc<uint8_t>(d, (size_t) hw.info.n_bytes);
            VXK_DCUDA(cudaMemcpy(d->head_w16_own, hw.data, (size_t) hw.info.n_bytes, cudaMemcpyHostToDevice));
            d->head_w16 = d->head_w16_own;
        } else {
            d->head_w16 = d->emb;
        }
    } else {
        dfail(VXK_STATUS_INVALID_ARGUMENT, hname + ": the head needs F16, BF16, Q8_0, Q4_K or Q6_K");
    }
    VXK_DCALL(vxk_head_create(&hc, &d->head), "vxk_head_create");

    // adapter
    if (d->cfg.enc_capacity > 0) {
        const TensorRef a0 = need(g, "adapter.0.weight");
        if (a0.info.n_dims != 2 || a0.info.ne[0] % 4) dfail(VXK_STATUS_INVALID_ARGUMENT, "adapter.0.weight shape");
        d->enc_dim = (int32_t) (a0.info.ne[0] / 4);
        const int64_t mid = a0.info.ne[1];
        d->ad0 = load_q(d, g, "adapter.0.weight", mid, 4 * (int64_t) d->enc_dim);
        d->ad2 = load_q(d, g, "adapter.2.weight", d->dim, mid);
        d->enc = dalloc<float>(d, (size_t) ps.max_streams * d->cfg.enc_capacity * d->enc_dim);
        VXK_DCUDA(cudaMemset(d->enc, 0, (size_t) ps.max_streams * d->cfg.enc_capacity * d->enc_dim * 4));
        d->ad_in = dalloc<float>(d, (size_t) ps.max_rows * 4 * d->enc_dim);
        d->ad_mid = dalloc<float>(d, (size_t) ps.max_rows * mid);
        d->ad_out = dalloc<float>(d, (size_t) ps.max_rows * d->dim);
        d->d_adapt = dalloc<vxk::AdaptRow>(d, (size_t) ps.max_rows);
    }
    d->audio = dalloc<float>(d, (size_t) ps.max_streams * d->cfg.audio_capacity * d->dim);
    VXK_DCUDA(cudaMemset(d->audio, 0, (size_t) ps.max_streams * d->cfg.audio_capacity * d->dim * 4));

    // scratch
    const size_t R = (size_t) ps.max_rows, C = (size_t) d->chunk;
    d->x = dalloc<float>(d, R * d->dim);
    d->xn = dalloc<float>(d, R * d->dim);
    d->q = dalloc<float>(d, R * qdim);
    d->k = dalloc<float>(d, R * kvdim);
    d->v = dalloc<float>(d, R * kvdim);
    d->att = dalloc<float>(d, R * qdim);
    d->proj = dalloc<float>(d, R * d->dim);
    d->gate = dalloc<float>(d, C * d->hidden);
    d->up = dalloc<float>(d, C * d->hidden);
    d->hn = dalloc<float>(d, (size_t) ps.max_streams * d->dim);
    d->d_rows = dalloc<vxk::DecRow>(d, R);
    d->stage_bytes = R * sizeof(vxk::DecRow);
    for (int i = 0; i < 2; ++i) {
        VXK_DCUDA(cudaHostAlloc(reinterpret_cast<void **>(&d->h_stage[i]), d->stage_bytes, cudaHostAllocDefault));
        VXK_DCUDA(cudaEventCreateWithFlags(&d->stage_ev[i], cudaEventDisableTiming));
    }
    VXK_DCUDA(cudaDeviceSynchronize());
}

// Products of `rows` rows in chunks: one activation quantization per chunk
// for the matrices of `ws` (split by family when they differ).
void products(vxk_decoder * d, vxk_qweight * const * ws, int n, const float * x, int64_t x_stride, int32_t rows,
              float * const * ys, const int64_t * y_strides, cudaStream_t cs) {
    bool same = true;
    const bool fam0 = vxk::qweight_shape(ws[0]).type == VXK_QTYPE_Q8_0;
    for (int i = 1; i < n; ++i) same = same && ((vxk::qweight_shape(ws[i]).type == VXK_QTYPE_Q8_0) == fam0);
    for (int32_t r0 = 0; r0 < rows; r0 += d->chunk) {
        const int32_t nr = std::min(d->chunk, rows - r0);
        float * yc[vxk::kQmmMaxGroup];
        for (int i = 0; i < n; ++i) yc[i] = ys[i] + (int64_t) r0 * y_strides[i];
        const float * xc = x + (int64_t) r0 * x_stride;
        if (same) {
            VXK_DCALL(vxk_qweight_matmul_group(ws, n, xc, nr, yc, cs), "quantized product");
        } else {
            for (int i = 0; i < n; ++i) VXK_DCALL(vxk_qweight_matmul(ws[i], xc, nr, yc[i], cs), "quantized product");
        }
    }
}

// The residual + norm in front of the group product ws: when that product of
// `rows` rows runs on the tcgen05 kernel in one call, the norm quantizes its
// rows straight into the product's activation tiles (np.out is not written)
// and the function returns true: the caller then runs
// qweight_matmul_group_prequantized as the very next launch.  Otherwise the
// plain norm into np.out.
bool norm_into(vxk_decoder * d, vxk::NormParams np, vxk_qweight * const * ws, int n, int32_t rows, cudaStream_t cs) {
    vxk::QtcTiles t{};
    if (!np.compact && rows <= d->chunk && d->dim % 256 == 0 && d->dim <= 8192 &&
        vxk::qweight_group_tiles(ws, n, rows, &t)) {
        np.out = nullptr;
        np.q_tiles = t.b;
        np.q_bmin = t.bmin;
        np.q_tiles8 = t.b8;
        np.q_dx = t.dx;
        np.q_npad = t.npad;
        np.q_rows_padded = t.rows_padded;
        VXK_DCUDA(vxk::launch_add_norm_quant(np, cs));
        return true;
    }
    VXK_DCUDA(vxk::launch_add_norm(np, cs));
    return false;
}

void forward(vxk_decoder * d, const int32_t * tokens, const int32_t * audio_slots, int32_t * argmax, float * logits,
             float * hidden, cudaStream_t cs) {
    if (!vxk::pool_batch_view(d->pool, &d->view)) dfail(VXK_STATUS_INVALID_STATE, "no batch is planned on the pool");
    if (!tokens || !audio_slots || !argmax) dfail(VXK_STATUS_INVALID_ARGUMENT, "null argument");
    const vxk::PoolBatchView & bv = d->view;
    const int32_t rows = (int32_t) bv.row_stream.size();
    const int32_t n_out = (int32_t) bv.last_rows.size();
    d->h_rows.assign((size_t) rows, vxk::DecRow{});
    for (int32_t r = 0; r < rows; ++r) {
        if (tokens[r] < 0 || tokens[r] >= d->vocab) dfail(VXK_STATUS_INVALID_ARGUMENT, "token out of range");
        if (audio_slots[r] < 0 || audio_slots[r] >= d->cfg.audio_capacity)
            dfail(VXK_STATUS_INVALID_ARGUMENT, "audio slot out of range");
        d->h_rows[(size_t) r] = vxk::DecRow{bv.row_stream[(size_t) r], tokens[r], audio_slots[r], -1};
    }
    for (int32_t i = 0; i < n_out; ++i) d->h_rows[(size_t) bv.last_rows[(size_t) i]].out_index = i;
    DevScope scope(d->ps.device);
    upload(d, d->h_rows.data(), (size_t) rows * sizeof(vxk::DecRow), d->d_rows, cs);

    const int32_t dim = d->dim, qdim = d->ps.n_q * d->ps.head_dim, kvdim = d->ps.n_kv * d->ps.head_dim;
    vxk::EmbedParams ep{};
    ep.emb = d->emb;
    ep.emb_row_bytes = d->emb_row_bytes;
    ep.emb_type = d->emb_type;
    ep.audio_cap = d->cfg.audio_capacity;
    ep.audio = d->audio;
    ep.rows = d->d_rows;
    ep.n_rows = rows;
    ep.dim = dim;
    ep.norm_w = d->attn_norm;
    ep.eps = d->eps;
    ep.x = d->x;
    ep.xn = d->xn;
    VXK_DCUDA(vxk::launch_embed_norm(ep, cs));

    bool qkv_tiles = false;  // the previous norm wrote this layer's q/k/v activation tiles
    for (int32_t l = 0; l < d->n_layers; ++l) {
        const Layer & L = d->layers[(size_t) l];
        {
            vxk_qweight * ws[3] = {L.q, L.k, L.v};
            float * ys[3] = {d->q, d->k, d->v};
            const int64_t st[3] = {qdim, kvdim, kvdim};
            if (qkv_tiles)
                VXK_DCALL((vxk_status) vxk::qweight_matmul_group_prequantized(ws, 3, rows, ys, nullptr, cs),
                          "quantized product");
            else
                products(d, ws, 3, d->xn, dim, rows, ys, st, cs);
        }
        // single-token rows on an f16 cache: the attention quantizes its output
        // rows into the o product's tiles in the same launch
        vxk_qweight * wo[1] = {L.o};
        vxk::QtcTiles ot{};
        const bool o_tiles = bv.single_token && rows <= d->chunk && vxk::pool_decode_quant_ok(d->pool) &&
                             vxk::qweight_group_tiles(wo, 1, rows, &ot);
        if (o_tiles) {
            VXK_DCALL((vxk_status) vxk::pool_decode_layer_quant(d->pool, l, d->q, d->k, d->v, nullptr, ot, cs),
                      "vxk_decode_layer");
        } else if (bv.single_token) {
            VXK_DCALL(vxk_decode_layer(d->pool, l, d->q, d->k, d->v, d->att, cs), "vxk_decode_layer");
        } else {
            VXK_DCALL(vxk_append_layer(d->pool, l, d->k, d->v, cs), "vxk_append_layer");
            VXK_DCALL(vxk_attend_layer(d->pool, l, d->q, d->att, cs), "vxk_attend_layer");
        }
        {
            float * ys[1] = {d->proj};
            const int64_t st[1] = {dim};
            if (o_tiles)
                VXK_DCALL((vxk_status) vxk::qweight_matmul_group_prequantized(wo, 1, rows, ys, nullptr, cs),
                          "quantized product");
            else
                products(d, wo, 1, d->att, qdim, rows, ys, st, cs);
        }
        vxk::NormParams np{};
        np.x = d->x;
        np.add = d->proj;
        np.w = d->ffn_norm + (int64_t) l * dim;
        np.ada = d->ada ? d->ada + (int64_t) l * dim : nullptr;
        np.out = d->xn;
        np.rows = d->d_rows;
        np.compact = 0;
        np.n_rows = rows;
        np.dim = dim;
        np.eps = d->eps;
        vxk_qweight * w13[2] = {L.w1, L.w3};
        const bool ffn_tiles = norm_into(d, np, w13, 2, rows, cs);
        for (int32_t r0 = 0; r0 < rows; r0 += d->chunk) {
            const int32_t nr = std::min(d->chunk, rows - r0);
            float * ys[2] = {d->gate, d->up};
            const int64_t st[2] = {d->hidden, d->hidden};
            if (ffn_tiles)  // rows <= chunk: one pass
                VXK_DCALL((vxk_status) vxk::qweight_matmul_group_prequantized(w13, 2, nr, ys, nullptr, cs),
                          "quantized product");
            else
                products(d, w13, 2, d->xn + (int64_t) r0 * dim, dim, nr, ys, st, cs);
            // w2 . (silu(gate) * up): SwiGLU inside w2's activation quantization
            VXK_DCALL((vxk_status) vxk::qweight_matmul_swiglu(L.w2, d->gate, d->up, nr, d->proj + (int64_t) r0 * dim,
                                                              cs),
                      "quantized product");
        }
        const bool last = l + 1 == d->n_layers;
        np.w = last ? d->dec_norm : d->attn_norm + (int64_t) (l + 1) * dim;
        np.ada = nullptr;
        np.out = last ? d->hn : d->xn;
        np.compact = last ? 1 : 0;
        if (last) {
            VXK_DCUDA(vxk::launch_add_norm(np, cs));
        } else {
            const Layer & N = d->layers[(size_t) l + 1];
            vxk_qweight * wn[3] = {N.q, N.k, N.v};
            qkv_tiles = norm_into(d, np, wn, 3, rows, cs);
        }
    }

    for (int32_t r0 = 0; r0 < n_out; r0 += vxk::kHeadRows) {
        const int32_t nr = std::min<int32_t>(vxk::kHeadRows, n_out - r0);
        float * lg = logits ? logits + (int64_t) r0 * d->vocab : nullptr;
        if (d->head_q) {
            VXK_DCALL(vxk_head_logits_argmax_q(d->head, d->head_q, d->hn + (int64_t) r0 * dim, nr, argmax + r0, lg, cs),
                      "vxk_head_logits_argmax_q");
        } else {
            VXK_DCALL(vxk_head_logits_argmax(d->head, d->head_w16, d->hn + (int64_t) r0 * dim, nr, argmax + r0, lg, cs),
                      "vxk_head_logits_argmax");
        }
    }
    if (hidden)
        VXK_DCUDA(cudaMemcpyAsync(hidden, d->hn, (size_t) n_out * dim * sizeof(float), cudaMemcpyDeviceToDevice, cs));
}

// Copies n rows between a device buffer and a ring at absolute position pos
// (slot = pos % cap, at most two segments).
void ring_copy(float * ring, int32_t cap, int32_t width, int64_t pos, int32_t n, float * rows, bool to_ring,
               cudaStream_t cs) {
    int32_t done = 0;
    while (done < n) {
        const int32_t slot = (int32_t) ((pos + done) % cap);
        const int32_t len = std::min(n - done, cap - slot);
        float * r = ring + (int64_t) slot * width;
        float * b = rows + (int64_t) done * width;
        const size_t bytes = (size_t) len * width * sizeof(float);
        VXK_DCUDA(cudaMemcpyAsync(to_ring ? r : b, to_ring ? b : r, bytes, cudaMemcpyDeviceToDevice, cs));
        done += len;
    }
}

void check_stream(const vxk_decoder * d, int32_t stream) {
    if (stream < 0 || stream >= d->ps.max_streams) dfail(VXK_STATUS_INVALID_ARGUMENT, "stream id out of range");
}

}  // namespace

extern "C" {

vxk_decoder_config vxk_decoder_default_config(void) {
    vxk_decoder_config c{};
    c.struct_size = sizeof(vxk_decoder_config);
    c.api_version = VXK_API_VERSION;
    c.audio_capacity = 256;
    c.enc_capacity = 256;
    c.time_value = 6.0f;
    return c;
}

vxk_status vxk_decoder_create(const vxk_gguf * g, vxk_pool * pool, const vxk_decoder_config * config,
                              vxk_decoder ** out) {
    if (out) *out = nullptr;
    auto set_error = [](const std::string & m) {
        std::lock_guard<std::mutex> lock(g_create_mutex);
        g_create_error = m;
    };
    if (!g || !pool || !out) {
        set_error("null argument");
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_decoder_config c = vxk_decoder_default_config();
    if (config) {
        if (config->struct_size < offsetof(vxk_decoder_config, reserved)) {
            set_error("config struct_size too small");
            return VXK_STATUS_INVALID_ARGUMENT;
        }
        std::memcpy(&c, config, std::min<size_t>(config->struct_size, sizeof(c)));
    }
    vxk_decoder * d = new (std::nothrow) vxk_decoder();
    if (!d) return VXK_STATUS_OUT_OF_MEMORY;
    d->cfg = c;
    const vxk_status st = dguarded(d, [&] { create(d, g, pool); });
    if (st != VXK_STATUS_OK) {
        set_error(d->last_error);
        destroy(d);
        return st;
    }
    *out = d;
    return VXK_STATUS_OK;
}

void vxk_decoder_destroy(vxk_decoder * d) { destroy(d); }

vxk_status vxk_decoder_last_error(const vxk_decoder * d, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    std::string m;
    if (d) {
        m = d->last_error;
    } else {
        std::lock_guard<std::mutex> lock(g_create_mutex);
        m = g_create_error;
    }
    const size_t n = std::min(m.size(), capacity - 1);
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_decoder_get_info(const vxk_decoder * d, vxk_decoder_info * out) {
    if (!d || !out) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_decoder_info i{};
    i.n_layers = d->n_layers;
    i.dim = d->dim;
    i.hidden = d->hidden;
    i.n_q_heads = d->ps.n_q;
    i.n_kv_heads = d->ps.n_kv;
    i.head_dim = d->ps.head_dim;
    i.vocab = d->vocab;
    i.ada_dim = d->ada ? d->ada_dim : 0;
    i.emb_type = d->head_type;
    i.max_rows = d->ps.max_rows;
    i.max_streams = d->ps.max_streams;
    i.audio_capacity = d->cfg.audio_capacity;
    i.enc_capacity = d->ad0 ? d->cfg.enc_capacity : 0;
    i.enc_dim = d->enc_dim;
    i.device_bytes = d->device_bytes;
    *out = i;
    return VXK_STATUS_OK;
}

vxk_status vxk_decoder_forward(vxk_decoder * d, const int32_t * tokens, const int32_t * audio_slots, int32_t * argmax,
                               float * logits, float * hidden, void * cuda_stream) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    return dguarded(d, [&] {
        forward(d, tokens, audio_slots, argmax, logits, hidden, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_decoder_write_enc(vxk_decoder * d, int32_t stream, int64_t frame, int32_t n, const float * rows,
                                 void * cuda_stream) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    return dguarded(d, [&] {
        if (!d->enc) dfail(VXK_STATUS_INVALID_STATE, "the decoder was created without the adapter");
        check_stream(d, stream);
        if (!rows || n < 1 || n > d->cfg.enc_capacity || frame < 0) dfail(VXK_STATUS_INVALID_ARGUMENT, "bad rows");
        DevScope scope(d->ps.device);
        ring_copy(d->enc + (int64_t) stream * d->cfg.enc_capacity * d->enc_dim, d->cfg.enc_capacity, d->enc_dim, frame,
                  n, const_cast<float *>(rows), true, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_decoder_write_audio(vxk_decoder * d, int32_t stream, int64_t pos, int32_t n, const float * rows,
                                   void * cuda_stream) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    return dguarded(d, [&] {
        check_stream(d, stream);
        if (!rows || n < 1 || n > d->cfg.audio_capacity || pos < 0) dfail(VXK_STATUS_INVALID_ARGUMENT, "bad rows");
        DevScope scope(d->ps.device);
        ring_copy(d->audio + (int64_t) stream * d->cfg.audio_capacity * d->dim, d->cfg.audio_capacity, d->dim, pos, n,
                  const_cast<float *>(rows), true, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_decoder_read_audio(vxk_decoder * d, int32_t stream, int64_t pos, int32_t n, float * rows,
                                  void * cuda_stream) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    return dguarded(d, [&] {
        check_stream(d, stream);
        if (!rows || n < 1 || n > d->cfg.audio_capacity || pos < 0) dfail(VXK_STATUS_INVALID_ARGUMENT, "bad rows");
        DevScope scope(d->ps.device);
        ring_copy(d->audio + (int64_t) stream * d->cfg.audio_capacity * d->dim, d->cfg.audio_capacity, d->dim, pos, n,
                  rows, false, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_decoder_adapt(vxk_decoder * d, int32_t n, const int32_t * streams, const int64_t * enc_frame,
                             const int64_t * audio_pos, void * cuda_stream) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    return dguarded(d, [&] {
        if (!d->ad0) dfail(VXK_STATUS_INVALID_STATE, "the decoder was created without the adapter");
        if (!streams || !enc_frame || !audio_pos || n < 1 || n > d->ps.max_rows)
            dfail(VXK_STATUS_INVALID_ARGUMENT, "n must be in [1, max_rows] with non-null arrays");
        d->h_adapt.resize((size_t) n);
        for (int32_t i = 0; i < n; ++i) {
            check_stream(d, streams[i]);
            if (enc_frame[i] < 0 || enc_frame[i] % 4 || audio_pos[i] < 0)
                dfail(VXK_STATUS_INVALID_ARGUMENT, "enc_frame must be a non-negative multiple of 4, audio_pos >= 0");
            d->h_adapt[(size_t) i] = vxk::AdaptRow{streams[i], (int32_t) (enc_frame[i] % d->cfg.enc_capacity),
                                                   (int32_t) (audio_pos[i] % d->cfg.audio_capacity), 0};
        }
        const cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        DevScope scope(d->ps.device);
        upload(d, d->h_adapt.data(), (size_t) n * sizeof(vxk::AdaptRow), d->d_adapt, cs);
        VXK_DCUDA(vxk::launch_adapter_gather(d->enc, d->cfg.enc_capacity, d->enc_dim, d->d_adapt, n, d->ad_in, cs));
        const vxk::QweightShape s0 = vxk::qweight_shape(d->ad0);
        {
            vxk_qweight * ws[1] = {d->ad0};
            float * ys[1] = {d->ad_mid};
            const int64_t st[1] = {s0.n_rows};
            products(d, ws, 1, d->ad_in, 4 * (int64_t) d->enc_dim, n, ys, st, cs);
        }
        VXK_DCUDA(vxk::launch_gelu_erf(d->ad_mid, (int64_t) n * s0.n_rows, cs));
        {
            vxk_qweight * ws[1] = {d->ad2};
            float * ys[1] = {d->ad_out};
            const int64_t st[1] = {d->dim};
            products(d, ws, 1, d->ad_mid, s0.n_rows, n, ys, st, cs);
        }
        VXK_DCUDA(vxk::launch_audio_scatter(d->ad_out, d->audio, d->cfg.audio_capacity, d->dim, d->d_adapt, n, cs));
    });
}

vxk_status vxk_decoder_sync(vxk_decoder * d, void * cuda_stream, int32_t timeout_ms) {
    if (!d) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_status st = vxk_sync(d->pool, cuda_stream, timeout_ms);
    if (st != VXK_STATUS_OK) {
        char buf[256] = {0};
        vxk_pool_last_error(d->pool, buf, sizeof(buf));
        d->last_error = std::string("pool: ") + buf;
        return st;
    }
    st = dguarded(d, [&] {
        DevScope scope(d->ps.device);
        int32_t err = 0;
        VXK_DCUDA(cudaMemcpy(&err, d->d_error, sizeof(err), cudaMemcpyDeviceToHost));
        if (err != 0) {
            VXK_DCUDA(cudaMemset(d->d_error, 0, sizeof(int32_t)));
            dfail(VXK_STATUS_TIMEOUT, "a quantized product kernel reported an expired bounded wait");
        }
    });
    if (st != VXK_STATUS_OK) return st;
    st = vxk_head_sync(d->head, cuda_stream, timeout_ms);
    if (st != VXK_STATUS_OK) d->last_error = "head reported a device error";
    return st;
}

}  // extern "C"
