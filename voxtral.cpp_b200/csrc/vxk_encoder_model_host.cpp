// Host runtime of the streaming encoder stack (include/vxk.h, vxk_encoder_*):
// the realtime model's encoder loaded from a GGUF file, run over the encoder
// pool's planned batch of many streams (build_encoder_steady_graph,
// src/voxtral.cpp:2386-2511, for any number of new frames per stream).
//
// One forward:
//   conv stem                         gelu(conv1(gelu(conv0(mel window)))) -> x
//   per layer l (products in calls of <= 512 rows):
//     xn = rms_norm(x) * attn_norm    (the previous layer's add_norm; the stem's for l = 0)
//     q, k, v = W{q,k,v} xn           one quantization for the three; q += bq, v += bv
//     attention                       vxk_enc_layer: RoPE, ring append, windowed MHA
//     x += Wo att + bo; xn = rms_norm(x) * ffn_norm
//     gate, up = W1 xn, W3 xn; x += W2 (silu(gate) * up) + b2
//     xn = rms_norm(x) * (the next attn_norm, or enc.norm into the output rows)
// The realtime encoder's norms are RMS norms without bias (enc_apply_norm with
// layernorm false, src/voxtral.cpp:1855-1861); a file whose enc.norm has a bias
// (the offline LayerNorm encoder) is refused.
#include "vxk.h"
#include "vxk_dequant.h"
#include "vxk_internal.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

namespace {

struct EncErr {
    vxk_status status;
    std::string message;
};

[[noreturn]] void efail2(vxk_status st, const std::string & m) { throw EncErr{st, m}; }

#define VXK_ECUDA(expr)                                                                                     \
    do {                                                                                                    \
        const cudaError_t e_ = (expr);                                                                      \
        if (e_ != cudaSuccess)                                                                              \
            efail2(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY : VXK_STATUS_BACKEND_ERROR,   \
                   std::string(#expr) + ": " + cudaGetErrorString(e_));                                     \
    } while (0)

#define VXK_ECALL(expr, what)                                                                               \
    do {                                                                                                    \
        const vxk_status s_ = (expr);                                                                       \
        if (s_ != VXK_STATUS_OK) efail2(s_, std::string(what) + " failed (" + vxk_status_string(s_) + ")"); \
    } while (0)

std::mutex g_enc_create_mutex;
std::string g_enc_create_error;

struct Scope {
    int prev = 0;
    explicit Scope(int d) {
        cudaGetDevice(&prev);
        cudaSetDevice(d);
    }
    ~Scope() { cudaSetDevice(prev); }
};

struct EncLayerW {
    vxk_qweight * q = nullptr;
    vxk_qweight * k = nullptr;
    vxk_qweight * v = nullptr;
    vxk_qweight * o = nullptr;
    vxk_qweight * w1 = nullptr;
    vxk_qweight * w3 = nullptr;
    vxk_qweight * w2 = nullptr;
    float * bq = nullptr;
    float * bv = nullptr;
    float * bo = nullptr;
    float * b2 = nullptr;
};

struct TRef {
    vxk_gguf_tensor info{};
    const uint8_t * data = nullptr;
};

bool tfind(const vxk_gguf * g, const std::string & name, TRef * out) {
    const int64_t i = vxk_gguf_find_tensor(g, name.c_str());
    if (i < 0 || vxk_gguf_get_tensor(g, i, &out->info) != VXK_STATUS_OK) return false;
    out->data = static_cast<const uint8_t *>(vxk_gguf_tensor_data(g, i));
    return out->data != nullptr;
}

TRef tneed(const vxk_gguf * g, const std::string & name) {
    TRef t;
    if (!tfind(g, name, &t)) efail2(VXK_STATUS_INVALID_ARGUMENT, "tensor " + name + " is missing");
    return t;
}

int64_t kint(const vxk_gguf * g, const char * key, int64_t def) {
    int64_t v = 0;
    return vxk_gguf_get_int(g, key, &v) == VXK_STATUS_OK ? v : def;
}

double kfloat(const vxk_gguf * g, const char * key, double def) {
    double v = 0;
    return vxk_gguf_get_float(g, key, &v) == VXK_STATUS_OK ? v : def;
}

// fp32 values of any F32 / F16 / BF16 tensor of n values.
std::vector<float> values(const TRef & t, int64_t n, const std::string & name) {
    if (t.info.type != 0 && t.info.type != 1 && t.info.type != 30)
        efail2(VXK_STATUS_INVALID_ARGUMENT, name + " must be F32, F16 or BF16");
    int64_t have = 1;
    for (int d = 0; d < t.info.n_dims; ++d) have *= t.info.ne[d];
    if (have != n) efail2(VXK_STATUS_INVALID_ARGUMENT, name + " has the wrong number of values");
    std::vector<float> out((size_t) n);
    for (int64_t i = 0; i < n; ++i) out[(size_t) i] = vxk::dequant_elem(t.data, t.info.type, i);
    return out;
}

}  // namespace

struct vxk_encoder {
    vxk_enc_pool * pool = nullptr;
    vxk::EncShape es{};
    int32_t dim = 0, hidden = 0, n_layers = 0, n_mel = 128, max_rows = 0, chunk = 64, max_win = 0;
    float eps = 1e-5f;
    std::vector<EncLayerW> layers;
    std::vector<vxk_qweight *> all_q;
    std::vector<void *> allocs;
    __half * w0 = nullptr;
    __half * w1 = nullptr;
    float * b0 = nullptr;
    float * b1 = nullptr;
    float * attn_norm = nullptr;
    float * ffn_norm = nullptr;
    float * enc_norm = nullptr;
    float * x = nullptr;
    float * xn = nullptr;
    float * q = nullptr;
    float * k = nullptr;
    float * v = nullptr;
    float * att = nullptr;
    float * proj = nullptr;
    float * gate = nullptr;
    float * up = nullptr;
    float * y0 = nullptr;
    vxk::ConvStream * d_conv = nullptr;
    int32_t * d_error = nullptr;
    uint8_t * h_stage[2] = {nullptr, nullptr};
    cudaEvent_t stage_ev[2] = {nullptr, nullptr};
    int stage_next = 0;
    size_t stage_bytes = 0;
    int64_t device_bytes = 0;
    vxk::EncBatchView view;
    std::vector<vxk::ConvStream> h_conv;
    std::string last_error;
};

namespace {

template <typename F>
vxk_status eg(vxk_encoder * e, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const EncErr & x) {
        if (e) e->last_error = x.message;
        return x.status;
    } catch (const std::bad_alloc &) {
        if (e) e->last_error = "host allocation failed";
        return VXK_STATUS_OUT_OF_MEMORY;
    } catch (...) {
        if (e) e->last_error = "unexpected exception";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

template <typename T>
T * ealloc(vxk_encoder * e, size_t count) {
    void * p = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    VXK_ECUDA(cudaMalloc(&p, bytes));
    e->allocs.push_back(p);
    e->device_bytes += (int64_t) bytes;
    return static_cast<T *>(p);
}

template <typename T>
T * eupload(vxk_encoder * e, const std::vector<T> & host) {
    T * d = ealloc<T>(e, host.size());
    VXK_ECUDA(cudaMemcpy(d, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice));
    return d;
}

void edestroy(vxk_encoder * e) {
    if (!e) return;
    Scope scope(e->es.device);
    for (vxk_qweight * w : e->all_q) {
        vxk::qweight_attach_error(w, nullptr);
        vxk_qweight_destroy(w);
    }
    for (void * p : e->allocs) cudaFree(p);
    if (e->d_error) cudaFree(e->d_error);
    for (int i = 0; i < 2; ++i) {
        if (e->h_stage[i]) cudaFreeHost(e->h_stage[i]);
        if (e->stage_ev[i]) cudaEventDestroy(e->stage_ev[i]);
    }
    delete e;
}

vxk_qweight * eload_q(vxk_encoder * e, const vxk_gguf * g, const std::string & name, int64_t rows, int64_t cols) {
    const TRef t = tneed(g, name);
    if (t.info.n_dims != 2 || t.info.ne[0] != cols || t.info.ne[1] != rows)
        efail2(VXK_STATUS_INVALID_ARGUMENT, name + " must be " + std::to_string(rows) + " x " + std::to_string(cols));
    if (t.info.type != VXK_QTYPE_Q8_0 && t.info.type != VXK_QTYPE_Q4_K && t.info.type != VXK_QTYPE_Q6_K)
        efail2(VXK_STATUS_INVALID_ARGUMENT, name + ": matrices must be Q8_0, Q4_K or Q6_K");
    vxk_qweight * w = nullptr;
    const vxk_status st = vxk_qweight_create_from_gguf(g, name.c_str(), e->es.device, e->chunk, &w);
    if (st != VXK_STATUS_OK) {
        char buf[512] = {0};
        vxk_qweight_last_error(nullptr, buf, sizeof(buf));
        efail2(st, name + ": " + buf);
    }
    e->all_q.push_back(w);
    vxk::qweight_attach_error(w, e->d_error);
    size_t packed = 0;
    if (vxk_qweight_packed_bytes((vxk_qtype) t.info.type, (int32_t) rows, (int32_t) cols, &packed) == VXK_STATUS_OK)
        e->device_bytes += (int64_t) packed;
    return w;
}

// Conv weights [out][in][k] (ggml ne = [k, in, out]) as f16 [in][k][out].
__half * load_conv(vxk_encoder * e, const TRef & t, int32_t in_ch, int32_t out_ch, const std::string & name) {
    if (t.info.n_dims != 3 || t.info.ne[0] != 3 || t.info.ne[1] != in_ch || t.info.ne[2] != out_ch)
        efail2(VXK_STATUS_INVALID_ARGUMENT, name + " must be [3][" + std::to_string(in_ch) + "][" +
                                               std::to_string(out_ch) + "] (ne)");
    const std::vector<float> w = values(t, (int64_t) 3 * in_ch * out_ch, name);
    std::vector<__half> tw((size_t) 3 * in_ch * out_ch);
    for (int32_t o = 0; o < out_ch; ++o)
        for (int32_t i = 0; i < in_ch; ++i)
            for (int32_t k = 0; k < 3; ++k)
                tw[((size_t) i * 3 + k) * out_ch + o] = __float2half_rn(w[((size_t) o * in_ch + i) * 3 + k]);
    return eupload(e, tw);
}

void ecreate(vxk_encoder * e, const vxk_gguf * g, vxk_enc_pool * pool, int32_t max_rows) {
    e->pool = pool;
    e->es = vxk::enc_pool_shape(pool);
    const vxk::EncShape & es = e->es;
    Scope scope(es.device);
    e->max_rows = max_rows > 0 ? max_rows : es.max_streams * 4;
    if (e->max_rows > es.max_streams * es.max_new) e->max_rows = es.max_streams * es.max_new;
    e->chunk = std::min<int32_t>(vxk::kQmmMaxRows, e->max_rows);
    e->max_win = 2 * es.max_new + 4;

    const TRef c0 = tneed(g, "enc.conv0.weight");
    e->dim = (int32_t) kint(g, "voxtral.encoder.dim", c0.info.n_dims == 3 ? c0.info.ne[2] : 0);
    e->n_mel = c0.info.n_dims == 3 ? (int32_t) c0.info.ne[1] : 0;
    e->n_layers = (int32_t) kint(g, "voxtral.encoder.n_layers", es.n_layers);
    const int64_t heads = kint(g, "voxtral.encoder.n_heads", es.n_heads);
    const int64_t kv_heads = kint(g, "voxtral.encoder.n_kv_heads", heads);
    const int64_t head_dim = kint(g, "voxtral.encoder.head_dim", es.head_dim);
    e->eps = (float) kfloat(g, "voxtral.encoder.norm_eps", 1e-5);
    const double theta = kfloat(g, "voxtral.encoder.rope_theta", es.rope_theta);
    if (e->n_layers != es.n_layers || heads != es.n_heads || kv_heads != heads || head_dim != es.head_dim)
        efail2(VXK_STATUS_INVALID_ARGUMENT, "the encoder pool's layers / heads / head_dim differ from the model's");
    if ((float) theta != es.rope_theta) efail2(VXK_STATUS_INVALID_ARGUMENT, "rope_theta differs from the pool's");
    if (e->dim % 256 || e->dim > 16384) efail2(VXK_STATUS_INVALID_ARGUMENT, "encoder dim must be a multiple of 256");
    TRef nb;
    if (tfind(g, "enc.norm.bias", &nb))
        efail2(VXK_STATUS_INVALID_ARGUMENT, "a LayerNorm (offline) encoder is not supported");
    const int32_t qdim = es.n_heads * es.head_dim;
    e->hidden = (int32_t) tneed(g, "enc.blk.0.ffn_w1.weight").info.ne[1];

    VXK_ECUDA(cudaMalloc(&e->d_error, sizeof(int32_t)));
    VXK_ECUDA(cudaMemset(e->d_error, 0, sizeof(int32_t)));

    e->w0 = load_conv(e, c0, e->n_mel, e->dim, "enc.conv0.weight");
    e->w1 = load_conv(e, tneed(g, "enc.conv1.weight"), e->dim, e->dim, "enc.conv1.weight");
    e->b0 = eupload(e, values(tneed(g, "enc.conv0.bias"), e->dim, "enc.conv0.bias"));
    e->b1 = eupload(e, values(tneed(g, "enc.conv1.bias"), e->dim, "enc.conv1.bias"));

    std::vector<float> an((size_t) e->n_layers * e->dim), fn((size_t) e->n_layers * e->dim);
    e->layers.resize((size_t) e->n_layers);
    for (int32_t l = 0; l < e->n_layers; ++l) {
        const std::string p = "enc.blk." + std::to_string(l) + ".";
        EncLayerW & L = e->layers[(size_t) l];
        L.q = eload_q(e, g, p + "attn_q.weight", qdim, e->dim);
        L.k = eload_q(e, g, p + "attn_k.weight", qdim, e->dim);
        L.v = eload_q(e, g, p + "attn_v.weight", qdim, e->dim);
        L.o = eload_q(e, g, p + "attn_o.weight", e->dim, qdim);
        L.w1 = eload_q(e, g, p + "ffn_w1.weight", e->hidden, e->dim);
        L.w3 = eload_q(e, g, p + "ffn_w3.weight", e->hidden, e->dim);
        L.w2 = eload_q(e, g, p + "ffn_w2.weight", e->dim, e->hidden);
        TRef t;
        if (tfind(g, p + "attn_q.bias", &t)) L.bq = eupload(e, values(t, qdim, p + "attn_q.bias"));
        if (tfind(g, p + "attn_v.bias", &t)) L.bv = eupload(e, values(t, qdim, p + "attn_v.bias"));
        if (tfind(g, p + "attn_o.bias", &t)) L.bo = eupload(e, values(t, e->dim, p + "attn_o.bias"));
        if (tfind(g, p + "ffn_w2.bias", &t)) L.b2 = eupload(e, values(t, e->dim, p + "ffn_w2.bias"));
        if (tfind(g, p + "attn_norm.bias", &t) || tfind(g, p + "ffn_norm.bias", &t))
            efail2(VXK_STATUS_INVALID_ARGUMENT, "a LayerNorm (offline) encoder is not supported");
        const std::vector<float> a = values(tneed(g, p + "attn_norm.weight"), e->dim, p + "attn_norm.weight");
        const std::vector<float> f = values(tneed(g, p + "ffn_norm.weight"), e->dim, p + "ffn_norm.weight");
        std::copy(a.begin(), a.end(), an.begin() + (size_t) l * e->dim);
        std::copy(f.begin(), f.end(), fn.begin() + (size_t) l * e->dim);
    }
    e->attn_norm = eupload(e, an);
    e->ffn_norm = eupload(e, fn);
    e->enc_norm = eupload(e, values(tneed(g, "enc.norm.weight"), e->dim, "enc.norm.weight"));

    const size_t R = (size_t) e->max_rows, C = (size_t) e->chunk;
    e->x = ealloc<float>(e, R * e->dim);
    e->xn = ealloc<float>(e, R * e->dim);
    e->q = ealloc<float>(e, R * qdim);
    e->k = ealloc<float>(e, R * qdim);
    e->v = ealloc<float>(e, R * qdim);
    e->att = ealloc<float>(e, R * qdim);
    e->proj = ealloc<float>(e, R * e->dim);
    e->gate = ealloc<float>(e, C * e->hidden);
    e->up = ealloc<float>(e, C * e->hidden);
    e->y0 = ealloc<float>(e, (size_t) es.max_streams * e->max_win * e->dim);
    e->d_conv = ealloc<vxk::ConvStream>(e, (size_t) es.max_streams);
    e->stage_bytes = (size_t) es.max_streams * sizeof(vxk::ConvStream);
    for (int i = 0; i < 2; ++i) {
        VXK_ECUDA(cudaHostAlloc(reinterpret_cast<void **>(&e->h_stage[i]), e->stage_bytes, cudaHostAllocDefault));
        VXK_ECUDA(cudaEventCreateWithFlags(&e->stage_ev[i], cudaEventDisableTiming));
    }
    VXK_ECUDA(cudaDeviceSynchronize());
}

void eproducts(vxk_encoder * e, vxk_qweight * const * ws, int n, const float * x, int64_t x_stride, int32_t rows,
               float * const * ys, const int64_t * y_strides, cudaStream_t cs,
               const float * const * biases = nullptr) {
    bool same = true;
    const bool fam0 = vxk::qweight_shape(ws[0]).type == VXK_QTYPE_Q8_0;
    for (int i = 1; i < n; ++i) same = same && ((vxk::qweight_shape(ws[i]).type == VXK_QTYPE_Q8_0) == fam0);
    for (int32_t r0 = 0; r0 < rows; r0 += e->chunk) {
        const int32_t nr = std::min(e->chunk, rows - r0);
        float * yc[vxk::kQmmMaxGroup];
        for (int i = 0; i < n; ++i) yc[i] = ys[i] + (int64_t) r0 * y_strides[i];
        const float * xc = x + (int64_t) r0 * x_stride;
        if (same) {
            VXK_ECALL((vxk_status) vxk::qweight_matmul_group_bias(ws, n, xc, nr, yc, biases, cs), "quantized product");
        } else {
            for (int i = 0; i < n; ++i)
                VXK_ECALL((vxk_status) vxk::qweight_matmul_group_bias(&ws[i], 1, xc, nr, &yc[i],
                                                                      biases ? &biases[i] : nullptr, cs),
                          "quantized product");
        }
    }
}

// The conv stem of the planned batch into x (rows of dim); returns the rows.
int32_t estem(vxk_encoder * e, const float * mel, float * x, cudaStream_t cs) {
    if (!vxk::enc_pool_batch_view(e->pool, &e->view)) efail2(VXK_STATUS_INVALID_STATE, "no batch is planned");
    if (!mel || !x) efail2(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
    const vxk::EncBatchView & bv = e->view;
    const int32_t rows = bv.rows;
    if (rows > e->max_rows)
        efail2(VXK_STATUS_INVALID_ARGUMENT, "batch rows exceed the encoder's max_rows (" +
                                                std::to_string(e->max_rows) + ")");
    const int32_t ns = (int32_t) bv.streams.size();
    e->h_conv.resize((size_t) ns);
    int32_t mel_off = 0, row0 = 0;
    for (int32_t i = 0; i < ns; ++i) {
        const int32_t win = 2 * bv.n_new[(size_t) i] + 4;
        e->h_conv[(size_t) i] = vxk::ConvStream{mel_off, win, bv.n_new[(size_t) i], row0};
        mel_off += e->n_mel * win;
        row0 += bv.n_new[(size_t) i];
    }
    Scope scope(e->es.device);
    {
        const size_t bytes = (size_t) ns * sizeof(vxk::ConvStream);
        const int i = e->stage_next;
        e->stage_next ^= 1;
        VXK_ECUDA(cudaEventSynchronize(e->stage_ev[i]));
        std::memcpy(e->h_stage[i], e->h_conv.data(), bytes);
        VXK_ECUDA(cudaMemcpyAsync(e->d_conv, e->h_stage[i], bytes, cudaMemcpyHostToDevice, cs));
        VXK_ECUDA(cudaEventRecord(e->stage_ev[i], cs));
    }
    vxk::ConvParams cp{};
    cp.mel = mel;
    cp.streams = e->d_conv;
    cp.n_streams = ns;
    cp.n_mel = e->n_mel;
    cp.dim = e->dim;
    cp.max_win = e->max_win;
    cp.w0 = e->w0;
    cp.b0 = e->b0;
    cp.w1 = e->w1;
    cp.b1 = e->b1;
    cp.y0 = e->y0;
    cp.x = x;
    cp.steady = 1;
    for (int32_t i = 0; i < ns; ++i) cp.steady = cp.steady && bv.n_new[(size_t) i] == 4;
    VXK_ECUDA(vxk::launch_conv_stem(cp, cs));
    return rows;
}

// The (residual +) norm in front of the group product ws: when that product of
// `rows` rows runs on the tcgen05 kernel in one call, the norm quantizes its
// rows straight into the product's activation tiles (np.out is not written)
// and the function returns true: the caller then runs
// qweight_matmul_group_prequantized as the very next launch.  Otherwise the
// plain norm into np.out.
bool enorm_into(vxk_encoder * e, vxk::NormParams np, vxk_qweight * const * ws, int n, int32_t rows, cudaStream_t cs) {
    vxk::QtcTiles t{};
    if (rows <= e->chunk && e->dim % 256 == 0 && e->dim <= 8192 && vxk::qweight_group_tiles(ws, n, rows, &t)) {
        np.out = nullptr;
        np.q_tiles = t.b;
        np.q_bmin = t.bmin;
        np.q_tiles8 = t.b8;
        np.q_dx = t.dx;
        np.q_npad = t.npad;
        np.q_rows_padded = t.rows_padded;
        VXK_ECUDA(vxk::launch_add_norm_quant(np, cs));
        return true;
    }
    VXK_ECUDA(vxk::launch_add_norm(np, cs));
    return false;
}

void eforward(vxk_encoder * e, const float * mel, float * out, cudaStream_t cs) {
    if (!out) efail2(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
    const int32_t rows = estem(e, mel, e->x, cs);
    const int32_t dim = e->dim, qdim = e->es.n_heads * e->es.head_dim;
    vxk::NormParams np{};
    np.x = e->x;
    np.rows = nullptr;
    np.n_rows = rows;
    np.dim = dim;
    np.eps = e->eps;
    np.w = e->attn_norm;
    np.out = e->xn;
    bool qkv_tiles = false;  // the previous norm wrote this layer's q/k/v activation tiles
    if (e->n_layers > 0) {
        vxk_qweight * w0[3] = {e->layers[0].q, e->layers[0].k, e->layers[0].v};
        qkv_tiles = enorm_into(e, np, w0, 3, rows, cs);
    } else {
        VXK_ECUDA(vxk::launch_add_norm(np, cs));
    }
    for (int32_t l = 0; l < e->n_layers; ++l) {
        const EncLayerW & L = e->layers[(size_t) l];
        {
            vxk_qweight * ws[3] = {L.q, L.k, L.v};
            float * ys[3] = {e->q, e->k, e->v};
            const int64_t st[3] = {qdim, qdim, qdim};
            const float * bs[3] = {L.bq, nullptr, L.bv};  // the q and v biases, added in the products' stores
            if (qkv_tiles)
                VXK_ECALL((vxk_status) vxk::qweight_matmul_group_prequantized(ws, 3, rows, ys, bs, cs),
                          "quantized product");
            else
                eproducts(e, ws, 3, e->xn, dim, rows, ys, st, cs, bs);
        }
        VXK_ECALL(vxk_enc_layer(e->pool, l, e->q, e->k, e->v, e->att, cs), "vxk_enc_layer");
        {
            vxk_qweight * ws[1] = {L.o};
            float * ys[1] = {e->proj};
            const int64_t st[1] = {dim};
            eproducts(e, ws, 1, e->att, qdim, rows, ys, st, cs);
        }
        np.add = e->proj;
        np.add_bias = L.bo;
        np.w = e->ffn_norm + (int64_t) l * dim;
        np.out = e->xn;
        vxk_qweight * w13[2] = {L.w1, L.w3};
        const bool ffn_tiles = enorm_into(e, np, w13, 2, rows, cs);
        for (int32_t r0 = 0; r0 < rows; r0 += e->chunk) {
            const int32_t nr = std::min(e->chunk, rows - r0);
            float * ys[2] = {e->gate, e->up};
            const int64_t st[2] = {e->hidden, e->hidden};
            if (ffn_tiles)  // rows <= chunk: one pass
                VXK_ECALL((vxk_status) vxk::qweight_matmul_group_prequantized(w13, 2, nr, ys, nullptr, cs),
                          "quantized product");
            else
                eproducts(e, w13, 2, e->xn + (int64_t) r0 * dim, dim, nr, ys, st, cs);
            VXK_ECALL((vxk_status) vxk::qweight_matmul_swiglu(L.w2, e->gate, e->up, nr, e->proj + (int64_t) r0 * dim,
                                                              cs),
                      "quantized product");
        }
        const bool last = l + 1 == e->n_layers;
        np.add = e->proj;
        np.add_bias = L.b2;
        np.w = last ? e->enc_norm : e->attn_norm + (int64_t) (l + 1) * dim;
        np.out = last ? out : e->xn;
        if (last) {
            VXK_ECUDA(vxk::launch_add_norm(np, cs));
        } else {
            const EncLayerW & N = e->layers[(size_t) l + 1];
            vxk_qweight * wn[3] = {N.q, N.k, N.v};
            qkv_tiles = enorm_into(e, np, wn, 3, rows, cs);
        }
    }
}

}  // namespace

extern "C" {

vxk_status vxk_encoder_create(const vxk_gguf * g, vxk_enc_pool * pool, int32_t max_rows, vxk_encoder ** out) {
    if (out) *out = nullptr;
    auto set_error = [](const std::string & m) {
        std::lock_guard<std::mutex> lock(g_enc_create_mutex);
        g_enc_create_error = m;
    };
    if (!g || !pool || !out || max_rows < 0) {
        set_error("null argument or negative max_rows");
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_encoder * e = new (std::nothrow) vxk_encoder();
    if (!e) return VXK_STATUS_OUT_OF_MEMORY;
    const vxk_status st = eg(e, [&] { ecreate(e, g, pool, max_rows); });
    if (st != VXK_STATUS_OK) {
        set_error(e->last_error);
        edestroy(e);
        return st;
    }
    *out = e;
    return VXK_STATUS_OK;
}

void vxk_encoder_destroy(vxk_encoder * e) { edestroy(e); }

vxk_status vxk_encoder_last_error(const vxk_encoder * e, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    std::string m;
    if (e) {
        m = e->last_error;
    } else {
        std::lock_guard<std::mutex> lock(g_enc_create_mutex);
        m = g_enc_create_error;
    }
    const size_t n = std::min(m.size(), capacity - 1);
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_encoder_get_info(const vxk_encoder * e, vxk_encoder_info * out) {
    if (!e || !out) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_encoder_info i{};
    i.n_layers = e->n_layers;
    i.dim = e->dim;
    i.hidden = e->hidden;
    i.n_heads = e->es.n_heads;
    i.head_dim = e->es.head_dim;
    i.n_mel = e->n_mel;
    i.max_rows = e->max_rows;
    i.device_bytes = e->device_bytes;
    *out = i;
    return VXK_STATUS_OK;
}

vxk_status vxk_encoder_forward(vxk_encoder * e, const float * mel, float * out, void * cuda_stream) {
    if (!e) return VXK_STATUS_INVALID_ARGUMENT;
    return eg(e, [&] { eforward(e, mel, out, static_cast<cudaStream_t>(cuda_stream)); });
}

vxk_status vxk_encoder_stem(vxk_encoder * e, const float * mel, float * out, void * cuda_stream) {
    if (!e) return VXK_STATUS_INVALID_ARGUMENT;
    return eg(e, [&] { estem(e, mel, out, static_cast<cudaStream_t>(cuda_stream)); });
}

vxk_status vxk_encoder_sync(vxk_encoder * e, void * cuda_stream, int32_t timeout_ms) {
    if (!e) return VXK_STATUS_INVALID_ARGUMENT;
    return eg(e, [&] {
        Scope scope(e->es.device);
        cudaEvent_t ev = nullptr;
        VXK_ECUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        cudaError_t q = cudaEventRecord(ev, static_cast<cudaStream_t>(cuda_stream));
        const auto t0 = std::chrono::steady_clock::now();
        while (q == cudaSuccess) {
            q = cudaEventQuery(ev);
            if (q == cudaSuccess) break;
            if (q != cudaErrorNotReady) break;
            q = cudaSuccess;
            const auto waited = std::chrono::steady_clock::now() - t0;
            if (waited > std::chrono::milliseconds(timeout_ms)) {
                cudaEventDestroy(ev);
                efail2(VXK_STATUS_TIMEOUT, "stream did not drain within the timeout");
            }
            // poll short waits (a step of a few ms); sleep between polls after 20 ms
            if (waited < std::chrono::milliseconds(20))
                std::this_thread::yield();
            else
                std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        cudaEventDestroy(ev);
        if (q != cudaSuccess) efail2(VXK_STATUS_BACKEND_ERROR, cudaGetErrorString(q));
        int32_t err[2] = {0, 0};
        VXK_ECUDA(cudaMemcpy(&err[0], vxk::enc_pool_error_word(e->pool), sizeof(int32_t), cudaMemcpyDeviceToHost));
        VXK_ECUDA(cudaMemcpy(&err[1], e->d_error, sizeof(int32_t), cudaMemcpyDeviceToHost));
        if (err[0] || err[1]) {
            VXK_ECUDA(cudaMemset(vxk::enc_pool_error_word(e->pool), 0, sizeof(int32_t)));
            VXK_ECUDA(cudaMemset(e->d_error, 0, sizeof(int32_t)));
            efail2(VXK_STATUS_TIMEOUT, "an encoder kernel reported an expired bounded wait");
        }
    });
}

}  // extern "C"
