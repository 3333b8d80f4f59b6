// Host runtime of the greedy head (include/vxk.h, vxk_head_*): tied logits
// and argmax of the decoder step (emit_logits_argmax, src/voxtral.cpp:2966-2972).
//
// The vocabulary is cut into tiles of tile_rows rows (a multiple of 32, at
// most 256: the N extent of one tcgen05.mma) so that the tiles split evenly
// into whole waves of the persistent one-CTA-per-SM grid: for 131072 rows on
// 148 SMs, 4 waves of 224-row tiles (586 tiles, at most 4 per CTA).
#include "vxk.h"
#include "vxk_internal.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

namespace {

thread_local std::string g_head_create_error;

struct HeadError {
    vxk_status status;
    std::string message;
};

[[noreturn]] void hfail(vxk_status s, const std::string & m) { throw HeadError{s, m}; }

#define VXK_HCUDA(expr)                                                                 \
    do {                                                                                \
        const cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                        \
            hfail(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY            \
                                                  : VXK_STATUS_BACKEND_ERROR,           \
                  std::string(#expr) + ": " + cudaGetErrorString(e_));                  \
        }                                                                               \
    } while (0)

class HeadDevice {
public:
    explicit HeadDevice(int d) {
        cudaGetDevice(&prev_);
        dev_ = d;
        if (prev_ != d) cudaSetDevice(d);
    }
    ~HeadDevice() {
        if (prev_ != dev_) cudaSetDevice(prev_);
    }

private:
    int prev_ = 0, dev_ = 0;
};

// 2-D tensor map {cols, rows} over a row-major 16-bit matrix, boxes of
// box_rows x 64 elements, 128-byte swizzle, zero fill past the edges.
// cuTensorMapEncodeTiled is a driver entry point, reached through the runtime
// so the library does not link libcuda.
void encode_rows_map(CUtensorMap * map, const void * base, int32_t dtype, int64_t cols, int64_t rows,
                     int32_t box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        void * fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            hfail(VXK_STATUS_BACKEND_ERROR, "cuTensorMapEncodeTiled is not available");
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const cuuint64_t dims[2] = {(cuuint64_t) cols, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t) box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode(map, dtype == VXK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              2, const_cast<void *>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) hfail(VXK_STATUS_BACKEND_ERROR, "cuTensorMapEncodeTiled failed for the greedy head");
}

}  // namespace

struct vxk_head {
    vxk_head_config cfg{};
    uint16_t * xh = nullptr;
    unsigned long long * best = nullptr;
    float * qlogits = nullptr;  // logits of the quantized path when the caller passes none
    int32_t * d_error = nullptr;
    cudaEvent_t ev_sync = nullptr;
    CUtensorMap map_x{};
    int32_t tile_rows = 0;
    int32_t n_tiles = 0;
    int32_t grid = 0;
    std::string last_error;
};

namespace {

template <typename F>
vxk_status hguarded(vxk_head * h, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const HeadError & e) {
        if (h) h->last_error = e.message;
        return e.status;
    } catch (const std::bad_alloc &) {
        if (h) h->last_error = "host out of memory";
        return VXK_STATUS_OUT_OF_MEMORY;
    } catch (...) {
        if (h) h->last_error = "internal error";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

void free_head(vxk_head * h) {
    if (!h) return;
    HeadDevice scope(h->cfg.device);
    if (h->xh) cudaFree(h->xh);
    if (h->best) cudaFree(h->best);
    if (h->qlogits) cudaFree(h->qlogits);
    if (h->d_error) cudaFree(h->d_error);
    if (h->ev_sync) cudaEventDestroy(h->ev_sync);
    delete h;
}

}  // namespace

extern "C" {

vxk_head_config vxk_head_default_config(void) {
    vxk_head_config c{};
    c.struct_size = sizeof(vxk_head_config);
    c.api_version = VXK_API_VERSION;
    c.device = 0;
    c.dim = 3072;
    c.vocab = 131072;
    c.dtype = VXK_DTYPE_F16;
    return c;
}

vxk_status vxk_head_create(const vxk_head_config * config, vxk_head ** out) {
    if (out) *out = nullptr;
    if (!config || !out) {
        g_head_create_error = "null argument";
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_head * h = new (std::nothrow) vxk_head();
    if (!h) return VXK_STATUS_OUT_OF_MEMORY;
    const vxk_status st = hguarded(h, [&] {
        const vxk_head_config & c = *config;
        if (c.struct_size < sizeof(vxk_head_config)) hfail(VXK_STATUS_INVALID_ARGUMENT, "config struct_size too small");
        if (c.dim < 64 || c.dim % 64 != 0) hfail(VXK_STATUS_INVALID_ARGUMENT, "dim must be a positive multiple of 64");
        if (c.vocab < 1) hfail(VXK_STATUS_INVALID_ARGUMENT, "vocab must be positive");
        if (c.dtype != VXK_DTYPE_F16 && c.dtype != VXK_DTYPE_BF16)
            hfail(VXK_STATUS_INVALID_ARGUMENT, "head weights must be F16 or BF16");
        h->cfg = c;
        int n_dev = 0;
        VXK_HCUDA(cudaGetDeviceCount(&n_dev));
        if (c.device < 0 || c.device >= n_dev) hfail(VXK_STATUS_INVALID_ARGUMENT, "no such CUDA device");
        HeadDevice scope(c.device);
        int sms = 0;
        VXK_HCUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c.device));
        if (sms < 1) hfail(VXK_STATUS_BACKEND_ERROR, "no multiprocessors");
        const int64_t waves = std::max<int64_t>(1, ((int64_t) c.vocab + (int64_t) sms * vxk::kHeadMaxTileRows - 1) /
                                                       ((int64_t) sms * vxk::kHeadMaxTileRows));
        int64_t rows = ((int64_t) c.vocab + sms * waves - 1) / (sms * waves);
        rows = (rows + 31) / 32 * 32;
        h->tile_rows = (int32_t) std::min<int64_t>(vxk::kHeadMaxTileRows, std::max<int64_t>(32, rows));
        h->n_tiles = (int32_t) (((int64_t) c.vocab + h->tile_rows - 1) / h->tile_rows);
        h->grid = std::min(sms, h->n_tiles);
        VXK_HCUDA(cudaMalloc(&h->xh, (size_t) vxk::kHeadRows * c.dim * sizeof(uint16_t)));
        VXK_HCUDA(cudaMalloc(&h->best, (size_t) vxk::kHeadRows * sizeof(unsigned long long)));
        VXK_HCUDA(cudaMalloc(&h->d_error, sizeof(int32_t)));
        VXK_HCUDA(cudaMemset(h->d_error, 0, sizeof(int32_t)));
        VXK_HCUDA(cudaEventCreateWithFlags(&h->ev_sync, cudaEventDisableTiming));
        encode_rows_map(&h->map_x, h->xh, (int32_t) c.dtype, c.dim, vxk::kHeadRows, 64);
    });
    if (st != VXK_STATUS_OK) {
        g_head_create_error = h->last_error;
        free_head(h);
        return st;
    }
    *out = h;
    return VXK_STATUS_OK;
}

void vxk_head_destroy(vxk_head * head) { free_head(head); }

vxk_status vxk_head_last_error(const vxk_head * head, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    const std::string & m = head ? head->last_error : g_head_create_error;
    const size_t n = std::min(capacity - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_head_logits_argmax(vxk_head * head, const void * w, const float * x, int32_t rows,
                                  int32_t * argmax, float * logits, void * cuda_stream) {
    if (!head) return VXK_STATUS_INVALID_ARGUMENT;
    return hguarded(head, [&] {
        const vxk_head_config & c = head->cfg;
        if (!w || !x || !argmax) hfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        if (rows < 1) hfail(VXK_STATUS_INVALID_ARGUMENT, "rows must be positive");
        if (reinterpret_cast<uintptr_t>(w) % 16 != 0) hfail(VXK_STATUS_INVALID_ARGUMENT, "w must be 16-byte aligned");
        HeadDevice scope(c.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        CUtensorMap map_w{};
        encode_rows_map(&map_w, w, (int32_t) c.dtype, c.dim, c.vocab, head->tile_rows);
        for (int32_t r0 = 0; r0 < rows; r0 += vxk::kHeadRows) {
            vxk::HeadParams p{};
            p.x = x + (int64_t) r0 * c.dim;
            p.xh = head->xh;
            p.best = head->best;
            p.argmax = argmax + r0;
            p.logits = logits ? logits + (int64_t) r0 * c.vocab : nullptr;
            p.error = head->d_error;
            p.vocab = c.vocab;
            p.dim = c.dim;
            p.n_rows = std::min<int32_t>(vxk::kHeadRows, rows - r0);
            p.tile_rows = head->tile_rows;
            p.n_tiles = head->n_tiles;
            p.dtype = (int32_t) c.dtype;
            VXK_HCUDA(vxk::launch_head(p, map_w, head->map_x, head->grid, cs));
        }
    });
}

vxk_status vxk_head_logits_argmax_q(vxk_head * head, vxk_qweight * w, const float * x, int32_t rows,
                                    int32_t * argmax, float * logits, void * cuda_stream) {
    if (!head) return VXK_STATUS_INVALID_ARGUMENT;
    return hguarded(head, [&] {
        const vxk_head_config & c = head->cfg;
        if (!w || !x || !argmax) hfail(VXK_STATUS_INVALID_ARGUMENT, "null argument");
        const vxk::QweightShape sh = vxk::qweight_shape(w);
        if (sh.device != c.device || sh.n_rows != c.vocab || sh.n_cols != c.dim)
            hfail(VXK_STATUS_INVALID_ARGUMENT, "the quantized embeddings must be vocab x dim on the head's device");
        if (rows < 1 || rows > vxk::kHeadRows || rows > sh.max_batch)
            hfail(VXK_STATUS_INVALID_ARGUMENT, "rows must be in [1, min(64, the matrix's max_batch)]");
        HeadDevice scope(c.device);
        cudaStream_t cs = static_cast<cudaStream_t>(cuda_stream);
        float * out = logits;
        if (!out) {
            if (!head->qlogits)
                VXK_HCUDA(cudaMalloc(&head->qlogits, (size_t) vxk::kHeadRows * c.vocab * sizeof(float)));
            out = head->qlogits;
        }
        const vxk_status st = vxk_qweight_matmul(w, x, rows, out, cuda_stream);
        if (st != VXK_STATUS_OK) hfail(st, "quantized logits product failed");
        VXK_HCUDA(vxk::launch_head_argmax(out, rows, c.vocab, head->best, argmax, cs));
    });
}

vxk_status vxk_head_sync(vxk_head * head, void * cuda_stream, int32_t timeout_ms) {
    if (!head) return VXK_STATUS_INVALID_ARGUMENT;
    return hguarded(head, [&] {
        HeadDevice scope(head->cfg.device);
        VXK_HCUDA(cudaEventRecord(head->ev_sync, static_cast<cudaStream_t>(cuda_stream)));
        const auto t0 = std::chrono::steady_clock::now();
        while (true) {
            const cudaError_t e = cudaEventQuery(head->ev_sync);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) hfail(VXK_STATUS_BACKEND_ERROR, cudaGetErrorString(e));
            const auto ms =
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if (ms > timeout_ms) hfail(VXK_STATUS_TIMEOUT, "stream did not drain within the timeout");
            // poll short waits (a step of a few ms); sleep between polls after 20 ms
            if (ms < 20)
                std::this_thread::yield();
            else
                std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        int32_t err = 0;
        VXK_HCUDA(cudaMemcpy(&err, head->d_error, sizeof(err), cudaMemcpyDeviceToHost));
        if (err != 0) {
            VXK_HCUDA(cudaMemset(head->d_error, 0, sizeof(int32_t)));
            hfail(VXK_STATUS_BACKEND_ERROR, "greedy head kernel reported a device error (bounded wait expired)");
        }
    });
}

}  // extern "C"
