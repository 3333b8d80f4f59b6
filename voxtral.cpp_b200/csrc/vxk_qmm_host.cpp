// Host runtime of the quantized-weight matrix product (include/vxk.h,
// vxk_qweight_*): the repack of GGUF rows into the device record layout,
// the product's scratch, and the split of the column range over CTAs.
//
// Record layout (one 16-row x 256-column tile, rows r = 0..15, lane L =
// 4g + c of the mma fragments, g = L / 4, c = L % 4):
//   Q8_0 (4352 B)  [8 blocks j][32 lanes][4 words i][4 bytes b]: int8
//                  W[g + 8(i%2)][32j + 4c + 16(i/2) + b], then [8 blocks][8 g]
//                  f16 pairs (d of row g, d of row g + 8).
//   Q4_K (2368 B)  [4 sub-block pairs p][32 lanes][4 words i][4 bytes b]:
//                  the 4-bit quants of sub-block 2p in the low nibble and of
//                  2p + 1 in the high nibble, each at the Q8_0 position
//                  (block = sub-block); then [16 rows] (d, dmin) f16 pairs,
//                  [16 rows][8] 6-bit scales and [16 rows][8] 6-bit mins as
//                  bytes (GGUF packs these 16 into 12 bytes per row).
//   Q6_K (3360 B)  [4 quads][32 lanes][4 sub-blocks][4 bytes b]: low 4 bits of
//                  the 16-column sub-block t = 4 quad + word: row g in the low
//                  nibble, row g + 8 in the high nibble, column 16t + 4c + b;
//                  then [2][32 lanes][4 pairs][4 bytes b]: the high 2 bits of
//                  sub-blocks 2P and 2P + 1 (P = 4 half + word), bits 0-1 / 2-3
//                  rows g / g + 8 of 2P, bits 4-5 / 6-7 of 2P + 1; then
//                  [16 rows][16] int8 scales, [16 rows] f16 d.
// Quants are stored as GGUF holds them (Q4_K 0..15, Q6_K 0..63 = q + 32).
#include "vxk.h"
#include "vxk_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_qw_create_error;

struct QwError {
    vxk_status status;
    std::string message;
};

[[noreturn]] void qfail(vxk_status s, const std::string & m) { throw QwError{s, m}; }

#define VXK_QCUDA(expr)                                                                 \
    do {                                                                                \
        const cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess) {                                                        \
            qfail(e_ == cudaErrorMemoryAllocation ? VXK_STATUS_OUT_OF_MEMORY            \
                                                  : VXK_STATUS_BACKEND_ERROR,           \
                  std::string(#expr) + ": " + cudaGetErrorString(e_));                  \
        }                                                                               \
    } while (0)

class QwDevice {
public:
    explicit QwDevice(int d) {
        cudaGetDevice(&prev_);
        dev_ = d;
        if (prev_ != d) cudaSetDevice(d);
    }
    ~QwDevice() {
        if (prev_ != dev_) cudaSetDevice(prev_);
    }

private:
    int prev_ = 0, dev_ = 0;
};

// A split stages its quantized rows in shared memory and a 64-row block is cut
// into at most 8 splits (one cluster): 64 column units at most.
constexpr int kMaxCols = 16384;

int64_t gguf_row_bytes(int type, int64_t k) {
    switch (type) {
        case VXK_QTYPE_Q8_0: return k / 32 * 34;
        case VXK_QTYPE_Q4_K: return k / 256 * 144;
        case VXK_QTYPE_Q6_K: return k / 256 * 210;
        default: return -1;
    }
}

void check_shape(int type, int32_t n_rows, int32_t n_cols) {
    if (vxk::qmm_record_bytes(type) == 0) qfail(VXK_STATUS_INVALID_ARGUMENT, "type must be Q8_0, Q4_K or Q6_K");
    if (n_rows < vxk::kQmmRows || n_rows % vxk::kQmmRows != 0)
        qfail(VXK_STATUS_INVALID_ARGUMENT, "n_rows must be a positive multiple of 64");
    if (n_cols < vxk::kQmmUnit || n_cols % vxk::kQmmUnit != 0 || n_cols > kMaxCols)
        qfail(VXK_STATUS_INVALID_ARGUMENT, "n_cols must be a multiple of 256 in [256, 16384]");
}

// Q4_K 6-bit scale and min of sub-block j from the 12 packed bytes.
void q4k_scale_min(const uint8_t * s, int j, uint8_t * sc, uint8_t * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t) ((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t) ((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

// One record: rows 16*tile .. +15, columns 256*u .. +255.
void repack_record(int type, const uint8_t * src, int64_t row_bytes, int64_t tile, int64_t u, uint8_t * out) {
    uint8_t val[16][256];
    if (type == VXK_QTYPE_Q8_0) {
        for (int rr = 0; rr < 16; ++rr) {
            const uint8_t * row = src + (tile * 16 + rr) * row_bytes;
            for (int j = 0; j < 8; ++j) {
                const uint8_t * blk = row + (u * 8 + j) * 34;
                std::memcpy(&val[rr][32 * j], blk + 2, 32);
                // f16 d pairs (row g, row g + 8) per block
                const int g = rr & 7, half = rr >> 3;
                std::memcpy(out + 4096 + (j * 8 + g) * 4 + half * 2, blk, 2);
            }
        }
        for (int j = 0; j < 8; ++j)
            for (int L = 0; L < 32; ++L)
                for (int i = 0; i < 4; ++i)
                    for (int b = 0; b < 4; ++b) {
                        const int g = L >> 2, c = L & 3;
                        out[j * 512 + L * 16 + i * 4 + b] = val[g + 8 * (i & 1)][32 * j + 4 * c + 16 * (i >> 1) + b];
                    }
        return;
    }
    if (type == VXK_QTYPE_Q4_K) {
        for (int rr = 0; rr < 16; ++rr) {
            const uint8_t * blk = src + (tile * 16 + rr) * row_bytes + u * 144;
            const uint8_t * qs = blk + 16;
            for (int i = 0; i < 4; ++i)
                for (int l = 0; l < 32; ++l) {
                    val[rr][64 * i + l] = qs[32 * i + l] & 0xF;
                    val[rr][64 * i + 32 + l] = qs[32 * i + l] >> 4;
                }
            std::memcpy(out + 2048 + rr * 4, blk, 4);  // d, dmin
            for (int j = 0; j < 8; ++j) q4k_scale_min(blk + 4, j, out + 2112 + rr * 8 + j, out + 2240 + rr * 8 + j);
        }
        for (int p = 0; p < 4; ++p)
            for (int L = 0; L < 32; ++L)
                for (int i = 0; i < 4; ++i)
                    for (int b = 0; b < 4; ++b) {
                        const int g = L >> 2, c = L & 3;
                        const int r = g + 8 * (i & 1), k = 4 * c + 16 * (i >> 1) + b;
                        out[p * 512 + L * 16 + i * 4 + b] =
                            (uint8_t) (val[r][32 * (2 * p) + k] | (val[r][32 * (2 * p + 1) + k] << 4));
                    }
        return;
    }
    // Q6_K
    for (int rr = 0; rr < 16; ++rr) {
        const uint8_t * blk = src + (tile * 16 + rr) * row_bytes + u * 210;
        for (int h = 0; h < 2; ++h) {
            const uint8_t * ql = blk + 64 * h;
            const uint8_t * qh = blk + 128 + 32 * h;
            for (int l = 0; l < 32; ++l) {
                val[rr][128 * h + l] = (uint8_t) ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4));
                val[rr][128 * h + l + 32] = (uint8_t) ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4));
                val[rr][128 * h + l + 64] = (uint8_t) ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4));
                val[rr][128 * h + l + 96] = (uint8_t) ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4));
            }
        }
        std::memcpy(out + 3072 + rr * 16, blk + 192, 16);
        std::memcpy(out + 3328 + rr * 2, blk + 208, 2);
    }
    for (int L = 0; L < 32; ++L) {
        const int g = L >> 2, c = L & 3;
        for (int t = 0; t < 16; ++t)
            for (int b = 0; b < 4; ++b) {
                const int k = 16 * t + 4 * c + b;
                out[(t >> 2) * 512 + L * 16 + (t & 3) * 4 + b] = (uint8_t) ((val[g][k] & 0xF) | ((val[g + 8][k] & 0xF) << 4));
            }
        for (int P = 0; P < 8; ++P)
            for (int b = 0; b < 4; ++b) {
                const int k0 = 16 * (2 * P) + 4 * c + b, k1 = k0 + 16;
                out[2048 + (P >> 2) * 512 + L * 16 + (P & 3) * 4 + b] =
                    (uint8_t) ((val[g][k0] >> 4) | ((val[g + 8][k0] >> 4) << 2) | ((val[g][k1] >> 4) << 4) |
                               ((val[g + 8][k1] >> 4) << 6));
            }
    }
}

int nt_for(int32_t rows) { return rows <= 8 ? 1 : rows <= 16 ? 2 : rows <= 32 ? 4 : 8; }

// Q6_K rows -> the tcgen05 layout (vxk_internal.h, kQtcRecordBytesQ6K): per
// 128-row block and unit, each row's 256 6-bit quants one per byte in column
// order (16-byte chunk c at c ^ (row % 8)), then its 16 int8 scales; (d, 0)
// pairs to `dd`.  The quant of element e of a GGUF block: low nibble of
// ql[64h + l] (parts 0, 1 of half h = e / 128, l = e % 32, part = (e / 32) % 4:
// ql[64h + 32 + l] for parts 1 and 3, high nibble for parts 2 and 3), high bits
// (qh[32h + l] >> 2 part) & 3.
void repack_q6k_tc(const uint8_t * src, int32_t n_rows, int32_t n_cols, uint8_t * rec, uint8_t * dd) {
    const int64_t units = n_cols / vxk::kQmmUnit;
    const int64_t rb = gguf_row_bytes(VXK_QTYPE_Q6_K, n_cols);
    for (int64_t b = 0; b < n_rows / 128; ++b)
        for (int64_t u = 0; u < units; ++u) {
            uint8_t * out = rec + (b * units + u) * vxk::kQtcRecordBytesQ6K;
            uint8_t * d = dd + ((b * units + u) * 128) * 4;
            for (int r = 0; r < 128; ++r) {
                const uint8_t * blk = src + (b * 128 + r) * rb + u * 210;
                const uint8_t * ql = blk;
                const uint8_t * qh = blk + 128;
                uint8_t q6[256];
                for (int e = 0; e < 256; ++e) {
                    const int h = e >> 7, part = (e >> 5) & 3, l = e & 31;
                    const uint8_t qb = ql[64 * h + 32 * (part & 1) + l];
                    const int lo = part < 2 ? (qb & 15) : (qb >> 4);
                    const int hi = (qh[32 * h + l] >> (2 * part)) & 3;
                    q6[e] = (uint8_t) (lo | (hi << 4));
                }
                for (int c = 0; c < 16; ++c)
                    std::memcpy(out + r * 256 + ((c ^ (r & 7)) << 4), q6 + 16 * c, 16);
                std::memcpy(out + 32768 + r * 16, blk + 192, 16);
                std::memcpy(d + r * 4, blk + 208, 2);
                d[r * 4 + 2] = d[r * 4 + 3] = 0;
            }
        }
}

// Q4_K rows -> the tcgen05 layout (vxk_internal.h, kQtcRecordBytes): per
// 128-row block and 256-column unit, each row's 128 quant bytes with 16-byte
// chunk c stored at chunk c ^ (row % 8), then each row's unpacked 6-bit
// scales and mins; the (d, dmin) pairs go to `dd` [block][unit][row].
void repack_q4k_tc(const uint8_t * src, int32_t n_rows, int32_t n_cols, uint8_t * rec, uint8_t * dd) {
    const int64_t units = n_cols / vxk::kQmmUnit;
    const int64_t rb = gguf_row_bytes(VXK_QTYPE_Q4_K, n_cols);
    for (int64_t b = 0; b < n_rows / 128; ++b)
        for (int64_t u = 0; u < units; ++u) {
            uint8_t * out = rec + (b * units + u) * vxk::kQtcRecordBytes;
            uint8_t * d = dd + ((b * units + u) * 128) * 4;
            for (int r = 0; r < 128; ++r) {
                const uint8_t * blk = src + (b * 128 + r) * rb + u * 144;
                for (int c = 0; c < 8; ++c) std::memcpy(out + r * 128 + ((c ^ (r & 7)) << 4), blk + 16 + 16 * c, 16);
                for (int j = 0; j < 8; ++j) q4k_scale_min(blk + 4, j, out + 16384 + r * 16 + j, out + 16384 + r * 16 + 8 + j);
                std::memcpy(d + r * 4, blk, 4);
            }
        }
}

}  // namespace

struct vxk_qweight {
    vxk_qweight_config cfg{};
    int32_t n_units = 0;
    int32_t nt_max = 0;
    int32_t sms = 0;
    uint8_t * w = nullptr;
    uint8_t * act = nullptr;
    float * act_d = nullptr;
    uint8_t * act_ms = nullptr;
    // tcgen05 form (Q4_K): records, (d, dmin) pairs and the f16 activation tiles
    uint8_t * w_tc = nullptr;
    uint8_t * dd_tc = nullptr;
    uint8_t * tc_b = nullptr;
    uint8_t * tc_bmin = nullptr;
    uint8_t * tc_b8 = nullptr;
    float * tc_dx = nullptr;
    int32_t * d_error = nullptr;
    int32_t * own_error = nullptr;   // d_error unless an owner attached a shared word
    cudaEvent_t ev_sync = nullptr;
    std::string last_error;
};

namespace {

template <typename F>
vxk_status qguarded(vxk_qweight * w, F && body) {
    try {
        body();
        return VXK_STATUS_OK;
    } catch (const QwError & e) {
        if (w) w->last_error = e.message;
        return e.status;
    } catch (const std::bad_alloc &) {
        if (w) w->last_error = "host out of memory";
        return VXK_STATUS_OUT_OF_MEMORY;
    } catch (...) {
        if (w) w->last_error = "internal error";
        return VXK_STATUS_INTERNAL_ERROR;
    }
}

void free_qweight(vxk_qweight * w) {
    if (!w) return;
    QwDevice scope(w->cfg.device);
    for (void * p : {(void *) w->w, (void *) w->act, (void *) w->act_d, (void *) w->act_ms, (void *) w->w_tc,
                     (void *) w->dd_tc, (void *) w->tc_b, (void *) w->tc_bmin, (void *) w->tc_b8, (void *) w->tc_dx, (void *) w->own_error})
        if (p) cudaFree(p);
    if (w->ev_sync) cudaEventDestroy(w->ev_sync);
    delete w;
}

// Column units per CTA for p.nt activation n-tiles over the group's 64-row
// blocks (p.mats).  A 64-row block is cut into at most 8 splits (one
// cluster).  For each split size that fits shared memory, the runtime says how
// many CTAs an SM holds; the plan minimises waves x (units per CTA + a fixed
// 1.5-unit cost of a CTA's start and cluster reduction), preferring fewer
// splits on ties (the rule was fitted to a sweep of split sizes on B200 at 16
// and 64 rows).
void plan_split(int32_t n_units, int32_t sms, vxk::QmmParams & p) {
    int64_t blocks = 0;
    for (int i = 0; i < p.n_mats; ++i) blocks += p.mats[i].n_rows / vxk::kQmmRows;
    int best_per = 0;
    double best_cost = 0.0;
    for (int per = 1; per <= n_units; ++per) {
        const int splits = (n_units + per - 1) / per;
        if (splits > vxk::kQmmMaxSplits) continue;
        if (per > 1 && (n_units + per - 2) / (per - 1) == splits) continue;  // same split count, more units
        const int smem = vxk::qmm_smem_bytes(p, per);
        if (smem > 232448) break;
        const int per_sm = vxk::qmm_ctas_per_sm(p, smem);
        if (per_sm < 1) continue;
        const int64_t slots = (int64_t) std::max(1, sms) * per_sm;
        const int64_t ctas = blocks * splits;
        // from 32 rows on the product is bound by instruction issue, and the
        // CTAs of a partial wave finish faster: count waves fractionally; at
        // 1-16 rows each CTA is latency-bound: count whole waves
        const double waves = p.nt >= 4 ? std::max(1.0, (double) ctas / (double) slots)
                                       : (double) ((ctas + slots - 1) / slots);
        const double cost = waves * (per + 1.5);
        if (best_per == 0 || cost < best_cost - 1e-9 || (cost <= best_cost + 1e-9 && splits < (n_units + best_per - 1) / best_per)) {
            best_per = per;
            best_cost = cost;
        }
    }
    if (best_per == 0) qfail(VXK_STATUS_INVALID_ARGUMENT, "no column split of this product fits shared memory");
    p.units_per_split = best_per;
    p.n_splits = (n_units + best_per - 1) / best_per;
}

vxk::QmmMat mat_of(const vxk_qweight * w, float * y, int32_t block0) {
    vxk::QmmMat m{};
    m.w = w->w;
    m.y = y;
    m.type = (int32_t) w->cfg.type;
    m.n_rows = w->cfg.n_rows;
    m.block0 = block0;
    return m;
}

// True when a product of `rows` rows with w runs on the tcgen05 kernel: Q4_K
// and Q6_K weights from 17 rows up, where the int8 mma.sync kernel is bound by
// instruction issue.
bool use_tc(const vxk_qweight * w, int32_t rows) { return w->w_tc && rows > 16; }

// Column units per CTA of the tcgen05 product (one 191 KB CTA per SM): the
// fewest whole waves x (units per CTA + 1.5), splits <= 8, fewer splits on
// ties; a wave holds as many clusters of `splits` CTAs as the runtime says fit.
void plan_split_tc(int32_t n_units, int32_t sms, int64_t blocks, vxk::QtcParams & p) {
    int best = 0;
    double best_cost = 0.0;
    for (int per = 1; per <= n_units; ++per) {
        const int splits = (n_units + per - 1) / per;
        if (splits > vxk::kQmmMaxSplits) continue;
        if (per > 1 && (n_units + per - 2) / (per - 1) == splits) continue;
        int clusters = vxk::qtc_max_active_clusters(p.npad, splits);
        if (clusters < 1) clusters = std::max(1, sms / splits);
        const int64_t waves = (blocks + clusters - 1) / clusters;
        const double cost = (double) waves * (per + 1.5);
        if (best == 0 || cost < best_cost - 1e-9) {
            best = per;
            best_cost = cost;
        }
    }
    p.units_per_split = best;
    p.n_splits = (n_units + best - 1) / best;
}

void run_tc(vxk_qweight * const * ws, int32_t n, const float * x, const float * x_up, int32_t rows,
            float * const * ys, const float * const * biases, int32_t * error, cudaStream_t stream,
            bool prequantized = false) {
    vxk_qweight * w0 = ws[0];
    vxk::QtcParams p{};
    p.n_mats = n;
    p.n_units = w0->n_units;
    p.rows = rows;
    p.npad = rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
    p.n_chunks = (rows + p.npad - 1) / p.npad;
    int32_t block0 = 0;
    for (int i = 0; i < n; ++i) {
        p.mats[i].w = ws[i]->w_tc;
        p.mats[i].dd = ws[i]->dd_tc;
        p.mats[i].y = ys[i];
        p.mats[i].n_rows = ws[i]->cfg.n_rows;
        p.mats[i].block0 = block0;
        p.mats[i].type = (int32_t) ws[i]->cfg.type;
        p.mats[i].bias = biases ? biases[i] : nullptr;
        block0 += ws[i]->cfg.n_rows / 128;
    }
    plan_split_tc(w0->n_units, w0->sms, (int64_t) block0 * p.n_chunks, p);
    p.x = x;
    p.x_up = x_up;
    // operand tiles of the types in the group: f16 (+ mins) for Q4_K, int8 for Q6_K
    bool q4 = false, q6 = false;
    for (int i = 0; i < n; ++i) (ws[i]->cfg.type == VXK_QTYPE_Q6_K ? q6 : q4) = true;
    p.b_tiles = q4 ? w0->tc_b : nullptr;
    p.bmin_tiles = q4 ? w0->tc_bmin : nullptr;
    p.b8_tiles = q6 ? w0->tc_b8 : nullptr;
    p.dx = w0->tc_dx;
    p.error = error;
    VXK_QCUDA(vxk::launch_qtc(p, stream, prequantized));
}

void run_sync(vxk_qweight * const * ws, int32_t n, const float * x, const float * x_up, int32_t rows,
              float * const * ys, int32_t * error, cudaStream_t stream) {
    vxk_qweight * w0 = ws[0];
    vxk::QmmParams p{};
    p.n_mats = n;
    p.n_units = w0->n_units;
    p.rows = rows;
    p.nt = nt_for(rows);
    int32_t block0 = 0;
    for (int i = 0; i < n; ++i) {
        p.mats[i] = mat_of(ws[i], ys[i], block0);
        block0 += ws[i]->cfg.n_rows / vxk::kQmmRows;
    }
    plan_split(w0->n_units, w0->sms, p);
    p.x = x;
    p.x_up = x_up;
    p.act = w0->act;
    p.act_d = w0->act_d;
    p.act_ms = w0->act_ms;
    p.error = error;
    VXK_QCUDA(vxk::launch_qmm(p, stream));
}

// Quantizes x and multiplies it by every matrix of ws (shared n_cols, device
// and activation family): the matrices that take the tcgen05 kernel in one
// launch, the others in one int8 mma.sync launch, each with its own
// quantization of x (the two kernels read different operand layouts).
// biases[i] (when given) is added to every row of ys[i]: in the tcgen05
// product's store, or by a separate kernel after the mma.sync product.
void run_group(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows, float * const * ys,
               cudaStream_t stream, const float * x_up = nullptr, const float * const * biases = nullptr) {
    // the quantization kernels read rows as float4
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(x_up) & 15))
        qfail(VXK_STATUS_INVALID_ARGUMENT, "x must be 16-byte aligned");
    vxk_qweight * tw[vxk::kQmmMaxGroup], * sw[vxk::kQmmMaxGroup];
    float * ty[vxk::kQmmMaxGroup], * sy[vxk::kQmmMaxGroup];
    const float * tb[vxk::kQmmMaxGroup], * sb[vxk::kQmmMaxGroup];
    int nt = 0, ns = 0;
    for (int i = 0; i < n; ++i) {
        const float * b = biases ? biases[i] : nullptr;
        if (use_tc(ws[i], rows)) {
            tw[nt] = ws[i];
            tb[nt] = b;
            ty[nt++] = ys[i];
        } else {
            sw[ns] = ws[i];
            sb[ns] = b;
            sy[ns++] = ys[i];
        }
    }
    if (nt) run_tc(tw, nt, x, x_up, rows, ty, tb, ws[0]->d_error, stream);
    // the int8 mma.sync kernel takes at most 64 rows per launch
    const int64_t K = ws[0]->cfg.n_cols;
    for (int32_t r0 = 0; ns && r0 < rows; r0 += vxk::kQmmMaxBatch) {
        const int32_t nr = std::min<int32_t>(vxk::kQmmMaxBatch, rows - r0);
        float * syc[vxk::kQmmMaxGroup];
        for (int i = 0; i < ns; ++i) syc[i] = sy[i] + (int64_t) r0 * sw[i]->cfg.n_rows;
        run_sync(sw, ns, x + (int64_t) r0 * K, x_up ? x_up + (int64_t) r0 * K : nullptr, nr, syc, ws[0]->d_error,
                 stream);
    }
    for (int i = 0; i < ns; ++i)
        if (sb[i]) VXK_QCUDA(vxk::launch_bias2(sy[i], sb[i], sw[i]->cfg.n_rows, nullptr, nullptr, 0, rows, stream));
}

// Argument checks of a group product (shared device, n_cols and activation
// family; rows within every matrix's max_batch).
void check_group(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows, float * const * ys) {
    vxk_qweight * w0 = ws[0];
    if (!x) qfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
    const bool fam0 = w0->cfg.type == VXK_QTYPE_Q8_0;
    for (int32_t i = 0; i < n; ++i) {
        const vxk_qweight_config & c = ws[i]->cfg;
        if (!ys[i]) qfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        if (c.device != w0->cfg.device || c.n_cols != w0->cfg.n_cols)
            qfail(VXK_STATUS_INVALID_ARGUMENT, "group matrices must share device and n_cols");
        if ((c.type == VXK_QTYPE_Q8_0) != fam0)
            qfail(VXK_STATUS_INVALID_ARGUMENT, "a group is all Q8_0 or all K-quants (one x quantization)");
        if (rows < 1 || rows > c.max_batch) qfail(VXK_STATUS_INVALID_ARGUMENT, "rows must be in [1, max_batch]");
    }
}

}  // namespace

namespace vxk {

QweightShape qweight_shape(const vxk_qweight * w) {
    return QweightShape{w->cfg.device, (int32_t) w->cfg.type, w->cfg.n_rows, w->cfg.n_cols, w->cfg.max_batch};
}

void qweight_attach_error(vxk_qweight * w, int32_t * word) { w->d_error = word ? word : w->own_error; }

int32_t qweight_matmul_swiglu(vxk_qweight * w, const float * gate, const float * up, int32_t rows, float * y,
                              cudaStream_t stream) {
    if (!w) return VXK_STATUS_INVALID_ARGUMENT;
    return qguarded(w, [&] {
        if (!gate || !up || !y) qfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        if (rows < 1 || rows > w->cfg.max_batch) qfail(VXK_STATUS_INVALID_ARGUMENT, "rows must be in [1, max_batch]");
        QwDevice scope(w->cfg.device);
        vxk_qweight * one[1] = {w};
        float * yv[1] = {y};
        run_group(one, 1, gate, rows, yv, stream, up);
    });
}

bool qweight_group_tiles(vxk_qweight * const * ws, int32_t n, int32_t rows, QtcTiles * t) {
    if (!ws || n < 1 || n > kQmmMaxGroup || !t) return false;
    for (int32_t i = 0; i < n; ++i) {
        const vxk_qweight * w = ws[i];
        if (!w || !use_tc(w, rows) || rows > w->cfg.max_batch || w->cfg.device != ws[0]->cfg.device ||
            w->cfg.n_cols != ws[0]->cfg.n_cols)
            return false;
    }
    const int32_t npad = rows <= 16 ? 16 : rows <= 32 ? 32 : 64;
    bool q4 = false, q6 = false;
    for (int32_t i = 0; i < n; ++i) (ws[i]->cfg.type == VXK_QTYPE_Q6_K ? q6 : q4) = true;
    t->b = q4 ? ws[0]->tc_b : nullptr;
    t->bmin = q4 ? ws[0]->tc_bmin : nullptr;
    t->b8 = q6 ? ws[0]->tc_b8 : nullptr;
    t->dx = ws[0]->tc_dx;
    t->npad = npad;
    t->rows_padded = npad * ((rows + npad - 1) / npad);
    return true;
}

int32_t qweight_matmul_group_prequantized(vxk_qweight * const * ws, int32_t n, int32_t rows, float * const * ys,
                                          const float * const * biases, cudaStream_t stream) {
    QtcTiles t{};
    if (!qweight_group_tiles(ws, n, rows, &t) || !ys) return VXK_STATUS_INVALID_ARGUMENT;
    return qguarded(ws[0], [&] {
        for (int32_t i = 0; i < n; ++i)
            if (!ys[i]) qfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        QwDevice scope(ws[0]->cfg.device);
        run_tc(ws, n, nullptr, nullptr, rows, ys, biases, ws[0]->d_error, stream, true);
    });
}

int32_t qweight_matmul_group_bias(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows,
                                  float * const * ys, const float * const * biases, cudaStream_t stream) {
    if (!ws || n < 1 || n > kQmmMaxGroup || !ys) return VXK_STATUS_INVALID_ARGUMENT;
    for (int32_t i = 0; i < n; ++i)
        if (!ws[i]) return VXK_STATUS_INVALID_ARGUMENT;
    return qguarded(ws[0], [&] {
        check_group(ws, n, x, rows, ys);
        QwDevice scope(ws[0]->cfg.device);
        run_group(ws, n, x, rows, ys, stream, nullptr, biases);
    });
}

}  // namespace vxk

extern "C" {

vxk_qweight_config vxk_qweight_default_config(void) {
    vxk_qweight_config c{};
    c.struct_size = sizeof(vxk_qweight_config);
    c.api_version = VXK_API_VERSION;
    c.device = 0;
    c.type = VXK_QTYPE_Q4_K;
    c.n_rows = 4096;
    c.n_cols = 3072;
    c.max_batch = 64;
    return c;
}

vxk_status vxk_qweight_packed_bytes(vxk_qtype type, int32_t n_rows, int32_t n_cols, size_t * out_bytes) {
    if (!out_bytes) return VXK_STATUS_INVALID_ARGUMENT;
    try {
        check_shape((int) type, n_rows, n_cols);
    } catch (const QwError & e) {
        return e.status;
    }
    *out_bytes = (size_t) (n_rows / 16) * (size_t) (n_cols / vxk::kQmmUnit) * (size_t) vxk::qmm_record_bytes((int) type);
    return VXK_STATUS_OK;
}

vxk_status vxk_qweight_repack(vxk_qtype type, int32_t n_rows, int32_t n_cols, const void * gguf_blocks,
                              size_t gguf_bytes, void * out, size_t out_bytes) {
    if (!gguf_blocks || !out) return VXK_STATUS_INVALID_ARGUMENT;
    try {
        check_shape((int) type, n_rows, n_cols);
        const int64_t rb = gguf_row_bytes((int) type, n_cols);
        if (gguf_bytes != (size_t) (rb * n_rows)) qfail(VXK_STATUS_INVALID_ARGUMENT, "gguf_bytes != n_rows * row bytes");
        size_t need = 0;
        vxk_qweight_packed_bytes(type, n_rows, n_cols, &need);
        if (out_bytes < need) return VXK_STATUS_BUFFER_TOO_SMALL;
        const int rec = vxk::qmm_record_bytes((int) type);
        const int64_t units = n_cols / vxk::kQmmUnit;
        const uint8_t * src = static_cast<const uint8_t *>(gguf_blocks);
        uint8_t * dst = static_cast<uint8_t *>(out);
        for (int64_t t = 0; t < n_rows / 16; ++t)
            for (int64_t u = 0; u < units; ++u) repack_record((int) type, src, rb, t, u, dst + (t * units + u) * rec);
    } catch (const QwError & e) {
        return e.status;
    } catch (...) {
        return VXK_STATUS_INTERNAL_ERROR;
    }
    return VXK_STATUS_OK;
}

vxk_status vxk_qweight_create(const vxk_qweight_config * config, const void * gguf_blocks, size_t gguf_bytes,
                              vxk_qweight ** out) {
    if (out) *out = nullptr;
    if (!config || !out || !gguf_blocks) {
        g_qw_create_error = "null argument";
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    vxk_qweight * w = new (std::nothrow) vxk_qweight();
    if (!w) return VXK_STATUS_OUT_OF_MEMORY;
    const vxk_status st = qguarded(w, [&] {
        const vxk_qweight_config & c = *config;
        if (c.struct_size < sizeof(vxk_qweight_config)) qfail(VXK_STATUS_INVALID_ARGUMENT, "config struct_size too small");
        check_shape((int) c.type, c.n_rows, c.n_cols);
        if (c.max_batch < 1 || c.max_batch > vxk::kQmmMaxRows)
            qfail(VXK_STATUS_INVALID_ARGUMENT, "max_batch must be in [1, 512]");
        const int64_t rb = gguf_row_bytes((int) c.type, c.n_cols);
        if (gguf_bytes != (size_t) (rb * c.n_rows)) qfail(VXK_STATUS_INVALID_ARGUMENT, "gguf_bytes != n_rows * row bytes");
        w->cfg = c;
        w->n_units = c.n_cols / vxk::kQmmUnit;
        w->nt_max = nt_for(std::min(c.max_batch, vxk::kQmmMaxBatch));
        int n_dev = 0;
        VXK_QCUDA(cudaGetDeviceCount(&n_dev));
        if (c.device < 0 || c.device >= n_dev) qfail(VXK_STATUS_INVALID_ARGUMENT, "no such CUDA device");
        QwDevice scope(c.device);
        VXK_QCUDA(cudaDeviceGetAttribute(&w->sms, cudaDevAttrMultiProcessorCount, c.device));
        size_t packed = 0;
        vxk_qweight_packed_bytes(c.type, c.n_rows, c.n_cols, &packed);
        std::vector<uint8_t> host(packed);
        const vxk_status rs = vxk_qweight_repack(c.type, c.n_rows, c.n_cols, gguf_blocks, gguf_bytes, host.data(), packed);
        if (rs != VXK_STATUS_OK) qfail(rs, "repack failed");
        VXK_QCUDA(cudaMalloc(&w->w, packed));
        VXK_QCUDA(cudaMemcpy(w->w, host.data(), packed, cudaMemcpyHostToDevice));
        const int64_t cols = (int64_t) w->nt_max * 8;
        VXK_QCUDA(cudaMalloc(&w->act, (size_t) w->n_units * w->nt_max * 2048));
        VXK_QCUDA(cudaMalloc(&w->act_d, (size_t) w->n_units * 8 * cols * sizeof(float)));
        VXK_QCUDA(cudaMalloc(&w->act_ms, (size_t) w->n_units * w->nt_max * 256));
        VXK_QCUDA(cudaMemset(w->act_ms, 0, (size_t) w->n_units * w->nt_max * 256));
        if ((c.type == VXK_QTYPE_Q4_K || c.type == VXK_QTYPE_Q6_K) && c.n_rows % 128 == 0) {
            const bool q6 = c.type == VXK_QTYPE_Q6_K;
            const size_t recs = (size_t) (c.n_rows / 128) * w->n_units;
            std::vector<uint8_t> hrec(recs * (q6 ? vxk::kQtcRecordBytesQ6K : vxk::kQtcRecordBytes)), hdd(recs * 128 * 4);
            if (q6)
                repack_q6k_tc(static_cast<const uint8_t *>(gguf_blocks), c.n_rows, c.n_cols, hrec.data(), hdd.data());
            else
                repack_q4k_tc(static_cast<const uint8_t *>(gguf_blocks), c.n_rows, c.n_cols, hrec.data(), hdd.data());
            VXK_QCUDA(cudaMalloc(&w->w_tc, hrec.size()));
            VXK_QCUDA(cudaMemcpy(w->w_tc, hrec.data(), hrec.size(), cudaMemcpyHostToDevice));
            VXK_QCUDA(cudaMalloc(&w->dd_tc, hdd.size()));
            VXK_QCUDA(cudaMemcpy(w->dd_tc, hdd.data(), hdd.size(), cudaMemcpyHostToDevice));
            const size_t chunks = (size_t) (c.max_batch + 63) / 64;  // 64-row chunks of one launch
            VXK_QCUDA(cudaMalloc(&w->tc_b, chunks * w->n_units * 64 * 512));
            VXK_QCUDA(cudaMalloc(&w->tc_bmin, chunks * w->n_units * 64 * 128));
            VXK_QCUDA(cudaMalloc(&w->tc_b8, chunks * w->n_units * 64 * 256));
            VXK_QCUDA(cudaMalloc(&w->tc_dx, chunks * w->n_units * 64 * sizeof(float)));
        }
        VXK_QCUDA(cudaMalloc(&w->d_error, sizeof(int32_t)));
        w->own_error = w->d_error;
        VXK_QCUDA(cudaMemset(w->d_error, 0, sizeof(int32_t)));
        VXK_QCUDA(cudaEventCreateWithFlags(&w->ev_sync, cudaEventDisableTiming));
        VXK_QCUDA(cudaDeviceSynchronize());
    });
    if (st != VXK_STATUS_OK) {
        g_qw_create_error = w->last_error;
        free_qweight(w);
        return st;
    }
    *out = w;
    return VXK_STATUS_OK;
}

void vxk_qweight_destroy(vxk_qweight * w) { free_qweight(w); }

vxk_status vxk_qweight_last_error(const vxk_qweight * w, char * buf, size_t capacity) {
    if (!buf || capacity == 0) return VXK_STATUS_INVALID_ARGUMENT;
    const std::string & m = w ? w->last_error : g_qw_create_error;
    const size_t n = std::min(capacity - 1, m.size());
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
    return m.size() < capacity ? VXK_STATUS_OK : VXK_STATUS_BUFFER_TOO_SMALL;
}

vxk_status vxk_qweight_matmul(vxk_qweight * w, const float * x, int32_t rows, float * y, void * cuda_stream) {
    if (!w) return VXK_STATUS_INVALID_ARGUMENT;
    return qguarded(w, [&] {
        const vxk_qweight_config & c = w->cfg;
        if (!x || !y) qfail(VXK_STATUS_INVALID_ARGUMENT, "null buffer");
        if (rows < 1 || rows > c.max_batch) qfail(VXK_STATUS_INVALID_ARGUMENT, "rows must be in [1, max_batch]");
        QwDevice scope(c.device);
        vxk_qweight * one[1] = {w};
        float * yv[1] = {y};
        run_group(one, 1, x, rows, yv, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_qweight_matmul_group(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows,
                                    float * const * ys, void * cuda_stream) {
    if (!ws || n < 1 || n > vxk::kQmmMaxGroup || !ys) return VXK_STATUS_INVALID_ARGUMENT;
    for (int32_t i = 0; i < n; ++i)
        if (!ws[i]) return VXK_STATUS_INVALID_ARGUMENT;
    vxk_qweight * w0 = ws[0];
    return qguarded(w0, [&] {
        check_group(ws, n, x, rows, ys);
        QwDevice scope(w0->cfg.device);
        run_group(ws, n, x, rows, ys, static_cast<cudaStream_t>(cuda_stream));
    });
}

vxk_status vxk_qweight_sync(vxk_qweight * w, void * cuda_stream, int32_t timeout_ms) {
    if (!w) return VXK_STATUS_INVALID_ARGUMENT;
    return qguarded(w, [&] {
        QwDevice scope(w->cfg.device);
        VXK_QCUDA(cudaEventRecord(w->ev_sync, static_cast<cudaStream_t>(cuda_stream)));
        const auto t0 = std::chrono::steady_clock::now();
        while (true) {
            const cudaError_t e = cudaEventQuery(w->ev_sync);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) qfail(VXK_STATUS_BACKEND_ERROR, cudaGetErrorString(e));
            const auto ms =
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if (ms > timeout_ms) qfail(VXK_STATUS_TIMEOUT, "stream did not drain within the timeout");
            // poll short waits (a step of a few ms); sleep between polls after 20 ms
            if (ms < 20)
                std::this_thread::yield();
            else
                std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        int32_t err = 0;
        VXK_QCUDA(cudaMemcpy(&err, w->d_error, sizeof(err), cudaMemcpyDeviceToHost));
        if (err != 0) {
            VXK_QCUDA(cudaMemset(w->d_error, 0, sizeof(int32_t)));
            qfail(VXK_STATUS_TIMEOUT, "quantized product kernel reported an expired bounded wait");
        }
    });
}

}  // extern "C"
