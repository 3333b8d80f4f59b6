// Internal declarations shared by the host runtime (vxk_pool.cpp,
// vxk_encoder_host.cpp) and the sm_100a kernels (vxk_decode.cu,
// vxk_encoder.cu).  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

struct vxk_qweight;
struct vxk_pool;
struct vxk_enc_pool;

namespace vxk {

// Decoder kernels are specialised for the Voxtral decoder head shape.
constexpr int kHeadDim = 128;     // head_dim of both Voxtral decoders
constexpr int kGroup = 4;         // query heads per kv head (32 / 8)
constexpr int kBlockTokens = 16;  // positions per page
constexpr int kQ8Block = 32;      // ggml QK8_0

// Row flag: the fused decode kernel appends this row's K/V before attending.
constexpr int32_t kRowAppend = 1;

// One query row of a planned batch (one new token of one stream).
struct RowDesc {
    int32_t stream;     // pool stream id (block-table row)
    int32_t pos;        // absolute position of the token
    int32_t win_start;  // oldest absolute position the row attends
    int32_t item_base;  // first work item of the row
    int32_t n_chunks;   // work items (splits) of the row
    int32_t flags;      // kRowAppend
    int32_t reserved0;
    int32_t reserved1;
};
static_assert(sizeof(RowDesc) == 32, "RowDesc layout");

// One split of one row: logical pages [page_begin, page_end).
struct WorkItem {
    int32_t row;
    int32_t chunk;
    int32_t page_begin;
    int32_t page_end;
};
static_assert(sizeof(WorkItem) == 16, "WorkItem layout");

// Block-table update (index into the [max_streams][bt_cap] table, page id).
struct TableUpdate {
    int32_t index;
    int32_t page;
};

// Partial record of one (work item, query head): acc[head_dim], m, l, pad.
constexpr int kPartialStride = kHeadDim + 4;

// Largest split (pages of one work item) the decode kernel accepts: 4 warps,
// each holding 4 page ids per lane.
constexpr int kMaxSplitPages = 512;

struct DecodeParams {
    // cache of one layer: one record per (page, kv head): the swizzled tile's
    // f32 / f16 values, or for q8_0 its int8 values followed by its f16 block
    // scales ([4 blocks][16 rows]), 2176 bytes
    uint8_t * k_data;
    uint8_t * v_data;
    int32_t n_blocks;
    int32_t n_kv;
    int32_t n_q;
    int32_t bt_cap;          // pages per stream ring
    const int32_t * block_table;
    const RowDesc * rows;
    const WorkItem * items;
    const int32_t * sched_offsets;  // [n_ctas + 1] per-CTA ranges of sched_units
    const int32_t * sched_units;    // unit = item * n_kv + kv head, per CTA in order
    int32_t n_ctas;
    int32_t n_rows;
    int32_t n_items;
    const float * q;         // [rows][n_q][head_dim]
    const float * k;         // [rows][n_kv][head_dim]
    const float * v;
    float * out;             // [rows][n_q][head_dim]
    const float2 * rope;     // [rope_rows][head_dim / 2] (cos, sin)
    int32_t rope_rows;
    float scale_log2;        // softmax scale * log2(e)
    float * partials;        // [n_items][n_q][kPartialStride]
    int32_t * counters;      // [max_rows][n_kv], zero between launches
    int32_t * error;         // device error word (0 = ok)
    int32_t fuse_append;     // 1: rows flagged kRowAppend append first
    int32_t dtype;           // 0 = f32, 1 = f16, 8 = q8_0
    // launch_decode_quant only: each row's output also quantized into the next
    // product's activation tiles (QtcTiles); out may then be nullptr
    uint8_t * q_tiles;
    uint8_t * q_bmin;
    uint8_t * q_tiles8;
    float * q_dx;
    int32_t q_npad;
    int32_t q_units;         // 256-column units of a row: n_q x head_dim / 256
};

struct AppendParams {
    uint8_t * k_data;  // records as in DecodeParams
    uint8_t * v_data;
    int32_t n_blocks;
    int32_t n_kv;
    int32_t bt_cap;
    const int32_t * block_table;
    const RowDesc * rows;
    int32_t n_rows;
    const float * k;
    const float * v;
    const float2 * rope;
    int32_t rope_rows;
    int32_t * error;
    int32_t dtype;
};

struct GatherParams {
    const uint8_t * k_data;  // records as in DecodeParams
    const uint8_t * v_data;
    int32_t n_blocks;
    int32_t n_kv;
    int32_t bt_cap;
    const int32_t * block_table;  // row of one stream
    int64_t pos_start;
    int32_t n;
    uint8_t * k_out;   // f16: [n][n_kv][hd] halves; q8_0: [n][n_kv][hd] int8
    uint8_t * v_out;
    uint8_t * k_scale_out;  // q8_0: [n][n_kv][hd/32] f16
    uint8_t * v_scale_out;
    int32_t dtype;
};

struct CompactParams {
    uint8_t * k_data;           // base of layer 0
    uint8_t * v_data;
    int64_t layer_data_bytes;   // bytes per layer of k_data
    int64_t page_data_bytes;    // bytes per page per layer (all kv heads' records)
    int32_t n_layers;
    const int2 * moves;         // (src, dst)
    int32_t n_moves;
};

// pdl: launch with programmatic stream serialization.  Only valid when the
// preceding kernel on the stream writes nothing the decode prologue reads
// (row/work descriptors, block table, cache pages of this layer).
cudaError_t launch_decode(const DecodeParams & p, cudaStream_t stream, bool pdl);
// launch_decode for an f16 cache with the quantization of the output rows into
// p.q_* (the o product's tiles) in the same launch.
cudaError_t launch_decode_quant(const DecodeParams & p, cudaStream_t stream, bool pdl);
cudaError_t launch_append(const AppendParams & p, cudaStream_t stream);
cudaError_t launch_table_updates(int32_t * table, const TableUpdate * updates, int32_t n,
                                 cudaStream_t stream);
cudaError_t launch_gather(const GatherParams & p, cudaStream_t stream);
cudaError_t launch_compact(const CompactParams & p, cudaStream_t stream);

// Fixed split scratch of vxk_decode_layer_static_scratch: partial records for
// up to 512 splits x 32 query heads, then arrival counters for up to 256 rows
// x 8 kv heads (8.66 MB of floats in total).
constexpr size_t kStaticScratchPartialFloats = (size_t) 512 * 32 * kPartialStride;
constexpr size_t kStaticScratchCounters = (size_t) 256 * 8;
constexpr size_t kStaticScratchFloats = kStaticScratchPartialFloats + kStaticScratchCounters;

// Same launch as launch_decode (without programmatic dependent launch), with
// the split scratch in the library's fixed device array instead of
// p.partials / p.counters.  Returns cudaErrorInvalidValue when the batch needs
// more scratch than the array holds.  Allocates nothing.
cudaError_t launch_decode_static_scratch(const DecodeParams & p, cudaStream_t stream);

// Launches one warp that waits, with the decode kernel's bounded wait, on an
// mbarrier nothing arrives on, and sets *error to the timeout code after
// limit_ns (test of the failure path).
cudaError_t launch_wait_probe(int32_t * error, uint64_t limit_ns, cudaStream_t stream);

// Shared-memory bytes the decode kernel needs, and how many of its CTAs are
// resident per SM on the current device (0 on error).
int decode_smem_bytes(int dtype);
int decode_ctas_per_sm(int dtype);

// ---------------------------------------------------------------------------
// Streaming encoder window attention
// ---------------------------------------------------------------------------

struct EncRowDesc {
    int32_t stream;
    int32_t pos;        // absolute frame of the query row
    int32_t win_start;  // max(0, pos - window + 1)
    int32_t slot;       // pos % capacity
};
static_assert(sizeof(EncRowDesc) == 16, "EncRowDesc layout");

struct EncParams {
    uint8_t * k_ring;       // [max_streams][n_layers][n_heads][ring_slots][head_dim] 16-bit, rows swizzled
    uint8_t * v_ring;
    int32_t n_layers;
    int32_t layer;
    int32_t n_heads;
    int32_t capacity;       // logical ring capacity (slot = position % capacity)
    int32_t ring_slots;     // stored rows per ring: round_up(capacity, 8), pad rows zero
    int32_t window;
    const EncRowDesc * rows;
    int32_t n_rows;
    const int32_t * group_first;  // first row of each (stream) group
    int32_t n_groups;
    // per group two int4: {first row | rows << 24, stream, first row's window
    // start, last row's position} and {first 8-slot box of the window walk
    // (window start % capacity rounded down to 8), boxes walked, last row's
    // slot, 0}: what the attention kernel needs of a group, without divisions
    // (rows of a group are consecutive positions)
    const int4 * groups;
    const float * q;        // [rows][n_heads][64]
    const float * k;
    const float * v;
    float * out;
    const float2 * rope;    // [rope_rows][32]
    int32_t rope_rows;
    float scale_log2;
    int32_t * error;
    int32_t dtype;          // 30 = bf16, 1 = f16, 0 = f32
    // 1 when every group is a whole stream (<= 8 new rows each): the attention
    // kernel then stores its own group's new K/V rows before loading the
    // window, and launch_enc_attention needs no launch_enc_append before it
    int32_t fuse_append;
    int32_t max_group_rows;  // most rows in one group of the batch (<= 8)
};

cudaError_t launch_enc_append(const EncParams & p, cudaStream_t stream);
cudaError_t launch_enc_attention(const EncParams & p, cudaStream_t stream);
int enc_smem_bytes();
// Most 128-key tiles one row group may span (window + 2*7 + capacity pad <= 768).
int enc_max_tiles();

// ---------------------------------------------------------------------------
// Greedy head: logits = W . x and argmax (vxk_head_*)
// ---------------------------------------------------------------------------

constexpr int kHeadRows = 64;          // batch rows per launch (M of the MMA)
constexpr int kHeadMaxTileRows = 256;  // vocabulary rows per tile (N of the MMA)

struct HeadParams {
    const float * x;              // [n_rows][dim] fp32
    uint16_t * xh;                // [64][dim] in W's 16-bit type
    unsigned long long * best;    // [64] packed (ordered logit, inverted index)
    int32_t * argmax;             // [n_rows]
    float * logits;               // [n_rows][vocab] fp32, or nullptr
    int32_t * error;              // device error word (0 = ok)
    int32_t vocab;
    int32_t dim;
    int32_t n_rows;               // 1 .. 64
    int32_t tile_rows;            // multiple of 32, <= 256
    int32_t n_tiles;
    int32_t dtype;                // 1 = f16, 30 = bf16
};

// tmw: 2-D tensor map {dim, vocab} over W with tile_rows x 64 boxes; tmx:
// {dim, 64} over xh with 64 x 64 boxes; both 128-byte swizzle.
cudaError_t launch_head(const HeadParams & p, const CUtensorMap & tmw, const CUtensorMap & tmx, int grid,
                        cudaStream_t stream);
int head_smem_bytes();
// Argmax of rows x vocab fp32 logits in device memory (first index of the
// largest value per row) through the per-row keys `best`.
cudaError_t launch_head_argmax(const float * logits, int32_t rows, int32_t vocab, unsigned long long * best,
                               int32_t * argmax, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Quantized-weight matrix product (vxk_qweight_*)
// ---------------------------------------------------------------------------

constexpr int kQmmRows = 64;       // weight rows per CTA (4 warps x 16-row tiles)
constexpr int kQmmUnit = 256;      // columns per record and per activation unit
constexpr int kQmmMaxBatch = 64;   // activation rows per mma.sync product (8 n-tiles of 8)
constexpr int kQmmMaxRows = 512;   // activation rows per vxk_qweight call (tcgen05: chunks of 64 in one launch)

constexpr int kQmmMaxGroup = 4;   // matrices sharing one activation quantization
constexpr int kQmmMaxSplits = 8;  // column splits of a 64-row block = CTAs of one (portable) cluster

// One weight matrix of a product group.
struct QmmMat {
    const uint8_t * w;         // records [n_rows / 16][n_units][record bytes]
    float * y;                 // [rows][n_rows] fp32
    int32_t type;              // 8 = Q8_0, 12 = Q4_K, 14 = Q6_K
    int32_t n_rows;            // a multiple of 64
    int32_t block0;            // first 64-row block of this matrix in the grid
    int32_t reserved;
};

struct QmmParams {
    QmmMat mats[kQmmMaxGroup]; // all Q8_0, or all K-quants (Q4_K / Q6_K): one x quantization
    int32_t n_mats;
    int32_t n_units;           // K / 256, shared by the group
    int32_t rows;              // activation rows, 1 .. nt * 8
    int32_t nt;                // n-tiles of 8 activation rows: 1, 2, 4 or 8
    int32_t units_per_split;   // column units per CTA
    int32_t n_splits;          // ceil(n_units / units_per_split) <= kQmmMaxSplits: one cluster
    const float * x;           // [rows][K] fp32
    const float * x_up;        // nullptr, or [rows][K]: the row is silu(x) * x_up (SwiGLU)
    uint8_t * act;             // [n_units][nt][8 blocks][32 lanes][8 B] int8 B fragments
    float * act_d;             // Q8_0: [n_units * 8][nt * 8]; K-quants: [n_units][nt * 8]
    uint8_t * act_ms;          // K-quants: [n_units][nt][32 lanes][8 B] sums of 32 quantized
                               // values as (h, l) int8 B fragments (zero-initialised)
    int32_t * error;           // device error word (0 = ok)
};

// tcgen05 form for Q4_K / Q6_K (vxk_qmm_tc.cu): records of 128 rows x 256 columns,
// [128 rows][128 quant bytes, 16-byte chunk c at c ^ (row % 8)] then
// [128 rows][6-bit scales[8], mins[8]]; (d, dmin) f16 pairs in a separate
// [blocks][units][128 rows] array read by the epilogue.
// Q6_K: [128 rows][256 bytes: the 6-bit quants q6 = q + 32, one per byte in
// column order, 16-byte chunk c at c ^ (row % 8)], then [128 rows][16 int8
// scales]; `dd` holds (d, 0).  One byte per quant (30% more than GGUF's
// 210 bytes per 256) so that forming the tensor-core operands takes no bit
// unpacking; the product is bound by that arithmetic, not by HBM.
constexpr int kQtcRecordBytes = 128 * 128 + 128 * 16;
constexpr int kQtcRecordBytesQ6K = 128 * 256 + 128 * 16;

struct QtcMat {
    const uint8_t * w;         // records [n_rows / 128][n_units][record bytes of the type]
    const uint8_t * dd;        // [n_rows / 128][n_units][128] (d, dmin) f16 pairs
    float * y;                 // [rows][n_rows] fp32
    int32_t n_rows;            // a multiple of 128
    int32_t block0;            // first 128-row block of this matrix in the grid
    int32_t type;              // 12 = Q4_K, 14 = Q6_K
    int32_t reserved;
    const float * bias;        // nullptr, or [n_rows] fp32 added to every row of y after the column sum
};

struct QtcParams {
    QtcMat mats[kQmmMaxGroup];
    int32_t n_mats;
    int32_t n_units;
    int32_t rows;              // activation rows, 1 .. npad
    int32_t npad;              // MMA N: rows padded to 16, 32 or 64
    int32_t n_chunks;          // row chunks of npad rows (more than one only with npad 64), grid z
    int32_t units_per_split;
    int32_t n_splits;          // <= kQmmMaxSplits: one cluster
    const float * x;           // [rows][K] fp32
    const float * x_up;        // nullptr, or [rows][K]: the row is silu(x) * x_up (SwiGLU)
    uint8_t * b_tiles;         // Q4_K operands: [n_units][npad x 256 f16, 4 SW128 atoms], or nullptr
    uint8_t * bmin_tiles;      // Q4_K: [n_units][npad rows x 16 f16, unswizzled K-major core matrices (32 B per row)]
    uint8_t * b8_tiles;        // Q6_K operands: [n_units][npad x 256 int8, 2 SW128 atoms], or nullptr
    float * dx;                // [n_units][npad]
    int32_t * error;
};

// Quantization of x into the f16 tiles, then the tcgen05 product; with
// prequantized, the product alone over tiles the previous launch on the stream
// wrote (launch_add_norm_quant).
cudaError_t launch_qtc(const QtcParams & p, cudaStream_t stream, bool prequantized = false);
// Clusters of cluster_y product CTAs the device runs at once (0 on error).
int qtc_max_active_clusters(int npad, int cluster_y);

// Shape of a quantized matrix (for the greedy head over quantized embeddings).
struct QweightShape {
    int32_t device, type, n_rows, n_cols, max_batch;
};
QweightShape qweight_shape(const vxk_qweight * w);
// Points the matrix's device error word at `word` (shared by an owner that
// reads one word for many matrices); nullptr restores its own.  The owner
// keeps `word` alive until the matrix is destroyed or detached.
void qweight_attach_error(vxk_qweight * w, int32_t * word);
// y = W (silu(gate) * up), the SwiGLU product computed inside the activation
// quantization (silu(g) = g / (1 + expf(-g)), each step rounded like the
// separate kernel would); 0 or a vxk_status number.
// Activation tiles of a tcgen05 group product (QtcParams b_tiles, bmin_tiles,
// dx of its first matrix) for `rows` rows, padded to npad x chunks.
struct QtcTiles {
    uint8_t * b;      // nullptr when no matrix of the group is Q4_K
    uint8_t * bmin;
    uint8_t * b8;     // nullptr when no matrix of the group is Q6_K
    float * dx;
    int32_t npad;
    int32_t rows_padded;
};
// True when the group product of ws over `rows` rows runs entirely on the
// tcgen05 kernel in one launch (every matrix a K-quant taking that kernel,
// shared device and n_cols, rows within every max_batch); then *t holds the
// tiles a producer writes before qweight_matmul_group_prequantized.
bool qweight_group_tiles(vxk_qweight * const * ws, int32_t n, int32_t rows, QtcTiles * t);
// The group product over the tiles the previous launch on `stream` wrote
// (no quantization launch); biases[i] as in qweight_matmul_group_bias.
int32_t qweight_matmul_group_prequantized(vxk_qweight * const * ws, int32_t n, int32_t rows, float * const * ys,
                                          const float * const * biases, cudaStream_t stream);
int32_t qweight_matmul_swiglu(vxk_qweight * w, const float * gate, const float * up, int32_t rows, float * y,
                              cudaStream_t stream);
// vxk_qweight_matmul_group, then y_i += bias_i on every row (ggml_mul_mat
// then ggml_add: one rounded fp32 add); biases or any bias_i may be nullptr.
// Matrices on the tcgen05 kernel add the bias in the product's store.
int32_t qweight_matmul_group_bias(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows,
                                  float * const * ys, const float * const * biases, cudaStream_t stream);
// silu(g) * u with separately rounded steps (ggml_silu then ggml_mul,
// src/voxtral.cpp:2877-2880), evaluated inside the activation quantization.
#ifdef __CUDACC__
__device__ __forceinline__ float swiglu_value(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
#endif

// Record bytes of one 16 x 256 tile (4352 / 2368 / 3360), 0 for other types.
int qmm_record_bytes(int type);
// Dynamic shared memory of the product kernel for the group's types, p.nt
// and `units` column units per split.
int qmm_smem_bytes(const QmmParams & p, int units);
// Resident product CTAs per SM for the family / p.nt at `smem` bytes.
int qmm_ctas_per_sm(const QmmParams & p, int smem);
// Activation quantization, then the product (both with programmatic
// dependent launch on `stream`; the product's splits as one cluster).
cudaError_t launch_qmm(const QmmParams & p, cudaStream_t stream);

// ---- whole decoder step (vxk_decoder.cu, vxk_decoder_host.cpp) ------------

// The pool's planned batch as the decoder needs it.
struct PoolBatchView {
    std::vector<int32_t> row_stream;  // per query row
    std::vector<int32_t> row_pos;
    std::vector<int32_t> last_rows;   // per planned stream: its last row
    bool single_token = false;
};
bool pool_batch_view(const vxk_pool * pool, PoolBatchView * out);

struct PoolShape {
    int32_t device, n_layers, n_q, n_kv, head_dim, max_streams, max_rows;
    float rope_theta;
};
PoolShape pool_shape(const vxk_pool * pool);
// True when pool_decode_layer_quant applies (an f16 cache, 4 query heads of
// 128 dims per kv head).
bool pool_decode_quant_ok(const vxk_pool * pool);
// vxk_decode_layer whose output rows are also quantized into `t` (the tiles
// of the o product, a one-matrix group over the same rows); out may be
// nullptr.  The product then runs as qweight_matmul_group_prequantized.
int32_t pool_decode_layer_quant(vxk_pool * pool, int32_t layer, const float * q, const float * k, const float * v,
                                float * out, const QtcTiles & t, cudaStream_t stream);

// One query row of a decoder forward.
struct DecRow {
    int32_t stream;
    int32_t token;
    int32_t audio_slot;
    int32_t out_index;  // this row's stream index in the plan when it is the stream's last row, else -1
};
static_assert(sizeof(DecRow) == 16, "DecRow layout");

// x = embedding row + audio row, xn = rms_norm(x) * w.
struct EmbedParams {
    const uint8_t * emb;      // tok_embeddings rows in their GGUF type
    int64_t emb_row_bytes;
    int32_t emb_type;         // ggml type: 0 F32, 1 F16, 8 Q8_0, 12 Q4_K, 14 Q6_K, 30 BF16
    int32_t audio_cap;
    const float * audio;      // [max_streams][audio_cap][dim]
    const DecRow * rows;
    int32_t n_rows;
    int32_t dim;
    const float * norm_w;
    float eps;
    float * x;                // [rows][dim] residual stream
    float * xn;               // [rows][dim]
};

// x += add (when add != nullptr; add + add_bias first when that is set);
// out = rms_norm(x) * w, then out + out * ada
// when ada != nullptr.  compact: only rows with out_index >= 0, written to
// out row out_index.
struct NormParams {
    float * x;
    const float * add;
    const float * add_bias;   // nullptr, or [dim]: x += (add + add_bias) (a product with its bias)
    const float * w;
    const float * ada;
    float * out;
    const DecRow * rows;
    int32_t compact;
    int32_t n_rows;
    int32_t dim;
    float eps;
    // launch_add_norm_quant only: the output rows quantized into a tcgen05
    // product's activation tiles (QtcTiles), out optional
    uint8_t * q_tiles;
    uint8_t * q_bmin;
    uint8_t * q_tiles8;
    float * q_dx;
    int32_t q_npad;
    int32_t q_rows_padded;     // q_npad x the product's row chunks
};

// One adapter group: 4 encoder frames of a stream into one audio slot.
struct AdaptRow {
    int32_t stream;
    int32_t enc_slot;     // slot of the group's first frame (a multiple of 4)
    int32_t audio_slot;
    int32_t reserved;
};
static_assert(sizeof(AdaptRow) == 16, "AdaptRow layout");

cudaError_t launch_embed_norm(const EmbedParams & p, cudaStream_t stream);
cudaError_t launch_add_norm(const NormParams & p, cudaStream_t stream);
// add_norm_kernel's rows quantized into p.q_tiles / q_bmin / q_dx (dim a
// multiple of 256, at most 8192; no compact rows).
cudaError_t launch_add_norm_quant(const NormParams & p, cudaStream_t stream);
// x = gelu_erf(x) over n values.
cudaError_t launch_gelu_erf(float * x, int64_t n, cudaStream_t stream);
// out[g] = the 4 frames of group g, concatenated ([n][4 * enc_dim]).
cudaError_t launch_adapter_gather(const float * enc, int32_t enc_cap, int32_t enc_dim, const AdaptRow * rows,
                                  int32_t n, float * out, cudaStream_t stream);
// audio[stream][audio_slot] = y[g] for each group.
cudaError_t launch_audio_scatter(const float * y, float * audio, int32_t audio_cap, int32_t dim,
                                 const AdaptRow * rows, int32_t n, cudaStream_t stream);

// ---- encoder stack (vxk_encoder_stack.cu, vxk_encoder_model_host.cpp) -------

struct EncBatchView {
    std::vector<int32_t> streams;   // per planned stream, plan order
    std::vector<int32_t> n_new;
    std::vector<int64_t> q_start;
    int32_t rows = 0;
};
struct EncShape {
    int32_t device, n_layers, n_heads, head_dim, max_streams, max_new;
    float rope_theta;
};
bool enc_pool_batch_view(const vxk_enc_pool * pool, EncBatchView * out);
EncShape enc_pool_shape(const vxk_enc_pool * pool);
int32_t * enc_pool_error_word(const vxk_enc_pool * pool);

// One planned stream's conv work: its mel window and output rows.
struct ConvStream {
    int32_t mel_offset;   // first float of its [n_mel][win] window in the mel buffer
    int32_t win;          // 2 n_new + 4 frames
    int32_t n_new;
    int32_t row0;         // its first output row
};
static_assert(sizeof(ConvStream) == 16, "ConvStream layout");

struct ConvParams {
    const float * mel;          // concatenated [n_mel][win] windows, channel-major
    const ConvStream * streams;
    int32_t n_streams;
    int32_t n_mel;
    int32_t dim;
    int32_t max_win;
    const __half * w0;          // conv0 weights [n_mel][3][dim] (f16, c fastest)
    const float * b0;           // [dim]
    const __half * w1;          // conv1 weights [dim][3][dim]
    const float * b1;
    float * y0;                 // [n_streams][max_win][dim] gelu(conv0), fp32
    float * x;                  // [rows][dim] encoder rows (gelu(conv1) at local 2 .. 2 + n_new - 1)
    int32_t steady;             // every stream has n_new = 4, in plan order (rows 4 s .. 4 s + 3)
};

cudaError_t launch_conv_stem(const ConvParams & p, cudaStream_t stream);
// y[r][i] += b[i] for rows of n values (ggml_add of a bias), two tensors at once.
cudaError_t launch_bias2(float * y0, const float * b0, int32_t n0, float * y1, const float * b1, int32_t n1,
                         int32_t rows, cudaStream_t stream);

}  // namespace vxk
