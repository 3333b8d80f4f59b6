/*
 * vx_oracle.h -- CPU restatement of voxtral.cpp's decoder KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code.  It is used by tests/ (as the checker), by
 * __graft_entry__.smoke() (as the checker) and by bench.py's cpu_baseline and
 * `--impl reference` legs (as the timed CPU restatement).
 *
 * Parity status (see the header of vx_oracle.c for the per-function notes):
 *   - decoder and encoder ring planners: PINNED by the expectations of the
 *     reference's own model-free tests (tests/cpp/test_decoder_kv.cpp:47-115,
 *     tests/cpp/test_encoder_kv.cpp:145-340), re-expressed in tests/.
 *   - f16 / bf16 round-to-nearest-even: pinned against numpy's float16 and a
 *     bit-level bf16 reference (tests/golden/).
 *   - q8_0 quantisation: pinned against gguf 0.19.0 quants.Q8_0, a third-party
 *     restatement of ggml's quantize_row_q8_0_ref (tests/golden/).
 *   - RoPE rounding and attention rounding: PARITY UNPINNED.  The arithmetic
 *     lives in ggml @5cecdad692d868e28dbd2f7c468504770108f30c, which the
 *     reference fetches at configure time (CMakeLists.txt:77-93) and which is
 *     absent here.  The oracle restates ggml's published CPU algorithm for
 *     rope mode 0 (cached theta by repeated fp32 multiplication, libm
 *     cosf/sinf, separately rounded x0*c - x1*s) and computes attention in
 *     fp64 as the exact-math target.
 */
#ifndef VX_ORACLE_H
#define VX_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type numbers for the cache formats (ggml.h enum ggml_type). */
#define VXO_F32  0
#define VXO_F16  1
#define VXO_Q8_0 8
#define VXO_BF16 30

/* ---- decoder ring (src/voxtral-internal.h:195-227) ---------------------- */
typedef struct vxo_dec_ring {
    int64_t capacity;
    int64_t used;
    int64_t oldest;   /* oldest_absolute_position */
    int64_t next;     /* next_absolute_position */
    int64_t wraps;
    int64_t evictions;
    int64_t bytes_moved;
    int64_t full_buffer_moves;
} vxo_dec_ring;

typedef struct vxo_seg { int32_t slot; int32_t len; } vxo_seg;

typedef struct vxo_dec_plan {
    int64_t absolute_start;
    int32_t n_new;
    int32_t write_nseg;
    vxo_seg write_seg[2];
    vxo_seg read_seg[2];
    int32_t read_nseg;
    int32_t wrapped;
    int64_t used_after;
    int64_t oldest_after;
    int64_t next_after;
    int64_t evicted;
} vxo_dec_plan;

int  vxo_dec_kv_plan(const vxo_dec_ring * ring, int64_t absolute_start,
                     int32_t n_new, vxo_dec_plan * out);
void vxo_dec_kv_commit(vxo_dec_ring * ring, const vxo_dec_plan * plan);

/* ---- encoder ring (src/voxtral-internal.h:404-435) ---------------------- */
typedef struct vxo_enc_plan {
    int64_t q_start;
    int32_t n_new;
    int32_t win_len;
    int64_t win_start;
    int64_t win_end;
    vxo_seg read_seg[2];
    int32_t read_nseg;
    int32_t read_wraps;
    vxo_seg write_seg[2];
    int32_t write_nseg;
    int32_t write_wraps;
    int64_t conv_mel_start;
    int64_t conv_mel_end;
    int32_t conv_slice_start;
    int32_t pad_;
    int64_t evicted;
} vxo_enc_plan;

int vxo_enc_kv_plan(int64_t q_start, int32_t n_new, int32_t capacity,
                    int32_t window, vxo_enc_plan * out);
int vxo_enc_kv_mask_allows(int64_t kv_abs, int64_t q_abs, int32_t window);

/* ---- element formats ---------------------------------------------------- */
uint16_t vxo_f32_to_f16(float x);
float    vxo_f16_to_f32(uint16_t h);
uint16_t vxo_f32_to_bf16(float x);
float    vxo_bf16_to_f32(uint16_t h);
void     vxo_f32_to_f16_n(const float * x, uint16_t * y, int64_t n);
void     vxo_f32_to_bf16_n(const float * x, uint16_t * y, int64_t n);

/* q8_0: blocks of 32 values, 34 bytes each {f16 d; int8 qs[32]}. */
void vxo_quantize_row_q8_0(const float * x, int64_t k, uint8_t * blocks);
void vxo_dequantize_row_q8_0(const uint8_t * blocks, int64_t k, float * y);

/* ---- RoPE mode 0 --------------------------------------------------------- */
/* cs receives n_dims floats: cos/sin interleaved per rotated pair. */
void vxo_rope_cache(int64_t pos, int32_t n_dims, float base, float * cs);
/* Rotate n_heads rows of head_dim values (adjacent pairs) at one position. */
void vxo_rope_apply(const float * x, int32_t n_heads, int32_t head_dim,
                    int64_t pos, float base, float * out);

/* Bytes of one cache row (n_kv heads x head_dim values) in a format. */
int64_t vxo_row_bytes(int32_t dtype, int32_t n_kv, int32_t head_dim);

/* One appended token: K is rotated at pos and stored, V is stored as-is. */
void vxo_kv_row(const float * k, const float * v, int32_t n_kv, int32_t head_dim,
                int64_t pos, float base, int32_t dtype,
                uint8_t * k_out, uint8_t * v_out);

/* n_rows appended tokens at consecutive positions pos0, pos0 + 1, ...:
 * vxo_kv_row on each; k/v [n_rows][n_kv][head_dim], outputs [n_rows][row bytes]. */
void vxo_kv_rows(const float * k, const float * v, int64_t n_rows, int32_t n_kv, int32_t head_dim,
                 int64_t pos0, float base, int32_t dtype, uint8_t * k_out, uint8_t * v_out);

/* Decode a stored row back to fp32 values (n_kv * head_dim). */
void vxo_row_to_f32(const uint8_t * row, int32_t dtype, int32_t n_kv,
                    int32_t head_dim, float * out);

/* Attention of one query row over n_keys stored rows (logical order), fp64
 * accumulation.  q: [n_q][head_dim] fp32 BEFORE RoPE when rope_q != 0.
 * GQA: query head h reads kv head h / (n_q / n_kv).  out: [n_q][head_dim]. */
void vxo_attn_row(const float * q, int64_t q_pos, float base, int32_t rope_q,
                  int32_t n_q, int32_t n_kv, int32_t head_dim,
                  const uint8_t * k_rows, const uint8_t * v_rows, int32_t dtype,
                  int64_t n_keys, float scale, float * out);

/* ---- timed CPU restatement of one decode step (bench baseline) ----------
 * Caches: per (stream, layer) a contiguous ring of `cap` rows, f16 bytes,
 * layout [stream][layer][kv_head][cap][head_dim].  For every stream and layer:
 * rotate and append K/V at pos[s] (slot pos % cap), then attend q over the
 * logical window [win_start[s], pos[s]] with fp32 online softmax.
 * q: [stream][layer][n_q][hd], k/v: [stream][layer][n_kv][hd], out like q.
 * Work is split over (stream, kv_head) with n_threads POSIX threads. */
void vxo_cpu_decode_step_f16(int32_t n_streams, int32_t n_layers, int32_t n_q,
                             int32_t n_kv, int32_t head_dim, int64_t cap,
                             uint16_t * k_cache, uint16_t * v_cache,
                             const float * q, const float * k, const float * v,
                             const int64_t * pos, const int64_t * win_start,
                             const float * rope_cs, int64_t rope_rows,
                             float scale, int32_t n_threads, float * out);

/* Same step for a cache of dtype VXO_F16 or VXO_Q8_0: rows of
 * vxo_row_bytes(dtype, 1, head_dim) bytes per kv head (q8_0: ggml blocks,
 * quantized on append, dequantized on read), layout
 * [stream][layer][kv_head][cap][row bytes]. */
void vxo_cpu_decode_step(int32_t dtype, int32_t n_streams, int32_t n_layers, int32_t n_q,
                         int32_t n_kv, int32_t head_dim, int64_t cap, uint8_t * k_cache,
                         uint8_t * v_cache, const float * q, const float * k, const float * v,
                         const int64_t * pos, const int64_t * win_start, const float * rope_cs,
                         int64_t rope_rows, float scale, int32_t n_threads, float * out);

/* Fill a rope cos/sin table [rows][head_dim] with vxo_rope_cache. */
void vxo_rope_table(int64_t rows, int32_t n_dims, float base, float * table);

/* Quantized-weight matrix product, ggml CPU semantics (vx_qmm.c).  Weight
 * types: 8 = Q8_0, 12 = Q4_K, 14 = Q6_K (GGUF block layouts). */
int64_t vxo_qrow_bytes(int32_t type, int64_t k);
void vxo_quantize_row_q8_K(const float * x, int64_t k, float * d, int8_t * q, int16_t * bsums);
void vxo_dequantize_row_w(int32_t type, const uint8_t * w, int64_t k, float * y);
int32_t vxo_qmatmul(int32_t type, const uint8_t * w, int32_t n, int32_t k, const float * x, int32_t rows,
                    double * y, double * mag);

#ifdef __cplusplus
}
#endif

#endif /* VX_ORACLE_H */
