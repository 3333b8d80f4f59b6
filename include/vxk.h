#ifndef VXK_H
#define VXK_H

/**
 * @file vxk.h
 * C ABI of the B200 (sm_100a) decoder KV-cache kernel layer for voxtral.cpp.
 *
 * This library replaces the ggml nodes that voxtral.cpp's decoder and
 * streaming encoder emit for their KV caches:
 *   - RoPE mode 0 on K and Q      (src/voxtral.cpp:2668-2671, 2463-2466)
 *   - K/V append into the cache   (src/voxtral.cpp:2677-2714 set_rows / cpy)
 *   - GQA attention over the cache (src/voxtral.cpp:2716-2854 flash_attn_ext)
 *   - encoder windowed attention  (src/voxtral.cpp:2459-2487)
 * and the host ring bookkeeping that drives them
 *   (src/voxtral.cpp:1590-1656, 3636-3692; src/voxtral-internal.h:193-227,
 *    381-435).
 *
 * Every function returns a vxk_status (numerically equal to the matching
 * voxtral_status of include/voxtral.h:97-110 where one exists), never throws,
 * and never frees caller memory.  Device pointers are plain CUDA device
 * addresses; `cuda_stream` is a cudaStream_t passed as void*.  Kernel
 * launches are asynchronous on that stream.  All calls on one pool must be
 * serialised by the caller, like calls on one voxtral_context
 * (include/voxtral.h:223).
 */

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#  define VXK_API __attribute__((visibility("default")))
#else
#  define VXK_API
#endif

#define VXK_API_VERSION 1u

#ifdef __cplusplus
extern "C" {
#endif

/** Status codes; 0..11 mirror voxtral_status (include/voxtral.h:97-110). */
typedef enum vxk_status {
    VXK_STATUS_OK = 0,
    VXK_STATUS_INVALID_ARGUMENT = 1,
    VXK_STATUS_INVALID_STATE = 2,
    VXK_STATUS_OUT_OF_MEMORY = 3,
    VXK_STATUS_NOT_READY = 5,
    VXK_STATUS_BACKEND_ERROR = 9,
    VXK_STATUS_INTERNAL_ERROR = 10,
    VXK_STATUS_BUFFER_TOO_SMALL = 11,
    VXK_STATUS_TIMEOUT = 12
} vxk_status;

/** Cache element formats; values are ggml_type numbers. */
typedef enum vxk_dtype {
    VXK_DTYPE_F32 = 0,
    VXK_DTYPE_F16 = 1,
    VXK_DTYPE_Q8_0 = 8,
    VXK_DTYPE_BF16 = 30
} vxk_dtype;

/** Returns a static name for a status ("ok", "invalid_argument", ...). */
VXK_API const char * vxk_status_string(vxk_status status);

/** Returns VXK_API_VERSION. */
VXK_API uint32_t vxk_api_version(void);

/* ======================================================================== */
/* Ring planners (host only, no device)                                     */
/* ======================================================================== */

/** Decoder ring state; replaces voxtral_decoder_kv_ring
 *  (src/voxtral-internal.h:195-204).  Positions are absolute; storage
 *  addressing is modulo `capacity`. */
typedef struct vxk_decoder_kv_ring {
    int64_t capacity;
    int64_t used;
    int64_t oldest_absolute_position;
    int64_t next_absolute_position;
    int64_t wraps;
    int64_t evictions;
    int64_t bytes_moved;
    int64_t full_buffer_moves;
} vxk_decoder_kv_ring;

/** One physical ring segment (src/voxtral-internal.h:206-209). */
typedef struct vxk_kv_seg {
    int32_t slot;
    int32_t len;
} vxk_kv_seg;

/** Decoder append plan; replaces voxtral_decoder_kv_plan_t
 *  (src/voxtral-internal.h:211-223). */
typedef struct vxk_decoder_kv_plan {
    int64_t absolute_start;
    int32_t n_new;
    int32_t write_nseg;
    vxk_kv_seg write_seg[2];
    vxk_kv_seg read_seg[2];   /* oldest -> newest logical order */
    int32_t read_nseg;
    int32_t wrapped;
    int64_t used_after;
    int64_t oldest_after;
    int64_t next_after;
    int64_t evicted;
} vxk_decoder_kv_plan;

/** Plans appending n_new tokens at absolute_start; replaces
 *  voxtral_decoder_kv_plan (src/voxtral.cpp:1618-1645).  Returns
 *  VXK_STATUS_INVALID_ARGUMENT for exactly the cases the reference rejects. */
VXK_API vxk_status vxk_decoder_kv_plan_make(const vxk_decoder_kv_ring * ring,
                                            int64_t absolute_start, int32_t n_new,
                                            vxk_decoder_kv_plan * out);

/** Commits a plan; replaces decoder_kv_commit_plan (src/voxtral.cpp:1647-1656). */
VXK_API vxk_status vxk_decoder_kv_plan_commit(vxk_decoder_kv_ring * ring,
                                              const vxk_decoder_kv_plan * plan);

/** Encoder ring plan; replaces voxtral_enc_kv_plan_t
 *  (src/voxtral-internal.h:404-428). */
typedef struct vxk_enc_kv_plan {
    int64_t q_start;
    int32_t n_new;
    int32_t win_len;
    int64_t win_start;
    int64_t win_end;
    vxk_kv_seg read_seg[2];
    int32_t read_nseg;
    int32_t read_wraps;
    vxk_kv_seg write_seg[2];
    int32_t write_nseg;
    int32_t write_wraps;
    int64_t conv_mel_start;
    int64_t conv_mel_end;
    int32_t conv_slice_start;
    int32_t reserved;
    int64_t evicted;
} vxk_enc_kv_plan;

/** Replaces voxtral_enc_kv_plan (src/voxtral.cpp:3656-3692). */
VXK_API vxk_status vxk_enc_kv_plan_make(int64_t q_start, int32_t n_new, int32_t capacity,
                                        int32_t window, vxk_enc_kv_plan * out);

/** Replaces voxtral_enc_kv_mask_allows (src/voxtral.cpp:3636-3638);
 *  returns 1 when a query at q_abs may attend a key at kv_abs. */
VXK_API int32_t vxk_enc_kv_mask_allows(int64_t kv_abs, int64_t q_abs, int32_t window);

/* ======================================================================== */
/* Decoder paged KV pool                                                    */
/* ======================================================================== */

/** Opaque per-device pool of KV pages shared by many streams. */
typedef struct vxk_pool vxk_pool;

/**
 * Pool configuration.  One page ("block") holds block_tokens consecutive
 * positions of one stream for every layer and kv head.  A stream's logical
 * position p lives in page block_table[stream][(p / block_tokens) %
 * (capacity / block_tokens)] at row p % block_tokens, so a stream is a ring of
 * `capacity` slots exactly like the reference's fixed decoder ring
 * (src/voxtral.cpp:413-427), with page indirection.
 */
typedef struct vxk_pool_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t device;
    int32_t n_layers;       /* 30 (3B offline) or 26 (4B realtime) */
    int32_t n_q_heads;      /* 32 */
    int32_t n_kv_heads;     /* 8 */
    int32_t head_dim;       /* 128 */
    int32_t block_tokens;   /* 16 */
    int32_t n_blocks;       /* physical pages in the pool */
    int32_t capacity;       /* per-stream ring capacity in tokens */
    int32_t max_streams;
    int32_t max_rows;       /* max query rows in one planned batch */
    int32_t max_position;   /* RoPE table rows: every position must be below */
    vxk_dtype dtype;        /* F16 (default), Q8_0, or F32 (the reference's exact
                               VOXTRAL_DECODER_KV_TYPE=f32 mode, src/voxtral.cpp:94-98) */
    float rope_theta;       /* 1e6 */
    uint32_t alloc_seed;    /* 0: pages handed out lowest index first; else a
                               seeded permutation (random block tables) */
    /* ---- fields after this line were added later; a caller whose
       struct_size ends before one gets that field's default ---- */
    int32_t split_pages;    /* 0 (default): the attention's split size is
                               chosen per batch from its pages and the
                               device's resident CTAs; n > 0: splits of n
                               pages (rounded up to a power of two, at most
                               512), still enlarged when a batch would need
                               more splits than the pool's scratch holds */
} vxk_pool_config;

/** Defaults: the 4B realtime decoder (26 layers, 32/8 heads x 128, 16-token
 *  pages, 8192-slot ring, f16, theta 1e6); n_blocks/max_streams sized for one
 *  stream. */
VXK_API vxk_pool_config vxk_pool_default_config(void);

/** Allocates the pool on `device` (pages zeroed once, like the reference's
 *  one-time cache clear at src/voxtral.cpp:1443-1465). */
VXK_API vxk_status vxk_pool_create(const vxk_pool_config * config, vxk_pool ** out_pool);
/** Frees the pool.  NULL is safe.  No work may be in flight on it. */
VXK_API void vxk_pool_destroy(vxk_pool * pool);
/** Copies the last error message of the pool (or of the last failed create
 *  when pool is NULL) into buf. */
VXK_API vxk_status vxk_pool_last_error(const vxk_pool * pool, char * buf, size_t capacity);

/** Pool occupancy counters. */
typedef struct vxk_pool_stats {
    int64_t pages_total;
    int64_t pages_used;
    int64_t pages_high_water;   /* 1 + highest physical page index in use */
    int64_t streams_open;
    int64_t compactions;
    int64_t pages_moved;
    int64_t bytes_moved;        /* device bytes copied by compaction */
    int64_t device_bytes;       /* bytes allocated on the device */
    int64_t kernel_launches;    /* kernels this pool has launched */
} vxk_pool_stats;

VXK_API vxk_status vxk_pool_get_stats(const vxk_pool * pool, vxk_pool_stats * out);

/** Opens a stream (an empty ring).  Replaces voxtral_ctx_decoder_begin_incremental
 *  (src/voxtral.cpp:5489-5496) for one stream. */
VXK_API vxk_status vxk_stream_open(vxk_pool * pool, int32_t * out_stream);
/** Closes a stream and returns its pages to the pool. */
VXK_API vxk_status vxk_stream_close(vxk_pool * pool, int32_t stream);
/** Logical reset (clear_kv_cache, src/voxtral.cpp:1590-1602): ring back to
 *  empty, pages returned, no device bytes touched. */
VXK_API vxk_status vxk_stream_reset(vxk_pool * pool, int32_t stream);
/** Copies the stream's ring counters (wraps, evictions, bytes_moved ...). */
VXK_API vxk_status vxk_stream_get_ring(const vxk_pool * pool, int32_t stream,
                                       vxk_decoder_kv_ring * out);
/** Window eviction: drops positions below new_oldest (which must lie in
 *  [oldest, next]); pages whose every slot is dropped go back to the pool.
 *  Counts the dropped positions as evictions. */
VXK_API vxk_status vxk_stream_evict(vxk_pool * pool, int32_t stream, int64_t new_oldest);

/**
 * Plans one batch: stream_ids[i] appends n_new[i] tokens at its next absolute
 * position (voxtral_decoder_kv_plan per stream, src/voxtral.cpp:5226-5231 and
 * 5170-5177), allocating pages as needed.  The batch's query rows are the new
 * tokens in order (stream by stream, position by position); row r of every
 * per-layer buffer belongs to that token.  Row descriptors and block-table
 * updates are copied to the device on cuda_stream.  A multi-token append
 * must not evict (the reference only prefills an empty ring).
 */
VXK_API vxk_status vxk_batch_plan(vxk_pool * pool, const int32_t * stream_ids,
                                  const int32_t * n_new, int32_t n_streams,
                                  void * cuda_stream);
/** Number of query rows of the planned batch. */
VXK_API vxk_status vxk_batch_rows(const vxk_pool * pool, int32_t * out_rows);
/** Commits every plan of the batch (decoder_kv_commit_plan). */
VXK_API vxk_status vxk_batch_commit(vxk_pool * pool);
/** Drops the planned batch without committing. */
VXK_API vxk_status vxk_batch_abort(vxk_pool * pool);

/**
 * One decoder layer of a single-token batch (every stream n_new == 1), fused:
 * rotate and append K/V at the new position, then GQA flash-decoding
 * attention over the window [oldest_after, position] including the new
 * token.  Replaces the RoPE + set_rows + flash_attn_ext nodes of
 * build_decoder_layer (src/voxtral.cpp:2663-2821) on the step graph.
 *   q   [rows][n_q_heads][head_dim]  fp32, before RoPE
 *   k,v [rows][n_kv_heads][head_dim] fp32, K before RoPE
 *   out [rows][n_q_heads][head_dim]  fp32
 */
VXK_API vxk_status vxk_decode_layer(vxk_pool * pool, int32_t layer, const float * q,
                                    const float * k, const float * v, float * out,
                                    void * cuda_stream);

/**
 * vxk_decode_layer with no device allocation behind it.  It has no
 * counterpart in the reference; it exists for callers that cannot call
 * cudaMalloc on their decode path: real-time audio threads, where cudaMalloc
 * may synchronise the whole device and has no latency bound, and host
 * applications whose device memory is already fully reserved by another
 * allocator.  The split scratch of the attention (per-split partial results
 * and arrival counters) lives in a fixed array inside libvxk.so (8.66 MB per
 * GPU that loads the library, held until the process exits) instead of
 * memory the library allocates; this call allocates nothing and calls no
 * allocating routine.
 *
 * Limits: a batch may need at most 512 x 32 x 132 partial floats (for 32
 * query heads: 512 splits) and 256 x 8 counters (256 rows of 8 kv heads);
 * larger batches return VXK_STATUS_INVALID_ARGUMENT with the sizes in the
 * pool's error message.  The batch must also pass the pool's own planning
 * limit, which vxk_decode_layer has too: its splits must fit the pool's
 * split bookkeeping (max(2048, 8 * max_rows) work items); otherwise the call
 * returns VXK_STATUS_INVALID_ARGUMENT ("batch windows exceed the split
 * scratch capacity").  The first call on a device looks up the array's
 * device address (with that device current) and remembers it for the life
 * of the process, so make that first call before any stream capture, and do
 * not reset the device (cudaDeviceReset) while libvxk.so is loaded: the
 * remembered address would no longer be valid.  Every call shares the one array and clears its
 * counters before launching; calls that overlap on the GPU (other streams,
 * other pools on the same device) race on it.  Arguments, results and the
 * launch are otherwise those of vxk_decode_layer.
 */
VXK_API vxk_status vxk_decode_layer_static_scratch(vxk_pool * pool, int32_t layer, const float * q,
                                                   const float * k, const float * v, float * out,
                                                   void * cuda_stream);

/** Appends the batch's new tokens to one layer (RoPE on K, f16/q8_0/f32 store);
 *  replaces src/voxtral.cpp:2663-2714 for prefill / multi-token batches. */
VXK_API vxk_status vxk_append_layer(vxk_pool * pool, int32_t layer, const float * k,
                                    const float * v, void * cuda_stream);

/** Causal attention of the batch's query rows over one layer's cache (row at
 *  position p attends [max(oldest, p - capacity + 1), p]); the prefill form of
 *  src/voxtral.cpp:2741-2760 with the mask of src/voxtral.cpp:3316-3323. */
VXK_API vxk_status vxk_attend_layer(vxk_pool * pool, int32_t layer, const float * q,
                                    float * out, void * cuda_stream);

/**
 * End-to-end single-token step from HOST buffers: plans stream_ids (n_new 1
 * each), copies every layer's q/k/v from host memory, runs all layers with
 * vxk_decode_layer, copies the outputs back, waits and commits.  Host buffers
 * are layer-major: h_q[layer][row][n_q_heads][head_dim], h_k/h_v
 * [layer][row][n_kv_heads][head_dim], h_out like h_q.  Pinned host memory
 * lets the copies overlap the layers.
 */
VXK_API vxk_status vxk_decode_step_host(vxk_pool * pool, const int32_t * stream_ids,
                                        int32_t n_streams, const float * h_q,
                                        const float * h_k, const float * h_v,
                                        float * h_out, void * cuda_stream);

/** Waits for cuda_stream with a bounded wait (timeout_ms) and reports any
 *  device-side error flag of the pool's kernels (VXK_STATUS_TIMEOUT or
 *  VXK_STATUS_BACKEND_ERROR). */
VXK_API vxk_status vxk_sync(vxk_pool * pool, void * cuda_stream, int32_t timeout_ms);

/**
 * Exercises the failure path of the pool's kernels without a fault: launches
 * one warp that waits, with the same bounded wait the decode kernel uses on
 * its copies, on a barrier that nothing completes; after limit_ms (1..1000)
 * it gives up and records a timeout in the pool's device error word, as a
 * decode launch whose page copies never landed would.  The next vxk_sync on
 * cuda_stream then returns VXK_STATUS_TIMEOUT and clears the word; the pool
 * stays usable.  No counterpart in the reference: it lets a host test that
 * its error handling sees device-side timeouts.
 */
VXK_API vxk_status vxk_pool_probe_wait_timeout(vxk_pool * pool, int32_t limit_ms, void * cuda_stream);

/** Page compaction: moves every live page above the lowest free pages down,
 *  rewriting block tables, so that used pages form a prefix of the pool.
 *  Counts the device bytes copied into the pool's and each moved stream's
 *  bytes_moved (include/voxtral-stream.h:129-131 metric). */
VXK_API vxk_status vxk_pool_compact(vxk_pool * pool, void * cuda_stream,
                                    int64_t * out_pages_moved, int64_t * out_bytes_moved);

/** Reads `n` logical positions [pos_start, pos_start+n) of one stream and
 *  layer back to host in ggml row layout: f16 rows of n_kv_heads*head_dim
 *  halves, or q8_0 rows of n_kv_heads*head_dim/32 blocks of 34 bytes
 *  {f16 d; int8 qs[32]}.  Positions must lie in the stream's window.
 *  Synchronises cuda_stream. */
VXK_API vxk_status vxk_read_rows(vxk_pool * pool, int32_t layer, int32_t stream,
                                 int64_t pos_start, int32_t n, void * k_out, void * v_out,
                                 void * cuda_stream);

/** Bytes of one ggml-layout row for the pool's dtype. */
VXK_API int64_t vxk_pool_row_bytes(const vxk_pool * pool);

/* ======================================================================== */
/* Streaming-encoder windowed attention                                     */
/* ======================================================================== */

/** Opaque encoder KV rings for many streams on one device. */
typedef struct vxk_enc_pool vxk_enc_pool;

typedef struct vxk_enc_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t device;
    int32_t n_layers;      /* 32 */
    int32_t n_heads;       /* 32 in the released model, 20 in the bench */
    int32_t head_dim;      /* 64 */
    int32_t window;        /* 750 (VOXTRAL_ENC_WINDOW) */
    int32_t capacity;      /* 878 (window + max_new) */
    int32_t max_streams;
    int32_t max_new;       /* rows per stream per batch, <= capacity - window */
    int32_t max_position;  /* RoPE table rows */
    vxk_dtype dtype;       /* BF16 (default here), F16, or F32 (the reference's default
                              encoder cache, src/voxtral.cpp:100-105: exact fp32
                              rows, attention on the CUDA cores) */
    float rope_theta;      /* 1e6 */
    int32_t reserved;
} vxk_enc_config;

VXK_API vxk_enc_config vxk_enc_default_config(void);
VXK_API vxk_status vxk_enc_create(const vxk_enc_config * config, vxk_enc_pool ** out);
VXK_API void vxk_enc_destroy(vxk_enc_pool * pool);
VXK_API vxk_status vxk_enc_last_error(const vxk_enc_pool * pool, char * buf, size_t capacity);
VXK_API vxk_status vxk_enc_stream_open(vxk_enc_pool * pool, int32_t * out_stream);
VXK_API vxk_status vxk_enc_stream_close(vxk_enc_pool * pool, int32_t stream);
VXK_API vxk_status vxk_enc_stream_reset(vxk_enc_pool * pool, int32_t stream);
/** Next absolute encoder frame of a stream and its eviction count. */
VXK_API vxk_status vxk_enc_stream_position(const vxk_enc_pool * pool, int32_t stream,
                                           int64_t * out_next, int64_t * out_evicted);

/** Plans n_new frames per stream (voxtral_enc_kv_plan per stream,
 *  src/voxtral.cpp:4072-4120); rows are stream-major like the decoder. */
VXK_API vxk_status vxk_enc_batch_plan(vxk_enc_pool * pool, const int32_t * stream_ids,
                                      const int32_t * n_new, int32_t n_streams,
                                      void * cuda_stream);
VXK_API vxk_status vxk_enc_batch_rows(const vxk_enc_pool * pool, int32_t * out_rows);
VXK_API vxk_status vxk_enc_batch_commit(vxk_enc_pool * pool);

/**
 * One encoder layer: rotate and store the batch's new K (V unrotated) at
 * slots abs % capacity, then masked attention of every new row over its
 * window [max(0, q - window + 1), q] (src/voxtral.cpp:2459-2487 with the
 * mask of src/voxtral.cpp:4104-4119), scale 1/sqrt(head_dim), MHA.
 *   q, out [rows][n_heads][head_dim] fp32; k, v [rows][n_heads][head_dim].
 * When every stream of the batch has at most 8 new rows (the steady chunk) and
 * the ring is 16-bit, this is one kernel launch (the store is fused into the
 * attention); otherwise two (store, then attention).  Either way q/k/v must be
 * complete on cuda_stream before the call's work starts.
 */
VXK_API vxk_status vxk_enc_layer(vxk_enc_pool * pool, int32_t layer, const float * q,
                                 const float * k, const float * v, float * out,
                                 void * cuda_stream);

/** Reads n slots' K/V rows [slot0, slot0+n) of one stream/layer (raw 16-bit
 *  elements, n_heads*head_dim per row).  Synchronises cuda_stream. */
VXK_API vxk_status vxk_enc_read_slots(vxk_enc_pool * pool, int32_t layer, int32_t stream,
                                      int32_t slot0, int32_t n, void * k_out, void * v_out,
                                      void * cuda_stream);

/* ======================================================================== */
/* Greedy head: tied logits and argmax                                      */
/* ======================================================================== */

/** Opaque greedy-head state for one device (scratch for a batch of rows). */
typedef struct vxk_head vxk_head;

typedef struct vxk_head_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t device;
    int32_t dim;           /* 3072 (decoder width); a multiple of 64 */
    int32_t vocab;         /* 131072 */
    vxk_dtype dtype;       /* F16 or BF16: the type W is stored in */
} vxk_head_config;

VXK_API vxk_head_config vxk_head_default_config(void);
VXK_API vxk_status vxk_head_create(const vxk_head_config * config, vxk_head ** out);
VXK_API void vxk_head_destroy(vxk_head * head);
VXK_API vxk_status vxk_head_last_error(const vxk_head * head, char * buf, size_t capacity);

/**
 * Greedy decoding head for a batch of rows: logits[r][v] = W[v] . x[r] and
 * argmax[r] = the first v with the largest logit.  Replaces
 * emit_logits_argmax (src/voxtral.cpp:2966-2972: ggml_mul_mat(tok_embeddings,
 * last_hidden) then ggml_argmax) for a tied embedding matrix stored as f16 or
 * bf16; x is rounded to W's type and products accumulate in fp32, like
 * ggml's f16 / bf16 dot products.
 *   w       [vocab][dim] f16 or bf16, device, 16-byte aligned
 *   x       [rows][dim] fp32, device (the final-norm output)
 *   argmax  [rows] int32, device
 *   logits  [rows][vocab] fp32, device, or NULL to skip writing them
 * Rows are processed 64 at a time (one pass over W per 64 rows).  Kernels
 * are asynchronous on cuda_stream; vxk_head_sync reports device errors.
 */
VXK_API vxk_status vxk_head_logits_argmax(vxk_head * head, const void * w, const float * x, int32_t rows,
                                          int32_t * argmax, float * logits, void * cuda_stream);

/** Bounded wait for cuda_stream, then the head's device error word
 *  (VXK_STATUS_TIMEOUT or VXK_STATUS_BACKEND_ERROR). */
VXK_API vxk_status vxk_head_sync(vxk_head * head, void * cuda_stream, int32_t timeout_ms);

typedef struct vxk_qweight vxk_qweight;

/**
 * The greedy head over GGUF-quantized tied embeddings (a Q4_K_M model stores
 * tok_embeddings as Q6_K: src/voxtral-quantize.cpp:146-148): logits = the
 * quantized product of x with W (vxk_qweight_matmul, ggml's arithmetic) and
 * argmax[r] = the first index of row r's largest logit (ggml_argmax).
 *   w       a vxk_qweight of vocab rows x dim columns on the head's device
 *   x       [rows][dim] fp32, device; rows <= 64 and <= w's max_batch
 *   argmax  [rows] int32, device
 *   logits  [rows][vocab] fp32, device, or NULL: the head then keeps them in a
 *           scratch it allocates on the first such call
 * Device errors: vxk_qweight_sync(w) for the product, vxk_head_sync(head).
 */
VXK_API vxk_status vxk_head_logits_argmax_q(vxk_head * head, vxk_qweight * w, const float * x, int32_t rows,
                                            int32_t * argmax, float * logits, void * cuda_stream);

/* ======================================================================== */
/* Quantized-weight matrix product (GGUF Q8_0 / Q4_K / Q6_K weights)        */
/* ======================================================================== */

/** GGUF block types of a weight matrix (ggml type ids). */
typedef enum vxk_qtype {
    VXK_QTYPE_Q8_0 = 8,   /* {f16 d; i8 q[32]}: 34 B per 32 values */
    VXK_QTYPE_Q4_K = 12,  /* {f16 d, dmin; u8 scales[12]; u8 q[128]}: 144 B per 256 */
    VXK_QTYPE_Q6_K = 14   /* {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d}: 210 B per 256 */
} vxk_qtype;

/* vxk_qweight (declared with the greedy head above): one quantized weight
 * matrix resident on a device, plus the scratch of its products (one product
 * at a time per matrix). */

typedef struct vxk_qweight_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t device;
    vxk_qtype type;
    int32_t n_rows;      /* output features N (ggml ne[1]); a multiple of 64 */
    int32_t n_cols;      /* input features K (ggml ne[0]); a multiple of 256, <= 16384 */
    int32_t max_batch;   /* activation rows per product, 1..512 (Q4_K / Q6_K from 17 rows: one
                            launch, 64-row chunks side by side; otherwise 64 rows per launch) */
    int32_t reserved;
} vxk_qweight_config;

VXK_API vxk_qweight_config vxk_qweight_default_config(void);

/**
 * Device layout of a weight: 16-row x 256-column tiles ("records"), ordered
 * [row tile][column tile], each holding the tile's quants in the register
 * order of the int8 tensor-core fragments, followed by its block scales
 * (Q4_K's 6-bit scales and mins unpacked to bytes).  Record bytes: Q8_0
 * 4352, Q4_K 2368, Q6_K 3360 (GGUF: 4352, 2304, 3360).  Pure host code.
 */
VXK_API vxk_status vxk_qweight_packed_bytes(vxk_qtype type, int32_t n_rows, int32_t n_cols, size_t * out_bytes);
VXK_API vxk_status vxk_qweight_repack(vxk_qtype type, int32_t n_rows, int32_t n_cols, const void * gguf_blocks,
                                      size_t gguf_bytes, void * out, size_t out_bytes);

/** Repacks the host GGUF rows (n_rows x row bytes, ggml row order) and
 *  uploads them; allocates the product scratch for max_batch rows.  Q4_K and
 *  Q6_K matrices whose n_rows is a multiple of 128 also keep the layout of the
 *  tensor-core product used from 17 rows (128-row x 256-column records: Q4_K
 *  1.03x and Q6_K 1.31x their GGUF bytes with the block scale pairs, Q6_K
 *  holding one quant per byte). */
VXK_API vxk_status vxk_qweight_create(const vxk_qweight_config * config, const void * gguf_blocks,
                                      size_t gguf_bytes, vxk_qweight ** out);
VXK_API void vxk_qweight_destroy(vxk_qweight * w);
VXK_API vxk_status vxk_qweight_last_error(const vxk_qweight * w, char * buf, size_t capacity);

/**
 * y[r][i] = W[i] . x[r] for r < rows, replacing ggml_mul_mat(W, x) of a
 * quantized W (src/voxtral.cpp:2659-2661, 2857, 2877-2881, 2955) with
 * ggml's CPU arithmetic: each x row is quantized like
 * quantize_row_q8_0_ref (Q8_0 weights) or quantize_row_q8_K_ref (K-quants),
 * block dot products are exact integers, and the blocks' scale factors are
 * applied in fp32.
 *   x [rows][n_cols] fp32, device, 16-byte aligned;  y [rows][n_rows] fp32, device.
 * Asynchronous on cuda_stream; vxk_qweight_sync reports device errors.
 */
VXK_API vxk_status vxk_qweight_matmul(vxk_qweight * w, const float * x, int32_t rows, float * y,
                                      void * cuda_stream);

/**
 * The same product for up to 4 matrices that share x (the q, k and v
 * projections of one layer: src/voxtral.cpp:2659-2661): x is quantized once
 * and one launch covers every matrix's rows.  All matrices are on one device
 * with equal n_cols and are all Q8_0 or all K-quants (Q4_K and Q6_K share
 * the Q8_K quantization of x); ys[i] is [rows][ws[i] n_rows].  Uses ws[0]'s
 * scratch and error word (read them with vxk_qweight_sync(ws[0], ...)).
 */
VXK_API vxk_status vxk_qweight_matmul_group(vxk_qweight * const * ws, int32_t n, const float * x, int32_t rows,
                                            float * const * ys, void * cuda_stream);

/* ======================================================================== */
/* GGUF model files                                                         */
/* ======================================================================== */

/** A GGUF file (v2/v3) mapped read-only: its metadata and tensor table, as the
 *  reference's loader reads them (src/voxtral.cpp:1040-1190). */
typedef struct vxk_gguf vxk_gguf;

typedef struct vxk_gguf_tensor {
    const char * name;   /* owned by the vxk_gguf */
    int32_t type;        /* ggml_type (0 F32, 1 F16, 8 Q8_0, 12 Q4_K, 14 Q6_K, 30 BF16, ...) */
    int32_t n_dims;
    int64_t ne[4];       /* ggml order: ne[0] is the row length; unused dims are 1 */
    uint64_t offset;     /* absolute file offset of the tensor's data */
    uint64_t n_bytes;    /* 0 for a ggml type this library does not know */
} vxk_gguf_tensor;

/** Metadata value types (GGUF): 0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32,
 *  7 bool, 8 string, 9 array, 10 u64, 11 i64, 12 f64. */
VXK_API vxk_status vxk_gguf_open(const char * path, vxk_gguf ** out);
VXK_API void vxk_gguf_close(vxk_gguf * g);
/** Last error of g, or of the last failed vxk_gguf_open when g is NULL. */
VXK_API vxk_status vxk_gguf_last_error(const vxk_gguf * g, char * buf, size_t capacity);
VXK_API uint32_t vxk_gguf_version(const vxk_gguf * g);
VXK_API int64_t vxk_gguf_n_tensors(const vxk_gguf * g);
VXK_API vxk_status vxk_gguf_get_tensor(const vxk_gguf * g, int64_t index, vxk_gguf_tensor * out);
/** Index of the named tensor, -1 when absent. */
VXK_API int64_t vxk_gguf_find_tensor(const vxk_gguf * g, const char * name);
/** Host pointer to a tensor's bytes inside the mapping (valid until close). */
VXK_API const void * vxk_gguf_tensor_data(const vxk_gguf * g, int64_t index);
VXK_API int64_t vxk_gguf_n_keys(const vxk_gguf * g);
VXK_API const char * vxk_gguf_key(const vxk_gguf * g, int64_t index);
/** Value type of a key, -1 when absent. */
VXK_API int32_t vxk_gguf_key_type(const vxk_gguf * g, const char * key);
/** Integer and bool values widened to int64 (gguf_get_val_i32 / _bool / ...). */
VXK_API vxk_status vxk_gguf_get_int(const vxk_gguf * g, const char * key, int64_t * out);
/** f32 / f64 values. */
VXK_API vxk_status vxk_gguf_get_float(const vxk_gguf * g, const char * key, double * out);
VXK_API vxk_status vxk_gguf_get_str(const vxk_gguf * g, const char * key, const char ** out);
/** Arrays: element type and count; numeric elements as raw little-endian
 *  bytes in the mapping (data NULL for string arrays: use _get_array_str). */
VXK_API vxk_status vxk_gguf_get_array(const vxk_gguf * g, const char * key, int32_t * elem_type, int64_t * count,
                                      const void ** data);
VXK_API vxk_status vxk_gguf_get_array_str(const vxk_gguf * g, const char * key, int64_t index, const char ** out);
/** vxk_qweight_create for a 2-D Q8_0 / Q4_K / Q6_K tensor of the file. */
VXK_API vxk_status vxk_qweight_create_from_gguf(const vxk_gguf * g, const char * tensor, int32_t device,
                                                int32_t max_batch, vxk_qweight ** out);

/** Bounded wait for cuda_stream, then the matrix's device error word. */
VXK_API vxk_status vxk_qweight_sync(vxk_qweight * w, void * cuda_stream, int32_t timeout_ms);

/* ======================================================================== */
/* Whole decoder step over a batch of streams, and the audio adapter ring    */
/* ======================================================================== */

/**
 * A decoder loaded from a GGUF model onto the pool's device: every layer's
 * quantized projections and FFN (Q8_0 / Q4_K / Q6_K), the norms, the time
 * conditioning, the tied (or untied output) head, the adapter and, per pool
 * stream, an encoder-output ring and an audio-embedding ring.  It runs
 * build_decoder_step_graph_reusable / build_decoder_prefill_graph
 * (src/voxtral.cpp:2900-2965, 3047-3104) for the pool's planned batch, with
 * the rows of many streams in one pass: x = tok_embeddings[token] +
 * audio_emb[slot], then per layer RMSNorm, q/k/v, RoPE + append + attention,
 * o + residual, RMSNorm, time scale (1 + ada), SwiGLU FFN + residual, and the
 * final norm, logits and argmax of each stream's last row.  Not thread-safe:
 * one caller (or vxk_batcher) at a time.
 */
typedef struct vxk_decoder vxk_decoder;

typedef struct vxk_decoder_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t audio_capacity;  /* audio-embedding ring slots per stream: 256 (VOXTRAL_AEMB_RING_CAP) */
    int32_t enc_capacity;    /* encoder-output ring frames per stream: 256 (VOXTRAL_ENC_OUT_RING_CAP);
                                0 = no adapter (adapter tensors not loaded) */
    float time_value;        /* time conditioning t: VOXTRAL_N_DELAY_TOKENS = 6 */
    int32_t reserved[3];
} vxk_decoder_config;

VXK_API vxk_decoder_config vxk_decoder_default_config(void);

/**
 * Loads the decoder of GGUF file g (keys voxtral.decoder.*, tensors
 * dec.blk.N.*, tok_embeddings.weight, dec.norm.weight, output.weight when
 * present, adapter.0/2.weight; src/voxtral.cpp:1097-1110, 1225-1252) for
 * pool, whose layers, heads and head_dim must match the file.  Projection,
 * FFN and adapter matrices must be Q8_0, Q4_K or Q6_K; the embeddings may
 * also be F16 or BF16; norms F32, F16 or BF16.  g may be closed afterwards.
 */
VXK_API vxk_status vxk_decoder_create(const vxk_gguf * g, vxk_pool * pool, const vxk_decoder_config * config,
                                      vxk_decoder ** out);
VXK_API void vxk_decoder_destroy(vxk_decoder * d);
/** Last error of d, or of the last failed vxk_decoder_create when d is NULL. */
VXK_API vxk_status vxk_decoder_last_error(const vxk_decoder * d, char * buf, size_t capacity);

typedef struct vxk_decoder_info {
    int32_t n_layers, dim, hidden, n_q_heads, n_kv_heads, head_dim, vocab, ada_dim;
    int32_t emb_type;        /* ggml type of tok_embeddings (or output.weight) */
    int32_t max_rows;        /* rows of one forward (the pool's max_rows) */
    int32_t max_streams;
    int32_t audio_capacity, enc_capacity, enc_dim;
    int64_t device_bytes;    /* weights, rings and scratch */
} vxk_decoder_info;

VXK_API vxk_status vxk_decoder_get_info(const vxk_decoder * d, vxk_decoder_info * out);

/**
 * One forward pass over the pool's planned batch (vxk_batch_plan; rows in
 * plan order, each stream's n_new rows at consecutive positions).  Host
 * arrays per row: tokens[rows] (0 <= token < vocab) and audio_slots[rows]
 * (the audio-embedding ring slot added to the row, audio_pos % capacity).
 * Device outputs per planned stream (its last row): argmax[n_streams] int32,
 * and optionally logits[n_streams][vocab] and hidden[n_streams][dim] (the
 * final-normed hidden state, decoder_hidden_diagnostic).  The KV caches are
 * appended; the caller commits (vxk_batch_commit) after vxk_decoder_sync.
 * Asynchronous on cuda_stream; allocates nothing after the first call with
 * a given row count.
 */
VXK_API vxk_status vxk_decoder_forward(vxk_decoder * d, const int32_t * tokens, const int32_t * audio_slots,
                                       int32_t * argmax, float * logits, float * hidden, void * cuda_stream);

/** Writes n encoder-output rows ([n][enc_dim] fp32, device memory) of stream
 *  into its ring at absolute frames frame .. frame+n-1 (slot = frame %
 *  enc_capacity); copy_chunk_to_enc_out_ring (src/voxtral.cpp:4018-4045). */
VXK_API vxk_status vxk_decoder_write_enc(vxk_decoder * d, int32_t stream, int64_t frame, int32_t n,
                                         const float * rows, void * cuda_stream);
/** Writes n audio-embedding rows ([n][dim] fp32, device memory) into stream's
 *  ring at absolute positions pos .. pos+n-1 (slot = pos % audio_capacity). */
VXK_API vxk_status vxk_decoder_write_audio(vxk_decoder * d, int32_t stream, int64_t pos, int32_t n,
                                           const float * rows, void * cuda_stream);

/**
 * The adapter over the encoder-output rings, n groups of any streams in one
 * pass (build_adapter_ring_graph_reusable, src/voxtral.cpp:2589-2620): group
 * g reads the 4 frames enc_frame[g] .. +3 of streams[g] (enc_frame a multiple
 * of 4), x = adapter.2 . gelu_erf(adapter.0 . concat(frames)), stored in the
 * stream's audio ring at audio_pos[g] % audio_capacity.  Host arrays; n in
 * [1, max_rows].
 */
VXK_API vxk_status vxk_decoder_adapt(vxk_decoder * d, int32_t n, const int32_t * streams,
                                     const int64_t * enc_frame, const int64_t * audio_pos, void * cuda_stream);

/** Reads n rows of a stream's audio ring back (device destination), for tests. */
VXK_API vxk_status vxk_decoder_read_audio(vxk_decoder * d, int32_t stream, int64_t pos, int32_t n, float * rows,
                                          void * cuda_stream);

/** Bounded wait for cuda_stream, then every device error word the decoder's
 *  launches use (pool, products, head). */
VXK_API vxk_status vxk_decoder_sync(vxk_decoder * d, void * cuda_stream, int32_t timeout_ms);

/* ======================================================================== */
/* Streaming encoder stack                                                   */
/* ======================================================================== */

/**
 * The realtime model's encoder loaded from a GGUF file onto an encoder pool's
 * device (tensors enc.conv0/1.*, enc.blk.N.*, enc.norm.weight; keys
 * voxtral.encoder.*, src/voxtral.cpp:1085-1095, 1190-1222).  One forward runs
 * build_encoder_steady_graph (src/voxtral.cpp:2386-2511) for the pool's planned
 * batch of many streams: the causal conv stem over each stream's Mel window,
 * then every layer (RMS norm, q/k/v with q and v biases, vxk_enc_layer's RoPE +
 * ring append + windowed attention, o with bias + residual, RMS norm, SwiGLU
 * FFN with the w2 bias + residual) and the final norm.  Projection and FFN
 * matrices must be Q8_0, Q4_K or Q6_K; conv weights, norms and biases F32,
 * F16 or BF16.  The offline LayerNorm encoder is refused.  Not thread-safe.
 */
typedef struct vxk_encoder vxk_encoder;

typedef struct vxk_encoder_info {
    int32_t n_layers, dim, hidden, n_heads, head_dim, n_mel, max_rows;
    int32_t reserved;
    int64_t device_bytes;
} vxk_encoder_info;

/** max_rows: rows of one forward (0: max_streams x 4, the steady step). */
VXK_API vxk_status vxk_encoder_create(const vxk_gguf * g, vxk_enc_pool * pool, int32_t max_rows,
                                      vxk_encoder ** out);
VXK_API void vxk_encoder_destroy(vxk_encoder * e);
/** Last error of e, or of the last failed vxk_encoder_create when e is NULL. */
VXK_API vxk_status vxk_encoder_last_error(const vxk_encoder * e, char * buf, size_t capacity);
VXK_API vxk_status vxk_encoder_get_info(const vxk_encoder * e, vxk_encoder_info * out);

/**
 * One forward over the encoder pool's planned batch (vxk_enc_batch_plan: n new
 * frames per stream at q_start).  mel (device): for each planned stream in
 * plan order its Mel window [n_mel][2 n + 4] fp32, channel-major, frames
 * 2 (q_start - 2) .. 2 (q_start + n) - 1 with zeros before frame 0 (the
 * reference's conv_cm, src/voxtral.cpp:4072-4101).  out (device): [rows][dim]
 * fp32, the final-normed encoder frames q_start .. q_start + n - 1 of each
 * stream, which vxk_decoder_write_enc stores for the adapter.  The rings are
 * appended; the caller commits (vxk_enc_batch_commit) after vxk_encoder_sync.
 */
VXK_API vxk_status vxk_encoder_forward(vxk_encoder * e, const float * mel, float * out, void * cuda_stream);
/** The conv stem alone for the planned batch (same arguments as
 *  vxk_encoder_forward): out [rows][dim] = gelu(conv1(gelu(conv0(mel)))) at
 *  each stream's new frames, before the first layer.  Touches no ring. */
VXK_API vxk_status vxk_encoder_stem(vxk_encoder * e, const float * mel, float * out, void * cuda_stream);
/** Bounded wait for cuda_stream, then the encoder pool's and the products'
 *  device error words. */
VXK_API vxk_status vxk_encoder_sync(vxk_encoder * e, void * cuda_stream, int32_t timeout_ms);

/* ======================================================================== */
/* Cross-context batcher                                                     */
/* ======================================================================== */

/**
 * Gathers the single-token decoder steps of many contexts into one batch per
 * GPU.  In the reference every voxtral_context runs its own step graph
 * (voxtral_ctx_decoder_step, src/voxtral-internal.h:243-251, called by
 * pump_incremental, src/voxtral-stream-decoder.cpp:92-98, 163-164, each
 * context on its own thread, include/voxtral.h:223); behind the unchanged C
 * ABI that call becomes vxk_batcher_step, which blocks its thread until the
 * batch holding its row has run.  A dispatcher thread inside the batcher
 * starts a batch when max_rows requests are queued, when `expected` are
 * queued, or max_wait_us after the oldest queued request, whichever comes
 * first; requests of one stream never share a batch.  Thread-safe.
 */
typedef struct vxk_batcher vxk_batcher;

typedef struct vxk_batcher_config {
    uint32_t struct_size;
    uint32_t api_version;
    int32_t max_rows;       /* rows per batch, 1..4096 */
    int32_t max_wait_us;    /* the oldest request waits at most this long for company */
    int32_t expected;       /* 0, or start as soon as this many requests are queued */
    int32_t timeout_ms;     /* bounded wait of vxk_batcher_step for its result */
} vxk_batcher_config;

VXK_API vxk_batcher_config vxk_batcher_default_config(void);

/** Runs one batch: n rows (stream, token, audio slot), writes each row's next
 *  token.  Called on the dispatcher thread, one batch at a time. */
typedef vxk_status (*vxk_batch_fn)(void * user, int32_t n, const int32_t * streams, const int32_t * tokens,
                                   const int32_t * audio_slots, int32_t * out_tokens);

VXK_API vxk_status vxk_batcher_create(const vxk_batcher_config * config, vxk_batch_fn fn, void * user,
                                      vxk_batcher ** out);
/**
 * A batcher whose batches run the decoder: vxk_batch_plan (one token per
 * stream), vxk_decoder_forward, the argmax read back (4 bytes per row),
 * vxk_decoder_sync, then vxk_batch_commit (vxk_batch_abort on failure), on
 * cuda_stream from the dispatcher thread.
 */
VXK_API vxk_status vxk_batcher_create_for_decoder(const vxk_batcher_config * config, vxk_decoder * d,
                                                  vxk_pool * pool, void * cuda_stream, vxk_batcher ** out);
/** Stops the dispatcher after the running batch; queued requests get
 *  VXK_STATUS_INVALID_STATE; returns once every vxk_batcher_step in progress
 *  has returned (none may start afterwards).  NULL is safe. */
VXK_API void vxk_batcher_destroy(vxk_batcher * b);

/** One decoder step of `stream` (its token and audio slot); blocks until the
 *  batch ran (out_token = the greedy next token) or timeout_ms passed
 *  (VXK_STATUS_TIMEOUT; the row still runs with its batch if already taken). */
VXK_API vxk_status vxk_batcher_step(vxk_batcher * b, int32_t stream, int32_t token, int32_t audio_slot,
                                    int32_t * out_token);

typedef struct vxk_batcher_stats {
    int64_t batches;
    int64_t rows;
    int64_t max_rows_seen;
    int64_t failed_batches;
    int64_t timeouts;
    double mean_wait_us;    /* request queued -> its batch started */
} vxk_batcher_stats;

VXK_API vxk_status vxk_batcher_get_stats(const vxk_batcher * b, vxk_batcher_stats * out);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* VXK_H */
