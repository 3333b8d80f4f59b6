/*
 * vx_cpu_step.c -- timed CPU restatement of one decoder KV step (bench only).
 *
 * TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline and `--impl reference`
 * legs time this; the product library never links it.  It follows the same
 * semantics as vx_oracle.c (rope mode 0 through a cos/sin table built with
 * vxo_rope_cache, f16 RNE append at slot pos % cap, GQA softmax attention
 * over the logical window [win_start, pos] with scale 1/sqrt(d)) but with the
 * fp32 online-softmax accumulation of ggml's CPU flash-attention loop
 * (running max M, running sum S, rescale on a new max), so it is a fair
 * multi-core CPU speed reference for src/voxtral.cpp:2629-2887.
 * The cache rows are f16 (ggml type 1) or q8_0 (ggml type 8: blocks of an
 * f16 scale and 32 int8, quantized on append by vxo_quantize_row_q8_0 and
 * dequantized on read).
 * Parallel over (stream, kv head) work items inside a layer, with a barrier
 * between layers, like ggml's per-op thread split.
 */
#include "vx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FLT16_MAX__)
typedef _Float16 vxo_half;
static inline float h2f(uint16_t h) {
    vxo_half x;
    memcpy(&x, &h, 2);
    return (float) x;
}
#else
static inline float h2f(uint16_t h) { return vxo_f16_to_f32(h); }
#endif

/* RoPE mode 0 on head_dim/2 adjacent pairs with each product and sum rounded
 * on its own (as vx_oracle.c and ggml's CPU rope), even though the rest of
 * this file is compiled with contraction for speed. */
__attribute__((noinline, optimize("fp-contract=off"))) static void rope_rotate(const float * x,
                                                                                const float * cs, int32_t hd,
                                                                                float * y) {
    for (int32_t i = 0; i < hd / 2; ++i) {
        const float c = cs[2 * i], sn = cs[2 * i + 1];
        const float x0 = x[2 * i], x1 = x[2 * i + 1];
        const float a = x0 * c, b = x1 * sn, e = x0 * sn, f = x1 * c;
        y[2 * i] = a - b;
        y[2 * i + 1] = e + f;
    }
}

typedef struct step_args {
    int32_t n_streams, n_layers, n_q, n_kv, hd;
    int64_t cap;
    int32_t dtype;      /* VXO_F16 or VXO_Q8_0 */
    int64_t row_bytes;  /* bytes of one kv head's row in the cache */
    uint8_t * kc;
    uint8_t * vc;
    const float * q;
    const float * k;
    const float * v;
    const int64_t * pos;
    const int64_t * win;
    const float * rope;
    int64_t rope_rows;
    float scale;
    float * out;
    int32_t n_threads;
    pthread_barrier_t * bar;
} step_args;

typedef struct thread_arg {
    const step_args * a;
    int32_t tid;
} thread_arg;

static void do_item(const step_args * a, int32_t layer, int32_t s, int32_t kvh) {
    const int32_t hd = a->hd;
    const int32_t group = a->n_q / a->n_kv;
    const int64_t p_new = a->pos[s];
    const float * cs = a->rope + (p_new < a->rope_rows ? p_new : 0) * hd;
    const int64_t base = (((int64_t) s * a->n_layers + layer) * a->n_kv + kvh) * a->cap;
    uint8_t * kc = a->kc + base * a->row_bytes;
    uint8_t * vc = a->vc + base * a->row_bytes;
    const int64_t sl = (int64_t) s * a->n_layers + layer;
    const int q8 = a->dtype == VXO_Q8_0;

    /* append: rotate K at p_new, store both rows (f16 RNE or q8_0) at slot p_new % cap */
    {
        const float * kr = a->k + (sl * a->n_kv + kvh) * hd;
        const float * vr = a->v + (sl * a->n_kv + kvh) * hd;
        uint8_t * kd = kc + (p_new % a->cap) * a->row_bytes;
        uint8_t * vd = vc + (p_new % a->cap) * a->row_bytes;
        float kx[256];
        rope_rotate(kr, cs, hd, kx);
        if (q8) {
            vxo_quantize_row_q8_0(kx, hd, kd);
            vxo_quantize_row_q8_0(vr, hd, vd);
        } else {
            for (int32_t i = 0; i < hd; ++i) ((uint16_t *) kd)[i] = vxo_f32_to_f16(kx[i]);
            for (int32_t i = 0; i < hd; ++i) ((uint16_t *) vd)[i] = vxo_f32_to_f16(vr[i]);
        }
    }

    float qr[8][256];
    float acc[8][256];
    float M[8], S[8];
    for (int32_t g = 0; g < group; ++g) {
        const float * qh = a->q + (sl * a->n_q + kvh * group + g) * hd;
        rope_rotate(qh, cs, hd, qr[g]);
        for (int32_t d = 0; d < hd; ++d) acc[g][d] = 0.0f;
        M[g] = -INFINITY;
        S[g] = 0.0f;
    }
    float kf[256], vf[256];
    for (int64_t p = a->win[s]; p <= p_new; ++p) {
        const uint8_t * kr = kc + (p % a->cap) * a->row_bytes;
        const uint8_t * vr = vc + (p % a->cap) * a->row_bytes;
        if (q8) {
            vxo_dequantize_row_q8_0(kr, hd, kf);
            vxo_dequantize_row_q8_0(vr, hd, vf);
        } else {
            for (int32_t d = 0; d < hd; ++d) kf[d] = h2f(((const uint16_t *) kr)[d]);
            for (int32_t d = 0; d < hd; ++d) vf[d] = h2f(((const uint16_t *) vr)[d]);
        }
        for (int32_t g = 0; g < group; ++g) {
            float sdot = 0.0f;
            for (int32_t d = 0; d < hd; ++d) sdot += qr[g][d] * kf[d];
            sdot *= a->scale;
            float ms = 1.0f, vs = 1.0f;
            if (sdot > M[g]) {
                ms = expf(M[g] - sdot);
                M[g] = sdot;
                for (int32_t d = 0; d < hd; ++d) acc[g][d] *= ms;
            } else {
                vs = expf(sdot - M[g]);
            }
            for (int32_t d = 0; d < hd; ++d) acc[g][d] += vs * vf[d];
            S[g] = S[g] * ms + vs;
        }
    }
    for (int32_t g = 0; g < group; ++g) {
        float * o = a->out + (sl * a->n_q + kvh * group + g) * hd;
        const float inv = S[g] > 0.0f ? 1.0f / S[g] : 0.0f;
        for (int32_t d = 0; d < hd; ++d) o[d] = acc[g][d] * inv;
    }
}

static void * worker(void * p) {
    const thread_arg * t = (const thread_arg *) p;
    const step_args * a = t->a;
    const int32_t items = a->n_streams * a->n_kv;
    for (int32_t layer = 0; layer < a->n_layers; ++layer) {
        for (int32_t it = t->tid; it < items; it += a->n_threads) {
            do_item(a, layer, it / a->n_kv, it % a->n_kv);
        }
        pthread_barrier_wait(a->bar);
    }
    return NULL;
}

void vxo_cpu_decode_step(int32_t dtype, int32_t n_streams, int32_t n_layers, int32_t n_q, int32_t n_kv,
                         int32_t head_dim, int64_t cap, uint8_t * k_cache, uint8_t * v_cache,
                         const float * q, const float * k, const float * v, const int64_t * pos,
                         const int64_t * win_start, const float * rope_cs, int64_t rope_rows, float scale,
                         int32_t n_threads, float * out) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (head_dim > 256 || n_q / n_kv > 8) return;
    if (dtype != VXO_F16 && !(dtype == VXO_Q8_0 && head_dim % 32 == 0)) return;
    pthread_barrier_t bar;
    pthread_barrier_init(&bar, NULL, (unsigned) n_threads);
    step_args a = {n_streams, n_layers, n_q, n_kv, head_dim, cap, dtype, vxo_row_bytes(dtype, 1, head_dim),
                   k_cache, v_cache, q, k, v, pos, win_start, rope_cs, rope_rows, scale, out, n_threads, &bar};
    pthread_t th[256];
    thread_arg ta[256];
    for (int32_t t = 0; t < n_threads; ++t) {
        ta[t].a = &a;
        ta[t].tid = t;
        if (t > 0) pthread_create(&th[t], NULL, worker, &ta[t]);
    }
    worker(&ta[0]);
    for (int32_t t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
    pthread_barrier_destroy(&bar);
}

void vxo_cpu_decode_step_f16(int32_t n_streams, int32_t n_layers, int32_t n_q, int32_t n_kv,
                             int32_t head_dim, int64_t cap, uint16_t * k_cache,
                             uint16_t * v_cache, const float * q, const float * k,
                             const float * v, const int64_t * pos, const int64_t * win_start,
                             const float * rope_cs, int64_t rope_rows, float scale,
                             int32_t n_threads, float * out) {
    vxo_cpu_decode_step(VXO_F16, n_streams, n_layers, n_q, n_kv, head_dim, cap, (uint8_t *) k_cache,
                        (uint8_t *) v_cache, q, k, v, pos, win_start, rope_cs, rope_rows, scale, n_threads, out);
}
