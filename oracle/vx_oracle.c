/*
 * vx_oracle.c -- CPU restatement of voxtral.cpp's decoder KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, smoke() and bench.py's CPU
 * legs.  The product library never links or calls it.  Built with
 * -ffp-contract=off so every fp32 operation below is rounded on its own.
 *
 * Per-function provenance (paths inside the reference project):
 *   vxo_dec_kv_plan / vxo_dec_kv_commit   src/voxtral.cpp:1604-1656
 *   vxo_enc_kv_plan / mask predicate      src/voxtral.cpp:3636-3692
 *   rope mode 0                           call site src/voxtral.cpp:2668-2671
 *                                         (n_dims=head_dim, mode 0, freq_base
 *                                         theta, freq_scale 1, ext_factor 0,
 *                                         attn_factor 1, beta 0/0); algorithm:
 *                                         ggml CPU rope (theta_scale =
 *                                         powf(base, -2/n_dims), theta_0 = pos,
 *                                         theta_{i+1} = theta_i * theta_scale,
 *                                         cosf/sinf, dst0 = x0*c - x1*s,
 *                                         dst1 = x0*s + x1*c)
 *   f16 append                            src/voxtral.cpp:2682-2713 (set_rows /
 *                                         cpy F32 -> F16, IEEE binary16 RNE)
 *   q8_0                                  ggml quantize_row_q8_0_ref (blocks of
 *                                         32: d = amax/127, id = d ? 1/d : 0,
 *                                         q = roundf(x*id)); the reference
 *                                         itself only quantises weights with it
 *                                         (src/voxtral-quantize.cpp:248)
 *   attention                             src/voxtral.cpp:2716-2854
 *                                         (flash_attn_ext, scale 1/sqrt(d),
 *                                         GQA head h -> kv head h/(n_q/n_kv))
 *
 * ggml @5cecdad692d868e28dbd2f7c468504770108f30c is not present on this
 * machine, so the rope and attention rounding are PARITY UNPINNED; the ring
 * planners, f16/bf16 and q8_0 are pinned (see vx_oracle.h).
 */
#include "vx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* decoder ring planner                                                    */
/* ---------------------------------------------------------------------- */

static int32_t dec_segments(int64_t start, int32_t len, int32_t cap, vxo_seg out[2]) {
    if (len <= 0) return 0;
    const int32_t slot = (int32_t) (start % cap);
    const int32_t room = cap - slot;
    const int32_t first = len < room ? len : room;
    out[0].slot = slot;
    out[0].len = first;
    if (first == len) return 1;
    out[1].slot = 0;
    out[1].len = len - first;
    return 2;
}

int vxo_dec_kv_plan(const vxo_dec_ring * r, int64_t start, int32_t n_new, vxo_dec_plan * o) {
    memset(o, 0, sizeof(*o));
    if (r->capacity <= 0 || r->used < 0 || r->used > r->capacity || r->oldest < 0 ||
        r->next < 0 || r->oldest + r->used != r->next || start != r->next ||
        n_new <= 0 || n_new > r->capacity) {
        return 0;
    }
    o->absolute_start = start;
    o->n_new = n_new;
    o->write_nseg = dec_segments(start, n_new, (int32_t) r->capacity, o->write_seg);
    o->next_after = start + n_new;
    o->used_after = r->used + n_new < r->capacity ? r->used + n_new : r->capacity;
    o->oldest_after = o->next_after - o->used_after;
    o->evicted = r->used + n_new - r->capacity > 0 ? r->used + n_new - r->capacity : 0;
    o->read_nseg = dec_segments(o->oldest_after, (int32_t) o->used_after,
                                (int32_t) r->capacity, o->read_seg);
    {
        const int64_t prev_cycle = start == 0 ? 0 : (start - 1) / r->capacity;
        const int64_t new_cycle = (o->next_after - 1) / r->capacity;
        o->wrapped = new_cycle > prev_cycle;
    }
    return 1;
}

void vxo_dec_kv_commit(vxo_dec_ring * r, const vxo_dec_plan * p) {
    r->used = p->used_after;
    r->oldest = p->oldest_after;
    r->next = p->next_after;
    r->evictions += p->evicted;
    if (p->wrapped) r->wraps += 1;
}

/* ---------------------------------------------------------------------- */
/* encoder ring planner                                                    */
/* ---------------------------------------------------------------------- */

int vxo_enc_kv_mask_allows(int64_t kv_abs, int64_t q_abs, int32_t window) {
    return kv_abs <= q_abs && kv_abs >= q_abs - (int64_t) (window - 1);
}

int vxo_enc_kv_plan(int64_t q_start, int32_t n_new, int32_t cap, int32_t window,
                    vxo_enc_plan * o) {
    memset(o, 0, sizeof(*o));
    if (n_new <= 0 || cap <= 0 || window <= 0) return 0;
    if (n_new > cap - window) return 0;
    if (q_start < 0) return 0;
    o->q_start = q_start;
    o->n_new = n_new;
    o->win_start = q_start - (int64_t) (window - 1) > 0 ? q_start - (int64_t) (window - 1) : 0;
    o->win_end = q_start + n_new;
    o->win_len = (int32_t) (o->win_end - o->win_start);
    o->read_nseg = dec_segments(o->win_start, o->win_len, cap, o->read_seg);
    o->read_wraps = o->read_nseg > 1;
    o->write_nseg = dec_segments(q_start, n_new, cap, o->write_seg);
    o->write_wraps = o->write_nseg > 1;
    o->conv_mel_start = 2 * (q_start - 2) > 0 ? 2 * (q_start - 2) : 0;
    o->conv_mel_end = 2 * (q_start + n_new);
    o->conv_slice_start = (int32_t) (q_start - o->conv_mel_start / 2);
    {
        const int64_t old_lo = q_start - window > 0 ? q_start - window : 0;
        const int64_t new_lo = o->win_end - window > 0 ? o->win_end - window : 0;
        o->evicted = new_lo - old_lo;
    }
    return 1;
}

/* ---------------------------------------------------------------------- */
/* element formats                                                         */
/* ---------------------------------------------------------------------- */

uint16_t vxo_f32_to_f16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t exp = (u >> 23) & 0xffu;
    const uint32_t mant = u & 0x7fffffu;
    if (exp == 0xffu) {
        if (mant) return (uint16_t) (sign | 0x7e00u | (mant >> 13));
        return (uint16_t) (sign | 0x7c00u);
    }
    const int32_t e = (int32_t) exp - 112; /* rebias 127 -> 15 */
    if (e >= 31) return (uint16_t) (sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t) sign;
        /* half subnormal: value = (1.mant) * 2^(e-14) in units of 2^-24 */
        const uint32_t full = mant | 0x800000u;
        const uint32_t shift = (uint32_t) (14 - e);
        uint32_t m = full >> shift;
        const uint32_t rem = full & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (m & 1u))) m += 1u;
        return (uint16_t) (sign | m);
    }
    uint32_t h = sign | ((uint32_t) e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u; /* may carry into inf */
    return (uint16_t) h;
}

float vxo_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t) h & 0x8000u) << 16;
    const uint32_t exp = ((uint32_t) h >> 10) & 0x1fu;
    const uint32_t mant = (uint32_t) h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (mant == 0) {
            u = sign;
        } else {
            float f = (float) mant * 5.9604644775390625e-08f; /* 2^-24, exact */
            memcpy(&u, &f, 4);
            u |= sign;
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (mant << 13);
    } else {
        u = sign | ((exp + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t vxo_f32_to_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t) ((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t) (u >> 16);
}

float vxo_bf16_to_f32(uint16_t h) {
    const uint32_t u = (uint32_t) h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void vxo_f32_to_f16_n(const float * x, uint16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = vxo_f32_to_f16(x[i]);
}

void vxo_f32_to_bf16_n(const float * x, uint16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = vxo_f32_to_bf16(x[i]);
}

void vxo_quantize_row_q8_0(const float * x, int64_t k, uint8_t * blocks) {
    const int64_t nb = k / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float * xb = x + b * 32;
        uint8_t * ob = blocks + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = vxo_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int j = 0; j < 32; ++j) {
            const float x0 = xb[j] * id;
            const int8_t q = (int8_t) roundf(x0);
            memcpy(ob + 2 + j, &q, 1);
        }
    }
}

void vxo_dequantize_row_q8_0(const uint8_t * blocks, int64_t k, float * y) {
    const int64_t nb = k / 32;
    for (int64_t b = 0; b < nb; ++b) {
        uint16_t dh;
        memcpy(&dh, blocks + b * 34, 2);
        const float d = vxo_f16_to_f32(dh);
        for (int j = 0; j < 32; ++j) {
            const int8_t q = (int8_t) blocks[b * 34 + 2 + j];
            y[b * 32 + j] = (float) q * d;
        }
    }
}

/* ---------------------------------------------------------------------- */
/* RoPE mode 0 (adjacent pairs)                                            */
/* ---------------------------------------------------------------------- */

void vxo_rope_cache(int64_t pos, int32_t n_dims, float base, float * cs) {
    const float theta_scale = powf(base, -2.0f / (float) n_dims);
    float theta = (float) pos;
    for (int32_t i = 0; i < n_dims / 2; ++i) {
        cs[2 * i + 0] = cosf(theta);
        cs[2 * i + 1] = sinf(theta);
        theta = theta * theta_scale;
    }
}

void vxo_rope_table(int64_t rows, int32_t n_dims, float base, float * table) {
    for (int64_t p = 0; p < rows; ++p) vxo_rope_cache(p, n_dims, base, table + p * n_dims);
}

void vxo_rope_apply(const float * x, int32_t n_heads, int32_t head_dim, int64_t pos,
                    float base, float * out) {
    float cs[512];
    vxo_rope_cache(pos, head_dim, base, cs);
    for (int32_t h = 0; h < n_heads; ++h) {
        const float * xr = x + (int64_t) h * head_dim;
        float * yr = out + (int64_t) h * head_dim;
        for (int32_t i = 0; i < head_dim / 2; ++i) {
            const float c = cs[2 * i], s = cs[2 * i + 1];
            const float x0 = xr[2 * i], x1 = xr[2 * i + 1];
            const float a = x0 * c;
            const float b = x1 * s;
            const float e = x0 * s;
            const float f = x1 * c;
            yr[2 * i + 0] = a - b;
            yr[2 * i + 1] = e + f;
        }
    }
}

/* ---------------------------------------------------------------------- */
/* cache rows                                                              */
/* ---------------------------------------------------------------------- */

int64_t vxo_row_bytes(int32_t dtype, int32_t n_kv, int32_t head_dim) {
    const int64_t n = (int64_t) n_kv * head_dim;
    switch (dtype) {
        case VXO_F32: return n * 4;
        case VXO_F16: return n * 2;
        case VXO_BF16: return n * 2;
        case VXO_Q8_0: return n / 32 * 34;
        default: return -1;
    }
}

static void store_row(const float * x, int64_t n, int32_t dtype, uint8_t * out) {
    switch (dtype) {
        case VXO_F32: memcpy(out, x, (size_t) n * 4); break;
        case VXO_F16: vxo_f32_to_f16_n(x, (uint16_t *) out, n); break;
        case VXO_BF16: vxo_f32_to_bf16_n(x, (uint16_t *) out, n); break;
        case VXO_Q8_0: vxo_quantize_row_q8_0(x, n, out); break;
        default: break;
    }
}

void vxo_kv_row(const float * k, const float * v, int32_t n_kv, int32_t head_dim,
                int64_t pos, float base, int32_t dtype, uint8_t * k_out, uint8_t * v_out) {
    float kr[8192];
    const int64_t n = (int64_t) n_kv * head_dim;
    vxo_rope_apply(k, n_kv, head_dim, pos, base, kr);
    store_row(kr, n, dtype, k_out);
    store_row(v, n, dtype, v_out);
}

void vxo_kv_rows(const float * k, const float * v, int64_t n_rows, int32_t n_kv, int32_t head_dim,
                 int64_t pos0, float base, int32_t dtype, uint8_t * k_out, uint8_t * v_out) {
    const int64_t vals = (int64_t) n_kv * head_dim;
    const int64_t rb = vxo_row_bytes(dtype, n_kv, head_dim);
    for (int64_t r = 0; r < n_rows; ++r)
        vxo_kv_row(k + r * vals, v + r * vals, n_kv, head_dim, pos0 + r, base, dtype, k_out + r * rb,
                   v_out + r * rb);
}

void vxo_row_to_f32(const uint8_t * row, int32_t dtype, int32_t n_kv, int32_t head_dim,
                    float * out) {
    const int64_t n = (int64_t) n_kv * head_dim;
    switch (dtype) {
        case VXO_F32: memcpy(out, row, (size_t) n * 4); break;
        case VXO_F16:
            for (int64_t i = 0; i < n; ++i) {
                uint16_t h;
                memcpy(&h, row + 2 * i, 2);
                out[i] = vxo_f16_to_f32(h);
            }
            break;
        case VXO_BF16:
            for (int64_t i = 0; i < n; ++i) {
                uint16_t h;
                memcpy(&h, row + 2 * i, 2);
                out[i] = vxo_bf16_to_f32(h);
            }
            break;
        case VXO_Q8_0: vxo_dequantize_row_q8_0(row, n, out); break;
        default: break;
    }
}

/* ---------------------------------------------------------------------- */
/* attention (fp64 accumulation)                                           */
/* ---------------------------------------------------------------------- */

void vxo_attn_row(const float * q, int64_t q_pos, float base, int32_t rope_q, int32_t n_q,
                  int32_t n_kv, int32_t head_dim, const uint8_t * k_rows,
                  const uint8_t * v_rows, int32_t dtype, int64_t n_keys, float scale,
                  float * out) {
    const int64_t row_bytes = vxo_row_bytes(dtype, n_kv, head_dim);
    const int64_t row_vals = (int64_t) n_kv * head_dim;
    const int32_t group = n_q / n_kv;
    float qr[8192];
    double acc[512];
    float * kf = (float *) malloc(sizeof(float) * (size_t) (n_keys > 0 ? n_keys : 1) * (size_t) row_vals);
    float * vf = (float *) malloc(sizeof(float) * (size_t) (n_keys > 0 ? n_keys : 1) * (size_t) row_vals);
    double * sc = (double *) malloc(sizeof(double) * (size_t) (n_keys > 0 ? n_keys : 1));
    if (!kf || !vf || !sc) {
        free(kf); free(vf); free(sc);
        return;
    }
    for (int64_t j = 0; j < n_keys; ++j) {
        vxo_row_to_f32(k_rows + j * row_bytes, dtype, n_kv, head_dim, kf + j * row_vals);
        vxo_row_to_f32(v_rows + j * row_bytes, dtype, n_kv, head_dim, vf + j * row_vals);
    }
    if (rope_q) {
        vxo_rope_apply(q, n_q, head_dim, q_pos, base, qr);
    } else {
        memcpy(qr, q, sizeof(float) * (size_t) n_q * head_dim);
    }
    for (int32_t h = 0; h < n_q; ++h) {
        const int32_t kvh = h / group;
        const float * qh = qr + (int64_t) h * head_dim;
        double m = -INFINITY;
        for (int64_t j = 0; j < n_keys; ++j) {
            const float * kr = kf + j * row_vals + (int64_t) kvh * head_dim;
            double s = 0.0;
            for (int32_t d = 0; d < head_dim; ++d) s += (double) qh[d] * (double) kr[d];
            s *= (double) scale;
            sc[j] = s;
            if (s > m) m = s;
        }
        double l = 0.0;
        for (int32_t d = 0; d < head_dim; ++d) acc[d] = 0.0;
        for (int64_t j = 0; j < n_keys; ++j) {
            const float * vr = vf + j * row_vals + (int64_t) kvh * head_dim;
            const double p = exp(sc[j] - m);
            l += p;
            for (int32_t d = 0; d < head_dim; ++d) acc[d] += p * (double) vr[d];
        }
        for (int32_t d = 0; d < head_dim; ++d) {
            out[(int64_t) h * head_dim + d] = n_keys > 0 ? (float) (acc[d] / l) : 0.0f;
        }
    }
    free(kf);
    free(vf);
    free(sc);
}
