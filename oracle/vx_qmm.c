/*
 * vx_qmm.c -- CPU restatement of ggml's quantized matrix product, the
 * arithmetic behind every ggml_mul_mat(W, x) of a quantized GGUF model in
 * voxtral.cpp: the decoder projections (src/voxtral.cpp:2659-2661 q/k/v,
 * 2857 o), the FFN (2877-2881), the adapter (2575-2580) and the tied
 * logits (2955).
 *
 * TEST INFRASTRUCTURE ONLY (the checker of vxk_qmatmul); the product never
 * links it.
 *
 * What ggml's CPU backend does for W (N rows x K, quantized) times x (f32):
 *   1. each row of x is quantized to the weight type's "vec dot" type:
 *      Q8_0 for Q8_0 weights, Q8_K for the K-quants (Q4_K, Q6_K);
 *   2. every output is a sum over blocks of exact integer dot products of the
 *      two quantized rows, scaled by the blocks' float factors.
 * ggml lives in a dependency that is absent here (ggml @5cecdad692d8, fetched
 * by CMakeLists.txt:77-93), so this file restates the published algorithms:
 *   - block layouts (GGUF): Q8_0 {f16 d; i8 q[32]} 34 B / 32 values;
 *     Q4_K {f16 d, dmin; u8 scales[12]; u8 q[128]} 144 B / 256;
 *     Q6_K {u8 ql[128]; u8 qh[64]; i8 scales[16]; f16 d} 210 B / 256.
 *     The decoders below are pinned against gguf 0.19.0 (gguf.quants), an
 *     independent numpy implementation of the same layouts (tests/).
 *   - quantize_row_q8_0_ref: per 32 values d = amax/127, id = d ? 1/d : 0,
 *     q = roundf(x*id), d stored as f16 (vx_oracle.c).
 *   - quantize_row_q8_K_ref: per 256 values, max = the value of largest
 *     magnitude (first one on ties), iscale = -127/max, q = min(127,
 *     nearest_int(iscale*x)) with round-half-to-even, d = 1/iscale (fp32),
 *     bsums = sums of 16 consecutive q.
 *   - vec_dot_q8_0_q8_0: sum over blocks of isum * (d_w * d_x).
 *   - vec_dot_q4_K_q8_K: per super-block, with d = d_w*d_x and
 *     dm = dmin_w*d_x: d * sum_j sc_j*isum_j - dm * sum_j m_j*(sum of the 32
 *     q8 of sub-block j).
 *   - vec_dot_q6_K_q8_K: per super-block, (d_w*d_x) * sum_g sc_g*isum_g over
 *     16 groups of 16 values, q6 in [-32, 31].
 * The scaled block terms are formed in fp32 as ggml forms them and summed in
 * fp64 here; ggml itself sums them in fp32 in an order that depends on the
 * SIMD path, so parity is checked against |sum| <= (terms + 4) * 2^-24 * mag,
 * mag = the sum of the terms' magnitudes (vxo_qmatmul returns both).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "vx_oracle.h"

enum { T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

static float f16_at(const uint8_t * p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return vxo_f16_to_f32(h);
}

/* ggml nearest_int: round half to even through the 1.5*2^23 magic number. */
static int nearest_int(float v) {
    const float m = v + 12582912.0f;
    int32_t i;
    memcpy(&i, &m, 4);
    return (i & 0x007fffff) - 0x00400000;
}

void vxo_quantize_row_q8_K(const float * x, int64_t k, float * d, int8_t * q, int16_t * bsums) {
    for (int64_t b = 0; b < k / 256; ++b) {
        const float * xb = x + b * 256;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 256; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                max = xb[j];
            }
        }
        if (amax == 0.0f) {
            d[b] = 0.0f;
            memset(q + b * 256, 0, 256);
            memset(bsums + b * 16, 0, 16 * sizeof(int16_t));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < 256; ++j) {
            const int v = nearest_int(iscale * xb[j]);
            q[b * 256 + j] = (int8_t) (v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int j = 0; j < 16; ++j) s += q[b * 256 + 16 * g + j];
            bsums[b * 16 + g] = (int16_t) s;
        }
        d[b] = 1.0f / iscale;
    }
}

/* Q4_K 6-bit scale and min of sub-block j from the 12 packed bytes. */
static void q4k_scale_min(const uint8_t * s, int j, int * sc, int * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Integer weights of one Q4_K super-block: w[e] in 0..15 for e in 0..255. */
static void q4k_values(const uint8_t * blk, int * w) {
    const uint8_t * qs = blk + 16;
    for (int i = 0; i < 4; ++i)
        for (int l = 0; l < 32; ++l) {
            w[64 * i + l] = qs[32 * i + l] & 0xF;
            w[64 * i + 32 + l] = qs[32 * i + l] >> 4;
        }
}

/* Integer weights of one Q6_K super-block: w[e] in -32..31. */
static void q6k_values(const uint8_t * blk, int * w) {
    for (int h = 0; h < 2; ++h) {
        const uint8_t * ql = blk + 64 * h;
        const uint8_t * qh = blk + 128 + 32 * h;
        for (int l = 0; l < 32; ++l) {
            w[128 * h + l] = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
            w[128 * h + l + 32] = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            w[128 * h + l + 64] = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            w[128 * h + l + 96] = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        }
    }
}

int64_t vxo_qrow_bytes(int32_t type, int64_t k) {
    switch (type) {
        case T_Q8_0: return k / 32 * 34;
        case T_Q4_K: return k / 256 * 144;
        case T_Q6_K: return k / 256 * 210;
        default: return -1;
    }
}

void vxo_dequantize_row_w(int32_t type, const uint8_t * w, int64_t k, float * y) {
    int v[256];
    if (type == T_Q8_0) {
        vxo_dequantize_row_q8_0(w, k, y);
        return;
    }
    for (int64_t b = 0; b < k / 256; ++b) {
        if (type == T_Q4_K) {
            const uint8_t * blk = w + b * 144;
            const float d = f16_at(blk), dmin = f16_at(blk + 2);
            q4k_values(blk, v);
            for (int j = 0; j < 8; ++j) {
                int sc, m;
                q4k_scale_min(blk + 4, j, &sc, &m);
                const float d1 = d * (float) sc, m1 = dmin * (float) m;
                for (int l = 0; l < 32; ++l) y[b * 256 + 32 * j + l] = d1 * (float) v[32 * j + l] - m1;
            }
        } else {
            const uint8_t * blk = w + b * 210;
            const float d = f16_at(blk + 208);
            const int8_t * sc = (const int8_t *) (blk + 192);
            q6k_values(blk, v);
            for (int e = 0; e < 256; ++e) y[b * 256 + e] = d * (float) sc[e / 16] * (float) v[e];
        }
    }
}

/* y[r*n + i] = sum over the blocks of row i of W and row r of x (see the
 * file header); mag[r*n + i] = sum of the terms' magnitudes; returns the
 * number of block terms per output, or -1 for an unknown type. */
int32_t vxo_qmatmul(int32_t type, const uint8_t * w, int32_t n, int32_t k, const float * x, int32_t rows,
                    double * y, double * mag) {
    const int64_t rb = vxo_qrow_bytes(type, k);
    if (rb < 0) return -1;
    int v[256];
    if (type == T_Q8_0) {
        const int nb = k / 32;
        uint8_t xq[34 * 512];  /* k <= 16384 */
        for (int32_t r = 0; r < rows; ++r) {
            vxo_quantize_row_q8_0(x + (int64_t) r * k, k, xq);
            for (int32_t i = 0; i < n; ++i) {
                const uint8_t * wr = w + (int64_t) i * rb;
                double acc = 0.0, m = 0.0;
                for (int b = 0; b < nb; ++b) {
                    int isum = 0;
                    for (int j = 0; j < 32; ++j)
                        isum += (int) (int8_t) wr[34 * b + 2 + j] * (int) (int8_t) xq[34 * b + 2 + j];
                    const float t = (float) isum * (f16_at(wr + 34 * b) * f16_at(xq + 34 * b));
                    acc += t;
                    m += fabs((double) t);
                }
                y[(int64_t) r * n + i] = acc;
                mag[(int64_t) r * n + i] = m;
            }
        }
        return nb;
    }
    const int nb = k / 256;
    float dx[64];
    int8_t qx[256 * 64];
    int16_t bs[16 * 64];  /* k <= 16384 */
    for (int32_t r = 0; r < rows; ++r) {
        vxo_quantize_row_q8_K(x + (int64_t) r * k, k, dx, qx, bs);
        for (int32_t i = 0; i < n; ++i) {
            const uint8_t * wr = w + (int64_t) i * rb;
            double acc = 0.0, m = 0.0;
            for (int b = 0; b < nb; ++b) {
                const int8_t * q8 = qx + 256 * b;
                if (type == T_Q4_K) {
                    const uint8_t * blk = wr + 144 * b;
                    q4k_values(blk, v);
                    int isc = 0, imn = 0;
                    for (int j = 0; j < 8; ++j) {
                        int sc, mn;
                        q4k_scale_min(blk + 4, j, &sc, &mn);
                        int s = 0;
                        for (int l = 0; l < 32; ++l) s += v[32 * j + l] * q8[32 * j + l];
                        isc += sc * s;
                        imn += mn * (bs[16 * b + 2 * j] + bs[16 * b + 2 * j + 1]);
                    }
                    const float d = f16_at(blk) * dx[b];
                    const float dm = f16_at(blk + 2) * dx[b];
                    const float t1 = d * (float) isc, t2 = dm * (float) imn;
                    acc += (double) t1 - (double) t2;
                    m += fabs((double) t1) + fabs((double) t2);
                } else {
                    const uint8_t * blk = wr + 210 * b;
                    const int8_t * sc = (const int8_t *) (blk + 192);
                    q6k_values(blk, v);
                    int is = 0;
                    for (int g = 0; g < 16; ++g) {
                        int s = 0;
                        for (int l = 0; l < 16; ++l) s += v[16 * g + l] * q8[16 * g + l];
                        is += sc[g] * s;
                    }
                    const float t = f16_at(blk + 208) * dx[b] * (float) is;
                    acc += t;
                    m += fabs((double) t);
                }
            }
            y[(int64_t) r * n + i] = acc;
            mag[(int64_t) r * n + i] = m;
        }
    }
    return type == T_Q4_K ? 2 * nb : nb;
}
