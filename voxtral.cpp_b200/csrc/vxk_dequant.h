// Element-wise dequantization of GGUF rows, shared by the decoder's
// embedding gather (device) and its load-time time-conditioning product
// (host).  Each value follows the expression order of ggml's CPU
// dequantizers so the results are bit-identical to them: dequantize_row_q8_0
// (y = q * d), dequantize_row_q4_K (d1 = d * sc, m1 = dmin * m, y = d1 * q -
// m1) and dequantize_row_q6_K (y = d * sc * q, left to right).  Products are
// rounded separately (no fused multiply-add).
#pragma once

#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define VXK_HD __host__ __device__ __forceinline__
#else
#define VXK_HD inline
#endif

namespace vxk {

VXK_HD float bits_to_float(uint32_t b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float f;
    memcpy(&f, &b, 4);
    return f;
#endif
}

VXK_HD float mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

VXK_HD float sub_rn(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}

// IEEE binary16 bits -> float (exact).
VXK_HD float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t m = h & 0x3FFu;
    if (e == 0) {
        // zero or subnormal: m * 2^-24, exact in float
        const float v = (float) m * 5.9604644775390625e-08f;
        return (h & 0x8000u) ? -v : v;
    }
    if (e == 31) return bits_to_float(sign | 0x7F800000u | (m << 13));
    return bits_to_float(sign | ((e + 112u) << 23) | (m << 13));
}

VXK_HD float bf16_to_float(uint16_t h) { return bits_to_float((uint32_t) h << 16); }

VXK_HD uint16_t load_u16(const uint8_t * p) { return (uint16_t) (p[0] | (p[1] << 8)); }

// Bytes of one row of `n` values of a ggml type (0 for types not handled here).
VXK_HD int64_t gguf_row_bytes(int type, int64_t n) {
    switch (type) {
    case 0: return n * 4;
    case 1:
    case 30: return n * 2;
    case 8: return n / 32 * 34;
    case 12: return n / 256 * 144;
    case 14: return n / 256 * 210;
    default: return 0;
    }
}

// Value e of a row stored as ggml type `type`.
VXK_HD float dequant_elem(const uint8_t * row, int type, int64_t e) {
    switch (type) {
    case 0: {
        uint32_t b = (uint32_t) row[4 * e] | ((uint32_t) row[4 * e + 1] << 8) | ((uint32_t) row[4 * e + 2] << 16) |
                     ((uint32_t) row[4 * e + 3] << 24);
        return bits_to_float(b);
    }
    case 1: return half_to_float(load_u16(row + 2 * e));
    case 30: return bf16_to_float(load_u16(row + 2 * e));
    case 8: {
        const uint8_t * b = row + (e / 32) * 34;
        const float d = half_to_float(load_u16(b));
        return mul_rn((float) (int8_t) b[2 + e % 32], d);
    }
    case 12: {
        const uint8_t * b = row + (e / 256) * 144;
        const float d = half_to_float(load_u16(b));
        const float dmin = half_to_float(load_u16(b + 2));
        const uint8_t * s = b + 4;
        const int w = (int) (e % 256);
        const int c = w / 64;
        const int hi = (w % 64) >= 32;
        const int l = w % 32;
        const int j = 2 * c + hi;
        int sc, m;
        if (j < 4) {
            sc = s[j] & 63;
            m = s[j + 4] & 63;
        } else {
            sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
            m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
        }
        const uint8_t qb = b[16 + 32 * c + l];
        const int q = hi ? (qb >> 4) : (qb & 0xF);
        const float d1 = mul_rn(d, (float) sc);
        const float m1 = mul_rn(dmin, (float) m);
        return sub_rn(mul_rn(d1, (float) q), m1);
    }
    case 14: {
        const uint8_t * b = row + (e / 256) * 210;
        const uint8_t * ql = b;
        const uint8_t * qh = b + 128;
        const int8_t * sc = reinterpret_cast<const int8_t *>(b + 192);
        const float d = half_to_float(load_u16(b + 208));
        const int w = (int) (e % 256);
        const int n = w / 128;
        const int g = (w % 128) / 32;
        const int l = w % 32;
        const uint8_t qlb = ql[64 * n + l + ((g & 1) ? 32 : 0)];
        const int low = g < 2 ? (qlb & 0xF) : (qlb >> 4);
        const int hb = (qh[32 * n + l] >> (2 * g)) & 3;
        const int q = (low | (hb << 4)) - 32;
        return mul_rn(mul_rn(d, (float) sc[8 * n + l / 16 + 2 * g]), (float) q);
    }
    default: return 0.0f;
    }
}

}  // namespace vxk
