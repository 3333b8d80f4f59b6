// Device code shared by the producers of the tcgen05 product's activation
// tiles (vxk_qmm_tc.cu: the quantization kernel; vxk_decoder.cu: the residual
// + RMS norm kernel that quantizes its output rows for the next product):
// quantize_row_q8_K_ref over one 256-column unit of one row, written as the f16
// B tile in the product's K order and the mins B row (operands of Q4_K
// matrices), as the int8 B tile in natural order (operands of Q6_K matrices),
// and d_x.  Included by .cu files only.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace vxk {

// K position (0..255, the order of the tensor-core operands) of element e of a
// 256-column unit.  Dequant word w (quant bytes 4w..4w+3 of the row, group
// g = w/8 of 64 elements, l = 4(w%8)) fills positions 8w..8w+7 with elements
// g*64 + {l, l+2, 32+l, 34+l, l+1, l+3, 33+l, 35+l}: the order in which
// masking the nibbles of one 32-bit word yields f16 pairs.
__device__ __forceinline__ int tc_position(int e) {
    const int g = e >> 6, within = e & 63;
    const int hi = within >= 32;
    const int l = within & 31;
    const int w = 8 * g + (l >> 2);
    const int bb = l & 3;
    const int s = (bb == 0 ? 0 : bb == 2 ? 1 : bb == 1 ? 4 : 5) + (hi ? 2 : 0);
    return 8 * w + s;
}

// Byte offset of K position p of operand row n in a unit tile of `rows` rows:
// 4 atoms of 64 positions, each [rows][128 B] with 128-byte swizzle.
__device__ __forceinline__ int tc_tile_off(int n, int p, int rows) {
    const int a = p >> 6, q = p & 63;
    return a * rows * 128 + (n >> 3) * 1024 + (n & 7) * 128 + ((((q >> 3) ^ (n & 7))) << 4) + (q & 7) * 2;
}

// Byte offset of K position k (0..255, the natural column order) of operand
// row n in an int8 unit tile of `rows` rows: 2 atoms of 128 positions, each
// [rows][128 B] with 128-byte swizzle.
__device__ __forceinline__ int tc8_tile_off(int n, int k, int rows) {
    return (k >> 7) * rows * 128 + (n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 4) & 7) ^ (n & 7)) << 4) + (k & 15);
}

// Columns of a unit that lane L holds: x[0..3] = eA .. eA + 3 and x[4..7] =
// eB .. eB + 3, eA = 64 (L / 8) + 4 (L % 8), eB = eA + 32, i.e. the elements of
// K positions 8L .. 8L + 7 (tc_position), so the lane's tile chunk is one
// 16-byte store.
__device__ __forceinline__ int qtc_lane_col_a(int lane) { return 64 * (lane >> 3) + 4 * (lane & 7); }

// One warp quantizes row r (of np padded rows) of one unit like
// quantize_row_q8_K_ref: iscale = -127 / (the value of largest magnitude,
// first column on ties), q = min(127, round-half-even(iscale x)), d = 1 /
// iscale (0 and all-zero q for a zero row).  Writes, when `tile` is given
// (operands of Q4_K matrices), the lane's 16-byte chunk of the f16 tile (unit
// tile base) and the row's mins B entries (the sums s_j of sub-blocks j = 2g,
// 2g + 1 as (l_j, h_j), s_j = 128 h_j + l_j; unit mins base `bmin`); when
// `tile8` is given (operands of Q6_K matrices), the lane's two 4-byte words of
// the int8 tile in natural column order; and, from lane 0, *dx = d.  Every
// lane of the warp calls it.
__device__ __forceinline__ void qtc_quantize_unit(const float (&x)[8], int lane, int r, int np, uint8_t * tile,
                                                  uint8_t * bmin, uint8_t * tile8, float * dx) {
    constexpr unsigned kAll = 0xffffffffu;
    const int g = lane >> 3;
    const int eA = qtc_lane_col_a(lane), eB = eA + 32;
    // the value of largest magnitude, first column on ties: key = |x| bits, then
    // the inverted column (non-negative floats order as integers)
    unsigned long long key = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int col = (i < 4 ? eA : eB) + (i & 3);
        const unsigned long long kx = ((unsigned long long) __float_as_uint(fabsf(x[i])) << 32) | (unsigned) (255 - col);
        key = kx > key ? kx : key;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(kAll, key, o);
        key = other > key ? other : key;
    }
    const int arg = 255 - (int) (key & 0xffffffffu);
    // the lane holding column arg, and which of its eight values it is
    const int a_within = arg & 63, a_hi = a_within >= 32 ? 1 : 0, a_l = a_within & 31;
    const int a_lane = 8 * (arg >> 6) + (a_l >> 2), a_idx = 4 * a_hi + (a_l & 3);
    float mine = x[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
        if (a_idx == i) mine = x[i];
    const float s_max = __shfl_sync(kAll, mine, a_lane);
    const float amax = __uint_as_float((unsigned) (key >> 32));
    int q[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float d = 0.0f;
    if (amax != 0.0f) {
        const float iscale = __fdiv_rn(-127.0f, s_max);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, x[i])));
        d = __fdiv_rn(1.0f, iscale);
    }
    if (tile8) {
        auto b4 = [](int a, int b, int c, int d) {
            return (uint32_t) (a & 0xff) | ((uint32_t) (b & 0xff) << 8) | ((uint32_t) (c & 0xff) << 16) |
                   ((uint32_t) (d & 0xff) << 24);
        };
        *reinterpret_cast<uint32_t *>(tile8 + tc8_tile_off(r, eA, np)) = b4(q[0], q[1], q[2], q[3]);
        *reinterpret_cast<uint32_t *>(tile8 + tc8_tile_off(r, eB, np)) = b4(q[4], q[5], q[6], q[7]);
    }
    if (lane == 0) *dx = d;
    if (!tile) return;
    // positions 8L + s hold elements A0, A2, B0, B2, A1, A3, B1, B3 (tc_position)
    auto h2 = [](int lo, int hi) {
        const __half2 v = __halves2half2(__int2half_rn(lo), __int2half_rn(hi));
        return *reinterpret_cast<const uint32_t *>(&v);
    };
    *reinterpret_cast<uint4 *>(tile + tc_tile_off(r, 8 * lane, np)) =
        make_uint4(h2(q[0], q[2]), h2(q[4], q[6]), h2(q[1], q[3]), h2(q[5], q[7]));
    // sums of sub-blocks 2g (the A quads) and 2g + 1 (the B quads) over the group's 8 lanes
    int sa = q[0] + q[1] + q[2] + q[3], sb = q[4] + q[5] + q[6] + q[7];
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        sa += __shfl_xor_sync(kAll, sa, o);
        sb += __shfl_xor_sync(kAll, sb, o);
    }
    if ((lane & 7) == 0) {
        // mins row: K position j = l_j, 8 + j = h_j (s_j = 128 h_j + l_j); unswizzled
        // K-major core matrices: row group r / 8 at 256 B, K half at 128 B, row r % 8 at 16 B
        uint8_t * mrow = bmin + (r >> 3) * 256 + (r & 7) * 16;
        *reinterpret_cast<__half *>(mrow + (2 * g) * 2) = __int2half_rn(sa & 127);
        *reinterpret_cast<__half *>(mrow + 128 + (2 * g) * 2) = __int2half_rn(sa >> 7);
        *reinterpret_cast<__half *>(mrow + (2 * g + 1) * 2) = __int2half_rn(sb & 127);
        *reinterpret_cast<__half *>(mrow + 128 + (2 * g + 1) * 2) = __int2half_rn(sb >> 7);
    }
}

}  // namespace vxk
