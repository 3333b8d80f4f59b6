// tcgen05 form of the quantized-weight product for Q4_K and Q6_K weights
// (vxk_qweight_matmul / _group, include/vxk.h): the same arithmetic as
// vxk_qmm.cu (ggml's CPU path: x quantized like quantize_row_q8_K_ref, exact
// integer block dots, fp32 block factors), for batches where the int8
// mma.sync kernel is bound by instruction issue.
//
// The sub-block scales are folded into the tensor-core operand instead of
// multiplying int32 results: a weight's 4-bit quant q times its 6-bit
// sub-block scale sc is an integer <= 945, exact in f16, and so are the
// quantized activations (|q8| <= 127); the fp32 accumulator of one unit holds
// sum_j sc_j * sum q4*q8 exactly while it stays below 2^24 (mean |q8| < 70).
// Q6_K's scaled quants p = sc*q reach 4096, past f16's exact integers; they
// become two 8-bit operands, hi = floor(p / 64) (s8) and 4 (p mod 64) (u8),
// multiplied by the int8 activations in kind::i8 MMAs (K = 32, int32
// accumulators) that the epilogue combines as 64 D_hi + D_lo / 4, an exact
// int32 sum (the activation tiles of Q6_K matrices are int8).
// Q4_K's mins term sum_j m_j * s_j (s_j = sums of 32 quantized activations)
// is one more K = 16 product: A = (m_0..m_7, 128 m_0..128 m_7), B = (l_0..l_7,
// h_0..h_7) with s_j = 128 h_j + l_j.  Per unit the epilogue applies
// d_x*d_w and d_x*dmin_w in fp32.
//
// CTA = 128 weight rows x a range of 256-column units x one chunk of up to 64
// activation rows (grid z: a product of more rows runs its 64-row chunks side
// by side in one launch); 16 warps:
//   warps 0-3, 12-15  dequant: thread = weight row (TMEM lane; warp w reaches
//               lanes 32 (w % 4) ..); per unit warps 0-3 turn the first half of
//               the row's quant bytes into TMEM columns 0-63 and warps 12-15
//               the second half into columns 64-127 (two dequant warps per
//               scheduler, so one's dependency chains hide behind the
//               other's): f16 pairs sc*q (Q4_K) or int8 quads hi, lo (Q6_K)
//               into TMEM (tcgen05.st); warps 0-3 also write the row's mins
//               row into shared memory (Q4_K)
//   warps 4-7   epilogue: thread = weight row; tcgen05.ld of the unit's
//               accumulators, fp32 block factors into registers
//   warp 8      bulk copies of the raw weight records (HBM stream, evict-first)
//   warp 9      bulk copies of the quantized activations (L2)
//   warps 10-11 tcgen05.mma issuers, warp 10 the even units and warp 11 the
//               odd ones (every buffer and barrier of a unit alternates with
//               its parity): Q4_K 16 kind::f16 MMAs (M = 128, N = rows padded
//               to 16, K = 16, A from TMEM) + 1 mins MMA per unit; Q6_K 2 x 8
//               kind::i8 MMAs (K = 32)
// Column splits of a 128-row block are one thread-block cluster and reduce
// their partial blocks through distributed shared memory, in split order.
#include "vxk_internal.h"
#include "vxk_qtc_quant.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

namespace vxk {
namespace {

constexpr int kThreads = 512;
constexpr int kRawStages = 4;
constexpr int kActStages = 2;  // = 2: a unit's stage is its parity, like its A and D buffers
constexpr int kMaxN = 64;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr unsigned kFull = 0xffffffffu;

// shared-memory map (offsets from a 1024-aligned base)
constexpr int kRawBytes = kQtcRecordBytesQ6K;                      // ring stage: the larger record
constexpr int kActB = kMaxN * 512;                                  // f16 B tile, 4 SW128 atoms
constexpr int kActBMin = kMaxN * 32;                                // mins B tile, 32 B per row (no swizzle)
constexpr int kActStage = kActB + kActBMin;
constexpr int kAMin = 128 * 32;                                     // mins A tile, 32 B per row (no swizzle)
constexpr int kOffRaw = 0;
constexpr int kOffAct = kOffRaw + kRawStages * kRawBytes;
constexpr int kOffAMin = kOffAct + kActStages * kActStage;
constexpr int kOffBar = kOffAMin + 2 * kAMin;
// barriers
constexpr int kBarRawFull = 0;
constexpr int kBarRawEmpty = kBarRawFull + kRawStages;
constexpr int kBarActFull = kBarRawEmpty + kRawStages;
constexpr int kBarActEmpty = kBarActFull + kActStages;
constexpr int kBarAFull = kBarActEmpty + kActStages;   // [2] A (TMEM) + mins A written
constexpr int kBarAEmpty = kBarAFull + 2;              // [2] MMAs of the unit done
constexpr int kBarDFull = kBarAEmpty + 2;              // [2] accumulators complete
constexpr int kBarDEmpty = kBarDFull + 2;              // [2] accumulators read
constexpr int kBarDrain = kBarDEmpty + 2;
constexpr int kNumBars = kBarDrain + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;       // tmem base, abort flag
constexpr int kSmem = kOffMisc + 16 + 1024;            // + alignment slack
static_assert(kSmem <= 232448, "tcgen05 quantized product exceeds 227 KB of shared memory");
static_assert(kActStages == 2, "the two MMA issuers split the units by parity");
static_assert(kRawStages * kRawBytes >= kMaxN * 128 * 4, "the reduction tile fits the raw ring");
static_assert(kOffAct % 1024 == 0 && kActStage % 1024 == 0, "128-byte swizzle atoms align");
// TMEM columns: A[b] 0..255 (128 each), D[b] 256..383, Dmin[b] (Q6_K: D_lo[b]) 384..511
constexpr int kTmemCols = 512;

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait shared by the roles: gives up when another role raised the
// CTA's abort flag, or after kWaitNs (then raises it and sets the error word).
__device__ __forceinline__ bool tc_wait(uint64_t * bar, uint32_t parity, volatile int32_t * abort_flag,
                                        int32_t * err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitNs) {
            *abort_flag = 1;
            if (err) atomicCAS(err, 0, 2);
            return false;
        }
    }
}

// Bounded wait that ignores the abort flag (copies and MMAs already in flight).
__device__ __forceinline__ void tc_drain(uint64_t * bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitNs) return;
    }
}

__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy(bool evict_first) {
    uint64_t policy;
    if (evict_first)
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    else
        asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// The same without swizzle: K-major core matrices of 8 rows x 16 B, lbo
// bytes between the two K halves of a row group, sbo between row groups.
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// D (TMEM) (+)= A (TMEM) . B (shared memory descriptor), kind::f16.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (TMEM) (+)= A (smem) . B (smem), kind::f16.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (TMEM) (+)= A (TMEM) . B (shared memory descriptor), kind::i8 (s32 D).
__device__ __forceinline__ void mma_ts_i8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 columns of 32 bits from registers into TMEM.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 16 columns of 32 bits from TMEM into registers; the caller
// waits (tcgen05.wait::ld) before using them, so several loads overlap.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// The same for 8 columns.
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_dsmem(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}


__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

// Sums column-major partial blocks [cols][R] of the S cluster CTAs (same
// shared-memory offset `local` in each) for elements [4*e0, 4*e1), in split
// order, four rows per load; every split's loads are issued before the sum;
// then adds bias[row0 + row] when bias is given.
template <int R>
__device__ __forceinline__ void cluster_reduce_store(uint32_t local, int S, int e0, int e1, int tid, int nthreads,
                                                     float * y, int64_t n_rows, int64_t row0, const float * bias) {
    const bool vec = (reinterpret_cast<uintptr_t>(y) & 15) == 0;
    for (int e = e0 + tid; e < e1; e += nthreads) {
        float4 v[kQmmMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kQmmMaxSplits; ++sp)
            if (sp < S) v[sp] = ld_dsmem_f32x4(map_dsmem(local + 16u * (uint32_t) e, (uint32_t) sp));
        float4 s = v[0];
#pragma unroll
        for (int sp = 1; sp < kQmmMaxSplits; ++sp)
            if (sp < S) {
                s.x += v[sp].x;
                s.y += v[sp].y;
                s.z += v[sp].z;
                s.w += v[sp].w;
            }
        const int col = (4 * e) / R, row = (4 * e) % R;
        if (bias) {
            const float * b = bias + row0 + row;
            s.x = __fadd_rn(s.x, b[0]);
            s.y = __fadd_rn(s.y, b[1]);
            s.z = __fadd_rn(s.z, b[2]);
            s.w = __fadd_rn(s.w, b[3]);
        }
        float * dst = y + (int64_t) col * n_rows + row0 + row;
        if (vec) {
            *reinterpret_cast<float4 *>(dst) = s;
        } else {
            dst[0] = s.x;
            dst[1] = s.y;
            dst[2] = s.z;
            dst[3] = s.w;
        }
    }
}


__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// ---------------------------------------------------------------------------
// Activation quantization for the tcgen05 product (quantize_row_q8_K_ref):
// f16 B tiles in the K order of tc_position (vxk_qtc_quant.h), the mins B rows
// (l_j, h_j) and d_x.  Grid (units, padded rows / 8), 256 threads: warp w
// quantizes row 8 y + w of unit x, lane L the columns of K positions 8L .. 8L
// + 7; every reduction is a warp shuffle.  Rows are read as float4 (16-byte
// aligned x, checked by the host).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qtc_act_kernel(const QtcParams p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int u = blockIdx.x, lane = threadIdx.x & 31;
    const int rg = blockIdx.y * 8 + (threadIdx.x >> 5);      // padded row over all chunks
    const int chunk = rg / p.npad, r = rg - chunk * p.npad;  // row r of 64-row chunk `chunk`
    const int64_t K = (int64_t) p.n_units * kQmmUnit;
    const int64_t cu = (int64_t) chunk * p.n_units + u;      // this chunk's unit
    // Lane L produces K positions 8L .. 8L + 7 of the unit's tile (one 16-byte
    // chunk): the elements 64g + l .. l + 3 and 64g + 32 + l .. + 3 (g = L / 8,
    // l = 4 (L % 8)) in the position order of tc_position, so it loads two
    // aligned float4 and stores the chunk at once.  x[0..3] = A, x[4..7] = B.
    const int eA = qtc_lane_col_a(lane), eB = eA + 32;  // element (column) indices of the two quads
    float x[8];
    if (rg < p.rows) {
        const float * row = p.x + (int64_t) rg * K + (int64_t) u * kQmmUnit;
        const float4 a = *reinterpret_cast<const float4 *>(row + eA), b = *reinterpret_cast<const float4 *>(row + eB);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        if (p.x_up) {
            const float * up = p.x_up + (int64_t) rg * K + (int64_t) u * kQmmUnit;
            const float4 c = *reinterpret_cast<const float4 *>(up + eA), e = *reinterpret_cast<const float4 *>(up + eB);
            const float uv[8] = {c.x, c.y, c.z, c.w, e.x, e.y, e.z, e.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = swiglu_value(x[i], uv[i]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.0f;
    }
    const int np = p.npad;
    qtc_quantize_unit(x, lane, r, np, p.b_tiles ? p.b_tiles + cu * np * 512 : nullptr,
                      p.bmin_tiles ? p.bmin_tiles + cu * np * 32 : nullptr,
                      p.b8_tiles ? p.b8_tiles + cu * np * 256 : nullptr, p.dx + cu * np + r);
}

// A Q6_K unit of row r into TMEM as int8 operands of kind::i8 MMAs: p = q sc
// (q = q6 - 32, sc the int8 scale of the 16-quant sub-block, |p| <= 4096) is
// split as p = 64 hi + lo with hi = floor(p / 64) in [-64, 64] (s8) and lo =
// p mod 64, stored as 4 lo (u8), hi at columns [abase, abase + 64) and 4 lo at
// [abase + 64, abase + 128); column t holds K positions 4t .. 4t + 3, the
// unit's elements in natural order.  The record holds one quant q6 per byte: a
// mask and a byte permute put the bytes (0, 2) and (1, 3) of a word in the
// 16-bit halves of two pair words, and one 32-bit multiply-add per pair word
// forms both 4 p + 32768 = 4 (q6 - 32) sc + 32768 in [16512, 49152] (no carry
// between the halves), whose high byte is hi + 128 and low byte 4 lo; byte
// permutes gather four of each into a word (hi + 128 turned into hi by
// flipping bit 7).  One call makes half `half` of the row: its elements
// 128 half .. 128 half + 127, hi columns 32 half + t and lo columns 64 + 32
// half + t.
__device__ __forceinline__ void dequant_q6_i8(const uint8_t * raw, int r, uint32_t abase, int half) {
    const uint8_t * qrow = raw + r * 256;
    // the scales of sub-blocks 8 half .. 8 half + 7: bytes 8 half .. of the row's 16
    const uint2 scv = *reinterpret_cast<const uint2 *>(raw + 32768 + r * 16 + 8 * half);
    const uint32_t scw[2] = {scv.x, scv.y};
    {
        uint32_t hi[32], lo[32];  // columns 32 half + t
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const int g = 8 * half + cc;  // sub-block g: chunk g, elements 16g .. 16g + 15
            const uint4 v = *reinterpret_cast<const uint4 *>(qrow + ((g ^ (r & 7)) << 4));
            const int sc = (int) (int8_t) (scw[cc >> 2] >> (8 * (cc & 3)));
            const uint32_t m4 = (uint32_t) (4 * sc);
            const uint32_t c4 = (uint32_t) (32768 - 128 * sc) * 0x00010001u;
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t r02 = (w[k] & 0x00FF00FFu) * m4 + c4;           // elements 4k, 4k + 2
                const uint32_t r13 = __byte_perm(w[k], 0u, 0x4341) * m4 + c4;  // elements 4k + 1, 4k + 3
                hi[4 * cc + k] = __byte_perm(r02, r13, 0x7351) ^ 0x80808080u;
                lo[4 * cc + k] = __byte_perm(r02, r13, 0x6240);
            }
        }
        tmem_st32(abase + 32 * half, hi);
        tmem_st32(abase + 64 + 32 * half, lo);
    }
}

// ---------------------------------------------------------------------------
// The product.
// ---------------------------------------------------------------------------
template <int N>
__global__ void __launch_bounds__(kThreads, 1) qtc_kernel(const QtcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t * bars = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(base + kOffMisc);
    volatile int32_t * abort_flag = reinterpret_cast<volatile int32_t *>(base + kOffMisc + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // this CTA: 128-row block of matrix m, units [u0, u0 + nu)
    QtcMat m = p.mats[0];
#pragma unroll
    for (int i = 1; i < kQmmMaxGroup; ++i)
        if (i < p.n_mats && (int) blockIdx.x >= p.mats[i].block0) m = p.mats[i];
    const int blk = (int) blockIdx.x - m.block0;
    const int split = (int) blockIdx.y;
    const int chunk = (int) blockIdx.z;                    // activation rows chunk * N ..
    const int64_t cbase = (int64_t) chunk * p.n_units;     // this chunk's unit index base
    const int u0 = split * p.units_per_split;
    const int nu = min(p.n_units, u0 + p.units_per_split) - u0;

    if (tid == 0) {
        for (int s = 0; s < kRawStages; ++s) {
            mbar_init(&bars[kBarRawFull + s], 1);
            mbar_init(&bars[kBarRawEmpty + s], 256);  // both dequant groups
        }
        for (int s = 0; s < kActStages; ++s) {
            mbar_init(&bars[kBarActFull + s], 1);
            mbar_init(&bars[kBarActEmpty + s], 1);         // MMA commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[kBarAFull + b], 256);     // both dequant groups
            mbar_init(&bars[kBarAEmpty + b], 1);
            mbar_init(&bars[kBarDFull + b], 1);
            mbar_init(&bars[kBarDEmpty + b], 128);
        }
        mbar_init(&bars[kBarDrain], 2);  // one commit per issuer
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    float * ptile = reinterpret_cast<float *>(base + kOffRaw);  // [N][128] partial block at the end

    if (warp < 4 || warp >= 12) {
        // ---------------- dequant: row r = 32 (warp % 4) + lane, column half hg ----------------
        const int hg = warp >> 3 & 1;  // warps 0-3: columns 0-63, warps 12-15: columns 64-127
        const int r = 32 * (warp & 3) + lane;
        const uint32_t lane_off = (uint32_t) (32 * (warp & 3)) << 16;
        const bool q6 = m.type == 14;
        for (int i = 0; i < nu; ++i) {
            const int s = i % kRawStages;
            if (!__all_sync(kFull, tc_wait(&bars[kBarRawFull + s], (uint32_t) (i / kRawStages) & 1u, abort_flag,
                                           p.error)))
                break;
            const uint8_t * raw = base + kOffRaw + s * kRawBytes;
            {
                const int b = i & 1;  // the A buffer of the unit's parity
                if (!__all_sync(kFull, tc_wait(&bars[kBarAEmpty + b], ((uint32_t) (i >> 1) & 1u) ^ 1u, abort_flag,
                                               p.error)))
                    break;
                tc_fence_after();
                if (q6) {
                    dequant_q6_i8(raw, r, tmem + 128 * b + lane_off, hg);
                } else {
                    const uint4 scm = *reinterpret_cast<const uint4 *>(raw + 16384 + r * 16);  // sc[8], mn[8]
                    const uint32_t mnw[2] = {scm.z, scm.w};
                    // this half's 4 sub-block scales (sub-blocks 4 hg .. 4 hg + 3) as f16
                    // pairs (s, s) by splicing each byte under the exponent of 1024 and
                    // subtracting 1024 (exact for s < 1024)
                    __half2 scl[4], sch[4];
                    {
                        const uint32_t scw = hg ? scm.y : scm.x;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const uint32_t bj = (scw >> (8 * j)) & 0xffu;
                            const uint32_t hb = bj | (bj << 16) | 0x64006400u;
                            scl[j] = __hsub2(*reinterpret_cast<const __half2 *>(&hb), __half2half2(__ushort_as_half(0x6400)));
                            // high nibbles come out as 1024 + 16 q: multiply by s / 16 (exact)
                            sch[j] = __hmul2(scl[j], __half2half2(__ushort_as_half(0x2c00)));
                        }
                    }
                    // 8 chunks of 16 B = 32 quant words -> 128 TMEM columns (4 per word);
                    // this group makes chunks 4 hg .. 4 hg + 3 (columns 64 hg ..).
                    // Word v holds bytes (b0, b1, b2, b3): the low nibbles of b0, b2 and their
                    // high nibbles, then the same of b1, b3 (v >> 8), each pair spliced under
                    // the f16 exponent of 1024 (high nibbles at 16x, which the scale absorbs);
                    // one fused multiply-add per pair removes the 1024 (or 1024 + 0) offset:
                    // (1024 + q) s - 1024 s and (1024 + 16 q) s/16 - 64 s are q s exactly.
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        const int half = 2 * hg + hh;  // columns 32 half ..
                        uint32_t cols[32];
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const int c = 2 * half + cc;  // chunk: words 4c .. 4c+3, group c / 2 = half
                            const uint4 v4 = *reinterpret_cast<const uint4 *>(raw + r * 128 + ((c ^ (r & 7)) << 4));
                            const __half2 slo = scl[2 * hh], shi = sch[2 * hh + 1];
                            const __half2 blo = __hmul2(scl[2 * hh], __half2half2(__ushort_as_half(0xe400)));     // -1024 s
                            const __half2 bhi = __hmul2(scl[2 * hh + 1], __half2half2(__ushort_as_half(0xd400))); // -64 s
                            const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const uint32_t v = vw[k], v8 = v >> 8;
                                const uint32_t h0 = (v & 0x000F000Fu) | 0x64006400u;
                                const uint32_t h1 = (v & 0x00F000F0u) | 0x64006400u;
                                const uint32_t h2 = (v8 & 0x000F000Fu) | 0x64006400u;
                                const uint32_t h3 = (v8 & 0x00F000F0u) | 0x64006400u;
                                cols[16 * cc + 4 * k + 0] = h2_bits(__hfma2(*reinterpret_cast<const __half2 *>(&h0), slo, blo));
                                cols[16 * cc + 4 * k + 1] = h2_bits(__hfma2(*reinterpret_cast<const __half2 *>(&h1), shi, bhi));
                                cols[16 * cc + 4 * k + 2] = h2_bits(__hfma2(*reinterpret_cast<const __half2 *>(&h2), slo, blo));
                                cols[16 * cc + 4 * k + 3] = h2_bits(__hfma2(*reinterpret_cast<const __half2 *>(&h3), shi, bhi));
                            }
                        }
                        tmem_st32(tmem + 128 * b + 32 * half + lane_off, cols);
                    }
                    // mins A row (warps 0-3): K 0..7 = m_j, K 8..15 = 128 m_j (f16, exact); unswizzled
                    // K-major core matrices: row group r / 8 at 256 B, K half at 128 B, row r % 8 at 16 B
                    if (hg == 0) {
                    uint8_t * amin = base + kOffAMin + b * kAMin + (r >> 3) * 256 + (r & 7) * 16;
                    uint32_t m0[4], m1[4];
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const float a0 = (float) ((mnw[(2 * jj) >> 2] >> (8 * ((2 * jj) & 3))) & 0xffu);
                        const float a1 = (float) ((mnw[(2 * jj + 1) >> 2] >> (8 * ((2 * jj + 1) & 3))) & 0xffu);
                        m0[jj] = h2_bits(__floats2half2_rn(a0, a1));
                        m1[jj] = h2_bits(__floats2half2_rn(128.0f * a0, 128.0f * a1));
                    }
                    *reinterpret_cast<uint4 *>(amin) = make_uint4(m0[0], m0[1], m0[2], m0[3]);
                    *reinterpret_cast<uint4 *>(amin + 128) = make_uint4(m1[0], m1[1], m1[2], m1[3]);
                    }
                }
                mbar_arrive(&bars[kBarRawEmpty + s]);  // the unit's raw bytes are read
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                mbar_arrive(&bars[kBarAFull + b]);
            }
        }
    } else if (warp < 8) {
        // ---------------- epilogue: row r = 32 (warp - 4) + lane ----------------
        const int q = warp & 3;
        const int r = 32 * q + lane;
        const uint32_t lane_off = (uint32_t) (32 * q) << 16;
        const uint32_t * dd = reinterpret_cast<const uint32_t *>(m.dd) + ((int64_t) blk * p.n_units + u0) * 128 + r;
        uint32_t ddn = nu > 0 ? __ldg(dd) : 0u;
        // d_x of each unit straight from global memory (written by the
        // quantization kernel: wait for it), so an activation stage is free
        // as soon as its MMAs complete.  Lane l holds d_x of activation rows l
        // and 32 + l (xa, xb), loaded one unit ahead; the FMAs take them by
        // shuffle, so no L2 round trip sits between the accumulators' arrival
        // and their use.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const float * dxu = p.dx + (cbase + u0) * N;
        float xa = 0.0f, xb = 0.0f;
        if (nu > 0) {
            if (lane < N) xa = __ldg(dxu + lane);
            if (N > 32) xb = __ldg(dxu + 32 + lane);
        }
        float acc[N];
#pragma unroll
        for (int j = 0; j < N; ++j) acc[j] = 0.0f;
        for (int i = 0; i < nu; ++i) {
            const int b = i & 1;
            const uint32_t ddc = ddn;
            float na = 0.0f, nb = 0.0f;
            if (i + 1 < nu) {
                ddn = __ldg(dd + (int64_t) (i + 1) * 128);
                if (lane < N) na = __ldg(dxu + (int64_t) (i + 1) * N + lane);
                if (N > 32) nb = __ldg(dxu + (int64_t) (i + 1) * N + 32 + lane);
            }
            const bool ok = tc_wait(&bars[kBarDFull + b], (uint32_t) (i >> 1) & 1u, abort_flag, p.error);
            if (!__all_sync(kFull, ok)) break;
            tc_fence_after();
            const float2 dw = __half22float2(*reinterpret_cast<const __half2 *>(&ddc));  // (d, dmin)
            // d_x of activation row e of this unit
            auto dxe = [&](int e) { return __shfl_sync(kFull, e < 32 ? xa : xb, e & 31); };
            if (m.type == 14) {
                // Q6_K: acc += (d_w * d_x) * (64 D_hi + D_lo / 4), an exact int32 sum;
                // 8 columns of D and D_lo in flight per wait (the 512-thread
                // launch leaves 128 registers a thread, 64 of them acc)
#pragma unroll
                for (int c0 = 0; c0 < N; c0 += 8) {
                    uint32_t v[8], lo[8];
                    tmem_ld8_nowait(tmem + 256 + 64 * b + c0 + lane_off, v);
                    tmem_ld8_nowait(tmem + 384 + 64 * b + c0 + lane_off, lo);
                    tmem_ld_wait();
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        acc[c0 + jj] = fmaf(__fmul_rn(dw.x, dxe(c0 + jj)),
                                            __int2float_rn(64 * (int) v[jj] + ((int) lo[jj] >> 2)), acc[c0 + jj]);
                }
            } else {
                // Q4_K: 8 columns of D and of Dmin in flight per wait
#pragma unroll
                for (int c0 = 0; c0 < N; c0 += 8) {
                    uint32_t v[8], mm[8];
                    tmem_ld8_nowait(tmem + 256 + 64 * b + c0 + lane_off, v);
                    tmem_ld8_nowait(tmem + 384 + 64 * b + c0 + lane_off, mm);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float x = dxe(c0 + j);
                        acc[c0 + j] = fmaf(-__fmul_rn(x, dw.y), __uint_as_float(mm[j]),
                                           fmaf(__fmul_rn(x, dw.x), __uint_as_float(v[j]), acc[c0 + j]));
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[kBarDEmpty + b]);
            xa = na;
            xb = nb;
        }
        // Partial block into the raw ring: every raw read of this CTA happened
        // before the last unit's MMAs, which this thread has waited for.
        if (!*abort_flag) {
#pragma unroll
            for (int j = 0; j < N; ++j) ptile[j * 128 + r] = acc[j];
        }
    } else if (warp == 8) {
        // ---------------- raw weight records (HBM) ----------------
        if (lane == 0) {
            const uint64_t pol = l2_policy(true);
            const uint32_t rec = m.type == 14 ? kQtcRecordBytesQ6K : kQtcRecordBytes;
            const uint8_t * src = m.w + ((int64_t) blk * p.n_units + u0) * rec;
            int i = 0;
            for (; i < nu; ++i) {
                const int s = i % kRawStages;
                if (!tc_wait(&bars[kBarRawEmpty + s], ((uint32_t) (i / kRawStages) & 1u) ^ 1u, abort_flag, p.error))
                    break;
                mbar_expect_tx(&bars[kBarRawFull + s], rec);
                bulk_g2s(base + kOffRaw + s * kRawBytes, src + (int64_t) i * rec, rec, &bars[kBarRawFull + s], pol);
            }
            if (*abort_flag)
                for (int d = i > kRawStages ? i - kRawStages : 0; d < i; ++d)
                    tc_drain(&bars[kBarRawFull + d % kRawStages], (uint32_t) (d / kRawStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---------------- quantized activations (L2), after the producer kernel ----------------
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0) {
            const uint64_t pol = l2_policy(false);
            const bool q6 = m.type == 14;
            int i = 0;
            for (; i < nu; ++i) {
                const int t = i % kActStages, u = u0 + i;
                if (!tc_wait(&bars[kBarActEmpty + t], ((uint32_t) (i / kActStages) & 1u) ^ 1u, abort_flag, p.error))
                    break;
                uint8_t * st = base + kOffAct + t * kActStage;
                if (q6) {  // the int8 tile
                    mbar_expect_tx(&bars[kBarActFull + t], (uint32_t) (N * 256));
                    bulk_g2s(st, p.b8_tiles + (cbase + u) * N * 256, N * 256, &bars[kBarActFull + t], pol);
                } else {   // the f16 tile and the mins tile
                    mbar_expect_tx(&bars[kBarActFull + t], (uint32_t) (N * 512 + N * 32));
                    bulk_g2s(st, p.b_tiles + (cbase + u) * N * 512, N * 512, &bars[kBarActFull + t], pol);
                    bulk_g2s(st + kActB, p.bmin_tiles + (cbase + u) * N * 32, N * 32, &bars[kBarActFull + t], pol);
                }
            }
            if (*abort_flag)
                for (int d = i > kActStages ? i - kActStages : 0; d < i; ++d)
                    tc_drain(&bars[kBarActFull + d % kActStages], (uint32_t) (d / kActStages) & 1u);
        }
        __syncwarp();
    } else if (warp < 12) {
        // ---------------- tcgen05.mma issuers (warps 10, 11) ----------------
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        if (lane == 0) {
            // Q4_K: fp32 D, f16 A and B; Q6_K: s32 D, s8 A and B; both K-major, N, M = 128
            const bool q6 = m.type == 14;
            const uint32_t idesc = q6 ? (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (N >> 3) << 17) |
                                            ((uint32_t) (128 >> 4) << 24)
                                      : (1u << 4) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (128 >> 4) << 24);
            // Q6_K's 4 lo operand is unsigned (u8 A, s8 B)
            const uint32_t idesc_lo = idesc & ~(1u << 7);
            // the units of this issuer's parity
            for (int i = warp - 10; i < nu; i += 2) {
                const int b = i & 1, t = i % kActStages;
                if (!tc_wait(&bars[kBarActFull + t], (uint32_t) (i / kActStages) & 1u, abort_flag, p.error)) break;
                if (!tc_wait(&bars[kBarDEmpty + b], ((uint32_t) (i >> 1) & 1u) ^ 1u, abort_flag, p.error)) break;
                if (!tc_wait(&bars[kBarAFull + b], (uint32_t) (i >> 1) & 1u, abort_flag, p.error)) break;
                tc_fence_after();
                const uint32_t bt = smem_u32(base + kOffAct + t * kActStage);
                const uint32_t dacc = tmem + 256 + 64 * b;
                // descriptors: the stage's base descriptor plus constant offsets (the
                // address field counts 16-byte units), so the issuing thread spends
                // one add per MMA
                const uint64_t bdesc0 = sw128_desc(bt, 16, 1024);
                const uint32_t a0 = tmem + 128 * b;
                if (q6) {
                    // K 32 per MMA (32 bytes of each operand row, like K 16 of f16):
                    // hi into D, lo into D_lo
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        const uint64_t bdesc = bdesc0 + (uint64_t) (((ks >> 2) * N * 128 + (ks & 3) * 32) >> 4);
                        mma_ts_i8(dacc, a0 + 8 * ks, bdesc, idesc, ks != 0);
                        mma_ts_i8(dacc + 128, a0 + 64 + 8 * ks, bdesc, idesc_lo, ks != 0);
                    }
                } else {
#pragma unroll
                    for (int ks = 0; ks < 16; ++ks)
                        mma_ts(dacc, a0 + 8 * ks, bdesc0 + (uint64_t) (((ks >> 2) * N * 128 + (ks & 3) * 32) >> 4),
                               idesc, ks != 0);
                    mma_ss(tmem + 384 + 64 * b, plain_desc(smem_u32(base + kOffAMin + b * kAMin), 128, 256),
                           plain_desc(bt + kActB, 128, 256), idesc, 0);
                }
                tc_commit(&bars[kBarAEmpty + b]);
                tc_commit(&bars[kBarActEmpty + t]);
                tc_commit(&bars[kBarDFull + b]);
            }
            // every MMA issued (by both issuers) completes before the CTA frees TMEM
            tc_commit(&bars[kBarDrain]);
            tc_drain(&bars[kBarDrain], 0);
        }
        __syncwarp();
    }

    // ---- results: the splits of a 128-row block are one cluster; each CTA
    // leaves its partial block [N columns][128 rows] in its own shared memory
    // (the drained raw ring) and, after a cluster barrier, sums slice `split`
    // of the block over all splits in split order (DSMEM).  Every thread of
    // every CTA reaches both cluster barriers. ----
    tc_fence_before();
    __syncthreads();
    const bool live = *abort_flag == 0;
    cluster_sync();
    if (live) {
        const int S = p.n_splits;
        const int rows_c = min(N, p.rows - chunk * N);
        const int E4 = rows_c * 128 / 4;
        const int e0 = (int) ((int64_t) E4 * split / S), e1 = (int) ((int64_t) E4 * (split + 1) / S);
        cluster_reduce_store<128>(smem_u32(ptile), S, e0, e1, tid, kThreads, m.y + (int64_t) chunk * N * m.n_rows,
                                  m.n_rows, (int64_t) blk * 128, m.bias);
    }
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

template <typename K>
cudaError_t launch_ex(K kernel, dim3 grid, unsigned block, size_t smem, cudaStream_t stream, const QtcParams & p,
                      unsigned cluster_y) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = cluster_y;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster_y > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int N>
cudaError_t launch_n(const QtcParams & p, cudaStream_t stream) {
    static bool raised[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!raised[dev]) {
        e = cudaFuncSetAttribute(qtc_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess) return e;
        raised[dev] = true;
    }
    const int blocks = p.mats[p.n_mats - 1].block0 + p.mats[p.n_mats - 1].n_rows / 128;
    return launch_ex(qtc_kernel<N>, dim3((unsigned) blocks, (unsigned) p.n_splits, (unsigned) p.n_chunks), kThreads,
                     kSmem, stream, p, (unsigned) p.n_splits);
}

template <int N>
int clusters_n(int cluster_y) {
    // The answer depends only on the device, the instantiation and the
    // cluster shape: asked of the runtime once, then remembered (the planner
    // asks for every candidate split on every product call).
    static std::atomic<int> memo[64][kQmmMaxSplits + 1];
    static bool raised[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cluster_y < 1 || cluster_y > kQmmMaxSplits) return 0;
    const int known = memo[dev][cluster_y].load(std::memory_order_relaxed);
    if (known > 0) return known;
    if (!raised[dev]) {
        if (cudaFuncSetAttribute(qtc_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
            return 0;
        raised[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1, (unsigned) cluster_y, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned) cluster_y;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, qtc_kernel<N>, &cfg) != cudaSuccess) return 0;
    if (n > 0) memo[dev][cluster_y].store(n, std::memory_order_relaxed);
    return n;
}

}  // namespace

int qtc_max_active_clusters(int npad, int cluster_y) {
    switch (npad) {
        case 16: return clusters_n<16>(cluster_y);
        case 32: return clusters_n<32>(cluster_y);
        default: return clusters_n<64>(cluster_y);
    }
}

cudaError_t launch_qtc(const QtcParams & p, cudaStream_t stream, bool prequantized) {
    if (p.n_chunks < 1 || (p.n_chunks > 1 && p.npad != 64) || p.rows <= p.npad * (p.n_chunks - 1))
        return cudaErrorInvalidValue;
    if (p.n_mats < 1 || p.n_mats > kQmmMaxGroup || p.rows < 1 || p.rows > p.npad * p.n_chunks || p.units_per_split < 1 ||
        p.n_splits < 1 || p.n_splits > kQmmMaxSplits || (int64_t) p.units_per_split * (p.n_splits - 1) >= p.n_units)
        return cudaErrorInvalidValue;
    if (p.npad != 16 && p.npad != 32 && p.npad != 64) return cudaErrorInvalidValue;
    for (int i = 0; i < p.n_mats; ++i) {
        if (p.mats[i].n_rows % 128 != 0) return cudaErrorInvalidValue;
        if (p.mats[i].type == 14 ? !p.b8_tiles : (!p.b_tiles || !p.bmin_tiles)) return cudaErrorInvalidValue;
    }
    if (!p.dx) return cudaErrorInvalidValue;
    if (!prequantized) {
        const cudaError_t e = launch_ex(qtc_act_kernel, dim3((unsigned) p.n_units, (unsigned) (p.npad * p.n_chunks / 8)),
                                        256, 0, stream, p, 1);
        if (e != cudaSuccess) return e;
    }
    switch (p.npad) {
        case 16: return launch_n<16>(p, stream);
        case 32: return launch_n<32>(p, stream);
        default: return launch_n<64>(p, stream);
    }
}

}  // namespace vxk
