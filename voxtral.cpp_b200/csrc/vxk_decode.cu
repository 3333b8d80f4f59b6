// sm_100a kernels of the decoder KV-cache path:
//   decode_kernel   fused RoPE + K/V append + split-K GQA flash-decoding
//                   attention with an in-kernel combine of the splits
//                   (replaces ggml_rope_ext + ggml_set_rows + ggml_flash_attn_ext
//                   of build_decoder_layer, src/voxtral.cpp:2663-2821)
//   append_kernel   RoPE + append of many tokens (prefill path,
//                   src/voxtral.cpp:2696-2713)
//   table_update_kernel, gather_kernel, compact_kernel: block-table upkeep,
//                   readback and page compaction.
//
// Cache layout (per layer): page-major [n_blocks][n_kv][tile], one tile = the
// 16 positions of one page for one kv head, stored contiguously so a single
// cp.async.bulk brings it into shared memory:
//   f16  tile: 16 rows x 256 B; the 16-byte chunk c of row r is stored at
//        chunk position c ^ (r & 7)  (4096 B)
//   q8_0 tile: 16 rows x 128 B int8 values, chunk c of row r at c ^ (r & 7)
//        (2048 B), then the ggml block scales as f16 [4 blocks][16 rows]
//        (128 B) in a parallel array.  V values are stored as the byte of
//        x + 128 (sign bit flipped); readback restores ggml's int8 bytes.
//   f32  tile: 16 rows x 512 B; chunk c (0-31) of row r stored at
//        c ^ (r & 7)  (8192 B).  The reference's f32 cache (its numerical
//        oracle mode) is exact, so its products run on the CUDA cores in fp32.
// The XOR swizzle makes the ldmatrix reads of the tensor-core tiles
// bank-conflict free without any shared-memory re-layout.
//
// The attention inner products run on the tensor cores with mma.sync
// m16n8k16 (f16 inputs, fp32 accumulation):
//   S^T[head][token] = Q[head][dim] . K^T      (A = Q, 4 real rows of 16)
//   O^T[dim][head]  += V^T[dim][token] . P^T   (B = P, 4 real columns of 8)
// q8_0 tiles are widened to f16 exactly in registers (int8 -> f16 magic
// numbers) and their ggml block scales are applied per 32-value block.
#include "vxk_internal.h"
#include "vxk_qtc_quant.h"

#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>

namespace vxk {
namespace {

constexpr int NT = 128;            // threads per CTA (4 warps)
constexpr int kWarps = NT / 32;
constexpr int kMaxChunkPages = 128;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier wait: 2 s

constexpr int kErrBadPage = 1;
constexpr int kErrTimeout = 2;
constexpr unsigned kFull = 0xffffffffu;

template <int DT> struct Cfg;
// kMinBlocks: resident CTAs per SM the launch bounds ask for.  The q8_0
// kernel is bound by instruction latency (two warps per scheduler left the
// dependency chains of its int8 dots and conversions exposed): three CTAs
// per SM with three stages each (161 registers, no spills) measured 0.83 of
// the copy peak on 128 streams at 8K-32K positions, against 0.75 for two
// CTAs with five stages.
// kTile: bytes of a tile's values; kScale: of its q8_0 block scales; kRec: the
// tile's record in the cache arrays (values, then scales: one bulk copy).
template <> struct Cfg<0> {
    static constexpr int kTile = kBlockTokens * kHeadDim * 4;   // 8192
    static constexpr int kScale = 0;
    static constexpr int kRec = kTile;
    static constexpr int kStages = 3;
    static constexpr int kMinBlocks = 1;
};
template <> struct Cfg<1> {
    static constexpr int kTile = kBlockTokens * kHeadDim * 2;   // 4096
    static constexpr int kScale = 0;
    static constexpr int kRec = kTile;
    static constexpr int kStages = 3;                            // per warp
    static constexpr int kMinBlocks = 2;
};
template <> struct Cfg<8> {
    static constexpr int kTile = kBlockTokens * kHeadDim;       // 2048
    static constexpr int kScale = kBlockTokens * (kHeadDim / kQ8Block) * 2;  // 128
    static constexpr int kRec = kTile + kScale;                             // 2176
    static constexpr int kStages = 3;
    static constexpr int kMinBlocks = 3;
};
template <int DT>
__host__ __device__ constexpr int stage_bytes() { return 2 * (Cfg<DT>::kTile + Cfg<DT>::kScale); }

constexpr int kPwFloats = kBlockTokens * kGroup + kGroup;

template <int DT>
struct __align__(128) Smem {
    uint8_t stage[kWarps][Cfg<DT>::kStages][stage_bytes<DT>()];  // [K tile|K scales|V tile|V scales]
    uint64_t full[kWarps][Cfg<DT>::kStages];
    float merge[kWarps * kGroup * kHeadDim];  // per-warp O^T, then split-combine weights
    uint8_t newk[kHeadDim * (DT == 0 ? 4 : 2)];  // appended row, plain order
    uint8_t newv[kHeadDim * (DT == 0 ? 4 : 2)];
    float qf[DT == 0 ? kGroup * kHeadDim : 1];     // f32: the unit's rotated, scaled queries
    float pw[DT == 0 ? kWarps * kPwFloats : 1];    // f32: per warp P[token][head], then alpha[head]
    uint16_t newk_scale[kHeadDim / kQ8Block];
    uint16_t newv_scale[kHeadDim / kQ8Block];
    float wm[kWarps][kGroup];        // per-warp running max / sum
    float wl[kWarps][kGroup];
    float red_m[kWarps][kGroup];     // combine reductions
    float red_l[kWarps][kGroup];
    int32_t abort_flag;
    int32_t last_flag;
};
static_assert(256 * kGroup <= kWarps * kGroup * kHeadDim, "combine weights fit in the merge buffer");

// Issue-side view of one work unit for one warp: pages of the split, kv head,
// and (per lane j) the page ids of the warp's pages j, j+32, j+64, j+96.
struct IssueUnit {
    int npages;
    int kvh;
    int pid[4];
};
static_assert(kMaxSplitPages <= kWarps * 4 * 32, "page ids per lane cover the largest split");

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

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
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

// Waits for a phase with a time bound; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on an
// mbarrier.  The K/V stream is read once per launch: evict-first in L2.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2,
                                        uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2,
                                          uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A(16x32 s8, row) * B(32x8 s8, col), exact int32 dot products.
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// Exact int8 -> f16 pairs from bytes stored as x + 128 (unsigned): splice
// them under the f16 exponent of 1024 (0x64), subtract 1024 + 128.  `sel`
// picks the two bytes (byte_perm selector with 4 = the 0x64 filler).
__device__ __forceinline__ uint32_t s8pair_to_h2(uint32_t biased, uint32_t sel) {
    const uint32_t h = __byte_perm(biased, 0x64646464u, sel);
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&h), __half2half2(__ushort_as_half(0x6480)));
    return h2_bits(r);
}

// RoPE mode 0 on one adjacent pair, each product and sum rounded on its own
// (ggml CPU rope: dst0 = x0*c - x1*s, dst1 = x0*s + x1*c).
__device__ __forceinline__ float2 rope_pair(float2 x, float2 cs) {
    float2 r;
    r.x = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    r.y = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    return r;
}

__device__ __forceinline__ void set_error(int32_t * err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Byte offset of element pair / chunk inside a swizzled tile row.
__device__ __forceinline__ int f16_chunk_off(int row, int chunk) { return row * 256 + ((chunk ^ (row & 7)) << 4); }
__device__ __forceinline__ int q8_chunk_off(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }
__device__ __forceinline__ int f32_chunk_off(int row, int chunk) { return row * 512 + ((chunk ^ (row & 7)) << 4); }

// ggml quantize_row_q8_0_ref on one 32-value block held as 16 pairs by 16
// consecutive lanes (lane group aligned to 16): d = amax/127,
// id = d ? 1/d : 0, q = roundf(x*id).
__device__ __forceinline__ void q8_pair(float2 x, char2 & q, float & d) {
    float a = fmaxf(fabsf(x.x), fabsf(x.y));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) a = fmaxf(a, __shfl_xor_sync(kFull, a, o));
    d = __fdiv_rn(a, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    q.x = static_cast<signed char>(static_cast<int>(roundf(__fmul_rn(x.x, id))));
    q.y = static_cast<signed char>(static_cast<int>(roundf(__fmul_rn(x.y, id))));
}

// Appends one (token, kv head) row with 128 threads: threads 0-63 rotate and
// store K pairs, threads 64-127 store V pairs, into the swizzled tile.  The
// stored values are also written, in plain order, to shared memory when sk is
// given (the fused decode patches them into its copy of the tile).
template <int DT>
__device__ __forceinline__ void append_head_row(const float * k, const float * v, const float2 * cs,
                                                uint8_t * k_data, uint8_t * v_data, int64_t tile, int tok, uint8_t * sk,
                                                uint8_t * sv, uint16_t * sks, uint16_t * svs) {
    const int tid = threadIdx.x;
    const bool is_k = tid < 64;
    const int i = is_k ? tid : tid - 64;  // pair index 0..63 (dims 2i, 2i+1)
    float2 x = reinterpret_cast<const float2 *>(is_k ? k : v)[i];
    if (is_k) x = rope_pair(x, cs[i]);
    if constexpr (DT == 0) {
        uint8_t * t = (is_k ? k_data : v_data) + tile * Cfg<0>::kTile;
        *reinterpret_cast<float2 *>(t + f32_chunk_off(tok, i >> 1) + (i & 1) * 8) = x;
        if (sk) reinterpret_cast<float2 *>(is_k ? sk : sv)[i] = x;
    } else if constexpr (DT == 1) {
        const __half2 h = __floats2half2_rn(x.x, x.y);
        uint8_t * t = (is_k ? k_data : v_data) + tile * Cfg<1>::kTile;
        *reinterpret_cast<__half2 *>(t + f16_chunk_off(tok, i >> 2) + (i & 3) * 4) = h;
        if (sk) reinterpret_cast<__half2 *>(is_k ? sk : sv)[i] = h;
    } else {
        char2 q;
        float d;
        q8_pair(x, q, d);
        uint8_t * t = (is_k ? k_data : v_data) + tile * Cfg<8>::kRec;
        if (!is_k) {
            // V values are stored with the sign bit flipped (the byte of x + 128):
            // the decode widens them to f16 without an XOR; readback flips back.
            q.x = (signed char) (q.x ^ 0x80);
            q.y = (signed char) (q.y ^ 0x80);
        }
        *reinterpret_cast<char2 *>(t + q8_chunk_off(tok, i >> 3) + (i & 7) * 2) = q;
        if (sk) reinterpret_cast<char2 *>(is_k ? sk : sv)[i] = q;
        if ((i & 15) == 0) {
            const __half dh = __float2half_rn(d);
            const int blk = i >> 4;
            uint8_t * sb = t + Cfg<8>::kTile;  // the record's scales follow its values
            reinterpret_cast<__half *>(sb)[blk * kBlockTokens + tok] = dh;
            if (sks) (is_k ? sks : svs)[blk] = __half_as_ushort(dh);
        }
    }
}

// The 4 heads x 128 dims of (row, kv head) held by thread t as o[h] = dim t of
// head h: staged in `buf` (512 floats) and quantized like
// quantize_row_q8_K_ref into units 2 kvh and 2 kvh + 1 of the next product's
// tiles (vxk_qtc_quant.h), one warp per unit.  Every thread of the CTA calls
// it; `buf` is free again when it returns.
__device__ __forceinline__ void quantize_out(const DecodeParams & p, float * buf, int row, int kvh,
                                             const float (&o)[kGroup]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int h = 0; h < kGroup; ++h) buf[h * kHeadDim + tid] = o[h];
    __syncthreads();
    if (warp < 2) {
        const int eA = qtc_lane_col_a(lane), eB = eA + 32;
        const float * u = buf + warp * 256;
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            x[i] = u[eA + i];
            x[4 + i] = u[eB + i];
        }
        const int np = p.q_npad, chunk = row / np, rr = row - chunk * np;
        const int64_t cu = (int64_t) chunk * p.q_units + 2 * kvh + warp;
        qtc_quantize_unit(x, lane, rr, np, p.q_tiles ? p.q_tiles + cu * np * 512 : nullptr,
                          p.q_bmin ? p.q_bmin + cu * np * 32 : nullptr,
                          p.q_tiles8 ? p.q_tiles8 + cu * np * 256 : nullptr, p.q_dx + cu * np + rr);
    }
    __syncthreads();
}

// Persistent flash-decoding kernel.  Grid = one CTA per resident slot; CTA b
// processes the work units (split, kv head) the host scheduled for it
// (sched_units[sched_offsets[b] .. sched_offsets[b+1]), longest-first greedy),
// one unit after the other.  Each warp streams its share of every unit's
// pages (pages warp, warp+4, ...) through its own ring of ST stages; the ring
// runs ahead across unit boundaries, so the next unit's pages are already in
// flight while the CTA merges and writes the current one.
// QUANT: the output of each (row, kv head) is also quantized into the next
// product's activation tiles (DecodeParams q_*), two 256-column units per kv
// head, by warps 0 and 1 after the row's last split.
template <int DT, bool QUANT>
__global__ void __launch_bounds__(NT, Cfg<DT>::kMinBlocks) decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem<DT> & S = *reinterpret_cast<Smem<DT> *>(smem_raw);
    constexpr int ST = Cfg<DT>::kStages;
    constexpr int TILE = Cfg<DT>::kTile;
    constexpr int SCALE = Cfg<DT>::kScale;
    constexpr int REC = Cfg<DT>::kRec;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int g = lane >> 2;     // mma group: head (QK rows) / dim (PV rows)
    const int c = lane & 3;      // mma thread-in-group: token pair / head pair
    const bool real = lane < 16; // lanes whose QK rows are real heads 0..3
    const int u0 = p.sched_offsets[blockIdx.x];
    const int nu = p.sched_offsets[blockIdx.x + 1] - u0;

    if (tid == 0) {
        for (int w = 0; w < kWarps; ++w)
            for (int s = 0; s < ST; ++s) mbar_init(&S.full[w][s], 1);
        S.abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    // ---- issue side (per warp, warp-uniform control, lane 0 copies) ---------
    const uint64_t policy = evict_first_policy();
    auto share_of = [&](int npages) { return npages > warp ? (npages - warp + kWarps - 1) / kWarps : 0; };
    // Descriptor of unit k for the issuing warp; lane j also fetches the page
    // ids of the warp's pages j + 32 r of that unit (splits <= kMaxSplitPages).
    auto fetch = [&](int k) -> IssueUnit {
        IssueUnit r{0, 0, {0, 0, 0, 0}};
        if (k >= nu) return r;
        const int uid = p.sched_units[u0 + k];
        const WorkItem it = p.items[uid / p.n_kv];
        const int stream = p.rows[it.row].stream;
        r.kvh = uid % p.n_kv;
        r.npages = it.page_end - it.page_begin;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int pi = warp + kWarps * (lane + 32 * j);
            if (pi < r.npages) {
                const int lp = it.page_begin + pi;
                int pg = p.block_table[(int64_t) stream * p.bt_cap + (lp % p.bt_cap)];
                if (pg < 0 || pg >= p.n_blocks) {
                    set_error(p.error, kErrBadPage);
                    pg = 0;
                }
                r.pid[j] = pg;
            }
        }
        return r;
    };
    IssueUnit cur = fetch(0);
    IssueUnit nxt = fetch(1);
    int iu = 0, ipi = 0, seq_issued = 0;
    int ist = 0;  // ring stage of copy seq_issued (seq_issued % ST, kept without a division)
    auto pump = [&](int seq_consumed) {
        while (iu < nu && seq_issued - seq_consumed < ST) {
            if (ipi >= share_of(cur.npages)) {
                ++iu;
                ipi = 0;
                cur = nxt;
                nxt = fetch(iu + 1);
                continue;
            }
            const int hi = ipi >> 5;
            const int reg = hi == 0 ? cur.pid[0] : hi == 1 ? cur.pid[1] : hi == 2 ? cur.pid[2] : cur.pid[3];
            const int pg = __shfl_sync(kFull, reg, ipi & 31);
            if (lane == 0) {
                const int st = ist;
                const int64_t tile = (int64_t) pg * p.n_kv + cur.kvh;
                uint64_t * bar = &S.full[warp][st];
                uint8_t * dst = S.stage[warp][st];
                // one copy per record: the stage is [K values | K scales | V values | V scales]
                mbar_expect_tx(bar, stage_bytes<DT>());
                bulk_g2s(dst, p.k_data + tile * REC, REC, bar, policy);
                bulk_g2s(dst + REC, p.v_data + tile * REC, REC, bar, policy);
            }
            ++seq_issued;
            ist = ist + 1 == ST ? 0 : ist + 1;
            ++ipi;
        }
    };
    pump(0);
    // Programmatic dependent launch: let the next launch on the stream start
    // its prologue (descriptors, block table, first page copies) while this
    // grid drains, and wait for the previous grid only now, before reading
    // the layer inputs (q/k/v) or touching the split scratch.  Both are
    // no-ops for a launch without the programmatic-serialization attribute.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int mi = lane >> 3;    // ldmatrix: matrix index of this lane's row address
    const int mrow = lane & 7;   //           row within that matrix
    int seq_consumed = 0;
    int cst = 0;        // ring stage of seq_consumed
    uint32_t cph = 0;   // and the parity of its fill ((seq_consumed / ST) & 1)
    for (int k = 0; k < nu; ++k) {
        const int uid = p.sched_units[u0 + k];
        const int item_idx = uid / p.n_kv;
        const int kvh = uid % p.n_kv;
        const WorkItem it = p.items[item_idx];
        const RowDesc rd = p.rows[it.row];
        const int last_page = rd.pos / kBlockTokens;
        const int n_pages = it.page_end - it.page_begin;
        const bool do_append = p.fuse_append && (rd.flags & kRowAppend) && (it.page_end - 1 == last_page);
        pump(seq_consumed);

        // Query fragments (A operand rows = heads; lanes 16-31 hold zero rows).
        // f16: a0 = dims 16ks+2c,+1 and a2 = dims 16ks+8+2c,+1 (mma k order);
        // q8_0: a0 = dims 16ks+4c,+1 and a2 = dims 16ks+4c+2,+3, the k order the
        // int8 ldmatrix delivers.  Scale*log2(e) is folded in.
        // f16: qa[ks] = the f16 A fragment (dims 16ks+2c,+1 | 16ks+8+2c,+1).
        // q8_0: the scores use exact int8 tensor-core dot products with the
        // int8 cache; each head's rotated, scaled query is split into two
        // int8 parts, q ~= qs * (254 * hi + lo) with qs = amax / (127 * 254),
        // hi in A rows 0-7 and lo in the (otherwise padding) rows 8-15, so one
        // m16n8k32 product yields both dots.  qa[ks][0] = hi, qa[ks][1] = lo
        // for dims 16ks+4c .. 16ks+4c+3 (the k order of the int8 ldmatrix).
        uint32_t qa[8][2];
        float qs = 0.0f;
        {
            const float * qrow = p.q + ((int64_t) it.row * p.n_q + (int64_t) kvh * kGroup + (g & 3)) * kHeadDim;
            const float2 * cs = p.rope + (int64_t) rd.pos * (kHeadDim / 2);
            if constexpr (DT == 0) {
                // the unit's four query heads, rotated and scaled, for all warps:
                // warp w writes head w (the previous unit's readers have passed
                // the barriers that end it)
                const float * qh = p.q + ((int64_t) it.row * p.n_q + (int64_t) kvh * kGroup + warp) * kHeadDim;
#pragma unroll
                for (int j = lane; j < kHeadDim / 2; j += 32) {
                    const float2 r = rope_pair(*reinterpret_cast<const float2 *>(qh + 2 * j), cs[j]);
                    *reinterpret_cast<float2 *>(S.qf + warp * kHeadDim + 2 * j) =
                        make_float2(r.x * p.scale_log2, r.y * p.scale_log2);
                }
                (void) qrow;
            } else if constexpr (DT == 1) {
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const int d0 = 16 * ks + 2 * c;
                    const int d1 = 16 * ks + 8 + 2 * c;
                    uint32_t v0 = 0, v1 = 0;
                    if (real) {
                        const float2 r0 = rope_pair(*reinterpret_cast<const float2 *>(qrow + d0), cs[d0 >> 1]);
                        const float2 r1 = rope_pair(*reinterpret_cast<const float2 *>(qrow + d1), cs[d1 >> 1]);
                        v0 = h2_bits(__floats2half2_rn(r0.x * p.scale_log2, r0.y * p.scale_log2));
                        v1 = h2_bits(__floats2half2_rn(r1.x * p.scale_log2, r1.y * p.scale_log2));
                    }
                    qa[ks][0] = v0;
                    qa[ks][1] = v1;
                }
            } else {
                float qv[8][4];
                float amax = 0.0f;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const int d0 = 16 * ks + 4 * c;
                    float2 r0 = make_float2(0.0f, 0.0f), r1 = make_float2(0.0f, 0.0f);
                    if (real) {
                        r0 = rope_pair(*reinterpret_cast<const float2 *>(qrow + d0), cs[d0 >> 1]);
                        r1 = rope_pair(*reinterpret_cast<const float2 *>(qrow + d0 + 2), cs[(d0 >> 1) + 1]);
                    }
                    qv[ks][0] = r0.x * p.scale_log2;
                    qv[ks][1] = r0.y * p.scale_log2;
                    qv[ks][2] = r1.x * p.scale_log2;
                    qv[ks][3] = r1.y * p.scale_log2;
#pragma unroll
                    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fabsf(qv[ks][j]));
                }
                // the head's 128 dims sit in the 4 lanes of one mma group
                amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
                const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
                qs = amax > 0.0f ? amax / (127.0f * 254.0f) : 0.0f;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    uint32_t hi = 0, lo = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float x = qv[ks][j] * inv;
                        const float h = rintf(x);                 // |h| <= 127
                        const float l = rintf((x - h) * 254.0f);  // |x - h| <= 1/2: |l| <= 127
                        hi |= ((uint32_t) (int32_t) h & 0xffu) << (8 * j);
                        lo |= ((uint32_t) (int32_t) l & 0xffu) << (8 * j);
                    }
                    qa[ks][0] = hi;
                    qa[ks][1] = lo;
                }
            }
        }
        if (do_append) {
            const int lp = last_page;
            int pg = p.block_table[(int64_t) rd.stream * p.bt_cap + (lp % p.bt_cap)];
            if (pg < 0 || pg >= p.n_blocks) {
                set_error(p.error, kErrBadPage);
                pg = 0;
            }
            const int64_t tile = (int64_t) pg * p.n_kv + kvh;
            const int64_t krow = ((int64_t) it.row * p.n_kv + kvh) * kHeadDim;
            append_head_row<DT>(p.k + krow, p.v + krow, p.rope + (int64_t) rd.pos * (kHeadDim / 2), p.k_data,
                                p.v_data, tile, rd.pos % kBlockTokens, S.newk, S.newv,
                                S.newk_scale, S.newv_scale);
        }
        __syncthreads();

        const int share = share_of(n_pages);
        // Replaces the stale copy of the appended row in a stage by the new values.
        auto patch = [&](uint8_t * sk, uint8_t * sv) {
            // Replace the stale copy of the appended row by the new values.
            const int t = rd.pos % kBlockTokens;
            if constexpr (DT == 0) {
                *reinterpret_cast<uint4 *>(sk + f32_chunk_off(t, lane)) =
                    *reinterpret_cast<const uint4 *>(S.newk + lane * 16);
                *reinterpret_cast<uint4 *>(sv + f32_chunk_off(t, lane)) =
                    *reinterpret_cast<const uint4 *>(S.newv + lane * 16);
            } else if constexpr (DT == 1) {
                const int ch = lane & 15;
                const uint4 val = *reinterpret_cast<const uint4 *>((lane < 16 ? S.newk : S.newv) + ch * 16);
                *reinterpret_cast<uint4 *>((lane < 16 ? sk : sv) + f16_chunk_off(t, ch)) = val;
            } else {
                if (lane < 16) {
                    const int ch = lane & 7;
                    const uint4 val = *reinterpret_cast<const uint4 *>((lane < 8 ? S.newk : S.newv) + ch * 16);
                    *reinterpret_cast<uint4 *>((lane < 8 ? sk : sv) + q8_chunk_off(t, ch)) = val;
                } else if (lane < 24) {
                    const int b = lane & 3;
                    const bool kk = lane < 20;
                    reinterpret_cast<uint16_t *>((kk ? sk : sv) + TILE)[b * kBlockTokens + t] =
                        kk ? S.newk_scale[b] : S.newv_scale[b];
                }
            }
            // The stage is refilled by the bulk-copy (async) proxy later:
            // order these generic-proxy writes before that.
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        };
        if constexpr (DT == 0) {
            // ---- f32 cache: fp32 products on the CUDA cores ---------------
            // Scores: lane (t = lane & 15, hp = lane >> 4) computes heads 2hp
            // and 2hp + 1 against token t of the page (its K row from shared
            // memory, the queries broadcast from S.qf).  Values: lane owns
            // dims 4 lane .. 4 lane + 3 of all four heads; the page's
            // probabilities and the rescale factors pass through S.pw.
            const int t = lane & 15;
            const int hp = lane >> 4;
            float m2[2] = {-INFINITY, -INFINITY};
            float l2[2] = {0.0f, 0.0f};
            float of[kGroup][4];
#pragma unroll
            for (int h = 0; h < kGroup; ++h) of[h][0] = of[h][1] = of[h][2] = of[h][3] = 0.0f;
            float * pw = S.pw + warp * kPwFloats;  // [token][head], then alpha[head]
            const float * qa0 = S.qf + (2 * hp) * kHeadDim;
            const float * qa1 = qa0 + kHeadDim;
            for (int i = 0; i < share; ++i) {
                const bool ready = mbar_wait(&S.full[warp][cst], cph, kWaitNs);
                if (!__all_sync(kFull, ready)) {
                    S.abort_flag = 1;
                    break;
                }
                const int lp = it.page_begin + warp + kWarps * i;
                uint8_t * sk = S.stage[warp][cst];
                uint8_t * sv = sk + TILE;
                if (do_append && lp == last_page) patch(sk, sv);
                float s0 = 0.0f, s1 = 0.0f;
#pragma unroll 8
                for (int ch = 0; ch < kHeadDim / 4; ++ch) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(sk + f32_chunk_off(t, ch));
                    const float4 a = *reinterpret_cast<const float4 *>(qa0 + 4 * ch);
                    const float4 b = *reinterpret_cast<const float4 *>(qa1 + 4 * ch);
                    s0 = fmaf(a.x, k4.x, s0);
                    s0 = fmaf(a.y, k4.y, s0);
                    s0 = fmaf(a.z, k4.z, s0);
                    s0 = fmaf(a.w, k4.w, s0);
                    s1 = fmaf(b.x, k4.x, s1);
                    s1 = fmaf(b.y, k4.y, s1);
                    s1 = fmaf(b.z, k4.z, s1);
                    s1 = fmaf(b.w, k4.w, s1);
                }
                const int pos = lp * kBlockTokens + t;
                if (pos < rd.win_start || pos > rd.pos) s0 = s1 = -INFINITY;
                float mx0 = s0, mx1 = s1;
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, o));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, o));
                }
                // every page of a split holds at least one position of the window
                const float mn0 = fmaxf(m2[0], mx0), mn1 = fmaxf(m2[1], mx1);
                const float al0 = exp2f(m2[0] - mn0), al1 = exp2f(m2[1] - mn1);
                const float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1);
                m2[0] = mn0;
                m2[1] = mn1;
                l2[0] = l2[0] * al0 + p0;
                l2[1] = l2[1] * al1 + p1;
                *reinterpret_cast<float2 *>(pw + t * kGroup + 2 * hp) = make_float2(p0, p1);
                if (t == 0) *reinterpret_cast<float2 *>(pw + kBlockTokens * kGroup + 2 * hp) = make_float2(al0, al1);
                __syncwarp();
                const float4 al = *reinterpret_cast<const float4 *>(pw + kBlockTokens * kGroup);
                const float alv[kGroup] = {al.x, al.y, al.z, al.w};
#pragma unroll
                for (int h = 0; h < kGroup; ++h) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) of[h][j] *= alv[h];
                }
#pragma unroll
                for (int tt = 0; tt < kBlockTokens; ++tt) {
                    const float4 v4 = *reinterpret_cast<const float4 *>(sv + f32_chunk_off(tt, lane));
                    const float4 pp = *reinterpret_cast<const float4 *>(pw + tt * kGroup);
                    const float pv[kGroup] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) {
                        of[h][0] = fmaf(pv[h], v4.x, of[h][0]);
                        of[h][1] = fmaf(pv[h], v4.y, of[h][1]);
                        of[h][2] = fmaf(pv[h], v4.z, of[h][2]);
                        of[h][3] = fmaf(pv[h], v4.w, of[h][3]);
                    }
                }
                __syncwarp();  // pw is rewritten by the next page
                ++seq_consumed;
                cst = cst + 1 == ST ? 0 : cst + 1;
                if (cst == 0) cph ^= 1u;
                pump(seq_consumed);
            }
            // ---- this warp's softmax state and O for the merge -----------------
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                l2[0] += __shfl_xor_sync(kFull, l2[0], o);
                l2[1] += __shfl_xor_sync(kFull, l2[1], o);
            }
            if (t == 0) {
                S.wm[warp][2 * hp] = m2[0];
                S.wm[warp][2 * hp + 1] = m2[1];
                S.wl[warp][2 * hp] = l2[0];
                S.wl[warp][2 * hp + 1] = l2[1];
            }
#pragma unroll
            for (int h = 0; h < kGroup; ++h)
                *reinterpret_cast<float4 *>(S.merge + (warp * kGroup + h) * kHeadDim + 4 * lane) =
                    make_float4(of[h][0], of[h][1], of[h][2], of[h][3]);
        } else {
            float o[8][4];
    #pragma unroll
            for (int mb = 0; mb < 8; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.0f;
            float m_run = -INFINITY;
            float l_part = 0.0f;
            // This lane's scores of head g for tokens 2c, 2c+1, 8+2c, 9+2c of one
            // page (log2 domain), masked to the row's window.
            auto page_scores = [&](const uint8_t * sk, int lp, float (&sc)[4]) {
                // ---- S^T = Q K^T for the page's 16 tokens (two n-blocks of 8) ---
                float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                float s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                const uint32_t kbase = smem_u32(sk);
                if constexpr (DT == 1) {
                    const int row = mrow + ((mi >> 1) << 3);
    #pragma unroll
                    for (int ks = 0; ks < 8; ++ks) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4(kbase + f16_chunk_off(row, 2 * ks + (mi & 1)), b0, b1, b2, b3);
                        mma16816(s0, qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
                        mma16816(s1, qa[ks][0], 0u, qa[ks][1], 0u, b2, b3);
                    }
                } else {
                    const int row = mrow + ((mi & 1) << 3);
                    const __half2 * dk = reinterpret_cast<const __half2 *>(sk + TILE);
    #pragma unroll
                    for (int blk = 0; blk < 4; ++blk) {
                        // w0 / w2: tokens 0-7, dims 0-15 / 16-31 of the block; w1 / w3: tokens 8-15
                        uint32_t w0, w1, w2, w3;
                        ldsm_x4(kbase + q8_chunk_off(row, 2 * blk + (mi >> 1)), w0, w1, w2, w3);
                        int t0[4], t1[4];
                        imma16832(t0, qa[2 * blk][0], qa[2 * blk][1], qa[2 * blk + 1][0], qa[2 * blk + 1][1], w0, w2);
                        imma16832(t1, qa[2 * blk][0], qa[2 * blk][1], qa[2 * blk + 1][0], qa[2 * blk + 1][1], w1, w3);
                        // t[0], t[1]: hi dots of head g, tokens 2c, 2c+1; t[2], t[3]: lo dots
                        const float2 d01 = __half22float2(dk[(blk * kBlockTokens + 2 * c) >> 1]);
                        const float2 d89 = __half22float2(dk[(blk * kBlockTokens + 8 + 2 * c) >> 1]);
                        s0[0] = fmaf((float) (t0[0] * 254 + t0[2]), d01.x, s0[0]);
                        s0[1] = fmaf((float) (t0[1] * 254 + t0[3]), d01.y, s0[1]);
                        s1[0] = fmaf((float) (t1[0] * 254 + t1[2]), d89.x, s1[0]);
                        s1[1] = fmaf((float) (t1[1] * 254 + t1[3]), d89.y, s1[1]);
                    }
                    s0[0] *= qs;
                    s0[1] *= qs;
                    s1[0] *= qs;
                    s1[1] *= qs;
                }

                const int tp = lp * kBlockTokens;
                sc[0] = s0[0];
                sc[1] = s0[1];
                sc[2] = s1[0];
                sc[3] = s1[1];
                // Only a page that the window cuts (a split's first page when the
                // ring has slid, the row's last page) needs the position mask; the
                // test is warp-uniform.  Lanes 16-31 (padding heads) are not
                // masked: their probabilities are forced to 0 below and they never
                // meet the real lanes in a reduction.
                if (tp < rd.win_start || tp + kBlockTokens - 1 > rd.pos) {
                    const int tk[4] = {2 * c, 2 * c + 1, 8 + 2 * c, 9 + 2 * c};
    #pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int pos = tp + tk[j];
                        if (pos < rd.win_start || pos > rd.pos) sc[j] = -INFINITY;
                    }
                }
            };
            // O^T += V^T P^T for one page, P as f16 pairs (tokens 2c,2c+1 | 8+2c,9+2c).
            auto page_values = [&](const uint8_t * sv, __half2 p01, __half2 p89) {
                // ---- O^T += V^T P^T ---------------------------------------------
                const uint32_t vbase = smem_u32(sv);
                if constexpr (DT == 1) {
                    const uint32_t b0 = h2_bits(p01), b1 = h2_bits(p89);
                    const int row = mrow + ((mi >> 1) << 3);
    #pragma unroll
                    for (int mb = 0; mb < 8; ++mb) {
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_t(vbase + f16_chunk_off(row, 2 * mb + (mi & 1)), a0, a1, a2, a3);
                        mma16816(o[mb], a0, a1, a2, a3, b0, b1);
                    }
                } else {
                    const int row = mrow + ((mi & 1) << 3);
                    const __half2 * dv = reinterpret_cast<const __half2 *>(sv + TILE);
                    // P as rounded for the row sum, x128 (exact) to keep P * d in the
                    // f16 normal range; the block scale is folded in with one f16 rounding
                    const __half2 p01s = __hmul2(p01, __float2half2_rn(128.0f));
                    const __half2 p89s = __hmul2(p89, __float2half2_rn(128.0f));
    #pragma unroll
                    for (int blk = 0; blk < 4; ++blk) {
                        const uint32_t b0 = h2_bits(__hmul2(p01s, dv[(blk * kBlockTokens + 2 * c) >> 1]));
                        const uint32_t b1 = h2_bits(__hmul2(p89s, dv[(blk * kBlockTokens + 8 + 2 * c) >> 1]));
                        uint32_t w0, w1, w2, w3;
                        ldsm_x4_t(vbase + q8_chunk_off(row, 2 * blk + (mi >> 1)), w0, w1, w2, w3);
                        mma16816(o[2 * blk], s8pair_to_h2(w0, 0x4240u), s8pair_to_h2(w0, 0x4341u),
                                 s8pair_to_h2(w1, 0x4240u), s8pair_to_h2(w1, 0x4341u), b0, b1);
                        mma16816(o[2 * blk + 1], s8pair_to_h2(w2, 0x4240u), s8pair_to_h2(w2, 0x4341u),
                                 s8pair_to_h2(w3, 0x4240u), s8pair_to_h2(w3, 0x4341u), b0, b1);
                    }
                }
            };
            // Pages are consumed one at a time (f16) or two at a time (q8_0: the two
            // pages' score, softmax and value work interleave, and the softmax
            // bookkeeping is shared).
            int i = 0;
            while (i < share) {
                const bool two = DT == 8 && i + 1 < share;
                const int stA = cst;
                const bool wrapA = cst + 1 == ST;
                const int stB = wrapA ? 0 : cst + 1;
                const uint32_t phB = wrapA ? cph ^ 1u : cph;
                bool ready = mbar_wait(&S.full[warp][stA], cph, kWaitNs);
                if (two) ready = ready && mbar_wait(&S.full[warp][stB], phB, kWaitNs);
                // the outcome is made warp-uniform so the warp never splits
                if (!__all_sync(kFull, ready)) {
                    S.abort_flag = 1;
                    break;
                }
                const int lpA = it.page_begin + warp + kWarps * i;
                const int lpB = lpA + kWarps;
                uint8_t * skA = S.stage[warp][stA];
                uint8_t * skB = S.stage[warp][stB];
                if (do_append && lpA == last_page) patch(skA, skA + TILE + SCALE);
                if (two && do_append && lpB == last_page) patch(skB, skB + TILE + SCALE);
                float scA[4], scB[4];
                page_scores(skA, lpA, scA);
                if (two) {
                    page_scores(skB, lpB, scB);
                } else {
    #pragma unroll
                    for (int j = 0; j < 4; ++j) scB[j] = -INFINITY;
                }

                // ---- online softmax (log2 domain) for head g --------------------
                float mx = fmaxf(fmaxf(fmaxf(scA[0], scA[1]), fmaxf(scA[2], scA[3])),
                                 fmaxf(fmaxf(scB[0], scB[1]), fmaxf(scB[2], scB[3])));
                mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
                const float m_new = fmaxf(m_run, mx);
                const float alpha = real ? exp2f(m_run - m_new) : 1.0f;
                float prA[4], prB[4];
    #pragma unroll
                for (int j = 0; j < 4; ++j) {
                    prA[j] = real ? exp2f(scA[j] - m_new) : 0.0f;
                    prB[j] = real ? exp2f(scB[j] - m_new) : 0.0f;
                }
                if (real) m_run = m_new;
                const __half2 p01A = __floats2half2_rn(prA[0], prA[1]);
                const __half2 p89A = __floats2half2_rn(prA[2], prA[3]);
                const __half2 p01B = __floats2half2_rn(prB[0], prB[1]);
                const __half2 p89B = __floats2half2_rn(prB[2], prB[3]);
                {
                    const float2 f0 = __half22float2(p01A), f1 = __half22float2(p89A);
                    float add = (f0.x + f0.y) + (f1.x + f1.y);
                    if (two) {
                        const float2 g0 = __half22float2(p01B), g1 = __half22float2(p89B);
                        add += (g0.x + g0.y) + (g1.x + g1.y);
                    }
                    l_part = l_part * alpha + add;
                }
                // rescale O^T columns (heads 2c, 2c+1) when any running max moved
                if (__any_sync(kFull, alpha != 1.0f)) {
                    const float a_lo = __shfl_sync(kFull, alpha, (8 * c) & 31);
                    const float a_hi = __shfl_sync(kFull, alpha, (8 * c + 4) & 31);
    #pragma unroll
                    for (int mb = 0; mb < 8; ++mb) {
                        o[mb][0] *= a_lo;
                        o[mb][1] *= a_hi;
                        o[mb][2] *= a_lo;
                        o[mb][3] *= a_hi;
                    }
                }
                page_values(skA + TILE + SCALE, p01A, p89A);
                if (two) page_values(skB + TILE + SCALE, p01B, p89B);
                __syncwarp();
                seq_consumed += two ? 2 : 1;
                if (two) {
                    const bool wrapB = stB + 1 == ST;
                    cst = wrapB ? 0 : stB + 1;
                    cph = wrapB ? phB ^ 1u : phB;
                } else {
                    cst = stB;
                    cph = phB;
                }
                i += two ? 2 : 1;
                pump(seq_consumed);
            }

            // ---- merge the 4 warps' partial softmax states -----------------------
            {
                float l_h = l_part + __shfl_xor_sync(kFull, l_part, 1);
                l_h += __shfl_xor_sync(kFull, l_h, 2);
                if (real && c == 0) {
                    S.wm[warp][g] = m_run;
                    S.wl[warp][g] = l_h;
                }
                if (c < 2) {
                    const float post = DT == 1 ? 1.0f : 1.0f / 128.0f;
    #pragma unroll
                    for (int mb = 0; mb < 8; ++mb) {
                        const int d0 = DT == 1 ? 16 * mb + g : 16 * mb + 2 * g;
                        const int d1 = DT == 1 ? 16 * mb + 8 + g : 16 * mb + 2 * g + 1;
                        float * h0 = S.merge + (warp * kGroup + 2 * c) * kHeadDim;
                        float * h1 = h0 + kHeadDim;
                        h0[d0] = o[mb][0] * post;
                        h1[d0] = o[mb][1] * post;
                        h0[d1] = o[mb][2] * post;
                        h1[d1] = o[mb][3] * post;
                    }
                }
            }
        }
        __syncthreads();
        if (S.abort_flag) {
            // Drain this warp's copies still in flight (bounded) before exiting.
            if (lane == 0) {
                for (int l = seq_consumed; l < seq_issued; ++l) mbar_wait(&S.full[warp][l % ST], (l / ST) & 1, kWaitNs);
                set_error(p.error, kErrTimeout);
            }
            return;
        }
        float M[kGroup], Lsum[kGroup], O[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            float mm = S.wm[0][h];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) mm = fmaxf(mm, S.wm[w][h]);
            float ls = 0.0f, os = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float wt = exp2f(S.wm[w][h] - mm);  // 0 for warps without pages
                ls += S.wl[w][h] * wt;
                os += S.merge[(w * kGroup + h) * kHeadDim + tid] * wt;
            }
            M[h] = mm;
            Lsum[h] = ls;
            O[h] = os;
        }
        // every thread has read the merge buffer before it is reused below
        __syncthreads();

        const int64_t out_base = ((int64_t) it.row * p.n_q + (int64_t) kvh * kGroup) * kHeadDim;
        if (rd.n_chunks == 1) {
            if constexpr (QUANT) {
                float o[kGroup];
#pragma unroll
                for (int h = 0; h < kGroup; ++h) o[h] = O[h] / Lsum[h];
                if (p.out)
#pragma unroll
                    for (int h = 0; h < kGroup; ++h) p.out[out_base + h * kHeadDim + tid] = o[h];
                quantize_out(p, S.merge, it.row, kvh, o);
            } else {
#pragma unroll
                for (int h = 0; h < kGroup; ++h) p.out[out_base + h * kHeadDim + tid] = O[h] / Lsum[h];
            }
            continue;
        }
        {
            float * part = p.partials + ((int64_t) item_idx * p.n_q + (int64_t) kvh * kGroup) * kPartialStride;
#pragma unroll
            for (int h = 0; h < kGroup; ++h) part[h * kPartialStride + tid] = O[h];
            if (tid < kGroup) {
                part[tid * kPartialStride + kHeadDim] = M[tid];
                part[tid * kPartialStride + kHeadDim + 1] = Lsum[tid];
            }
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const int prev = atomicAdd(&p.counters[it.row * p.n_kv + kvh], 1);
            S.last_flag = (prev == rd.n_chunks - 1);
        }
        __syncthreads();
        if (!S.last_flag) continue;
        __threadfence();

        // ---- last split of the (row, kv head): combine all splits -----------
        const int nc = rd.n_chunks;
        float * comb_w = S.merge;  // [split][head] weights
        auto part_at = [&](int cc, int h) -> const float * {
            return p.partials + ((int64_t) (rd.item_base + cc) * p.n_q + (int64_t) kvh * kGroup + h) * kPartialStride;
        };
        float lm[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) lm[h] = -INFINITY;
        for (int cc = tid; cc < nc; cc += NT) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h) lm[h] = fmaxf(lm[h], __ldcg(part_at(cc, h) + kHeadDim));
        }
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) lm[h] = fmaxf(lm[h], __shfl_xor_sync(kFull, lm[h], off));
        }
        if (lane == 0) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h) S.red_m[warp][h] = lm[h];
        }
        __syncthreads();
        float Mx[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            Mx[h] = S.red_m[0][h];
#pragma unroll
            for (int w = 1; w < kWarps; ++w) Mx[h] = fmaxf(Mx[h], S.red_m[w][h]);
        }
        float ls[kGroup] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int cc = tid; cc < nc; cc += NT) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h) {
                const float * pc = part_at(cc, h);
                const float w = exp2f(__ldcg(pc + kHeadDim) - Mx[h]);
                ls[h] += __ldcg(pc + kHeadDim + 1) * w;
                comb_w[cc * kGroup + h] = w;
            }
        }
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) ls[h] += __shfl_xor_sync(kFull, ls[h], off);
        }
        if (lane == 0) {
#pragma unroll
            for (int h = 0; h < kGroup; ++h) S.red_l[warp][h] = ls[h];
        }
        __syncthreads();
        float o[kGroup];
#pragma unroll
        for (int h = 0; h < kGroup; ++h) {
            float Lt = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) Lt += S.red_l[w][h];
            float acc = 0.0f;
            for (int cc = 0; cc < nc; ++cc) acc = fmaf(comb_w[cc * kGroup + h], __ldcg(part_at(cc, h) + tid), acc);
            o[h] = acc / Lt;
            if (!QUANT || p.out) p.out[out_base + h * kHeadDim + tid] = o[h];
        }
        if (tid == 0) p.counters[it.row * p.n_kv + kvh] = 0;
        // the weights in the merge buffer are read before the next unit writes it
        __syncthreads();
        if constexpr (QUANT) quantize_out(p, S.merge, it.row, kvh, o);
    }
}

template <int DT>
__global__ void __launch_bounds__(NT) append_kernel(const AppendParams p) {
    const int row = blockIdx.x / p.n_kv;
    const int kvh = blockIdx.x % p.n_kv;
    if (row >= p.n_rows) return;
    const RowDesc rd = p.rows[row];
    const int lp = rd.pos / kBlockTokens;
    const int pg = p.block_table[(int64_t) rd.stream * p.bt_cap + (lp % p.bt_cap)];
    if (pg < 0 || pg >= p.n_blocks) {
        if (threadIdx.x == 0) set_error(p.error, kErrBadPage);
        return;
    }
    const int64_t tile = (int64_t) pg * p.n_kv + kvh;
    const int64_t krow = ((int64_t) row * p.n_kv + kvh) * kHeadDim;
    append_head_row<DT>(p.k + krow, p.v + krow, p.rope + (int64_t) rd.pos * (kHeadDim / 2), p.k_data, p.v_data,
                        tile, rd.pos % kBlockTokens, nullptr, nullptr, nullptr, nullptr);
}

__global__ void table_update_kernel(int32_t * table, const TableUpdate * up, int32_t n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) table[up[i].index] = up[i].page;
}

// Reads rows back in plain order (un-swizzled): one CTA per (position, head).
template <int DT>
__global__ void gather_kernel(const GatherParams p) {
    const int r = blockIdx.x / p.n_kv;
    const int kvh = blockIdx.x % p.n_kv;
    if (r >= p.n) return;
    const int64_t pos = p.pos_start + r;
    const int64_t lp = pos / kBlockTokens;
    const int pg = p.block_table[lp % p.bt_cap];
    if (pg < 0 || pg >= p.n_blocks) return;
    const int64_t tile = (int64_t) pg * p.n_kv + kvh;
    const int tok = (int) (pos % kBlockTokens);
    constexpr int row_bytes = DT == 0 ? kHeadDim * 4 : DT == 1 ? kHeadDim * 2 : kHeadDim;
    constexpr int chunks = row_bytes / 16;
    const int64_t dst = ((int64_t) r * p.n_kv + kvh) * row_bytes;
    const uint8_t * kt = p.k_data + tile * Cfg<DT>::kRec;
    const uint8_t * vt = p.v_data + tile * Cfg<DT>::kRec;
    for (int ch = threadIdx.x; ch < chunks; ch += blockDim.x) {
        const int off = DT == 0 ? f32_chunk_off(tok, ch) : DT == 1 ? f16_chunk_off(tok, ch) : q8_chunk_off(tok, ch);
        *reinterpret_cast<uint4 *>(p.k_out + dst + ch * 16) = *reinterpret_cast<const uint4 *>(kt + off);
        uint4 vv = *reinterpret_cast<const uint4 *>(vt + off);
        if constexpr (DT == 8) {  // q8_0 V bytes are stored as x + 128
            vv.x ^= 0x80808080u;
            vv.y ^= 0x80808080u;
            vv.z ^= 0x80808080u;
            vv.w ^= 0x80808080u;
        }
        *reinterpret_cast<uint4 *>(p.v_out + dst + ch * 16) = vv;
    }
    if constexpr (DT == 8) {
        constexpr int nb = kHeadDim / kQ8Block;
        const int64_t sdst = ((int64_t) r * p.n_kv + kvh) * nb;
        const uint16_t * ks = reinterpret_cast<const uint16_t *>(kt + Cfg<8>::kTile);
        const uint16_t * vs = reinterpret_cast<const uint16_t *>(vt + Cfg<8>::kTile);
        for (int b = threadIdx.x; b < nb; b += blockDim.x) {
            reinterpret_cast<uint16_t *>(p.k_scale_out)[sdst + b] = ks[b * kBlockTokens + tok];
            reinterpret_cast<uint16_t *>(p.v_scale_out)[sdst + b] = vs[b * kBlockTokens + tok];
        }
    }
}

// One CTA per (move, layer, K|V): copies a page's bytes of every kv head.
__global__ void __launch_bounds__(256) compact_kernel(const CompactParams p) {
    const int m = blockIdx.x;
    const int layer = blockIdx.y;
    const bool is_v = blockIdx.z != 0;
    if (m >= p.n_moves) return;
    const int2 mv = p.moves[m];
    {
        uint8_t * base = (is_v ? p.v_data : p.k_data) + (int64_t) layer * p.layer_data_bytes;
        const uint4 * src = reinterpret_cast<const uint4 *>(base + (int64_t) mv.x * p.page_data_bytes);
        uint4 * dst = reinterpret_cast<uint4 *>(base + (int64_t) mv.y * p.page_data_bytes);
        const int64_t n = p.page_data_bytes / 16;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

template <int DT, bool QUANT = false>
cudaError_t launch_decode_t(const DecodeParams & p, cudaStream_t stream, bool pdl) {
    const int smem = (int) sizeof(Smem<DT>);
    // The opt-in is per device; remember which devices have it.
    static unsigned long long configured = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64 || !(configured & (1ull << dev))) {
        e = cudaFuncSetAttribute(decode_kernel<DT, QUANT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) configured |= 1ull << dev;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned) p.n_ctas);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_kernel<DT, QUANT>, p);
}

// Failure-path probe: a warp waits, with the decode kernel's own bounded
// wait, on an mbarrier that nothing arrives on; when the limit passes it sets
// the error word exactly as a decode launch whose copies never land would.
__global__ void wait_probe_kernel(int32_t * error, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    const bool landed = __all_sync(kFull, mbar_wait(&bar, 0, limit_ns));
    if (!landed && threadIdx.x == 0) set_error(error, kErrTimeout);
}

}  // namespace

cudaError_t launch_wait_probe(int32_t * error, uint64_t limit_ns, cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>(error, limit_ns);
    return cudaGetLastError();
}

int decode_smem_bytes(int dtype) {
    return dtype == 8 ? (int) sizeof(Smem<8>) : dtype == 0 ? (int) sizeof(Smem<0>) : (int) sizeof(Smem<1>);
}

template <int DT>
int ctas_per_sm_t() {
    int n = 0;
    if (cudaFuncSetAttribute(decode_kernel<DT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sizeof(Smem<DT>)) !=
        cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<DT, false>, NT, sizeof(Smem<DT>)) != cudaSuccess) return 0;
    return n;
}

int decode_ctas_per_sm(int dtype) {
    if (dtype == 8) return ctas_per_sm_t<8>();
    if (dtype == 0) return ctas_per_sm_t<0>();
    return ctas_per_sm_t<1>();
}

cudaError_t launch_decode(const DecodeParams & p, cudaStream_t stream, bool pdl) {
    if (p.n_items <= 0 || p.n_ctas <= 0) return cudaSuccess;
    if (p.dtype == 8) return launch_decode_t<8>(p, stream, pdl);
    if (p.dtype == 0) return launch_decode_t<0>(p, stream, pdl);
    return launch_decode_t<1>(p, stream, pdl);
}

cudaError_t launch_decode_quant(const DecodeParams & p, cudaStream_t stream, bool pdl) {
    if (p.dtype != 1 || !p.q_dx || (!p.q_tiles && !p.q_tiles8) || (p.q_tiles && !p.q_bmin) ||
        (p.q_npad != 16 && p.q_npad != 32 && p.q_npad != 64) || p.q_units != p.n_q * kHeadDim / 256 ||
        p.n_q != p.n_kv * kGroup)
        return cudaErrorInvalidValue;
    if (p.n_items <= 0 || p.n_ctas <= 0) return cudaSuccess;
    return launch_decode_t<1, true>(p, stream, pdl);
}

// ---------------------------------------------------------------------------
// Fixed split scratch for callers that must not allocate device memory.
//
// The decode kernel keeps per-split partial results and per-(row, kv head)
// arrival counters in scratch memory.  vxk_decode_layer_static_scratch uses
// this file-scope array for them instead of memory allocated by the library,
// so a call performs no device allocation at all.  The array is part of the
// module image: every GPU that loads libvxk.so holds its
// kStaticScratchFloats * 4 bytes (about 8.7 MB) until the process exits.
// Every call shares it, so two such calls that overlap on the GPU (different
// streams, or different pools on one device) race on it.
// ---------------------------------------------------------------------------
namespace {
static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];
}  // namespace

// Device address of g_static_scratch on the current device.  Host code may not
// use the symbol itself as a device pointer, so the address is looked up once
// per device (with that device current) and remembered.
static cudaError_t static_scratch_address(float ** out) {
    static std::mutex mu;
    static float * addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && addr[dev]) {
        *out = addr[dev];
        return cudaSuccess;
    }
    void * ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) addr[dev] = static_cast<float *>(ptr);
    *out = static_cast<float *>(ptr);
    return cudaSuccess;
}

cudaError_t launch_decode_static_scratch(const DecodeParams & params, cudaStream_t stream) {
    if (params.n_items <= 0 || params.n_ctas <= 0) return cudaSuccess;
    if ((size_t) params.n_items * params.n_q * kPartialStride > kStaticScratchPartialFloats ||
        (size_t) params.n_rows * params.n_kv > kStaticScratchCounters)
        return cudaErrorInvalidValue;
    float * base = nullptr;
    cudaError_t e = static_scratch_address(&base);
    if (e != cudaSuccess) return e;
    DecodeParams p = params;
    p.partials = base;
    p.counters = reinterpret_cast<int32_t *>(base + kStaticScratchPartialFloats);
    // The array keeps the previous call's contents; the arrival counters must
    // start at zero (partials are written before they are read).
    e = cudaMemsetAsync(p.counters, 0, (size_t) p.n_rows * p.n_kv * sizeof(int32_t), stream);
    if (e != cudaSuccess) return e;
    if (p.dtype == 8) return launch_decode_t<8>(p, stream, false);
    if (p.dtype == 0) return launch_decode_t<0>(p, stream, false);
    return launch_decode_t<1>(p, stream, false);
}

cudaError_t launch_append(const AppendParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    const dim3 grid((unsigned) (p.n_rows * p.n_kv));
    if (p.dtype == 8) {
        append_kernel<8><<<grid, NT, 0, stream>>>(p);
    } else if (p.dtype == 0) {
        append_kernel<0><<<grid, NT, 0, stream>>>(p);
    } else {
        append_kernel<1><<<grid, NT, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_table_updates(int32_t * table, const TableUpdate * updates, int32_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    table_update_kernel<<<(n + 255) / 256, 256, 0, stream>>>(table, updates, n);
    return cudaGetLastError();
}

cudaError_t launch_gather(const GatherParams & p, cudaStream_t stream) {
    if (p.n <= 0) return cudaSuccess;
    const dim3 grid((unsigned) (p.n * p.n_kv));
    if (p.dtype == 8) {
        gather_kernel<8><<<grid, 32, 0, stream>>>(p);
    } else if (p.dtype == 0) {
        gather_kernel<0><<<grid, 32, 0, stream>>>(p);
    } else {
        gather_kernel<1><<<grid, 32, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_compact(const CompactParams & p, cudaStream_t stream) {
    if (p.n_moves <= 0) return cudaSuccess;
    const dim3 grid((unsigned) p.n_moves, (unsigned) p.n_layers, 2);
    compact_kernel<<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace vxk
