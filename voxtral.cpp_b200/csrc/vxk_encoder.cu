// sm_100a kernels of the streaming-encoder KV ring:
//   enc_append_kernel  RoPE on K + 16-bit store of K/V at slot pos % capacity
//                      (set_rows of src/voxtral.cpp:2474-2479)
//   enc_tc_kernel      masked window attention of up to 8 new rows of one
//                      stream over [max(0, q - window + 1), q]
//                      (src/voxtral.cpp:2480-2487, mask of
//                      src/voxtral.cpp:4104-4119), scale 1/sqrt(64), on the
//                      5th-generation tensor cores (tcgen05.mma, TMEM
//                      accumulators) fed by TMA tensor copies.
//
// Ring layout: [stream][layer][head][capacity][64] 16-bit, one (stream,
// layer, head) ring = capacity x 128-byte rows.  A TMA tensor map views all
// rings as a 3-D tensor {64, capacity, rings}; boxes of 8 slots x 64 dims land
// in shared memory in the 128-byte-swizzled canonical layout the tensor
// cores read.  The window is walked in boxes through a virtual ring of
// round_up(capacity, 8) slots: slots past the real capacity read as zeros
// (TMA out-of-bounds fill) and are masked.
//
// One CTA = one (row group, head), 5 warps:
//   warp 4     TMA producer and tcgen05.mma issuer (one elected lane)
//   warps 0-3  own TMEM lane quadrants 0-3: softmax and epilogue
// Two phases, exact softmax (no online rescaling):
//   S^T[key][query] = K . Q^T   (M=128 keys per tile, N=8 queries, K=64)
//   softmax over all keys of the window, P^T to shared memory
//   O^T[dim][query] += V^T . P^T (M=64 dims, N=8, K=128 keys per tile)
// bf16 operands carry 8 mantissa bits, so Q and P are each split into a bf16
// high part and the bf16 residual (x = hi + lo) and both parts are
// multiplied; products accumulate in fp32.
#include "vxk_internal.h"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace vxk {
namespace {

constexpr int kEncHd = 64;
constexpr int kTcThreads = 160;
constexpr int kTcStages = 4;
constexpr int kTcMaxTiles = 6;          // keys per group <= 6 x 128
constexpr int kTcBoxes = 16;            // 8-slot boxes per 128-key tile
constexpr int kTcStageBytes = 16384;    // 128 keys x 128 B
constexpr uint64_t kTcWaitNs = 2000000000ull;
constexpr unsigned kFull = 0xffffffffu;

// shared-memory map (offsets from a 1024-aligned base)
constexpr int kOffStage = 0;
constexpr int kOffQ = kTcStages * kTcStageBytes;                 // Q^T hi, lo: 2 x 1 KB
constexpr int kOffP = kOffQ + 2048;                              // P^T hi, lo: tiles x 2 x 2 KB
constexpr int kOffBar = kOffP + kTcMaxTiles * 2 * 2048;
constexpr int kNumBars = 2 * kTcStages + 4;                      // full, mma, q, s, p, o
constexpr int kOffMisc = kOffBar + kNumBars * 8;                 // tmem addr, abort
constexpr int kOffRed = kOffMisc + 16;                           // [2][4 warps][8]
constexpr int kTcSmem = kOffRed + 2 * 4 * 8 * 4 + 1024;          // + alignment slack

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

// Bounded wait on an mbarrier phase; false after kTcWaitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kTcWaitNs) return false;
    }
}

// 3-D TMA tile load (no multicast) into shared memory, counted on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void * dst, const CUtensorMap * map, int c0, int c1, int c2,
                                            uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// descriptor version 1, base offset 0.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// D(tmem) (+)= A(smem) * B(smem), kind::f16, fp32 accumulate.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier when all tcgen05 ops issued so far by this thread finish.
__device__ __forceinline__ void tc_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 8 columns of 32 bits from TMEM into registers.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float2 enc_rope_pair(float2 x, float2 cs) {
    float2 r;
    r.x = __fsub_rn(__fmul_rn(x.x, cs.x), __fmul_rn(x.y, cs.y));
    r.y = __fadd_rn(__fmul_rn(x.x, cs.y), __fmul_rn(x.y, cs.x));
    return r;
}

template <int DT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (DT == 30) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    } else {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    }
}

template <int DT>
__device__ __forceinline__ uint16_t to16(float a) {
    if constexpr (DT == 30) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(a));
    } else {
        return __half_as_ushort(__float2half_rn(a));
    }
}

template <int DT>
__device__ __forceinline__ float from16(uint16_t u) {
    if constexpr (DT == 30) {
        return __bfloat162float(__ushort_as_bfloat16(u));
    } else {
        return __half2float(__ushort_as_half(u));
    }
}

__device__ __forceinline__ int64_t ring_index(const EncParams & p, int stream, int head) {
    return ((int64_t) stream * p.n_layers + p.layer) * p.n_heads + head;
}

// One CTA per row; thread t < 32*n_heads handles one (head, pair).
template <int DT>
__global__ void enc_append_kernel(const EncParams p) {
    const int r = blockIdx.x;
    if (r >= p.n_rows) return;
    const EncRowDesc rd = p.rows[r];
    const float2 * cs = p.rope + (int64_t) rd.pos * (kEncHd / 2);
    for (int idx = threadIdx.x; idx < p.n_heads * (kEncHd / 2); idx += blockDim.x) {
        const int h = idx / (kEncHd / 2);
        const int i = idx % (kEncHd / 2);
        const int64_t src = ((int64_t) r * p.n_heads + h) * kEncHd + 2 * i;
        const float2 kx = enc_rope_pair(*reinterpret_cast<const float2 *>(p.k + src), cs[i]);
        const float2 vx = *reinterpret_cast<const float2 *>(p.v + src);
        const int64_t dst = (ring_index(p, rd.stream, h) * p.capacity + rd.slot) * kEncHd + 2 * i;
        reinterpret_cast<uint32_t *>(p.k_ring)[dst / 2] = pack2<DT>(kx.x, kx.y);
        reinterpret_cast<uint32_t *>(p.v_ring)[dst / 2] = pack2<DT>(vx.x, vx.y);
    }
}

template <int DT>
__global__ void __launch_bounds__(kTcThreads) enc_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                                                            const __grid_constant__ CUtensorMap tmv,
                                                            const EncParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * stages = base + kOffStage;
    uint8_t * qt = base + kOffQ;
    uint8_t * pt = base + kOffP;
    uint64_t * full = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint64_t * mmab = full + kTcStages;
    uint64_t * q_bar = mmab + kTcStages;
    uint64_t * s_bar = q_bar + 1;
    uint64_t * p_bar = q_bar + 2;
    uint64_t * o_bar = q_bar + 3;
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(base + kOffMisc);
    int32_t * abort_flag = reinterpret_cast<int32_t *>(base + kOffMisc + 4);
    float * red = reinterpret_cast<float *>(base + kOffRed);  // [2][4][8]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int grp = blockIdx.x / p.n_heads;
    const int h = blockIdx.x % p.n_heads;
    if (grp >= p.n_groups) return;
    const int r0 = p.group_first[grp];
    const int nr = p.group_first[grp + 1] - r0;  // <= 8 rows
    const EncRowDesc first = p.rows[r0];
    const EncRowDesc last = p.rows[r0 + nr - 1];
    const int ring = (int) ring_index(p, first.stream, h);
    const int cap = p.capacity;
    const int vslots = (cap + 7) & ~7;           // virtual ring of whole boxes
    const int ws = first.win_start;
    const int we = last.pos;
    const int s0 = (ws % cap) & ~7;               // first box slot
    const int nb = (((we % cap) - s0 + vslots) % vslots) / 8 + 1;
    const int T = (nb + kTcBoxes - 1) / kTcBoxes; // host guarantees T <= kTcMaxTiles
    constexpr uint32_t fmt = DT == 30 ? 1u : 0u;  // BF16 / F16 operands
    const uint32_t idesc_qk = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 17) | (8u << 24);
    const uint32_t idesc_pv = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (1u << 17) | (4u << 24);

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&mmab[s], 1);
        }
        mbar_init(q_bar, 128);
        mbar_init(s_bar, 1);
        mbar_init(p_bar, 128);
        mbar_init(o_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 64;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_tmem = tmem;        // S^T tile t in columns 8t .. 8t+7
    const uint32_t o_tmem = tmem + 48;   // O^T in columns 48 .. 55

    if (warp == 4) {
        // ---------------- producer / MMA issuer ----------------
        if (lane == 0) {
            const int nloads = 2 * T;  // K tiles, then V tiles
            auto issue = [&](int L) {
                const bool is_v = L >= T;
                const int t = is_v ? L - T : L;
                const int st = L % kTcStages;
                uint8_t * dst = stages + st * kTcStageBytes;
                mbar_expect_tx(&full[st], kTcStageBytes);
#pragma unroll 1
                for (int b = 0; b < kTcBoxes; ++b) {
                    const int gb = t * kTcBoxes + b;
                    const int slot = gb < nb ? (s0 + 8 * gb) % vslots : 0;
                    tma_load_3d(dst + b * 1024, is_v ? &tmv : &tmk, 0, slot, ring, &full[st]);
                }
            };
            int issued = 0;
            while (issued < nloads && issued < kTcStages) issue(issued++);
            bool ok = mbar_wait(q_bar, 0);
            tc_fence_after();
            int L = 0;
            for (; ok && L < nloads; ++L) {
                const int st = L % kTcStages;
                if (L == T) {
                    ok = mbar_wait(p_bar, 0);
                    tc_fence_after();
                    if (!ok) break;
                }
                if (!mbar_wait(&full[st], (L / kTcStages) & 1)) {
                    ok = false;
                    break;
                }
                const uint32_t sa = smem_u32(stages + st * kTcStageBytes);
                if (L < T) {
                    // S^T tile L = K . (Q_hi + Q_lo)^T
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            tc_mma(s_tmem + 8 * L, sw128_desc(sa + ks * 32, 16, 1024),
                                   sw128_desc(smem_u32(qt + part * 1024) + ks * 32, 16, 1024), idesc_qk,
                                   (part | ks) != 0);
                        }
                    }
                } else {
                    // O^T += V^T . (P_hi + P_lo)^T for tile t
                    const int t = L - T;
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
                        const uint32_t pb = smem_u32(pt + (t * 2 + part) * 2048);
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks) {
                            tc_mma(o_tmem, sw128_desc(sa + ks * 2048, 16, 1024),
                                   sw128_desc(pb + (ks >> 2) * 1024 + (ks & 3) * 32, 16, 1024), idesc_pv,
                                   (t | part | ks) != 0);
                        }
                    }
                }
                tc_commit(&mmab[st]);
                if (L == T - 1) tc_commit(s_bar);
                if (L == nloads - 1) tc_commit(o_bar);
                if (issued < nloads) {
                    // refill this stage once the MMAs reading it are done
                    if (!mbar_wait(&mmab[st], (L / kTcStages) & 1)) {
                        ok = false;
                        break;
                    }
                    issue(issued++);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                if (p.error) atomicCAS(p.error, 0, 2);
                // wake the consumers, then drain the copies not yet consumed
                tc_commit(s_bar);
                tc_commit(o_bar);
                for (int l = L; l < issued; ++l) mbar_wait(&full[l % kTcStages], (l / kTcStages) & 1);
            }
        }
        __syncwarp();
    } else {
        // ---------------- softmax / epilogue warps 0-3 ----------------
        // Q^T (hi, lo): 8 rows x 64 dims, 128-byte swizzled K-major rows.
        for (int idx = tid; idx < 8 * 32; idx += 128) {
            const int j = idx >> 5;
            const int i = idx & 31;  // pair: dims 2i, 2i+1
            float2 qv = make_float2(0.0f, 0.0f);
            if (j < nr) {
                const EncRowDesc rd = p.rows[r0 + j];
                const float2 x = *reinterpret_cast<const float2 *>(p.q + ((int64_t) (r0 + j) * p.n_heads + h) * kEncHd + 2 * i);
                const float2 rr = enc_rope_pair(x, p.rope[(int64_t) rd.pos * (kEncHd / 2) + i]);
                qv = make_float2(rr.x * p.scale_log2, rr.y * p.scale_log2);
            }
            const uint16_t hx = to16<DT>(qv.x), hy = to16<DT>(qv.y);
            const uint16_t lx = to16<DT>(qv.x - from16<DT>(hx)), ly = to16<DT>(qv.y - from16<DT>(hy));
            const int off = j * 128 + (((i >> 2) ^ j) << 4) + (i & 3) * 4;
            *reinterpret_cast<uint32_t *>(qt + off) = (uint32_t) hx | ((uint32_t) hy << 16);
            *reinterpret_cast<uint32_t *>(qt + 1024 + off) = (uint32_t) lx | ((uint32_t) ly << 16);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(q_bar);

        float sv[kTcMaxTiles][8];
        const bool have_s = mbar_wait(s_bar, 0);
        tc_fence_after();
        const uint32_t lane_off = (uint32_t) (32 * warp) << 16;
#pragma unroll
        for (int t = 0; t < kTcMaxTiles; ++t) {
            if (t < T) tmem_ld8(s_tmem + lane_off + 8 * t, sv[t]);
        }
        int qpos[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) qpos[j] = j < nr ? p.rows[r0 + j].pos : -1;
        const int r = 32 * warp + lane;  // key row within a tile
        float mx[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx[j] = -INFINITY;
#pragma unroll
        for (int t = 0; t < kTcMaxTiles; ++t) {
            if (t >= T) break;
            const int gb = t * kTcBoxes + (r >> 3);
            const int slot = (s0 + 8 * gb) % vslots + (r & 7);
            bool valid = have_s && !*abort_flag && gb < nb && slot < cap;
            const int kp = we - (((we % cap) - slot + cap) % cap);
            valid = valid && kp >= ws;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const bool ok = valid && j < nr && kp <= qpos[j] && kp >= qpos[j] - (p.window - 1);
                sv[t][j] = ok ? sv[t][j] : -INFINITY;
                mx[j] = fmaxf(mx[j], sv[t][j]);
            }
        }
        // per-query max over the 128 consumer threads
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx[j] = fmaxf(mx[j], __shfl_xor_sync(kFull, mx[j], o));
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) red[warp * 8 + j] = mx[j];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        float M[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            M[j] = fmaxf(fmaxf(red[j], red[8 + j]), fmaxf(red[16 + j], red[24 + j]));
            if (M[j] == -INFINITY) M[j] = 0.0f;  // padding queries
        }
        float ls[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ls[j] = 0.0f;
#pragma unroll
        for (int t = 0; t < kTcMaxTiles; ++t) {
            if (t >= T) break;
            uint8_t * ph = pt + (t * 2) * 2048 + (r >> 6) * 1024;
            uint8_t * pl = ph + 2048;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float e = exp2f(sv[t][j] - M[j]);
                const uint16_t hi = to16<DT>(e);
                const float ehi = from16<DT>(hi);
                const uint16_t lo = to16<DT>(e - ehi);
                ls[j] += ehi + from16<DT>(lo);
                const int off = j * 128 + ((((r & 63) >> 3) ^ j) << 4) + (r & 7) * 2;
                *reinterpret_cast<uint16_t *>(ph + off) = hi;
                *reinterpret_cast<uint16_t *>(pl + off) = lo;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(p_bar);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ls[j] += __shfl_xor_sync(kFull, ls[j], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) red[32 + warp * 8 + j] = ls[j];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool have_o = mbar_wait(o_bar, 0);
        tc_fence_after();
        float ov[8];
        tmem_ld8(o_tmem + lane_off, ov);
        if (have_o && !*abort_flag && lane < 16) {
            const int dim = 16 * warp + lane;  // M=64 accumulator rows sit in lanes 0-15 of each quadrant
            for (int j = 0; j < nr; ++j) {
                const float L = red[32 + j] + red[40 + j] + red[48 + j] + red[56 + j];
                p.out[((int64_t) (r0 + j) * p.n_heads + h) * kEncHd + dim] = ov[j] / L;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 64;" ::"r"(tmem) : "memory");
    }
}

}  // namespace

int enc_smem_bytes() { return kTcSmem; }

int enc_max_tiles() { return kTcMaxTiles; }

cudaError_t launch_enc_append(const EncParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    if (p.dtype == 30) {
        enc_append_kernel<30><<<p.n_rows, 256, 0, stream>>>(p);
    } else {
        enc_append_kernel<1><<<p.n_rows, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_enc_attention(const EncParams & p, const CUtensorMap & tmk, const CUtensorMap & tmv,
                                 cudaStream_t stream) {
    if (p.n_groups <= 0) return cudaSuccess;
    const unsigned grid = (unsigned) (p.n_groups * p.n_heads);
    cudaError_t e;
    if (p.dtype == 30) {
        e = cudaFuncSetAttribute(enc_tc_kernel<30>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        if (e != cudaSuccess) return e;
        enc_tc_kernel<30><<<grid, kTcThreads, kTcSmem, stream>>>(tmk, tmv, p);
    } else {
        e = cudaFuncSetAttribute(enc_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        if (e != cudaSuccess) return e;
        enc_tc_kernel<1><<<grid, kTcThreads, kTcSmem, stream>>>(tmk, tmv, p);
    }
    return cudaGetLastError();
}

}  // namespace vxk
