// sm_100a kernels of the streaming-encoder KV ring:
//   enc_append_kernel  RoPE on K + 16-bit store of K/V at slot pos % capacity
//                      (set_rows of src/voxtral.cpp:2474-2479)
//   enc_tc_kernel      masked window attention of up to 8 new rows of one
//                      stream over [max(0, q - window + 1), q]
//                      (src/voxtral.cpp:2480-2487, mask of
//                      src/voxtral.cpp:4104-4119), scale 1/sqrt(64), on the
//                      5th-generation tensor cores (tcgen05.mma, TMEM
//                      accumulators) fed by TMA bulk copies.
//
// Ring layout: [stream][layer][head][ring_slots][64] 16-bit, ring_slots =
// round_up(capacity, 8); the pad slots stay zero.  Rows are stored
// pre-swizzled: the 16-byte chunk c of slot s sits at chunk c ^ (s & 7).  A
// run of slots that starts at a multiple of 8 therefore lands, by a plain
// 1-D bulk copy into a 1024-byte-aligned buffer, in exactly the 128-byte
// swizzled K-major layout the tensor cores read, and a 128-key tile is one
// bulk copy (two where it crosses the end of the ring) instead of sixteen
// tensor-map boxes.
//
// Work unit = (row group, head).  Persistent CTAs, one per SM, walk their
// units through a warp-specialised pipeline (12 warps):
//   warp 8     TMA producer: 16 KB stages (128 keys of K or V) into a
//              10-stage shared-memory ring.  One thread issues every copy,
//              and a copy's issue costs about as long as its bytes take at
//              the SM's share of HBM, so this thread's path is kept free of
//              waits other than for ring slots: group descriptors come
//              precomputed from the host (no divisions, no dependent loads)
//   warp 9     tcgen05.mma issuer of S^T = K.Q^T (one lane), tile by tile
//   warp 11    tcgen05.mma issuer of O^T += V^T.P^T (one lane): the two
//              products of consecutive units are issued side by side
//   warp 10    Q^T producer (RoPE, scale, bf16 hi/lo split)
//   warps 0-3  own TMEM lane quadrants 0-3: softmax and epilogue of the
//              even units of the CTA; warps 4-7 the same for the odd units
//              (one set's softmax and epilogue take about a unit's copy time)
// With fuse_append (every group a whole stream) all warps but the producer
// first store the new K/V rows of the CTA's units into the ring (replacing
// enc_append_kernel's launch); the producer copies the tiles holding new
// rows after their signal.
// Per unit, two phases with an exact softmax (no online rescaling):
//   S^T[key][query] = K . Q^T    (M=128 keys per tile, N=16 = 8 queries x
//                                 {hi, lo}, K=64 dims: 4 MMAs per tile)
//   softmax over all keys of the window, P^T to shared memory
//   O^T[dim][query] += V^T . P^T (per tile 4 MMAs of M=128 = the dims of
//                                 keys 0-63 and of keys 64-127, N=32, K=16)
// Q, S, P and O are double-buffered by unit parity, so the tensor cores
// compute unit i+1's scores while the softmax warps work on unit i, and the
// ring keeps up to 160 KB of K/V reads in flight per SM.
// bf16 operands carry 8 mantissa bits, so Q and P are each split into a bf16
// high part and the bf16 residual (x = hi + lo) and both parts are
// multiplied; products accumulate in fp32.
//
// f32 rings (the reference's default encoder cache, src/voxtral.cpp:100-105)
// keep fp32 rows (256 B, the 16-byte chunk c of slot s at chunk c ^ (s & 7))
// and take enc_f32_kernel: the same units on the CUDA cores in fp32, one
// 128-thread CTA per unit, 128-key tiles of K then V by bulk copy into two
// shared-memory buffers, scores one key per thread, an exact softmax over the
// window, and P.V with each thread owning 4 dims of every row over an eighth
// of the keys.
#include "vxk_internal.h"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace vxk {
namespace {

constexpr int kEncHd = 64;
constexpr int kTcSets = 2;              // softmax/epilogue warp sets (4 warps each)
constexpr int kTcThreads = 128 * kTcSets + 128;
constexpr int kWarpProducer = 4 * kTcSets, kWarpS = kWarpProducer + 1, kWarpQ = kWarpProducer + 2,
              kWarpPV = kWarpProducer + 3;
constexpr int kTcStages = 10;
constexpr int kTcMaxTiles = 6;          // keys per group <= 6 x 128
constexpr int kTcBoxes = 16;            // 8-slot boxes per 128-key tile
constexpr int kTcStageBytes = 16384;    // 128 keys x 128 B
constexpr int kTmemCols = 512;          // S^T 2 sets x 96 columns, O^T 2 sets x 4 accumulators x 32
constexpr uint64_t kTcWaitNs = 2000000000ull;
constexpr unsigned kFull = 0xffffffffu;

// shared-memory map (offsets from a 1024-aligned base)
constexpr int kOffStage = 0;
constexpr int kOffQ = kTcStages * kTcStageBytes;                 // Q^T [2 sets][hi, lo] x 1 KB
constexpr int kPBuf = kTcMaxTiles * 4096;                        // P^T [tiles][key half][hi, lo] x 1 KB
constexpr int kOffP = kOffQ + 2 * 2048;                          // 2 sets of kPBuf
constexpr int kOffBar = kOffP + 2 * kPBuf;
// mbarrier indices
constexpr int kBarFull = 0;                    // stage landed (TMA tx count)
constexpr int kBarEmpty = kTcStages;           // stage consumed (tcgen05.commit)
constexpr int kBarQFull = 2 * kTcStages;       // [2] Q^T written
constexpr int kBarQEmpty = kBarQFull + 2;      // [2] S MMAs done reading Q^T
constexpr int kBarSFull = kBarQEmpty + 2;      // [2] S^T complete in TMEM
constexpr int kBarSEmpty = kBarSFull + 2;      // [2] S^T read by the softmax warps
constexpr int kBarPFull = kBarSEmpty + 2;      // [2] P^T written
constexpr int kBarPEmpty = kBarPFull + 2;      // [2] PV MMAs done reading P^T
constexpr int kBarOFull = kBarPEmpty + 2;      // [2] O^T complete in TMEM
constexpr int kBarOEmpty = kBarOFull + 2;      // [2] O^T read by the epilogue
constexpr int kBarDrain = kBarOEmpty + 2;      // all MMAs of the CTA done (both issuers)
constexpr int kBarRows = kBarDrain + 1;        // every unit's new K/V rows are in the ring (fuse_append)
constexpr int kNumBars = kBarRows + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;                 // tmem addr, abort flag
constexpr int kOffRed = kOffMisc + 16;                           // max [2][4][8], sums [2][4][8]
constexpr int kOffEpi = kOffRed + (64 + 64) * 4;                 // [2 sets] O^T of keys 64-127 [8 queries][64 dims]
constexpr int kTcSmem = kOffEpi + 2 * 8 * 64 * 4 + 1024;         // + alignment slack
static_assert(kTcSmem <= 232448, "encoder attention exceeds 227 KB of shared memory");

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

// 1-D bulk copy global -> this CTA's shared memory, completion counted on an
// mbarrier; each ring row is read once per layer: evict-first in L2.
__device__ __forceinline__ void bulk_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar,
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

// 32 lanes x 16 columns of 32 bits from TMEM into registers.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// The same load without the wait (tcgen05.wait::ld before using the values).
__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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
    // Launched with programmatic stream serialization: wait for the previous
    // grid (whatever produced k/v) before reading anything, then let the
    // attention launch start its prologue.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
        // byte 4i of the row = chunk i / 4, stored at chunk (i / 4) ^ (slot & 7)
        const int64_t row = ring_index(p, rd.stream, h) * p.ring_slots + rd.slot;
        if constexpr (DT == 0) {
            // dims 2i, 2i+1 = bytes 8i of the 256-byte row: chunk i / 2
            const int64_t dst = row * (kEncHd * 4) + ((((i >> 1) ^ (rd.slot & 7))) << 4) + (i & 1) * 8;
            *reinterpret_cast<float2 *>(p.k_ring + dst) = kx;
            *reinterpret_cast<float2 *>(p.v_ring + dst) = vx;
        } else {
            const int64_t dst = row * (kEncHd * 2) + ((((i >> 2) ^ (rd.slot & 7))) << 4) + (i & 3) * 4;
            *reinterpret_cast<uint32_t *>(p.k_ring + dst) = pack2<DT>(kx.x, kx.y);
            *reinterpret_cast<uint32_t *>(p.v_ring + dst) = pack2<DT>(vx.x, vx.y);
        }
    }
}

// Bounded wait on an mbarrier phase shared by the kernel's roles: gives up
// when another role has raised the CTA's abort flag, or after kTcWaitNs, in
// which case it raises the flag and sets the device error word.
__device__ __forceinline__ bool enc_wait(uint64_t * bar, uint32_t parity, volatile int32_t * abort_flag,
                                         int32_t * err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kTcWaitNs) {
            *abort_flag = 1;
            if (err) atomicCAS(err, 0, 2);
            return false;
        }
    }
}

// Bounded wait that ignores the abort flag: used to let copies and MMAs that
// are already in flight finish before the CTA exits.
__device__ __forceinline__ void enc_drain(uint64_t * bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kTcWaitNs) return;
    }
}

// One unit of work: the rows of one group (<= 8 new frames of one stream) and
// one head, attending the union of their windows, walked as nb 8-slot boxes
// from slot s0 of the virtual ring, in T tiles of 16 boxes.
struct EncUnit {
    int r0, nr, h, ws, we, wem, s0, nb, T;
    int64_t ring;  // ring index (stream, layer, head)
};

// Walks the units u0, u0 + step, ... of a CTA (unit = group * n_heads + head)
// without divisions, loading each group's 32-byte descriptor (EncParams::groups)
// one unit ahead so that its latency overlaps the current unit.
struct UnitWalk {
    int u, grp, h, dg, dh, step, n_units, n_heads;
    int4 a, b;
    __device__ __forceinline__ void init(const EncParams & p, int u0, int step_, int n_units_) {
        u = u0;
        step = step_;
        n_units = n_units_;
        n_heads = p.n_heads;
        grp = u0 / n_heads;
        h = u0 - grp * n_heads;
        dg = step / n_heads;
        dh = step - dg * n_heads;
        if (u < n_units) fetch(p);
    }
    __device__ __forceinline__ void fetch(const EncParams & p) {
        a = __ldg(p.groups + 2 * grp);
        b = __ldg(p.groups + 2 * grp + 1);
    }
    __device__ __forceinline__ bool more() const { return u < n_units; }
    // the current unit; then moves to the next and starts loading its descriptor
    __device__ __forceinline__ EncUnit take(const EncParams & p) {
        EncUnit U;
        U.h = h;
        U.r0 = a.x & 0xffffff;
        U.nr = (int) ((unsigned) a.x >> 24);
        U.ring = ((int64_t) a.y * p.n_layers + p.layer) * p.n_heads + h;
        U.ws = a.z;
        U.we = a.w;
        U.s0 = b.x;
        U.nb = b.y;
        U.wem = b.z;
        U.T = (U.nb + kTcBoxes - 1) / kTcBoxes;  // host guarantees T <= kTcMaxTiles
        u += step;
        h += dh;
        grp += dg;
        if (h >= n_heads) {
            h -= n_heads;
            ++grp;
        }
        if (u < n_units) fetch(p);
        return U;
    }
};

// Persistent, warp-specialised window attention.  CTA b handles units b,
// b + gridDim.x, ...; unit i of a CTA uses buffer set i & 1 of Q, S, P and O,
// so that unit i+1's S = K.Q^T runs on the tensor cores while the softmax
// warps work on unit i.  Stage order through the shared-memory ring:
// K(0), K(1), V(0), K(2), V(1), ..., V(last).
template <int DT>
__global__ void __launch_bounds__(kTcThreads, 1) enc_tc_kernel(const EncParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * stages = base + kOffStage;
    uint8_t * qbuf = base + kOffQ;
    uint8_t * pbuf = base + kOffP;
    uint64_t * bars = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(base + kOffMisc);
    volatile int32_t * abort_flag = reinterpret_cast<volatile int32_t *>(base + kOffMisc + 4);
    float * redmax = reinterpret_cast<float *>(base + kOffRed);  // [2 sets][4 warps][8]
    float * redsum = redmax + 64;                                // [2 sets][4 warps][8]
    float * epi_all = reinterpret_cast<float *>(base + kOffEpi); // [2 sets][8][64]

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int cap = p.capacity;
    const int vslots = p.ring_slots;  // round_up(capacity, 8): the ring walked in whole boxes
    const int n_units = p.n_groups * p.n_heads;
    const int stride = (int) gridDim.x;
    if ((int) blockIdx.x >= n_units) return;

    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&bars[kBarFull + s], 1);
            mbar_init(&bars[kBarEmpty + s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[kBarQFull + b], 1);
            mbar_init(&bars[kBarQEmpty + b], 1);
            mbar_init(&bars[kBarSFull + b], 1);
            mbar_init(&bars[kBarSEmpty + b], 128);
            mbar_init(&bars[kBarPFull + b], 128);
            mbar_init(&bars[kBarPEmpty + b], 1);
            mbar_init(&bars[kBarOFull + b], 1);
            mbar_init(&bars[kBarOEmpty + b], 128);

        }
        mbar_init(&bars[kBarDrain], 2);
        mbar_init(&bars[kBarRows], kTcThreads / 32 - 1);
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
    // Launched with programmatic stream serialization: only the barrier setup
    // and the TMEM allocation above overlap the previous grid; every global
    // read (rows, q, the rings the append kernel just wrote) comes after this.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (p.fuse_append && warp != kWarpProducer) {
        // Fused append (the set_rows of src/voxtral.cpp:2474-2479): every warp but
        // the producer stores the new K (rotated) and V rows of some of the CTA's
        // units into the ring, lane l dims 2l, 2l + 1 of each row; no other unit
        // reads a unit's (stream, head) ring.  The producer copies the tiles that
        // hold new rows only after all warps have signalled.
        constexpr int kStoreWarps = kTcThreads / 32 - 1;
        constexpr int kRowBytes = kEncHd * 2;
        UnitWalk W;
        W.init(p, blockIdx.x + (warp < kWarpProducer ? warp : warp - 1) * stride, kStoreWarps * stride, n_units);
        while (W.more()) {
            const EncUnit U = W.take(p);
            const int pos0 = U.we - U.nr + 1;
            int slot0 = U.wem - U.nr + 1;  // = pos0 % capacity (rows are consecutive positions)
            slot0 = slot0 < 0 ? slot0 + cap : slot0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j < U.nr) {
                    const int64_t src = ((int64_t) (U.r0 + j) * p.n_heads + U.h) * kEncHd + 2 * lane;
                    const float2 kr = enc_rope_pair(*reinterpret_cast<const float2 *>(p.k + src),
                                                    p.rope[(int64_t) (pos0 + j) * (kEncHd / 2) + lane]);
                    const float2 vx = *reinterpret_cast<const float2 *>(p.v + src);
                    const int slot = slot0 + j < cap ? slot0 + j : slot0 + j - cap;
                    // byte 4 lane of the row = chunk lane / 4, stored at chunk (lane / 4) ^ (slot & 7)
                    const int64_t dst =
                        (U.ring * vslots + slot) * kRowBytes + (((lane >> 2) ^ (slot & 7)) << 4) + (lane & 3) * 4;
                    *reinterpret_cast<uint32_t *>(p.k_ring + dst) = pack2<DT>(kr.x, kr.y);
                    *reinterpret_cast<uint32_t *>(p.v_ring + dst) = pack2<DT>(vx.x, vx.y);
                }
            }
        }
        // the producer's bulk copies (async proxy) read these rows after the signal
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarRows]);
    }
    // TMEM columns (N = 16: 8 queries' hi parts, then their lo parts):
    //   S^T of set b, tile t      at 96 b + 16 t
    //   O^T of set b, accumulator a at 192 + 128 b + 32 a: an M = 128 x N = 32 block whose
    //   lanes 0-63 x columns 0-15 hold dims 0-63 over keys 0-63 of each tile and lanes
    //   64-127 x columns 16-31 dims 0-63 over keys 64-127 (the other quarters are unused
    //   cross products); accumulators and halves are summed in the epilogue

    if (warp == kWarpProducer) {
        // ---------------- TMA producer ----------------
        // One thread issues every copy: its per-tile path is kept short (a
        // running stage and phase, ring bases computed once per unit), since
        // the copies of a unit are issued back to back at the HBM rate.
        if (lane == 0) {
            uint32_t c = 0;           // copies issued
            int st = 0;               // = c % kTcStages
            uint32_t ph = 0;          // = (c / kTcStages) & 1
            bool ok = true;
            const uint64_t policy = evict_first_policy();
            constexpr int kRowBytes = kEncHd * 2;
            const int64_t ring_bytes = (int64_t) vslots * kRowBytes;
            // tile t of a unit whose ring starts at `ring`: 128 consecutive slots from
            // s0 + 128 t, wrapping at the ring's end (rows past the window are read and masked)
            auto load = [&](const uint8_t * ring, int s0, int t) -> bool {
                if (!enc_wait(&bars[kBarEmpty + st], ph ^ 1, abort_flag, p.error)) return false;
                uint8_t * dst = stages + st * kTcStageBytes;
                uint64_t * full = &bars[kBarFull + st];
                mbar_expect_tx(full, kTcStageBytes);
                int slot = s0 + 128 * t;
                slot = slot >= vslots ? slot - vslots : slot;
                const int n = min(128, vslots - slot);
                bulk_load(dst, ring + slot * kRowBytes, (uint32_t) (n * kRowBytes), full, policy);
                if (n < 128) bulk_load(dst + n * kRowBytes, ring, (uint32_t) ((128 - n) * kRowBytes), full, policy);
                ++c;
                if (++st == kTcStages) {
                    st = 0;
                    ph ^= 1;
                }
                return true;
            };
            const uint8_t * pv_ring = nullptr;  // V ring and geometry of the previous unit
            int p_s0 = 0, p_T = 0;
            bool rows_ready = !p.fuse_append;
            UnitWalk W;
            W.init(p, blockIdx.x, stride, n_units);
            for (int i = 0; ok && W.more(); ++i) {
                const EncUnit U = W.take(p);
                const uint8_t * k_ring = p.k_ring + U.ring * ring_bytes;
                // with fuse_append the tiles from the one holding the unit's first
                // new row on are copied after the other warps stored the rows
                int t_new = U.T;
                if (p.fuse_append) {
                    int first = U.wem - U.nr + 1;
                    first = first < 0 ? first + cap : first;
                    int off = first - U.s0;
                    off = off < 0 ? off + vslots : off;
                    t_new = off >> 7;
                }
                for (int t = 0; ok && t < U.T; ++t) {
                    if (t == t_new && !rows_ready) {
                        ok = enc_wait(&bars[kBarRows], 0, abort_flag, p.error);
                        rows_ready = true;
                    }
                    ok = ok && load(k_ring, U.s0, t);
                }
                for (int t = 0; ok && t < p_T; ++t) ok = load(pv_ring, p_s0, t);
                pv_ring = p.v_ring + U.ring * ring_bytes;
                p_s0 = U.s0;
                p_T = U.T;
            }
            for (int t = 0; ok && t < p_T; ++t) ok = load(pv_ring, p_s0, t);
            if (!ok || *abort_flag) {
                // let every issued copy land before the CTA exits
                for (uint32_t d = c > (uint32_t) kTcStages ? c - kTcStages : 0; d < c; ++d)
                    enc_drain(&bars[kBarFull + d % kTcStages], (d / kTcStages) & 1);
            }
        }
        __syncwarp();
    } else if (warp == kWarpS || warp == kWarpPV) {
        // ---------------- tcgen05.mma issuers of S and PV ----------------
        if (lane == 0) {
            const bool s_role = warp == kWarpS;
            constexpr uint32_t fmt = DT == 30 ? 1u : 0u;  // BF16 / F16 operands
            // fp32 accumulate.  S: M = 128 keys, N = 16, K-major A.  PV: M = 128 (dims of
            // keys 0-63, then dims of keys 64-127: the V tile's two 64-key halves are two
            // MN atoms 8 KB apart), N = 32, MN-major A.
            const uint32_t idesc_qk = (1u << 4) | (fmt << 7) | (fmt << 10) | (2u << 17) | (8u << 24);
            const uint32_t idesc_pv = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (4u << 17) | (8u << 24);
            uint32_t c = 0;
            auto s_unit = [&](const EncUnit & U, int i) -> bool {
                const int b = i & 1;
                const uint32_t k = (uint32_t) (i >> 1) & 1;
                if (!enc_wait(&bars[kBarQFull + b], k, abort_flag, p.error)) return false;
                if (!enc_wait(&bars[kBarSEmpty + b], k ^ 1, abort_flag, p.error)) return false;
                tc_fence_after();
                const uint32_t qa = smem_u32(qbuf + b * 2048);
                const uint32_t sd = tmem + 96 * b;
                uint64_t bq[4];
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) bq[ks] = sw128_desc(qa + ks * 32, 16, 1024);
                // each tile as soon as it lands (its stage is released by the commit)
                for (int t = 0; t < U.T; ++t) {
                    const int st = (int) (c % kTcStages);
                    if (!enc_wait(&bars[kBarFull + st], (c / kTcStages) & 1, abort_flag, p.error)) return false;
                    tc_fence_after();
                    const uint64_t ka = sw128_desc(smem_u32(stages + st * kTcStageBytes), 16, 1024);
                    // S^T tile = K . [Q_hi; Q_lo]^T; +2 in the descriptor = +32 bytes (16 dims)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) tc_mma(sd + 16 * t, ka + 2 * ks, bq[ks], idesc_qk, ks != 0);
                    tc_commit(&bars[kBarEmpty + st]);
                    ++c;
                }
                tc_commit(&bars[kBarQEmpty + b]);
                tc_commit(&bars[kBarSFull + b]);
                return true;
            };
            auto pv_unit = [&](const EncUnit & U, int i) -> bool {
                const int b = i & 1;
                const uint32_t k = (uint32_t) (i >> 1) & 1;
                if (!enc_wait(&bars[kBarPFull + b], k, abort_flag, p.error)) return false;
                if (!enc_wait(&bars[kBarOEmpty + b], k ^ 1, abort_flag, p.error)) return false;
                tc_fence_after();
                const uint32_t pa = smem_u32(pbuf + b * kPBuf);
                const uint32_t od = tmem + 192 + 128 * b;
                for (int t = 0; t < U.T; ++t) {
                    const int st = (int) (c % kTcStages);
                    if (!enc_wait(&bars[kBarFull + st], (c / kTcStages) & 1, abort_flag, p.error)) return false;
                    tc_fence_after();
                    const uint32_t sa = smem_u32(stages + st * kTcStageBytes);
                    // acc ks += [V^T(keys 16ks..) ; V^T(keys 64+16ks..)] . [P^T(keys 16ks..) | P^T(keys 64+16ks..)]
                    // B rows: P_hi, P_lo of keys 16ks.., then P_hi, P_lo of keys 64+16ks.. (8 rows each)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        tc_mma(od + 32 * ks, sw128_desc(sa + ks * 2048, 8192, 1024),
                               sw128_desc(pa + t * 4096 + ks * 32, 16, 1024), idesc_pv, t != 0);
                    }
                    tc_commit(&bars[kBarEmpty + st]);
                    ++c;
                }
                tc_commit(&bars[kBarPEmpty + b]);
                tc_commit(&bars[kBarOFull + b]);
                return true;
            };
            // Ring loads in the producer's order: K tiles of unit i at [kc, kc + T_i),
            // then V tiles of unit i - 1 at [kc + T_i, kc + T_i + T_(i-1)); each
            // issuer walks the same sequence and consumes its own tiles.
            bool ok = true;
            EncUnit prev{};
            int i = 0;
            uint32_t kc = 0;
            UnitWalk W;
            W.init(p, blockIdx.x, stride, n_units);
            for (; ok && W.more(); ++i) {
                const EncUnit U = W.take(p);
                if (s_role) {
                    c = kc;
                    ok = s_unit(U, i);
                } else if (i > 0) {
                    c = kc + (uint32_t) U.T;
                    ok = pv_unit(prev, i - 1);
                }
                kc += (uint32_t) U.T + (i > 0 ? (uint32_t) prev.T : 0u);
                prev = U;
            }
            if (!s_role && ok && i > 0) {
                c = kc;
                pv_unit(prev, i - 1);
            }
            // every MMA issued so far completes before the CTA frees TMEM
            // (the barrier completes once both issuers' MMAs are done)
            tc_commit(&bars[kBarDrain]);
            enc_drain(&bars[kBarDrain], 0);
        }
        __syncwarp();
    } else if (warp == kWarpQ) {
        // ---------------- Q^T (hi, lo) producer ----------------
        // 8 query rows x 64 dims per unit, rotated, scaled by log2(e)/sqrt(64),
        // 128-byte swizzled K-major rows.  Lane l handles dims 2l, 2l+1 of every
        // row; rows of a group are consecutive positions ending at U.we.
        UnitWalk W;
        W.init(p, blockIdx.x, stride, n_units);
        for (int i = 0; W.more(); ++i) {
            const EncUnit U = W.take(p);
            const int b = i & 1;
            const uint32_t k = (uint32_t) (i >> 1) & 1;
            const int pos0 = U.we - U.nr + 1;
            float2 xq[8], cs[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                xq[j] = cs[j] = make_float2(0.0f, 0.0f);
                if (j < U.nr) {
                    xq[j] = *reinterpret_cast<const float2 *>(p.q + ((int64_t) (U.r0 + j) * p.n_heads + U.h) * kEncHd +
                                                                2 * lane);
                    cs[j] = p.rope[(int64_t) (pos0 + j) * (kEncHd / 2) + lane];
                }
            }
            if (!__all_sync(kFull, enc_wait(&bars[kBarQEmpty + b], k ^ 1, abort_flag, p.error))) break;
            uint8_t * qb = qbuf + b * 2048;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float2 qv = make_float2(0.0f, 0.0f);
                if (j < U.nr) {
                    const float2 rr = enc_rope_pair(xq[j], cs[j]);
                    qv = make_float2(rr.x * p.scale_log2, rr.y * p.scale_log2);
                }
                const uint16_t hx = to16<DT>(qv.x), hy = to16<DT>(qv.y);
                const uint16_t lx = to16<DT>(qv.x - from16<DT>(hx)), ly = to16<DT>(qv.y - from16<DT>(hy));
                const int off = j * 128 + (((lane >> 2) ^ j) << 4) + (lane & 3) * 4;
                *reinterpret_cast<uint32_t *>(qb + off) = (uint32_t) hx | ((uint32_t) hy << 16);
                *reinterpret_cast<uint32_t *>(qb + 1024 + off) = (uint32_t) lx | ((uint32_t) ly << 16);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kBarQFull + b]);
        }
    } else {
        // ---------------- softmax and epilogue, warps 0-7 ----------------
        // Set `set` (warps 4 set .. 4 set + 3) takes the CTA's units i with
        // i & 1 == set, i.e. buffer set b = set of Q, S, P and O.  Thread r
        // owns key row r of every tile (TMEM lane r, quadrant warp & 3).  The
        // loop never leaves early, so the set's named barrier stays matched;
        // after an abort every wait returns at once and no result is written.
        const int set = warp >> 2;
        const int wq = warp & 3;
        const uint32_t lane_off = (uint32_t) (32 * wq) << 16;
        const int r = 32 * wq + lane;
        float * epi = epi_all + set * 8 * 64;
        float * rmax = redmax + set * 32;
        auto epilogue = [&](const EncUnit & U, int j) {
            const int b = j & 1;
            const uint32_t k = (uint32_t) (j >> 1) & 1;
            const bool have_o = __all_sync(kFull, enc_wait(&bars[kBarOFull + b], k, abort_flag, p.error));
            tc_fence_after();
            float ov[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) ov[q] = 0.0f;
            const int half = wq >> 1;  // lanes 0-63: keys 0-63 of each tile; lanes 64-127: keys 64-127
            if (have_o) {
                uint32_t acc[4][16];
#pragma unroll
                for (int a = 0; a < 4; ++a) tmem_ld16_nw(tmem + 192 + 128 * b + 32 * a + 16 * half + lane_off, acc[a]);
                tmem_wait_ld();
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int q = 0; q < 8; ++q) ov[q] += __uint_as_float(acc[a][q]) + __uint_as_float(acc[a][8 + q]);
            }
            tc_fence_before();
            mbar_arrive(&bars[kBarOEmpty + b]);
            const int dim = 32 * (wq & 1) + lane;
            if (half) {
#pragma unroll
                for (int q = 0; q < 8; ++q) epi[q * 64 + dim] = ov[q];
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory");
            if (!half && have_o && !*abort_flag) {
                const float * ls = redsum + b * 32;
                for (int q = 0; q < U.nr; ++q) {
                    const float L = ls[q] + ls[8 + q] + ls[16 + q] + ls[24 + q];
                    p.out[((int64_t) (U.r0 + q) * p.n_heads + U.h) * kEncHd + dim] = (ov[q] + epi[q * 64 + dim]) / L;
                }
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory");  // epi is rewritten by the next epilogue
        };
        UnitWalk W;
        W.init(p, blockIdx.x + set * stride, kTcSets * stride, n_units);
        EncUnit prev{};
        int iprev = -1;
        for (int i = set; W.more(); i += kTcSets) {
            const EncUnit U = W.take(p);
            const int b = i & 1;
            const uint32_t k = (uint32_t) (i >> 1) & 1;
            float sv[kTcMaxTiles][8];
            const bool have_s = __all_sync(kFull, enc_wait(&bars[kBarSFull + b], k, abort_flag, p.error));
            tc_fence_after();
#pragma unroll
            for (int t = 0; t < kTcMaxTiles; ++t) {
                if (have_s && t < U.T) {
                    float sr[16];
                    tmem_ld16(tmem + 96 * b + lane_off + 16 * t, sr);
#pragma unroll
                    for (int q = 0; q < 8; ++q) sv[t][q] = sr[q] + sr[8 + q];
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[kBarSEmpty + b]);
            int qpos[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) qpos[q] = q < U.nr ? U.we - U.nr + 1 + q : -1;
            float mx[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) mx[q] = -INFINITY;
            // slot and absolute position of key row r: for the boxes walked
            // (gb < nb) s0 + 8 gb < 2 vslots and (we % cap) - slot + cap lies in
            // (0, 2 cap), so one conditional subtraction replaces each modulo;
            // the other rows are masked whatever they compute
            const int wem = U.wem;
#pragma unroll
            for (int t = 0; t < kTcMaxTiles; ++t) {
                if (t >= U.T) break;
                const int gb = t * kTcBoxes + (r >> 3);
                int sb = U.s0 + 8 * gb;
                sb = sb >= vslots ? sb - vslots : sb;
                const int slot = sb + (r & 7);
                bool valid = have_s && gb < U.nb && slot < cap;
                int back = wem - slot + cap;
                back = back >= cap ? back - cap : back;
                const int kp = U.we - back;
                valid = valid && kp >= U.ws;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const bool ok = valid && q < U.nr && kp <= qpos[q] && kp >= qpos[q] - (p.window - 1);
                    sv[t][q] = ok ? sv[t][q] : -INFINITY;
                    mx[q] = fmaxf(mx[q], sv[t][q]);
                }
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) mx[q] = fmaxf(mx[q], __shfl_xor_sync(kFull, mx[q], o));
            }
            if (lane == 0) {
#pragma unroll
                for (int q = 0; q < 8; ++q) rmax[wq * 8 + q] = mx[q];
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory");
            float M[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                M[q] = fmaxf(fmaxf(rmax[q], rmax[8 + q]), fmaxf(rmax[16 + q], rmax[24 + q]));
                if (M[q] == -INFINITY) M[q] = 0.0f;  // padding queries
            }
            // P of set b is free once the PV MMAs of unit i-2 completed
            enc_wait(&bars[kBarPEmpty + b], k ^ 1, abort_flag, p.error);
            float ls[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) ls[q] = 0.0f;
            uint8_t * pb = pbuf + b * kPBuf;
#pragma unroll
            for (int t = 0; t < kTcMaxTiles; ++t) {
                if (t >= U.T) break;
                // B operand rows 0-7 = P_hi of queries 0-7, rows 8-15 = P_lo
                uint8_t * ph = pb + t * 4096 + (r >> 6) * 2048;
                uint8_t * pl = ph + 1024;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float e = exp2f(sv[t][q] - M[q]);
                    const uint16_t hi = to16<DT>(e);
                    const float ehi = from16<DT>(hi);
                    const uint16_t lo = to16<DT>(e - ehi);
                    ls[q] += ehi + from16<DT>(lo);
                    const int off = q * 128 + ((((r & 63) >> 3) ^ q) << 4) + (r & 7) * 2;
                    *reinterpret_cast<uint16_t *>(ph + off) = hi;
                    *reinterpret_cast<uint16_t *>(pl + off) = lo;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&bars[kBarPFull + b]);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) ls[q] += __shfl_xor_sync(kFull, ls[q], o);
            }
            if (lane == 0) {
#pragma unroll
                for (int q = 0; q < 8; ++q) redsum[b * 32 + wq * 8 + q] = ls[q];
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + set) : "memory");
            if (kTcSets == 2) {
                // this set's next unit is two units away: finish this one first
                epilogue(U, i);
            } else {
                // one set: the previous unit's products are done by now
                if (iprev >= 0) epilogue(prev, iprev);
                prev = U;
                iprev = i;
            }
        }
        if (kTcSets == 1 && iprev >= 0) epilogue(prev, iprev);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}


// ---------------------------------------------------------------------------
// f32 rings: window attention on the CUDA cores
// ---------------------------------------------------------------------------
constexpr int kF32Threads = 128;
constexpr int kF32Tile = 128;                  // keys per stage
constexpr int kF32MaxKeys = 768;               // window - 1 + 8 rows fits (host checks <= 752)
constexpr int kF32Rows = 8;                    // rows per group (kEncRowsPerGroup)
// Kernel variants: R = rows per group the scores are kept for (8, or 4 for the
// steady chunk, whose smaller score buffer leaves room for a third stage at two
// CTAs per SM), NS = 128-key stages in flight.
constexpr int kF32RowBytes = kEncHd * 4;       // 256

template <int R, int NS>
struct __align__(128) EncF32Smem {
    float kv[NS][kF32Tile * kEncHd];           // 128-key stages (rows swizzled as in the ring)
    float s[kF32MaxKeys][R];                   // scores, then probabilities: [key][row]
    float q[kEncHd][R];                        // rotated, scaled queries: [dim][row]
    float red[kF32Threads / 32][R];
    float inv_l[R];
    uint64_t full[NS];
    int32_t abort_flag;
};
static_assert(sizeof(float) * kF32Rows * 8 * kEncHd <= sizeof(float) * kF32Tile * kEncHd,
              "P.V partial sums fit one stage buffer");

// One CTA per unit (row group of <= 8 rows of one stream, head).  The unit's
// keys stream through two 128-key stages (K stages, then V stages); thread 0
// refills a stage as soon as every thread has finished with it.  Row bounds
// and ring slots come from the group descriptor (rows of a group are
// consecutive positions), with no division per key.  Measured and dropped:
// five 64-key stages with two threads per key (slower: the kernel is bound
// by the latency of its shared-memory loads and FMA chains, not by copies in
// flight).
template <int R, int NS>
__global__ void __launch_bounds__(kF32Threads) enc_f32_kernel(const EncParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    EncF32Smem<R, NS> & S = *reinterpret_cast<EncF32Smem<R, NS> *>(smem_raw);
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    if (tid == 0) {
        for (int st = 0; st < NS; ++st) mbar_init(&S.full[st], 1);
        S.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // nothing an earlier grid writes is read before this point
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int u = blockIdx.x;
    const int grp = u / p.n_heads;
    const int h = u - grp * p.n_heads;
    const int4 ga = __ldg(p.groups + 2 * grp), gb = __ldg(p.groups + 2 * grp + 1);
    const int r0 = ga.x & 0xffffff;
    const int nr = (int) ((unsigned) ga.x >> 24);
    const int ws = ga.z;
    const int we = ga.w;
    const int nkeys = we - ws + 1;
    if (nr < 1 || nr > R || nkeys < 1 || nkeys > kF32MaxKeys) {
        if (tid == 0 && p.error) atomicCAS(p.error, 0, 1);
        return;
    }
    const int cap = p.capacity;
    int slot0 = gb.z - (nkeys - 1);  // ws % capacity: the window is shorter than the ring
    slot0 = slot0 < 0 ? slot0 + cap : slot0;
    const int T = (nkeys + kF32Tile - 1) / kF32Tile;  // stages of K, then as many of V
    const int64_t ring = ring_index(p, ga.y, h);
    const uint64_t policy = evict_first_policy();
    // stage j < T: K keys [64 j, ...); stage j >= T: V keys [64 (j - T), ...)
    auto issue = [&](int j) {
        const int jj = j < T ? j : j - T;
        const int k0 = jj * kF32Tile;
        const int n = min(kF32Tile, nkeys - k0);
        int slot = slot0 + k0;
        slot = slot >= cap ? slot - cap : slot;
        const int run = min(n, cap - slot);
        const uint8_t * base = (j < T ? p.k_ring : p.v_ring) + ring * p.ring_slots * (int64_t) kF32RowBytes;
        uint64_t * bar = &S.full[j % NS];
        float * dst = S.kv[j % NS];
        mbar_expect_tx(bar, (uint32_t) (n * kF32RowBytes));
        bulk_load(dst, base + (int64_t) slot * kF32RowBytes, (uint32_t) (run * kF32RowBytes), bar, policy);
        if (n > run) bulk_load(dst + run * kEncHd, base, (uint32_t) ((n - run) * kF32RowBytes), bar, policy);
    };
    int issued = 0;  // thread 0: stages issued so far
    if (tid == 0)
        for (; issued < NS && issued < 2 * T; ++issued) issue(issued);
    // queries: thread t -> row t / 16, dims 4 (t % 16) .. + 3
    {
        const int r = tid >> 4;
        const int c = tid & 15;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < nr) {
            const int pos = we - (nr - 1) + r;
            const float * qr = p.q + ((int64_t) (r0 + r) * p.n_heads + h) * kEncHd + 4 * c;
            const float2 * cs = p.rope + (int64_t) pos * (kEncHd / 2) + 2 * c;
            const float2 a = enc_rope_pair(*reinterpret_cast<const float2 *>(qr), cs[0]);
            const float2 b = enc_rope_pair(*reinterpret_cast<const float2 *>(qr + 2), cs[1]);
            v = make_float4(a.x * p.scale_log2, a.y * p.scale_log2, b.x * p.scale_log2, b.y * p.scale_log2);
        }
        if (r < R) {
            S.q[4 * c + 0][r] = v.x;
            S.q[4 * c + 1][r] = v.y;
            S.q[4 * c + 2][r] = v.z;
            S.q[4 * c + 3][r] = v.w;
        }
    }
    // row r attends [max(0, pos_r - window + 1), pos_r], pos_r = we - (nr - 1) + r
    int lo[R], hi[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        hi[r] = r < nr ? we - (nr - 1) + r : -1;
        lo[r] = max(0, hi[r] - (p.window - 1));
    }
    __syncthreads();
    float acc[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.0f;
    const int c4 = tid & 15;     // P.V: dims 4 c4 .. + 3
    const int kg = tid >> 4;     //       keys kg, kg + 8, ... of each stage
    bool ok = true;
    int j = 0;
    for (; j < 2 * T; ++j) {
        // stage (j - 1) % S was released by the barrier that ended iteration j - 1
        if (tid == 0 && j > 0 && j + NS - 1 < 2 * T) issue(issued++);
        const bool landed = enc_wait(&S.full[j % NS], (uint32_t) ((j / NS) & 1), &S.abort_flag, p.error);
        if (!__syncthreads_and(landed ? 1 : 0)) {
            ok = false;
            break;
        }
        const float * buf = S.kv[j % NS];
        if (j < T) {
            // ---- scores of key 128 j + tid for every row ------------------------
            const int ki = j * kF32Tile + tid;
            if (ki < nkeys) {
                int slot = slot0 + ki;
                slot = slot >= cap ? slot - cap : slot;
                const int sw = slot & 7;
                float sc[R];
#pragma unroll
                for (int r = 0; r < R; ++r) sc[r] = 0.0f;
                const float * kr = buf + tid * kEncHd;
#pragma unroll 4
                for (int c = 0; c < kEncHd / 4; ++c) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(kr + 4 * (c ^ sw));
                    const float kd[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
                    for (int d = 0; d < 4; ++d) {
                        const float4 qa = *reinterpret_cast<const float4 *>(&S.q[4 * c + d][0]);
                        sc[0] = fmaf(qa.x, kd[d], sc[0]);
                        sc[1] = fmaf(qa.y, kd[d], sc[1]);
                        sc[2] = fmaf(qa.z, kd[d], sc[2]);
                        sc[3] = fmaf(qa.w, kd[d], sc[3]);
                        if constexpr (R > 4) if (nr > 4) {
                            const float4 qb = *reinterpret_cast<const float4 *>(&S.q[4 * c + d][4]);
                            sc[4] = fmaf(qb.x, kd[d], sc[4]);
                            sc[5] = fmaf(qb.y, kd[d], sc[5]);
                            sc[6] = fmaf(qb.z, kd[d], sc[6]);
                            sc[7] = fmaf(qb.w, kd[d], sc[7]);
                        }
                    }
                }
                const int kp = ws + ki;
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (!(kp >= lo[r] && kp <= hi[r])) sc[r] = -INFINITY;
                *reinterpret_cast<float4 *>(&S.s[ki][0]) = make_float4(sc[0], sc[1], sc[2], sc[3]);
                if constexpr (R > 4)
                    *reinterpret_cast<float4 *>(&S.s[ki][4]) = make_float4(sc[4], sc[5], sc[6], sc[7]);
            }
        } else {
            // ---- P.V over this stage's keys kg, kg + 8, ... --------------------
            const int k0 = (j - T) * kF32Tile;
            const int n = min(kF32Tile, nkeys - k0);
            int slot = slot0 + k0 + kg;
            slot = slot >= cap ? slot - cap : slot;
            for (int i = kg; i < n; i += kF32Threads / 16) {
                const int ki = k0 + i;
                const int sw = slot & 7;
                slot += kF32Threads / 16;
                slot = slot >= cap ? slot - cap : slot;
                const float4 v4 = *reinterpret_cast<const float4 *>(buf + i * kEncHd + 4 * (c4 ^ sw));
                const float4 pa = *reinterpret_cast<const float4 *>(&S.s[ki][0]);
                const float pr[4] = {pa.x, pa.y, pa.z, pa.w};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    acc[r][0] = fmaf(pr[r], v4.x, acc[r][0]);
                    acc[r][1] = fmaf(pr[r], v4.y, acc[r][1]);
                    acc[r][2] = fmaf(pr[r], v4.z, acc[r][2]);
                    acc[r][3] = fmaf(pr[r], v4.w, acc[r][3]);
                }
                if constexpr (R > 4) if (nr > 4) {
                    const float4 pb = *reinterpret_cast<const float4 *>(&S.s[ki][4]);
                    const float pq[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        acc[4 + r][0] = fmaf(pq[r], v4.x, acc[4 + r][0]);
                        acc[4 + r][1] = fmaf(pq[r], v4.y, acc[4 + r][1]);
                        acc[4 + r][2] = fmaf(pq[r], v4.z, acc[4 + r][2]);
                        acc[4 + r][3] = fmaf(pq[r], v4.w, acc[4 + r][3]);
                    }
                }
            }
        }
        __syncthreads();
        if (j == T - 1) {
            // ---- exact softmax over the window, per row ------------------------
            float mx[R];
#pragma unroll
            for (int r = 0; r < R; ++r) mx[r] = -INFINITY;
            for (int ki = tid; ki < nkeys; ki += kF32Threads) {
#pragma unroll
                for (int r = 0; r < R; ++r) mx[r] = fmaxf(mx[r], S.s[ki][r]);
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) mx[r] = fmaxf(mx[r], __shfl_xor_sync(kFull, mx[r], o));
            }
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) S.red[warp][r] = mx[r];
            }
            __syncthreads();
            float M[R], ls[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                M[r] = fmaxf(fmaxf(S.red[0][r], S.red[1][r]), fmaxf(S.red[2][r], S.red[3][r]));
                ls[r] = 0.0f;
            }
            __syncthreads();
            for (int ki = tid; ki < nkeys; ki += kF32Threads) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    // every real row holds its own position: M[r] is finite
                    const float e = r < nr ? exp2f(S.s[ki][r] - M[r]) : 0.0f;
                    S.s[ki][r] = e;
                    ls[r] += e;
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) ls[r] += __shfl_xor_sync(kFull, ls[r], o);
            }
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; ++r) S.red[warp][r] = ls[r];
            }
            __syncthreads();
            if (tid < R) {
                const float l = (S.red[0][tid] + S.red[1][tid]) + (S.red[2][tid] + S.red[3][tid]);
                S.inv_l[tid] = l > 0.0f ? 1.0f / l : 0.0f;
            }
            __syncthreads();
        }
    }
    if (!ok) {
        // let the copies in flight (stages j .. issued - 1) land before the CTA exits
        if (tid == 0)
            for (int d = j; d < issued; ++d) enc_drain(&S.full[d % NS], (uint32_t) ((d / NS) & 1));
        return;
    }
    // ---- sum the key groups' partial products -----------------------------
    float * part = S.kv[0];  // [kg][row][dim]
#pragma unroll
    for (int r = 0; r < R; ++r)
        *reinterpret_cast<float4 *>(part + (kg * R + r) * kEncHd + 4 * c4) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    __syncthreads();
    {
        const int r = tid >> 4;
        if (r < nr) {
            float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int g = 0; g < kF32Threads / 16; ++g) {
                const float4 x = *reinterpret_cast<const float4 *>(part + (g * R + r) * kEncHd + 4 * c4);
                o.x += x.x;
                o.y += x.y;
                o.z += x.z;
                o.w += x.w;
            }
            const float il = S.inv_l[r];
            *reinterpret_cast<float4 *>(p.out + ((int64_t) (r0 + r) * p.n_heads + h) * kEncHd + 4 * c4) =
                make_float4(o.x * il, o.y * il, o.z * il, o.w * il);
        }
    }
}
}  // namespace

int enc_smem_bytes() { return kTcSmem; }

int enc_max_tiles() { return kTcMaxTiles; }

// Both encoder kernels wait (griddepcontrol.wait) before reading anything an
// earlier grid may write, so they are always launched with programmatic
// stream serialization: their launch and prologue overlap the previous grid.
template <typename K>
cudaError_t launch_pdl(K kernel, unsigned grid, unsigned block, size_t smem, cudaStream_t stream, const EncParams & p) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

cudaError_t launch_enc_append(const EncParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    if (p.dtype == 30) return launch_pdl(enc_append_kernel<30>, (unsigned) p.n_rows, 256, 0, stream, p);
    if (p.dtype == 0) return launch_pdl(enc_append_kernel<0>, (unsigned) p.n_rows, 256, 0, stream, p);
    return launch_pdl(enc_append_kernel<1>, (unsigned) p.n_rows, 256, 0, stream, p);
}

cudaError_t launch_enc_attention(const EncParams & p, cudaStream_t stream) {
    if (p.n_groups <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const int units = p.n_groups * p.n_heads;
    if (p.dtype == 0) {
        if (p.max_group_rows <= 4) {
            const int smem = (int) sizeof(EncF32Smem<4, 3>);
            e = cudaFuncSetAttribute(enc_f32_kernel<4, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            return launch_pdl(enc_f32_kernel<4, 3>, (unsigned) units, kF32Threads, (size_t) smem, stream, p);
        }
        const int smem = (int) sizeof(EncF32Smem<8, 2>);
        e = cudaFuncSetAttribute(enc_f32_kernel<8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        return launch_pdl(enc_f32_kernel<8, 2>, (unsigned) units, kF32Threads, (size_t) smem, stream, p);
    }
    // persistent: one CTA per SM (the shared-memory ring allows no second)
    const unsigned grid = (unsigned) (units < sms ? units : sms);
    if (p.dtype == 30) {
        e = cudaFuncSetAttribute(enc_tc_kernel<30>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        if (e != cudaSuccess) return e;
        return launch_pdl(enc_tc_kernel<30>, grid, kTcThreads, kTcSmem, stream, p);
    } else {
        e = cudaFuncSetAttribute(enc_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
        if (e != cudaSuccess) return e;
        return launch_pdl(enc_tc_kernel<1>, grid, kTcThreads, kTcSmem, stream, p);
    }
}

}  // namespace vxk
