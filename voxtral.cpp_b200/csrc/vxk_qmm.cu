// Quantized-weight matrix product y = x . W^T for GGUF Q8_0 / Q4_K / Q6_K
// weights (vxk_qweight_matmul, include/vxk.h), with the arithmetic of
// ggml's CPU backend: x rows quantized to Q8_0 / Q8_K, exact integer block
// dot products, block scales applied in fp32.  Replaces the ggml_mul_mat of
// the decoder projections (src/voxtral.cpp:2659-2661, 2857), FFN (2877-2881),
// adapter (2575-2580) and tied logits (2955) of a quantized model.
//
// Two kernels per product:
//   qmm_act_kernel  quantizes the activation rows (one CTA per 256-column
//                   unit and row) into int8 tensor-core B fragments plus
//                   their scales (and, for Q4_K, the 32-value sums the
//                   sub-block mins multiply);
//   qmm_kernel      one warp per 16-row weight tile streams the tile's
//                   records (16 rows x 256 columns, fragment order) through
//                   its own ring of bulk copies and multiplies them with the
//                   CTA's staged activations on the int8 tensor cores
//                   (mma.sync m16n8k32; m16n8k16 for Q6_K's 16-value
//                   sub-blocks); sub-block scales are applied to the int32
//                   results, block scales in fp32.  The column range can be
//                   split over the CTAs of a thread-block cluster, which sum
//                   their partial blocks through distributed shared memory
//                   in split order.
// The weight stream is the HBM traffic (4352 / 2368 / 3360 bytes per 4096
// weights); activations are a few hundred KB and stay in L2.
#include "vxk_internal.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

namespace vxk {
namespace {

constexpr int kThreads = 128;  // 4 warps, one 16-row tile each
constexpr int kStages = 4;     // weight records in flight per warp
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kErrTimeout = 2;
constexpr unsigned kFull = 0xffffffffu;

__host__ __device__ constexpr int rec_bytes(int type) {
    return type == 8 ? 4352 : type == 12 ? 2368 : type == 14 ? 3360 : 0;
}

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
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > kWaitNs) return false;
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

// Barrier over the CTAs of this thread-block cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory offset in cluster CTA `rank`, and a load from it.
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
// order, four rows per load; every split's loads are issued before the sum.
template <int R>
__device__ __forceinline__ void cluster_reduce_store(uint32_t local, int S, int e0, int e1, int tid, int nthreads,
                                                     float * y, int64_t n_rows, int64_t row0) {
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


__device__ __forceinline__ void set_error(int32_t * err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// D = A(16x32 s8, row) * B(32x8 s8, col), int32.
__device__ __forceinline__ void imma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D = A(16x16 s8, row) * B(16x8 s8, col), int32.
__device__ __forceinline__ void imma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// Four unsigned bytes in 0..63 minus 32 each, as four int8 (no borrow: the
// top bit of every byte is set before the subtraction and flipped after).
__device__ __forceinline__ uint32_t sub32x4(uint32_t v) {
    return ((v | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
}

__device__ __forceinline__ int byte_s(uint32_t w, int i) { return (int) (int8_t) (w >> (8 * i)); }
__device__ __forceinline__ int byte_u(uint32_t w, int i) { return (int) ((w >> (8 * i)) & 0xffu); }

// ---------------------------------------------------------------------------
// Activation quantization.  FAM 0: quantize_row_q8_0_ref per 32 values
// (d = amax/127, id = d ? 1/d : 0, q = roundf(x*id), d kept as its f16);
// FAM 1: quantize_row_q8_K_ref per 256 values (max = the value of largest
// magnitude, first on ties; iscale = -127/max; q = min(127, round-half-even
// (iscale*x)); d = 1/iscale), plus the sums s_j of the 32 q of each sub-block
// j that Q4_K's mins multiply, as s_j = 128 h_j + l_j (h_j in [-32, 31], l_j
// in [0, 127]): two int8 B fragments of an m16n8k16 product whose k is j
// (lanes with k >= 8 hold zeros, written once when the scratch is created).
// Grid (units, nt*8 rows), 256 threads: thread t holds column 256u + t.
// Rows past p.rows are written as zeros.
// ---------------------------------------------------------------------------
template <int FAM>
__global__ void __launch_bounds__(256) qmm_act_kernel(const QmmParams p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int u = blockIdx.x, r = blockIdx.y, t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const int64_t K = (int64_t) p.n_units * kQmmUnit;
    const int ncol = p.nt * 8;
    const int64_t xi = (int64_t) r * K + (int64_t) u * kQmmUnit + t;
    const float x = r < p.rows ? (p.x_up ? swiglu_value(p.x[xi], p.x_up[xi]) : p.x[xi]) : 0.0f;
    int q = 0;
    if constexpr (FAM == 0) {
        float amax = fabsf(x);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        q = (int) roundf(__fmul_rn(x, id));
        if (lane == 0) p.act_d[((int64_t) u * 8 + warp) * ncol + r] = __half2float(__float2half_rn(d));
    } else {
        __shared__ unsigned long long red[8];
        __shared__ float s_max;
        // key: |x| bits (non-negative floats order as integers), then the
        // inverted column so that the first column wins a tie
        unsigned long long key = ((unsigned long long) __float_as_uint(fabsf(x)) << 32) | (unsigned) (255 - t);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(kFull, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0) red[warp] = key;
        __syncthreads();
        unsigned long long best = red[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) best = red[w] > best ? red[w] : best;
        const int arg = 255 - (int) (best & 0xffffffffu);
        if (t == arg) s_max = x;
        __syncthreads();
        const float amax = __uint_as_float((unsigned) (best >> 32));
        float d = 0.0f;
        if (amax != 0.0f) {
            const float iscale = __fdiv_rn(-127.0f, s_max);
            q = min(127, __float2int_rn(__fmul_rn(iscale, x)));
            d = __fdiv_rn(1.0f, iscale);
        }
        int s = q;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
        if (lane == 0) {
            // B fragment b0 of column r, k = j: lane 4*(r%8) + j/4, byte j%4
            uint8_t * ms = p.act_ms + (((int64_t) u * p.nt + (r >> 3)) * 32 + 4 * (r & 7) + (warp >> 2)) * 8;
            ms[warp & 3] = (uint8_t) (int8_t) (s >> 7);
            ms[4 + (warp & 3)] = (uint8_t) (s & 127);
        }
        if (t == 0) p.act_d[(int64_t) u * ncol + r] = d;
    }
    // B fragment of block j = t / 32 for batch row r: lane 4*(r%8) + (k%16)/4,
    // byte 4*(k/16) + k%4, k = t % 32
    const int kk = t & 31;
    const int fl = 4 * (r & 7) + ((kk & 15) >> 2);
    const int fb = ((kk >> 4) << 2) + (kk & 3);
    p.act[((((int64_t) u * p.nt + (r >> 3)) * 8 + warp) * 32 + fl) * 8 + fb] = (uint8_t) (int8_t) q;
}

// ---------------------------------------------------------------------------
// The product.  Shared memory: [4 warps][kStages][record] weight rings, then
// the split's activations: B fragments [units][NT][8 blocks][32 lanes][8 B],
// scales (Q8_0 [units*8][NT*8], K-quants [units][NT*8] fp32), Q4_K sums of 32
// q as (h, l) B fragments [units][NT][32 lanes][8 B]; then mbarriers.
// ---------------------------------------------------------------------------
template <int WT, int NT>
struct QmmLayout {
    static constexpr int kRec = rec_bytes(WT);
    static constexpr int kRing = 4 * kStages * kRec;
    static constexpr int kActPerUnit = NT * 8 * 256;
    static constexpr int kScalePerUnit = (WT == 8 ? 8 : 1) * NT * 8 * 4;
    static constexpr int kSumPerUnit = WT == 12 ? NT * 32 * 8 : 0;
    static constexpr int kPerUnit = kActPerUnit + kScalePerUnit + kSumPerUnit;
    static int bytes(int units) { return kRing + units * kPerUnit + 256; }
};

// One CTA: 64 rows (row block rb) of matrix m over the split's column units.
template <int WT, int NT>
__device__ __forceinline__ void qmm_cta(const QmmParams & p, const QmmMat & m, const int rb, uint8_t * smem) {
    using L = QmmLayout<WT, NT>;
    constexpr int REC = L::kRec;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const int split = blockIdx.y;
    const int u0 = split * p.units_per_split;
    const int nu = min(p.n_units, u0 + p.units_per_split) - u0;
    const int cap = p.units_per_split;
    uint8_t * ring = smem;
    uint8_t * sact = smem + L::kRing;
    float * sd = reinterpret_cast<float *>(sact + cap * L::kActPerUnit);
    uint8_t * sms = reinterpret_cast<uint8_t *>(sd) + cap * L::kScalePerUnit;
    uint64_t * bars = reinterpret_cast<uint64_t *>(sms + cap * L::kSumPerUnit);
    // bars[w * kStages + s]: weight ring stages; bars[16]: activations
    int32_t * s_abort = reinterpret_cast<int32_t *>(bars + 4 * kStages + 1);
    if (tid == 0) {
        for (int i = 0; i < 4 * kStages + 1; ++i) mbar_init(&bars[i], 1);
        *s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // ---- weight ring of this warp's tile (weights are constant: the copies
    // may start before the previous kernel on the stream has finished) ----
    const int tile = rb * 4 + warp;
    const uint8_t * wt = m.w + ((int64_t) tile * p.n_units + u0) * REC;
    uint8_t * wring = ring + warp * kStages * REC;
    uint64_t * wbar = bars + warp * kStages;
    const uint64_t pol_w = l2_policy(true);
    int issued = 0;
    auto pump = [&](int consumed) {
        while (issued < nu && issued - consumed < kStages) {
            if (lane == 0) {
                const int st = issued % kStages;
                mbar_expect_tx(&wbar[st], REC);
                bulk_g2s(wring + st * REC, wt + (int64_t) issued * REC, REC, &wbar[st], pol_w);
            }
            ++issued;
        }
    };
    pump(0);

    // ---- the split's activations, written by the quantization kernel ----
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) {
        const uint64_t pol_a = l2_policy(false);
        const uint32_t a_bytes = nu * L::kActPerUnit, d_bytes = nu * L::kScalePerUnit,
                       s_bytes = nu * L::kSumPerUnit;
        mbar_expect_tx(&bars[4 * kStages], a_bytes + d_bytes + s_bytes);
        bulk_g2s(sact, p.act + (int64_t) u0 * L::kActPerUnit, a_bytes, &bars[4 * kStages], pol_a);
        bulk_g2s(sd, reinterpret_cast<const uint8_t *>(p.act_d) + (int64_t) u0 * L::kScalePerUnit, d_bytes,
                 &bars[4 * kStages], pol_a);
        if constexpr (WT == 12)
            bulk_g2s(sms, p.act_ms + (int64_t) u0 * L::kSumPerUnit, s_bytes,
                     &bars[4 * kStages], pol_a);
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    bool ok = __all_sync(kFull, mbar_wait(&bars[4 * kStages], 0));
    int consumed = 0;
    for (int i = 0; ok && i < nu; ++i) {
        const int st = i % kStages;
        if (!__all_sync(kFull, mbar_wait(&wbar[st], (uint32_t) (i / kStages) & 1u))) {
            ok = false;
            break;
        }
        const uint8_t * rec = wring + st * REC;
        const uint8_t * ua = sact + i * L::kActPerUnit;
        auto bfrag = [&](int n, int j) {
            return *reinterpret_cast<const uint2 *>(ua + ((n * 8 + j) * 32 + lane) * 8);
        };
        if constexpr (WT == 8) {
            // Q8_0: 8 blocks of 32 columns, one k32 product per block and n-tile,
            // scaled by d_w * d_x of the block
            const uint32_t * dws = reinterpret_cast<const uint32_t *>(rec + 4096);
            const float * dx = sd + i * 8 * NT * 8;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint4 a = *reinterpret_cast<const uint4 *>(rec + j * 512 + lane * 16);
                const uint32_t dwp = dws[j * 8 + g];
                const float2 dw = __half22float2(*reinterpret_cast<const __half2 *>(&dwp));
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    const uint2 b = bfrag(n, j);
                    int cc[4];
                    imma_k32(cc, a.x, a.y, a.z, a.w, b.x, b.y);
                    const float2 d = *reinterpret_cast<const float2 *>(dx + j * NT * 8 + n * 8 + 2 * c);
                    acc[n][0] = fmaf((float) cc[0], __fmul_rn(dw.x, d.x), acc[n][0]);
                    acc[n][1] = fmaf((float) cc[1], __fmul_rn(dw.x, d.y), acc[n][1]);
                    acc[n][2] = fmaf((float) cc[2], __fmul_rn(dw.y, d.x), acc[n][2]);
                    acc[n][3] = fmaf((float) cc[3], __fmul_rn(dw.y, d.y), acc[n][3]);
                }
            }
        } else if constexpr (WT == 12) {
            // Q4_K: 8 sub-blocks of 32 columns with 6-bit scales (int32 sums),
            // mins times the activation's 32-value sums, then
            // d_x*d_w * isum - d_x*dmin_w * msum
            const uint32_t ddg = *reinterpret_cast<const uint32_t *>(rec + 2048 + g * 4);
            const uint32_t ddh = *reinterpret_cast<const uint32_t *>(rec + 2048 + (g + 8) * 4);
            const uint2 scg = *reinterpret_cast<const uint2 *>(rec + 2112 + g * 8);
            const uint2 sch = *reinterpret_cast<const uint2 *>(rec + 2112 + (g + 8) * 8);
            const uint2 mng = *reinterpret_cast<const uint2 *>(rec + 2240 + g * 8);
            const uint2 mnh = *reinterpret_cast<const uint2 *>(rec + 2240 + (g + 8) * 8);
            int isum[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n) isum[n][0] = isum[n][1] = isum[n][2] = isum[n][3] = 0;
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                const uint4 v = *reinterpret_cast<const uint4 *>(rec + pr * 512 + lane * 16);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int s = 2 * pr + h;
                    const uint32_t a0 = (v.x >> (4 * h)) & 0x0f0f0f0fu, a1 = (v.y >> (4 * h)) & 0x0f0f0f0fu;
                    const uint32_t a2 = (v.z >> (4 * h)) & 0x0f0f0f0fu, a3 = (v.w >> (4 * h)) & 0x0f0f0f0fu;
                    const int sg = byte_u(s < 4 ? scg.x : scg.y, s & 3);
                    const int sh = byte_u(s < 4 ? sch.x : sch.y, s & 3);
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const uint2 b = bfrag(n, s);
                        int cc[4];
                        imma_k32(cc, a0, a1, a2, a3, b.x, b.y);
                        isum[n][0] += sg * cc[0];
                        isum[n][1] += sg * cc[1];
                        isum[n][2] += sh * cc[2];
                        isum[n][3] += sh * cc[3];
                    }
                }
            }
            const float2 dg = __half22float2(*reinterpret_cast<const __half2 *>(&ddg));
            const float2 dh = __half22float2(*reinterpret_cast<const __half2 *>(&ddh));
            const float * dx = sd + i * NT * 8;
            // mins: sum_j m_j * s_j = 128 * (m . h) + (m . l), k = j on the
            // tensor cores (A: the row's 8 mins in k 0..7, zero above)
            const uint32_t am0 = c == 0 ? mng.x : c == 1 ? mng.y : 0u;
            const uint32_t am1 = c == 0 ? mnh.x : c == 1 ? mnh.y : 0u;
            const uint8_t * um = sms + i * L::kSumPerUnit;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const uint2 bm = *reinterpret_cast<const uint2 *>(um + (n * 32 + lane) * 8);
                int mh[4], ml[4];
                imma_k16(mh, am0, am1, bm.x);
                imma_k16(ml, am0, am1, bm.y);
                const int col = n * 8 + 2 * c;
                const float2 d = *reinterpret_cast<const float2 *>(dx + col);
                acc[n][0] = fmaf(-__fmul_rn(d.x, dg.y), (float) (128 * mh[0] + ml[0]),
                                 fmaf(__fmul_rn(d.x, dg.x), (float) isum[n][0], acc[n][0]));
                acc[n][1] = fmaf(-__fmul_rn(d.y, dg.y), (float) (128 * mh[1] + ml[1]),
                                 fmaf(__fmul_rn(d.y, dg.x), (float) isum[n][1], acc[n][1]));
                acc[n][2] = fmaf(-__fmul_rn(d.x, dh.y), (float) (128 * mh[2] + ml[2]),
                                 fmaf(__fmul_rn(d.x, dh.x), (float) isum[n][2], acc[n][2]));
                acc[n][3] = fmaf(-__fmul_rn(d.y, dh.y), (float) (128 * mh[3] + ml[3]),
                                 fmaf(__fmul_rn(d.y, dh.x), (float) isum[n][3], acc[n][3]));
            }
        } else {
            // Q6_K: 16 sub-blocks of 16 columns with int8 scales; 6-bit quants
            // rebuilt from the low-nibble and high-2-bit planes, minus 32
            const uint4 scg = *reinterpret_cast<const uint4 *>(rec + 3072 + g * 16);
            const uint4 sch = *reinterpret_cast<const uint4 *>(rec + 3072 + (g + 8) * 16);
            const float dwg = __half2float(*reinterpret_cast<const __half *>(rec + 3328 + g * 2));
            const float dwh = __half2float(*reinterpret_cast<const __half *>(rec + 3328 + (g + 8) * 2));
            const uint32_t scgw[4] = {scg.x, scg.y, scg.z, scg.w};
            const uint32_t schw[4] = {sch.x, sch.y, sch.z, sch.w};
            int isum[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n) isum[n][0] = isum[n][1] = isum[n][2] = isum[n][3] = 0;
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
                const uint4 rl = *reinterpret_cast<const uint4 *>(rec + qd * 512 + lane * 16);
                const uint4 hq = *reinterpret_cast<const uint4 *>(rec + 2048 + (qd >> 1) * 512 + lane * 16);
                const uint32_t rlw[4] = {rl.x, rl.y, rl.z, rl.w};
                const uint32_t hw[2] = {(qd & 1) ? hq.z : hq.x, (qd & 1) ? hq.w : hq.y};
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    const int t = 4 * qd + tt;
                    const uint32_t hp = hw[tt >> 1];
                    const bool odd = tt & 1;
                    const uint32_t h0 = (odd ? hp : hp << 4) & 0x30303030u;
                    const uint32_t h1 = (odd ? hp >> 2 : hp << 2) & 0x30303030u;
                    const uint32_t a0 = sub32x4((rlw[tt] & 0x0f0f0f0fu) | h0);
                    const uint32_t a1 = sub32x4(((rlw[tt] >> 4) & 0x0f0f0f0fu) | h1);
                    const int sg = byte_s(scgw[t >> 2], t & 3);
                    const int sh = byte_s(schw[t >> 2], t & 3);
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const uint2 b = bfrag(n, t >> 1);
                        int cc[4];
                        imma_k16(cc, a0, a1, odd ? b.y : b.x);
                        isum[n][0] += sg * cc[0];
                        isum[n][1] += sg * cc[1];
                        isum[n][2] += sh * cc[2];
                        isum[n][3] += sh * cc[3];
                    }
                }
            }
            const float * dx = sd + i * NT * 8;
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const float2 d = *reinterpret_cast<const float2 *>(dx + n * 8 + 2 * c);
                acc[n][0] = fmaf(__fmul_rn(dwg, d.x), (float) isum[n][0], acc[n][0]);
                acc[n][1] = fmaf(__fmul_rn(dwg, d.y), (float) isum[n][1], acc[n][1]);
                acc[n][2] = fmaf(__fmul_rn(dwh, d.x), (float) isum[n][2], acc[n][2]);
                acc[n][3] = fmaf(__fmul_rn(dwh, d.y), (float) isum[n][3], acc[n][3]);
            }
        }
        __syncwarp();
        consumed = i + 1;
        pump(consumed);
    }
    if (!ok) {
        // drain this warp's copies still in flight (bounded), then report
        if (lane == 0) {
            for (int l = consumed; l < issued; ++l) mbar_wait(&wbar[l % kStages], (uint32_t) (l / kStages) & 1u);
            set_error(p.error, kErrTimeout);
            atomicExch(s_abort, 1);
        }
    }

    // ---- results.  The splits of a 64-row block are one thread-block
    // cluster: each CTA writes its partial block [columns][64 rows] into its
    // own shared memory (the drained weight ring); after a cluster barrier
    // CTA r sums slice r of the block over all splits, in split order, from
    // the members' shared memory (DSMEM), and writes y.  Every CTA reaches
    // both cluster barriers on every path (a CTA whose waits expired writes
    // nothing; the error word reports it). ----
    float * ptile = reinterpret_cast<float *>(ring);  // [NT * 8][64]
    __syncthreads();
    const bool live = *s_abort == 0;
    if (live) {
        const int r0 = warp * 16 + g;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int col = n * 8 + 2 * c;
            ptile[col * kQmmRows + r0] = acc[n][0];
            ptile[(col + 1) * kQmmRows + r0] = acc[n][1];
            ptile[col * kQmmRows + r0 + 8] = acc[n][2];
            ptile[(col + 1) * kQmmRows + r0 + 8] = acc[n][3];
        }
    }
    cluster_sync();
    if (live) {
        const int S = p.n_splits;
        const int E4 = p.rows * kQmmRows / 4;
        const int e0 = (int) ((int64_t) E4 * split / S), e1 = (int) ((int64_t) E4 * (split + 1) / S);
        cluster_reduce_store<kQmmRows>(smem_u32(ptile), S, e0, e1, tid, kThreads, m.y, m.n_rows,
                                       (int64_t) rb * kQmmRows);
    }
    cluster_sync();  // no CTA leaves while another still reads its shared memory
}

// The product over a group of matrices that share x (one weight type family):
// blockIdx.x runs over the matrices' 64-row blocks in order, blockIdx.y over
// the column splits.
template <int FAM, int NT>
__global__ void __launch_bounds__(kThreads, 1) qmm_kernel(const QmmParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    QmmMat m = p.mats[0];
#pragma unroll
    for (int i = 1; i < kQmmMaxGroup; ++i)
        if (i < p.n_mats && (int) blockIdx.x >= p.mats[i].block0) m = p.mats[i];
    const int rb = (int) blockIdx.x - m.block0;
    if constexpr (FAM == 0) {
        qmm_cta<8, NT>(p, m, rb, smem);
    } else {
        if (m.type == 12)
            qmm_cta<12, NT>(p, m, rb, smem);
        else
            qmm_cta<14, NT>(p, m, rb, smem);
    }
}

// Launch with programmatic dependent launch and, when cluster_y > 1, a
// thread-block cluster of (1, cluster_y, 1).
template <typename K>
cudaError_t launch_pdl(K kernel, dim3 grid, unsigned block, size_t smem, cudaStream_t stream, const QmmParams & p,
                       unsigned cluster_y = 1) {
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

template <int WT>
int layout_bytes(int nt, int units) {
    switch (nt) {
        case 1: return QmmLayout<WT, 1>::bytes(units);
        case 2: return QmmLayout<WT, 2>::bytes(units);
        case 4: return QmmLayout<WT, 4>::bytes(units);
        default: return QmmLayout<WT, 8>::bytes(units);
    }
}

int layout_bytes_type(int type, int nt, int units) {
    switch (type) {
        case 8: return layout_bytes<8>(nt, units);
        case 12: return layout_bytes<12>(nt, units);
        case 14: return layout_bytes<14>(nt, units);
        default: return 0;
    }
}

// The shared-memory cap of an instantiation is raised once per device.
template <int FAM, int NT>
cudaError_t raise_smem() {
    static bool raised[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!raised[dev]) {
        e = cudaFuncSetAttribute(qmm_kernel<FAM, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
        if (e != cudaSuccess) return e;
        raised[dev] = true;
    }
    return cudaSuccess;
}

template <int FAM, int NT>
cudaError_t launch_fam(const QmmParams & p, int smem, cudaStream_t stream) {
    cudaError_t e = raise_smem<FAM, NT>();
    if (e != cudaSuccess) return e;
    const int blocks = p.mats[p.n_mats - 1].block0 + p.mats[p.n_mats - 1].n_rows / kQmmRows;
    return launch_pdl(qmm_kernel<FAM, NT>, dim3((unsigned) blocks, (unsigned) p.n_splits), kThreads, (size_t) smem,
                      stream, p, (unsigned) p.n_splits);
}

// Resident CTAs per SM for a shared-memory size: asked of the runtime once per
// (device, size in 1 KB steps) and remembered, since the planner asks for
// every candidate split on every product call.
template <int FAM, int NT>
int ctas_fam(int smem) {
    static std::atomic<int> memo[64][233];
    if (raise_smem<FAM, NT>() != cudaSuccess) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || smem < 0 || smem > 232448) return 0;
    const int key = (smem + 1023) / 1024;
    std::atomic<int> & slot = memo[dev][key];
    const int known = slot.load(std::memory_order_relaxed);
    if (known > 0 && (known >> 20) == (smem & 0x3ff) + 1) return known & 0xfffff;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qmm_kernel<FAM, NT>, kThreads, (size_t) smem) != cudaSuccess)
        return 0;
    if (n > 0 && n < (1 << 20)) slot.store(((smem & 0x3ff) + 1) << 20 | n, std::memory_order_relaxed);
    return n;
}

template <int FAM>
cudaError_t launch_nt(const QmmParams & p, int smem, cudaStream_t stream) {
    switch (p.nt) {
        case 1: return launch_fam<FAM, 1>(p, smem, stream);
        case 2: return launch_fam<FAM, 2>(p, smem, stream);
        case 4: return launch_fam<FAM, 4>(p, smem, stream);
        case 8: return launch_fam<FAM, 8>(p, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <int FAM>
int ctas_nt(int nt, int smem) {
    switch (nt) {
        case 1: return ctas_fam<FAM, 1>(smem);
        case 2: return ctas_fam<FAM, 2>(smem);
        case 4: return ctas_fam<FAM, 4>(smem);
        default: return ctas_fam<FAM, 8>(smem);
    }
}

}  // namespace

int qmm_record_bytes(int type) { return rec_bytes(type); }

int qmm_smem_bytes(const QmmParams & p, int units) {
    int b = 0;
    for (int i = 0; i < p.n_mats; ++i) b = std::max(b, layout_bytes_type(p.mats[i].type, p.nt, units));
    return b;
}

int qmm_ctas_per_sm(const QmmParams & p, int smem) {
    return p.mats[0].type == 8 ? ctas_nt<0>(p.nt, smem) : ctas_nt<1>(p.nt, smem);
}

cudaError_t launch_qmm(const QmmParams & p, cudaStream_t stream) {
    if (p.n_mats < 1 || p.n_mats > kQmmMaxGroup || p.rows < 1 || p.rows > p.nt * 8 || p.units_per_split < 1 ||
        p.n_splits < 1 || p.n_splits > kQmmMaxSplits ||
        (int64_t) p.units_per_split * (p.n_splits - 1) >= p.n_units)
        return cudaErrorInvalidValue;
    const int fam = p.mats[0].type == 8 ? 0 : 1;
    for (int i = 0; i < p.n_mats; ++i)
        if (p.mats[i].n_rows % kQmmRows != 0 || (p.mats[i].type == 8 ? 0 : 1) != fam) return cudaErrorInvalidValue;
    const int smem = qmm_smem_bytes(p, p.units_per_split);
    if (smem <= 0 || smem > 232448) return cudaErrorInvalidValue;
    const dim3 agrid((unsigned) p.n_units, (unsigned) (p.nt * 8));
    cudaError_t e = fam == 0 ? launch_pdl(qmm_act_kernel<0>, agrid, 256, 0, stream, p)
                             : launch_pdl(qmm_act_kernel<1>, agrid, 256, 0, stream, p);
    if (e != cudaSuccess) return e;
    return fam == 0 ? launch_nt<0>(p, smem, stream) : launch_nt<1>(p, smem, stream);
}

}  // namespace vxk
