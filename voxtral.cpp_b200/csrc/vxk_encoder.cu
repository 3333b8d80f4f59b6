// sm_100a kernels of the streaming-encoder KV ring:
//   enc_append_kernel     RoPE on K + 16-bit store of K/V at slot pos % capacity
//                         (set_rows of src/voxtral.cpp:2474-2479)
//   enc_attention_kernel  masked window attention of a stream's new rows over
//                         [max(0, q - window + 1), q] (src/voxtral.cpp:2480-2487,
//                         mask of src/voxtral.cpp:4104-4119), scale 1/sqrt(64).
//
// Ring layout: [stream][layer][head][capacity][64] 16-bit, so one (stream,
// layer, head) ring is a contiguous 878 x 128-byte region.
#include "vxk_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace vxk {
namespace {

constexpr int kEncHd = 64;
constexpr int kEncNT = 128;
constexpr int kEncRows = 16;     // query rows per CTA
constexpr int kEncKeys = 64;     // keys per tile

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
__device__ __forceinline__ float2 unpack2(uint32_t u) {
    if constexpr (DT == 30) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
    } else {
        return __half22float2(*reinterpret_cast<const __half2 *>(&u));
    }
}

__device__ __forceinline__ int64_t ring_base(const EncParams & p, int stream, int head) {
    return (((int64_t) stream * p.n_layers + p.layer) * p.n_heads + head) * (int64_t) p.capacity;
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
        const int64_t dst = (ring_base(p, rd.stream, h) + rd.slot) * kEncHd + 2 * i;
        reinterpret_cast<uint32_t *>(p.k_ring)[dst / 2] = pack2<DT>(kx.x, kx.y);
        reinterpret_cast<uint32_t *>(p.v_ring)[dst / 2] = pack2<DT>(vx.x, vx.y);
    }
}

// One CTA per (row group, head).  A row group is <= 16 consecutive rows of one
// stream; the CTA streams the union of their windows through shared memory in
// 64-key tiles with an fp32 online softmax per row.
template <int DT>
__global__ void __launch_bounds__(kEncNT) enc_attention_kernel(const EncParams p) {
    __shared__ __align__(16) float qs[kEncRows][kEncHd];
    __shared__ __align__(16) uint32_t ks[kEncKeys][kEncHd / 2 + 1];
    __shared__ __align__(16) uint32_t vs[kEncKeys][kEncHd / 2];
    __shared__ float sc[kEncRows][kEncKeys];
    __shared__ float row_m[kEncRows], row_l[kEncRows], row_a[kEncRows];

    const int grp = blockIdx.x / p.n_heads;
    const int h = blockIdx.x % p.n_heads;
    if (grp >= p.n_groups) return;
    const int r0 = p.group_first[grp];
    const int r1 = p.group_first[grp + 1];
    const int nr = r1 - r0;
    const int tid = threadIdx.x;
    const EncRowDesc first = p.rows[r0];
    const EncRowDesc last = p.rows[r1 - 1];
    const int64_t base = ring_base(p, first.stream, h);

    for (int idx = tid; idx < kEncRows * (kEncHd / 2); idx += kEncNT) {
        const int r = idx / (kEncHd / 2);
        const int i = idx % (kEncHd / 2);
        float2 q = make_float2(0.0f, 0.0f);
        if (r < nr) {
            const EncRowDesc rd = p.rows[r0 + r];
            const float2 x = *reinterpret_cast<const float2 *>(p.q + ((int64_t) (r0 + r) * p.n_heads + h) * kEncHd + 2 * i);
            q = enc_rope_pair(x, p.rope[(int64_t) rd.pos * (kEncHd / 2) + i]);
        }
        qs[r][2 * i] = q.x * p.scale_log2;
        qs[r][2 * i + 1] = q.y * p.scale_log2;
    }
    if (tid < kEncRows) {
        row_m[tid] = -INFINITY;
        row_l[tid] = 0.0f;
    }
    // Output accumulators: thread owns row tid/8, dims 8*(tid%8)..+7.
    const int orow = tid >> 3;
    const int od = (tid & 7) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    __syncthreads();

    const int64_t ws = first.win_start;
    const int64_t we = last.pos;  // inclusive
    for (int64_t k0 = ws; k0 <= we; k0 += kEncKeys) {
        const int nk = (int) (we - k0 + 1 < kEncKeys ? we - k0 + 1 : kEncKeys);
        for (int idx = tid; idx < kEncKeys * (kEncHd / 8); idx += kEncNT) {
            const int kk = idx / (kEncHd / 8);
            const int c = idx % (kEncHd / 8);
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (kk < nk) {
                const int64_t slot = (k0 + kk) % p.capacity;
                const int64_t off = (base + slot) * kEncHd + 8 * c;
                kv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(p.k_ring) + off);
                vv = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(p.v_ring) + off);
            }
            ks[kk][4 * c + 0] = kv.x;
            ks[kk][4 * c + 1] = kv.y;
            ks[kk][4 * c + 2] = kv.z;
            ks[kk][4 * c + 3] = kv.w;
            *reinterpret_cast<uint4 *>(&vs[kk][4 * c]) = vv;
        }
        __syncthreads();
        // scores: thread owns key tid%64 for rows (tid/64)*8 .. +7
        {
            const int kk = tid & 63;
            const int rb = (tid >> 6) * 8;
            float s[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) s[r] = 0.0f;
#pragma unroll 8
            for (int i = 0; i < kEncHd / 2; ++i) {
                const float2 kf = unpack2<DT>(ks[kk][i]);
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    s[r] = fmaf(qs[rb + r][2 * i], kf.x, s[r]);
                    s[r] = fmaf(qs[rb + r][2 * i + 1], kf.y, s[r]);
                }
            }
            const int64_t kabs = k0 + kk;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                bool ok = kk < nk && (rb + r) < nr;
                if (ok) {
                    const int64_t qabs = p.rows[r0 + rb + r].pos;
                    ok = kabs <= qabs && kabs >= qabs - (p.window - 1);
                }
                sc[rb + r][kk] = ok ? s[r] : -INFINITY;
            }
        }
        __syncthreads();
        // per-row online softmax over the tile: warp w handles rows 4w..4w+3
        {
            const int w = tid >> 5, lane = tid & 31;
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                const int r = w * 4 + rr;
                float a = sc[r][lane], b = sc[r][lane + 32];
                float m = fmaxf(a, b);
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float m_old = row_m[r];
                const float m_new = fmaxf(m_old, m);
                const float ea = m_new == -INFINITY ? 0.0f : exp2f(a - m_new);
                const float eb = m_new == -INFINITY ? 0.0f : exp2f(b - m_new);
                sc[r][lane] = ea;
                sc[r][lane + 32] = eb;
                float l = ea + eb;
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
                __syncwarp();
                if (lane == 0) {
                    const float alpha = m_new == -INFINITY ? 1.0f : exp2f(m_old - m_new);
                    row_a[r] = alpha;
                    row_l[r] = row_l[r] * alpha + l;
                    row_m[r] = m_new;
                }
            }
        }
        __syncthreads();
        {
            const float alpha = row_a[orow];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] *= alpha;
            for (int kk = 0; kk < nk; ++kk) {
                const float pr = sc[orow][kk];
                const uint4 vv = *reinterpret_cast<const uint4 *>(&vs[kk][od / 2]);
                const float2 a = unpack2<DT>(vv.x), b = unpack2<DT>(vv.y), c = unpack2<DT>(vv.z), d = unpack2<DT>(vv.w);
                acc[0] = fmaf(pr, a.x, acc[0]);
                acc[1] = fmaf(pr, a.y, acc[1]);
                acc[2] = fmaf(pr, b.x, acc[2]);
                acc[3] = fmaf(pr, b.y, acc[3]);
                acc[4] = fmaf(pr, c.x, acc[4]);
                acc[5] = fmaf(pr, c.y, acc[5]);
                acc[6] = fmaf(pr, d.x, acc[6]);
                acc[7] = fmaf(pr, d.y, acc[7]);
            }
        }
        __syncthreads();
    }
    if (orow < nr) {
        const float inv = 1.0f / row_l[orow];
        float * o = p.out + ((int64_t) (r0 + orow) * p.n_heads + h) * kEncHd + od;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = acc[i] * inv;
    }
}

}  // namespace

int enc_smem_bytes() { return 0; }

cudaError_t launch_enc_append(const EncParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    if (p.dtype == 30) {
        enc_append_kernel<30><<<p.n_rows, 256, 0, stream>>>(p);
    } else {
        enc_append_kernel<1><<<p.n_rows, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_enc_attention(const EncParams & p, cudaStream_t stream) {
    if (p.n_groups <= 0) return cudaSuccess;
    const unsigned grid = (unsigned) (p.n_groups * p.n_heads);
    if (p.dtype == 30) {
        enc_attention_kernel<30><<<grid, kEncNT, 0, stream>>>(p);
    } else {
        enc_attention_kernel<1><<<grid, kEncNT, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace vxk
