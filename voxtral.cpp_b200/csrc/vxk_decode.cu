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
// Cache layout (per layer): page-major [n_blocks][n_kv][16 tokens][128] so one
// (page, kv head) tile is a contiguous 4 KiB (f16) or 2 KiB + 128 B (q8_0)
// region that one cp.async.bulk copies into shared memory.
#include "vxk_internal.h"

#include <cuda_fp16.h>
#include <stdint.h>

namespace vxk {
namespace {

constexpr int NT = 128;            // threads per CTA
constexpr int kStages = 8;         // bulk-copy ring depth
constexpr int kGroupPages = 16;    // pages whose scores are held at once
constexpr int kGroupTokens = kGroupPages * kBlockTokens;
constexpr int kMaxChunkPages = 128;
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded mbarrier wait: 2 s

constexpr int kErrBadPage = 1;
constexpr int kErrTimeout = 2;

template <int DT> struct Fmt;
template <> struct Fmt<1> {
    static constexpr int kData = kBlockTokens * kHeadDim * 2;  // 4096
    static constexpr int kStage = kData;
};
template <> struct Fmt<8> {
    static constexpr int kData = kBlockTokens * kHeadDim;                       // 2048
    static constexpr int kScale = kBlockTokens * (kHeadDim / kQ8Block) * 2;     // 128
    static constexpr int kStage = kData + kScale;                               // 2176
};

template <int DT>
struct __align__(128) Smem {
    uint8_t stage[kStages][Fmt<DT>::kStage];
    uint64_t full[kStages];
    float scores[kGroupTokens * kGroup];     // also the combine weights
    uint8_t newk[kHeadDim * 2];
    uint8_t newv[kHeadDim * 2];
    uint16_t newk_scale[kHeadDim / kQ8Block];
    uint16_t newv_scale[kHeadDim / kQ8Block];
    int32_t pages[kMaxChunkPages];
    float red_m[NT / 32][kGroup];
    float red_l[NT / 32][kGroup];
    float comb_m[kGroup];
    float comb_l[kGroup];
    int32_t abort_flag;
    int32_t last_flag;
};
static_assert(sizeof(float) * 8 * kGroup * kHeadDim <= sizeof(uint8_t) * kStages * Fmt<8>::kStage,
              "acc reduction buffer must fit in the stage ring");

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
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

// 1-D bulk copy global -> shared, completion counted on an mbarrier.  The
// K/V stream is read once per launch, so it is marked evict-first in L2.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes,
                                         uint64_t * bar, uint64_t policy) {
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

__device__ __forceinline__ void h8_to_f8(const uint4 & u, float * f) {
    const __half2 * h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// Exact int8 -> fp32 for the 4 signed bytes of a word: bias to unsigned,
// splice under the exponent of 2^23, subtract (2^23 + 128).
__device__ __forceinline__ void s8x4_to_f4(uint32_t w, float * f) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7540u)) - 8388736.0f;
    f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7541u)) - 8388736.0f;
    f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7542u)) - 8388736.0f;
    f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7543u)) - 8388736.0f;
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

// ggml quantize_row_q8_0_ref on one 32-value block held as 16 pairs by 16
// consecutive lanes (lane group aligned to 16): d = amax/127,
// id = d ? 1/d : 0, q = roundf(x*id).
__device__ __forceinline__ void q8_pair(float2 x, char2 & q, float & d) {
    float a = fmaxf(fabsf(x.x), fabsf(x.y));
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    d = __fdiv_rn(a, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    q.x = static_cast<signed char>(static_cast<int>(roundf(__fmul_rn(x.x, id))));
    q.y = static_cast<signed char>(static_cast<int>(roundf(__fmul_rn(x.y, id))));
}

// Appends one (token, kv head) row with 128 threads: threads 0-63 rotate and
// store K pairs, threads 64-127 store V pairs.  Writes the stored values also
// to shared memory (newk/newv) when smem pointers are given.
template <int DT>
__device__ __forceinline__ void append_head_row(const float * k, const float * v,
                                                const float2 * cs, uint8_t * k_data,
                                                uint8_t * v_data, uint8_t * k_scale,
                                                uint8_t * v_scale, int64_t tile, int tok,
                                                uint8_t * sk, uint8_t * sv, uint16_t * sks,
                                                uint16_t * svs) {
    const int tid = threadIdx.x;
    const bool is_k = tid < 64;
    const int i = is_k ? tid : tid - 64;  // pair index 0..63
    float2 x = reinterpret_cast<const float2 *>(is_k ? k : v)[i];
    if (is_k) x = rope_pair(x, cs[i]);
    if constexpr (DT == 1) {
        const __half2 h = __floats2half2_rn(x.x, x.y);
        uint8_t * base = (is_k ? k_data : v_data) + (tile * kBlockTokens + tok) * (kHeadDim * 2);
        reinterpret_cast<__half2 *>(base)[i] = h;
        if (sk) reinterpret_cast<__half2 *>(is_k ? sk : sv)[i] = h;
    } else {
        char2 q;
        float d;
        q8_pair(x, q, d);
        uint8_t * base = (is_k ? k_data : v_data) + (tile * kBlockTokens + tok) * kHeadDim;
        reinterpret_cast<char2 *>(base)[i] = q;
        if (sk) reinterpret_cast<char2 *>(is_k ? sk : sv)[i] = q;
        if ((i & 15) == 0) {
            const __half dh = __float2half_rn(d);
            const int blk = i >> 4;
            uint8_t * sb = (is_k ? k_scale : v_scale) +
                           (tile * kBlockTokens + tok) * (kHeadDim / kQ8Block) * 2;
            reinterpret_cast<__half *>(sb)[blk] = dh;
            if (sks) (is_k ? sks : svs)[blk] = __half_as_ushort(dh);
        }
    }
}

// Query dims owned by lane j (0..7) of a token group, slot s (0..15).
template <int DT>
__device__ __forceinline__ int q_dim(int j, int s) {
    if constexpr (DT == 1) {
        return (s < 8) ? 8 * j + s : 64 + 8 * j + (s - 8);
    } else {
        return 16 * j + s;
    }
}

// Reduce-scatter of 4 per-head partial dot products across the 8 lanes of a
// token group: returns the full sum of head hsel(j) = 2*bit2(j) + bit1(j).
__device__ __forceinline__ float reduce_scatter4(const float s[4], int j) {
    const bool hi2 = (j & 4) != 0;
    float k0 = hi2 ? s[2] : s[0];
    float k1 = hi2 ? s[3] : s[1];
    const float o0 = hi2 ? s[0] : s[2];
    const float o1 = hi2 ? s[1] : s[3];
    k0 += __shfl_xor_sync(0xffffffffu, o0, 4);
    k1 += __shfl_xor_sync(0xffffffffu, o1, 4);
    const bool hi1 = (j & 2) != 0;
    float r = hi1 ? k1 : k0;
    const float o = hi1 ? k0 : k1;
    r += __shfl_xor_sync(0xffffffffu, o, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    return r;
}

template <int DT>
__global__ void __launch_bounds__(NT, 4) decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem<DT> & S = *reinterpret_cast<Smem<DT> *>(smem_raw);
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int kvh = blockIdx.x % p.n_kv;
    const int item_idx = blockIdx.x / p.n_kv;
    if (item_idx >= p.n_items) return;
    const WorkItem it = p.items[item_idx];
    const RowDesc rd = p.rows[it.row];
    const int last_page = rd.pos / kBlockTokens;
    const int n_pages = it.page_end - it.page_begin;
    const bool do_append =
        p.fuse_append && (rd.flags & kRowAppend) && (it.page_end - 1 == last_page);
    const int64_t kv_stride_tiles = p.n_kv;

    for (int i = tid; i < n_pages; i += NT) {
        const int lp = it.page_begin + i;
        int pg = p.block_table[(int64_t) rd.stream * p.bt_cap + (lp % p.bt_cap)];
        if (pg < 0 || pg >= p.n_blocks) {
            set_error(p.error, kErrBadPage);
            pg = 0;
        }
        S.pages[i] = pg;
    }
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&S.full[s], 1);
        S.abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    const int total = 2 * n_pages;
    const uint64_t policy = evict_first_policy();
    int issued = 0;  // meaningful in thread 0 only
    auto issue = [&](int L) {
        const int gi = L / (2 * kGroupPages);
        const int base = gi * 2 * kGroupPages;
        const int np = min(kGroupPages, n_pages - gi * kGroupPages);
        const int r = L - base;
        const bool is_v = r >= np;
        const int pi = is_v ? r - np : r;
        const int64_t tile = (int64_t) S.pages[gi * kGroupPages + pi] * kv_stride_tiles + kvh;
        const int st = L % kStages;
        uint64_t * bar = &S.full[st];
        if constexpr (DT == 1) {
            mbar_expect_tx(bar, Fmt<1>::kData);
            bulk_g2s(S.stage[st], (is_v ? p.v_data : p.k_data) + tile * Fmt<1>::kData,
                     Fmt<1>::kData, bar, policy);
        } else {
            mbar_expect_tx(bar, Fmt<8>::kData + Fmt<8>::kScale);
            bulk_g2s(S.stage[st], (is_v ? p.v_data : p.k_data) + tile * Fmt<8>::kData,
                     Fmt<8>::kData, bar, policy);
            bulk_g2s(S.stage[st] + Fmt<8>::kData,
                     (is_v ? p.v_scale : p.k_scale) + tile * Fmt<8>::kScale, Fmt<8>::kScale,
                     bar, policy);
        }
    };
    if (tid == 0) {
        const int n0 = min(kStages, total);
        for (int L = 0; L < n0; ++L) issue(L);
        issued = n0;
    }

    // Query prologue: rotate this lane's 16 dims of the group's 4 heads and
    // fold in scale*log2(e).
    const int t = tid >> 3;   // token in page (QK phase)
    const int j = tid & 7;    // lane in token group
    float qv[kGroup][16];
    {
        const float * qrow = p.q + ((int64_t) it.row * p.n_q + (int64_t) kvh * kGroup) * kHeadDim;
        const float2 * cs = p.rope + (int64_t) rd.pos * (kHeadDim / 2);
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
#pragma unroll
            for (int s = 0; s < 16; s += 2) {
                const int d = q_dim<DT>(j, s);
                const float2 x = *reinterpret_cast<const float2 *>(qrow + g * kHeadDim + d);
                const float2 r = rope_pair(x, cs[d >> 1]);
                qv[g][s] = r.x * p.scale_log2;
                qv[g][s + 1] = r.y * p.scale_log2;
            }
        }
    }
    if (do_append) {
        const int tok = rd.pos % kBlockTokens;
        const int64_t tile = (int64_t) S.pages[n_pages - 1] * kv_stride_tiles + kvh;
        const int64_t krow = ((int64_t) it.row * p.n_kv + kvh) * kHeadDim;
        append_head_row<DT>(p.k + krow, p.v + krow, p.rope + (int64_t) rd.pos * (kHeadDim / 2),
                            p.k_data, p.v_data, p.k_scale, p.v_scale, tile, tok, S.newk,
                            S.newv, S.newk_scale, S.newv_scale);
    }
    __syncthreads();

    float m_run[kGroup], l_run[kGroup];
    float acc[kGroup][8];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[g][i] = 0.0f;
    }
    const int g8 = tid >> 4;   // token pair (PV phase)
    const int j16 = tid & 15;  // 8-dim slice (PV phase)
    const int n_groups = (n_pages + kGroupPages - 1) / kGroupPages;
    bool aborted = false;
    int L = 0;

    for (int gi = 0; gi < n_groups && !aborted; ++gi) {
        const int np = min(kGroupPages, n_pages - gi * kGroupPages);
        // ---- K phase: scores of the group's tokens --------------------------
        for (int pi = 0; pi < np; ++pi, ++L) {
            const int st = L % kStages;
            if (!mbar_wait(&S.full[st], (L / kStages) & 1, kWaitNs)) S.abort_flag = 1;
            const int lp = it.page_begin + gi * kGroupPages + pi;
            const bool patch = do_append && lp == last_page && t == rd.pos % kBlockTokens;
            float s[kGroup];
            if constexpr (DT == 1) {
                const uint8_t * row = S.stage[st] + t * (kHeadDim * 2);
                uint4 a = *reinterpret_cast<const uint4 *>(row + 16 * j);
                uint4 b = *reinterpret_cast<const uint4 *>(row + 128 + 16 * j);
                if (patch) {
                    a = *reinterpret_cast<const uint4 *>(S.newk + 16 * j);
                    b = *reinterpret_cast<const uint4 *>(S.newk + 128 + 16 * j);
                }
                float kf[16];
                h8_to_f8(a, kf);
                h8_to_f8(b, kf + 8);
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        s0 = fmaf(qv[g][i], kf[i], s0);
                        s1 = fmaf(qv[g][8 + i], kf[8 + i], s1);
                    }
                    s[g] = s0 + s1;
                }
            } else {
                const uint8_t * row = S.stage[st] + t * kHeadDim;
                uint4 a = *reinterpret_cast<const uint4 *>(row + 16 * j);
                const uint16_t * sc = reinterpret_cast<const uint16_t *>(S.stage[st] + Fmt<8>::kData);
                uint16_t dbits = sc[t * (kHeadDim / kQ8Block) + (j >> 1)];
                if (patch) {
                    a = *reinterpret_cast<const uint4 *>(S.newk + 16 * j);
                    dbits = S.newk_scale[j >> 1];
                }
                const float d = __half2float(__ushort_as_half(dbits));
                float kf[16];
                s8x4_to_f4(a.x, kf);
                s8x4_to_f4(a.y, kf + 4);
                s8x4_to_f4(a.z, kf + 8);
                s8x4_to_f4(a.w, kf + 12);
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        s0 = fmaf(qv[g][i], kf[i], s0);
                        s1 = fmaf(qv[g][8 + i], kf[8 + i], s1);
                    }
                    s[g] = (s0 + s1) * d;
                }
            }
            const float tot = reduce_scatter4(s, j);
            if ((j & 1) == 0) {
                const int h = ((j >> 2) & 1) * 2 + ((j >> 1) & 1);
                const int tp = lp * kBlockTokens + t;
                const bool valid = tp >= rd.win_start && tp <= rd.pos;
                S.scores[(pi * kBlockTokens + t) * kGroup + h] = valid ? tot : -INFINITY;
            }
            __syncthreads();
            if (S.abort_flag) {
                aborted = true;
                break;
            }
            if (tid == 0 && issued < total) issue(issued++);
        }
        if (aborted) break;

        // ---- softmax of the group (log2 domain), merged into the run -------
        {
            const int n_tok = np * kBlockTokens;
            const int h = tid & 3;
            float lm = -INFINITY;
            for (int k2 = tid >> 2; k2 < n_tok; k2 += NT / 4) lm = fmaxf(lm, S.scores[k2 * kGroup + h]);
            lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 4));
            lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 8));
            lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 16));
            if (lane < 4) S.red_m[warp][lane] = lm;
            __syncthreads();
            float m_new[kGroup];
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
                float mg = S.red_m[0][g];
#pragma unroll
                for (int w = 1; w < NT / 32; ++w) mg = fmaxf(mg, S.red_m[w][g]);
                m_new[g] = fmaxf(m_run[g], mg);
            }
            const float mh = h == 0 ? m_new[0] : h == 1 ? m_new[1] : h == 2 ? m_new[2] : m_new[3];
            float ls = 0.0f;
            for (int k2 = tid >> 2; k2 < n_tok; k2 += NT / 4) {
                const float e = exp2f(S.scores[k2 * kGroup + h] - mh);
                S.scores[k2 * kGroup + h] = e;
                ls += e;
            }
            ls += __shfl_xor_sync(0xffffffffu, ls, 4);
            ls += __shfl_xor_sync(0xffffffffu, ls, 8);
            ls += __shfl_xor_sync(0xffffffffu, ls, 16);
            if (lane < 4) S.red_l[warp][lane] = ls;
            __syncthreads();
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
                float lg = 0.0f;
#pragma unroll
                for (int w = 0; w < NT / 32; ++w) lg += S.red_l[w][g];
                const float alpha = exp2f(m_run[g] - m_new[g]);
                l_run[g] = l_run[g] * alpha + lg;
                m_run[g] = m_new[g];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[g][i] *= alpha;
            }
        }

        // ---- V phase: acc += p * V ----------------------------------------
        for (int pi = 0; pi < np; ++pi, ++L) {
            const int st = L % kStages;
            if (!mbar_wait(&S.full[st], (L / kStages) & 1, kWaitNs)) S.abort_flag = 1;
            const int lp = it.page_begin + gi * kGroupPages + pi;
            const int patch_tok = (do_append && lp == last_page) ? rd.pos % kBlockTokens : -1;
            const int t0 = g8, t1 = g8 + 8;
            const float4 pa = *reinterpret_cast<const float4 *>(&S.scores[(pi * kBlockTokens + t0) * kGroup]);
            const float4 pb = *reinterpret_cast<const float4 *>(&S.scores[(pi * kBlockTokens + t1) * kGroup]);
            float fa[8], fb[8];
            float wa[kGroup] = {pa.x, pa.y, pa.z, pa.w};
            float wb[kGroup] = {pb.x, pb.y, pb.z, pb.w};
            if constexpr (DT == 1) {
                uint4 va = *reinterpret_cast<const uint4 *>(S.stage[st] + t0 * (kHeadDim * 2) + 16 * j16);
                uint4 vb = *reinterpret_cast<const uint4 *>(S.stage[st] + t1 * (kHeadDim * 2) + 16 * j16);
                if (t0 == patch_tok) va = *reinterpret_cast<const uint4 *>(S.newv + 16 * j16);
                if (t1 == patch_tok) vb = *reinterpret_cast<const uint4 *>(S.newv + 16 * j16);
                h8_to_f8(va, fa);
                h8_to_f8(vb, fb);
            } else {
                uint2 va = *reinterpret_cast<const uint2 *>(S.stage[st] + t0 * kHeadDim + 8 * j16);
                uint2 vb = *reinterpret_cast<const uint2 *>(S.stage[st] + t1 * kHeadDim + 8 * j16);
                const uint16_t * sc = reinterpret_cast<const uint16_t *>(S.stage[st] + Fmt<8>::kData);
                uint16_t da = sc[t0 * (kHeadDim / kQ8Block) + (j16 >> 2)];
                uint16_t db = sc[t1 * (kHeadDim / kQ8Block) + (j16 >> 2)];
                if (t0 == patch_tok) {
                    va = *reinterpret_cast<const uint2 *>(S.newv + 8 * j16);
                    da = S.newv_scale[j16 >> 2];
                }
                if (t1 == patch_tok) {
                    vb = *reinterpret_cast<const uint2 *>(S.newv + 8 * j16);
                    db = S.newv_scale[j16 >> 2];
                }
                s8x4_to_f4(va.x, fa);
                s8x4_to_f4(va.y, fa + 4);
                s8x4_to_f4(vb.x, fb);
                s8x4_to_f4(vb.y, fb + 4);
                const float dfa = __half2float(__ushort_as_half(da));
                const float dfb = __half2float(__ushort_as_half(db));
#pragma unroll
                for (int g = 0; g < kGroup; ++g) {
                    wa[g] *= dfa;
                    wb[g] *= dfb;
                }
            }
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    acc[g][i] = fmaf(wa[g], fa[i], acc[g][i]);
                    acc[g][i] = fmaf(wb[g], fb[i], acc[g][i]);
                }
            }
            __syncthreads();
            if (S.abort_flag) {
                aborted = true;
                break;
            }
            if (tid == 0 && issued < total) issue(issued++);
        }
    }

    if (aborted) {
        // Drain the copies still in flight (bounded) before the CTA exits.
        if (tid == 0) {
            for (int l = L + 1; l < issued; ++l) mbar_wait(&S.full[l % kStages], (l / kStages) & 1, kWaitNs);
            set_error(p.error, kErrTimeout);
        }
        return;
    }

    // ---- reduce acc over the 8 token pairs, emit output or partial ---------
    float * red = reinterpret_cast<float *>(&S.stage[0][0]);  // [8][4][128]
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        float4 * dst = reinterpret_cast<float4 *>(red + (g8 * kGroup + g) * kHeadDim + 8 * j16);
        dst[0] = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
        dst[1] = make_float4(acc[g][4], acc[g][5], acc[g][6], acc[g][7]);
    }
    __syncthreads();
    float o[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        float sum = 0.0f;
#pragma unroll
        for (int q2 = 0; q2 < 8; ++q2) sum += red[(q2 * kGroup + g) * kHeadDim + tid];
        o[g] = sum;
    }
    const int64_t out_base = ((int64_t) it.row * p.n_q + (int64_t) kvh * kGroup) * kHeadDim;
    if (rd.n_chunks == 1) {
#pragma unroll
        for (int g = 0; g < kGroup; ++g) p.out[out_base + g * kHeadDim + tid] = o[g] / l_run[g];
        return;
    }
    {
        float * part = p.partials + ((int64_t) item_idx * p.n_q + (int64_t) kvh * kGroup) * kPartialStride;
#pragma unroll
        for (int g = 0; g < kGroup; ++g) part[g * kPartialStride + tid] = o[g];
        if (tid < kGroup) {
            part[tid * kPartialStride + kHeadDim] = m_run[tid];
            part[tid * kPartialStride + kHeadDim + 1] = l_run[tid];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const int prev = atomicAdd(&p.counters[it.row * p.n_kv + kvh], 1);
        S.last_flag = (prev == rd.n_chunks - 1);
    }
    __syncthreads();
    if (!S.last_flag) return;
    __threadfence();

    // ---- last split of the (row, kv head): combine all splits --------------
    const int nc = rd.n_chunks;
    auto part_at = [&](int c, int g) -> const float * {
        return p.partials +
               ((int64_t) (rd.item_base + c) * p.n_q + (int64_t) kvh * kGroup + g) * kPartialStride;
    };
    {
        float lm[kGroup];
#pragma unroll
        for (int g = 0; g < kGroup; ++g) lm[g] = -INFINITY;
        for (int c = tid; c < nc; c += NT) {
#pragma unroll
            for (int g = 0; g < kGroup; ++g) lm[g] = fmaxf(lm[g], __ldcg(part_at(c, g) + kHeadDim));
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) lm[g] = fmaxf(lm[g], __shfl_xor_sync(0xffffffffu, lm[g], off));
        }
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < kGroup; ++g) S.red_m[warp][g] = lm[g];
        }
        __syncthreads();
        float M[kGroup];
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            M[g] = S.red_m[0][g];
#pragma unroll
            for (int w = 1; w < NT / 32; ++w) M[g] = fmaxf(M[g], S.red_m[w][g]);
        }
        float ls[kGroup] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int c = tid; c < nc; c += NT) {
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
                const float * pc = part_at(c, g);
                const float w = exp2f(__ldcg(pc + kHeadDim) - M[g]);
                ls[g] += __ldcg(pc + kHeadDim + 1) * w;
                S.scores[c * kGroup + g] = w;
            }
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) ls[g] += __shfl_xor_sync(0xffffffffu, ls[g], off);
        }
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < kGroup; ++g) S.red_l[warp][g] = ls[g];
        }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            float Lsum = 0.0f;
#pragma unroll
            for (int w = 0; w < NT / 32; ++w) Lsum += S.red_l[w][g];
            const float inv = 1.0f / Lsum;
            float acc2 = 0.0f;
            for (int c = 0; c < nc; ++c) acc2 = fmaf(S.scores[c * kGroup + g], __ldcg(part_at(c, g) + tid), acc2);
            p.out[out_base + g * kHeadDim + tid] = acc2 * inv;
        }
    }
    if (tid == 0) p.counters[it.row * p.n_kv + kvh] = 0;
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
    append_head_row<DT>(p.k + krow, p.v + krow, p.rope + (int64_t) rd.pos * (kHeadDim / 2),
                        p.k_data, p.v_data, p.k_scale, p.v_scale, tile, rd.pos % kBlockTokens,
                        nullptr, nullptr, nullptr, nullptr);
}

__global__ void table_update_kernel(int32_t * table, const TableUpdate * up, int32_t n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) table[up[i].index] = up[i].page;
}

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
    constexpr int row_bytes = DT == 1 ? kHeadDim * 2 : kHeadDim;
    const int64_t src = (tile * kBlockTokens + tok) * row_bytes;
    const int64_t dst = ((int64_t) r * p.n_kv + kvh) * row_bytes;
    for (int b = threadIdx.x; b < row_bytes / 4; b += blockDim.x) {
        reinterpret_cast<uint32_t *>(p.k_out + dst)[b] = reinterpret_cast<const uint32_t *>(p.k_data + src)[b];
        reinterpret_cast<uint32_t *>(p.v_out + dst)[b] = reinterpret_cast<const uint32_t *>(p.v_data + src)[b];
    }
    if constexpr (DT == 8) {
        constexpr int nsb = (kHeadDim / kQ8Block) * 2;
        const int64_t ssrc = (tile * kBlockTokens + tok) * nsb;
        const int64_t sdst = ((int64_t) r * p.n_kv + kvh) * nsb;
        for (int b = threadIdx.x; b < nsb / 2; b += blockDim.x) {
            reinterpret_cast<uint16_t *>(p.k_scale_out + sdst)[b] = reinterpret_cast<const uint16_t *>(p.k_scale + ssrc)[b];
            reinterpret_cast<uint16_t *>(p.v_scale_out + sdst)[b] = reinterpret_cast<const uint16_t *>(p.v_scale + ssrc)[b];
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
    if (p.page_scale_bytes > 0) {
        uint8_t * base = (is_v ? p.v_scale : p.k_scale) + (int64_t) layer * p.layer_scale_bytes;
        const uint4 * src = reinterpret_cast<const uint4 *>(base + (int64_t) mv.x * p.page_scale_bytes);
        uint4 * dst = reinterpret_cast<uint4 *>(base + (int64_t) mv.y * p.page_scale_bytes);
        const int64_t n = p.page_scale_bytes / 16;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

}  // namespace

int decode_smem_bytes(int dtype) {
    return dtype == 8 ? (int) sizeof(Smem<8>) : (int) sizeof(Smem<1>);
}

cudaError_t launch_decode(const DecodeParams & p, cudaStream_t stream) {
    if (p.n_items <= 0) return cudaSuccess;
    const dim3 grid((unsigned) (p.n_items * p.n_kv));
    if (p.dtype == 8) {
        const int smem = (int) sizeof(Smem<8>);
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        decode_kernel<8><<<grid, NT, smem, stream>>>(p);
    } else {
        const int smem = (int) sizeof(Smem<1>);
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        decode_kernel<1><<<grid, NT, smem, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    const dim3 grid((unsigned) (p.n_rows * p.n_kv));
    if (p.dtype == 8) {
        append_kernel<8><<<grid, NT, 0, stream>>>(p);
    } else {
        append_kernel<1><<<grid, NT, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_table_updates(int32_t * table, const TableUpdate * updates, int32_t n,
                                 cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    table_update_kernel<<<(n + 255) / 256, 256, 0, stream>>>(table, updates, n);
    return cudaGetLastError();
}

cudaError_t launch_gather(const GatherParams & p, cudaStream_t stream) {
    if (p.n <= 0) return cudaSuccess;
    const dim3 grid((unsigned) (p.n * p.n_kv));
    if (p.dtype == 8) {
        gather_kernel<8><<<grid, 64, 0, stream>>>(p);
    } else {
        gather_kernel<1><<<grid, 64, 0, stream>>>(p);
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
