// sm_100a greedy head: logits = W . x for every row of a decode batch and
// their argmax, the tail of the decoder step
//   ggml_mul_mat(tok_embeddings, last_hidden) + ggml_argmax
//   (emit_logits_argmax, src/voxtral.cpp:2966-2972)
// for a tied embedding matrix W [vocab][dim] stored as f16 or bf16.
//
// The batch's rows (up to 64, converted to W's 16-bit type like ggml's f16 /
// bf16 vec_dot does) are the M = 64 operand of tcgen05.mma, and a slice of
// `tile_rows` vocabulary rows of W is the N operand (N <= 256), so each MMA
// instruction covers a wide slice of the vocabulary and an epilogue thread owns
// one batch row: it scans that row's logits in TMEM for the largest value
// (first index on ties, as ggml_argmax) without any cross-thread reduction and
// folds the result into a global 64-bit (ordered value, inverted index)
// maximum with one atomicMax per row and tile.
//
// Persistent kernel, one CTA per SM, 6 warps:
//   warp 0     TMA producer: per 64-element K chunk, the 64 x 64 x-block and
//              the tile_rows x 64 W-block (128-byte swizzle) into a 5-stage ring
//   warp 1     tcgen05.mma issuer (one lane): D[64 rows][tile_rows] in TMEM,
//              double-buffered across tiles (2 x 256 columns)
//   warps 2-5  epilogue: TMEM lane quadrants; M = 64 puts batch row 16q + l in
//              lane l (l < 16) of quadrant q
#include "vxk_internal.h"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

namespace vxk {
namespace {

constexpr int kHeadThreads = 192;
constexpr int kHeadStages = 5;
constexpr int kChunk = 64;                        // K elements per stage (one 128-byte row)
constexpr int kXBytes = kHeadRows * 128;          // x block of a stage: 8 KB
constexpr int kStageBytes = kXBytes + kHeadMaxTileRows * 128;  // + W block: 40 KB
constexpr int kTmemCols = 512;                    // two D buffers of up to 256 fp32 columns
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr unsigned kFull = 0xffffffffu;

// shared-memory map (offsets from a 1024-aligned base)
constexpr int kBarFull = 0;
constexpr int kBarEmpty = kHeadStages;
constexpr int kBarDFull = 2 * kHeadStages;        // [2] D of a tile complete
constexpr int kBarDEmpty = kBarDFull + 2;         // [2] D read by the epilogue
constexpr int kBarDrain = kBarDEmpty + 2;
constexpr int kNumBars = kBarDrain + 1;
constexpr int kOffBar = kHeadStages * kStageBytes;
constexpr int kOffMisc = kOffBar + kNumBars * 8;  // tmem base, abort flag
constexpr int kHeadSmem = kOffMisc + 16 + 1024;   // + alignment slack
static_assert(kHeadSmem <= 232448, "greedy head exceeds 227 KB of shared memory");

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
__device__ __forceinline__ bool head_wait(uint64_t * bar, uint32_t parity, volatile int32_t * abort_flag,
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
__device__ __forceinline__ void head_drain(uint64_t * bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitNs) return;
    }
}

// 2-D TMA tile load into this CTA's shared memory, counted on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int c0, int c1, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle, descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 columns of 32 bits from TMEM into registers.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Monotonic key: larger logit first, then smaller vocabulary index.
__device__ __forceinline__ unsigned long long best_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long) u << 32) | (unsigned long long) (0xFFFFFFFFu - (uint32_t) idx);
}

template <int DT>
__device__ __forceinline__ uint16_t to16(float a) {
    if constexpr (DT == 30) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(a));
    } else {
        return __half_as_ushort(__float2half_rn(a));
    }
}

// x [n_rows][dim] fp32 -> xh [64][dim] in W's type (rows past n_rows zero);
// clears the per-row best keys.
template <int DT>
__global__ void head_prep_kernel(const HeadParams p) {
    const int r = blockIdx.y;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < p.dim) {
        const float v = r < p.n_rows ? p.x[(int64_t) r * p.dim + k] : 0.0f;
        p.xh[(int64_t) r * p.dim + k] = to16<DT>(v);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) p.best[r] = 0ull;
}

__global__ void head_finish_kernel(const HeadParams p) {
    const int r = threadIdx.x;
    if (r < p.n_rows) p.argmax[r] = (int32_t) (0xFFFFFFFFu - (uint32_t) (p.best[r] & 0xFFFFFFFFull));
}

template <int DT>
__global__ void __launch_bounds__(kHeadThreads, 1) head_kernel(const __grid_constant__ CUtensorMap tmw,
                                                               const __grid_constant__ CUtensorMap tmx,
                                                               const HeadParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t * bars = reinterpret_cast<uint64_t *>(base + kOffBar);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(base + kOffMisc);
    volatile int32_t * abort_flag = reinterpret_cast<volatile int32_t *>(base + kOffMisc + 4);

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int n_chunks = p.dim / kChunk;
    const int stride = (int) gridDim.x;
    const int w_bytes = p.tile_rows * 128;
    if ((int) blockIdx.x >= p.n_tiles) return;

    if (tid == 0) {
        for (int s = 0; s < kHeadStages; ++s) {
            mbar_init(&bars[kBarFull + s], 1);
            mbar_init(&bars[kBarEmpty + s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[kBarDFull + b], 1);
            mbar_init(&bars[kBarDEmpty + b], 128);
        }
        mbar_init(&bars[kBarDrain], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Launched with programmatic stream serialization: only the setup above
    // overlaps the previous grid (the conversion of x).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            uint32_t c = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += stride) {
                for (int ch = 0; ok && ch < n_chunks; ++ch) {
                    const int st = (int) (c % kHeadStages);
                    if (!head_wait(&bars[kBarEmpty + st], ((c / kHeadStages) & 1) ^ 1, abort_flag, p.error)) {
                        ok = false;
                        break;
                    }
                    uint8_t * dst = base + st * kStageBytes;
                    mbar_expect_tx(&bars[kBarFull + st], (uint32_t) (kXBytes + w_bytes));
                    tma_load_2d(dst, &tmx, ch * kChunk, 0, &bars[kBarFull + st]);
                    tma_load_2d(dst + kXBytes, &tmw, ch * kChunk, tile * p.tile_rows, &bars[kBarFull + st]);
                    ++c;
                }
            }
            if (!ok || *abort_flag) {
                for (uint32_t d = c > (uint32_t) kHeadStages ? c - kHeadStages : 0; d < c; ++d)
                    head_drain(&bars[kBarFull + d % kHeadStages], (d / kHeadStages) & 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- tcgen05.mma issuer ----------------
        if (lane == 0) {
            constexpr uint32_t fmt = DT == 30 ? 1u : 0u;
            // fp32 accumulate, K-major A (x) and B (W), N = tile_rows, M = 64
            const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t) (p.tile_rows >> 3) << 17) |
                                   ((uint32_t) (kHeadRows >> 4) << 24);
            uint32_t c = 0;
            int t = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < p.n_tiles; tile += stride, ++t) {
                const int b = t & 1;
                if (!head_wait(&bars[kBarDEmpty + b], ((t >> 1) & 1) ^ 1, abort_flag, p.error)) break;
                tc_fence_after();
                const uint32_t d = tmem + 256 * b;
                for (int ch = 0; ch < n_chunks; ++ch) {
                    const int st = (int) (c % kHeadStages);
                    if (!head_wait(&bars[kBarFull + st], (c / kHeadStages) & 1, abort_flag, p.error)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t xa = smem_u32(base + st * kStageBytes);
                    const uint32_t wb = xa + kXBytes;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        tc_mma(d, sw128_desc(xa + ks * 32, 16, 1024), sw128_desc(wb + ks * 32, 16, 1024), idesc,
                               (ch | ks) != 0);
                    }
                    tc_commit(&bars[kBarEmpty + st]);
                    ++c;
                }
                if (ok) tc_commit(&bars[kBarDFull + b]);
            }
            tc_commit(&bars[kBarDrain]);
            head_drain(&bars[kBarDrain], 0);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue warps 2-5 ----------------
        // Quadrant q holds batch rows 16q .. 16q+15 in its lanes 0-15.
        const int q = warp & 3;
        const int row = 16 * q + lane;
        const bool real = lane < 16 && row < p.n_rows;
        const uint32_t lane_off = (uint32_t) (32 * q) << 16;
        const bool vec_store = (p.vocab & 3) == 0;
        int t = 0;
        for (int tile = blockIdx.x; tile < p.n_tiles; tile += stride, ++t) {
            const int b = t & 1;
            const bool have = __all_sync(kFull, head_wait(&bars[kBarDFull + b], (t >> 1) & 1, abort_flag, p.error));
            tc_fence_after();
            const int col0 = tile * p.tile_rows;
            float best_v = -INFINITY;
            int best_i = -1;
            for (int c0 = 0; have && c0 < p.tile_rows; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + 256 * b + c0 + lane_off, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int col = col0 + c0 + j;
                    if (col < p.vocab && v[j] > best_v) {
                        best_v = v[j];
                        best_i = col;
                    }
                }
                if (p.logits && real) {
                    float * dst = p.logits + (int64_t) row * p.vocab + col0 + c0;
                    if (vec_store && col0 + c0 + 32 <= p.vocab) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + c0 + j < p.vocab) dst[j] = v[j];
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&bars[kBarDEmpty + b]);
            if (have && real && best_i >= 0 && !*abort_flag) atomicMax(&p.best[row], best_key(best_v, best_i));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// Argmax of logits already in memory (the head over quantized embeddings):
// every CTA scans a slice of one row and folds the first index of its largest
// value into the row's key.  Grid (slices, rows).
__global__ void __launch_bounds__(256) head_argmax_kernel(const float * logits, int32_t vocab,
                                                          unsigned long long * best) {
    __shared__ unsigned long long red[8];
    const int r = blockIdx.y;
    const float * row = logits + (int64_t) r * vocab;
    unsigned long long key = 0ull;  // below every value's key
    for (int i = blockIdx.x * 256 + threadIdx.x; i < vocab; i += gridDim.x * 256) {
        const unsigned long long k = best_key(row[i], i);
        key = k > key ? k : key;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(kFull, key, o);
        key = other > key ? other : key;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) key = red[w] > key ? red[w] : key;
        key = red[0] > key ? red[0] : key;
        atomicMax(&best[r], key);
    }
}

__global__ void head_keys_to_ids_kernel(const unsigned long long * best, int32_t rows, int32_t * argmax) {
    const int r = threadIdx.x;
    if (r < rows) argmax[r] = (int32_t) (0xFFFFFFFFu - (uint32_t) (best[r] & 0xFFFFFFFFull));
}

template <typename K>
cudaError_t launch_pdl(K kernel, dim3 grid, unsigned block, size_t smem, cudaStream_t stream, bool pdl,
                       const CUtensorMap * tmw, const CUtensorMap * tmx, const HeadParams & p) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, *tmw, *tmx, p);
}

}  // namespace

int head_smem_bytes() { return kHeadSmem; }

cudaError_t launch_head_argmax(const float * logits, int32_t rows, int32_t vocab, unsigned long long * best,
                               int32_t * argmax, cudaStream_t stream) {
    if (rows <= 0 || rows > kHeadRows || vocab <= 0) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(best, 0, (size_t) rows * sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    const int slices = std::max(1, std::min(64, (vocab + 2047) / 2048));
    head_argmax_kernel<<<dim3((unsigned) slices, (unsigned) rows), 256, 0, stream>>>(logits, vocab, best);
    head_keys_to_ids_kernel<<<1, kHeadRows, 0, stream>>>(best, rows, argmax);
    return cudaGetLastError();
}

cudaError_t launch_head(const HeadParams & p, const CUtensorMap & tmw, const CUtensorMap & tmx, int grid,
                        cudaStream_t stream) {
    if (p.n_rows <= 0 || p.n_rows > kHeadRows) return cudaErrorInvalidValue;
    // 1. x -> 16-bit rows of the MMA operand, best keys cleared
    const dim3 pg((unsigned) ((p.dim + 255) / 256), (unsigned) kHeadRows);
    if (p.dtype == 30) {
        head_prep_kernel<30><<<pg, 256, 0, stream>>>(p);
    } else {
        head_prep_kernel<1><<<pg, 256, 0, stream>>>(p);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // 2. logits and per-tile maxima (programmatic launch: prologue overlaps step 1)
    if (p.dtype == 30) {
        e = cudaFuncSetAttribute(head_kernel<30>, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmem);
        if (e != cudaSuccess) return e;
        e = launch_pdl(head_kernel<30>, dim3((unsigned) grid), kHeadThreads, kHeadSmem, stream, true, &tmw, &tmx, p);
    } else {
        e = cudaFuncSetAttribute(head_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kHeadSmem);
        if (e != cudaSuccess) return e;
        e = launch_pdl(head_kernel<1>, dim3((unsigned) grid), kHeadThreads, kHeadSmem, stream, true, &tmw, &tmx, p);
    }
    if (e != cudaSuccess) return e;
    // 3. keys -> token ids
    head_finish_kernel<<<1, kHeadRows, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace vxk
