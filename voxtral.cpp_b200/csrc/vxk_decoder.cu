// Row-wise kernels of the whole decoder step (voxtral.cpp's
// build_decoder_layer, src/voxtral.cpp:2630-2886, and the step graph around
// it, 3047-3104), and of the adapter ring (2589-2620).  The matrix products,
// the attention and the head run in their own kernels; these are the pieces
// between them, each one pass over a row that stays in L2:
//   embed_norm_kernel  x = tok_embeddings[token] + audio_emb[slot] (ggml_get_rows
//                      of the GGUF type, ggml_add), xn = rms_norm(x) * attn_norm
//   add_norm_kernel    x += proj (ggml_add), out = rms_norm(x) * w, optional
//                      out + out * ada (the time conditioning, 2862-2874)
//   add_norm_quant_kernel  the same, with the output rows quantized straight
//                      into the next tcgen05 product's activation tiles
//   gelu_erf_kernel    the adapter's and time MLP's ggml_gelu_erf
//   adapter gather / audio scatter: 4 encoder frames per group, audio ring rows
//
// RMS norm follows ggml's CPU rms_norm: the squares are rounded in fp32 and
// summed in fp64, mean = (float) (sum / n), scale = 1 / sqrtf(mean + eps),
// y = x * scale, then * w; every product and sum is rounded separately.
#include "vxk_dequant.h"
#include "vxk_internal.h"
#include "vxk_qtc_quant.h"

namespace vxk {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ double block_sum(double v, double * red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    // fixed order over the warps, so every thread gets the same sum
    for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
    return t;
}

__device__ __forceinline__ float rms_scale(double sum, int dim, float eps) {
    const float mean = (float) (sum / (double) dim);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

__global__ void __launch_bounds__(kNormThreads) embed_norm_kernel(EmbedParams p) {
    __shared__ double red[kNormThreads / 32];
    const int r = blockIdx.x;
    const DecRow row = p.rows[r];
    const uint8_t * emb = p.emb + (int64_t) row.token * p.emb_row_bytes;
    const float * audio = p.audio + ((int64_t) row.stream * p.audio_cap + row.audio_slot) * p.dim;
    float * x = p.x + (int64_t) r * p.dim;
    double sum = 0.0;
    for (int i = threadIdx.x; i < p.dim; i += kNormThreads) {
        const float v = __fadd_rn(dequant_elem(emb, p.emb_type, i), audio[i]);
        x[i] = v;
        sum += (double) __fmul_rn(v, v);
    }
    sum = block_sum(sum, red);
    const float scale = rms_scale(sum, p.dim, p.eps);
    float * xn = p.xn + (int64_t) r * p.dim;
    for (int i = threadIdx.x; i < p.dim; i += kNormThreads) xn[i] = __fmul_rn(__fmul_rn(x[i], scale), p.norm_w[i]);
}

// One row per CTA; V float4 per thread held in registers, every load issued
// before the first store (x and add may not be assumed apart otherwise).
// Launched as a programmatic dependent of the previous kernel: nothing is read
// or written before griddepcontrol.wait (the producer grid has completed and
// its memory is visible); the next launch may start right after.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <int V>
__global__ void __launch_bounds__(kNormThreads) add_norm_kernel(NormParams p) {
    __shared__ double red[kNormThreads / 32];
    pdl_enter();
    const int r = blockIdx.x;
    int out_row = r;
    if (p.compact) {
        out_row = p.rows[r].out_index;
        if (out_row < 0) return;  // the last norm: only each stream's last row goes on
    }
    const int n4 = p.dim / 4;
    float4 * x = reinterpret_cast<float4 *>(p.x + (int64_t) r * p.dim);
    const float4 * add = p.add ? reinterpret_cast<const float4 *>(p.add + (int64_t) r * p.dim) : nullptr;
    const float4 * ab = p.add_bias ? reinterpret_cast<const float4 *>(p.add_bias) : nullptr;
    float4 v[V];
    float4 a[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n4) {
            v[j] = x[i];
            if (add) a[j] = add[i];
        }
    }
    if (add && ab) {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int i = threadIdx.x + j * kNormThreads;
            if (i < n4) {
                const float4 bb = ab[i];
                a[j].x = __fadd_rn(a[j].x, bb.x);
                a[j].y = __fadd_rn(a[j].y, bb.y);
                a[j].z = __fadd_rn(a[j].z, bb.z);
                a[j].w = __fadd_rn(a[j].w, bb.w);
            }
        }
    }
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n4) {
            if (add) {
                v[j].x = __fadd_rn(v[j].x, a[j].x);
                v[j].y = __fadd_rn(v[j].y, a[j].y);
                v[j].z = __fadd_rn(v[j].z, a[j].z);
                v[j].w = __fadd_rn(v[j].w, a[j].w);
                x[i] = v[j];
            }
            sum += (double) __fmul_rn(v[j].x, v[j].x);
            sum += (double) __fmul_rn(v[j].y, v[j].y);
            sum += (double) __fmul_rn(v[j].z, v[j].z);
            sum += (double) __fmul_rn(v[j].w, v[j].w);
        }
    }
    sum = block_sum(sum, red);
    const float scale = rms_scale(sum, p.dim, p.eps);
    const float4 * w = reinterpret_cast<const float4 *>(p.w);
    const float4 * ada = p.ada ? reinterpret_cast<const float4 *>(p.ada) : nullptr;
    float4 * out = reinterpret_cast<float4 *>(p.out + (int64_t) out_row * p.dim);
#pragma unroll
    for (int j = 0; j < V; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < n4) {
            const float4 wv = w[i];
            float4 y;
            y.x = __fmul_rn(__fmul_rn(v[j].x, scale), wv.x);
            y.y = __fmul_rn(__fmul_rn(v[j].y, scale), wv.y);
            y.z = __fmul_rn(__fmul_rn(v[j].z, scale), wv.z);
            y.w = __fmul_rn(__fmul_rn(v[j].w, scale), wv.w);
            if (ada) {
                const float4 av = ada[i];
                y.x = __fadd_rn(y.x, __fmul_rn(y.x, av.x));
                y.y = __fadd_rn(y.y, __fmul_rn(y.y, av.y));
                y.z = __fadd_rn(y.z, __fmul_rn(y.z, av.z));
                y.w = __fadd_rn(y.w, __fmul_rn(y.w, av.w));
            }
            out[i] = y;
        }
    }
}

// add_norm_kernel's arithmetic with the output quantized for the tcgen05
// product that takes it (vxk_qtc_quant.h) instead of stored: one CTA per row
// (padded to the product's rows; padding rows get zero tiles), one warp per
// 256-column unit, lane L holding the columns of the unit's K positions 8L ..
// 8L + 7, so the row never leaves registers between the norm and the tiles.
// The squares are summed in fp64 per lane, over the warp and then over the
// warps in a fixed order.
__global__ void __launch_bounds__(1024) add_norm_quant_kernel(NormParams p) {
    __shared__ double red[32];
    pdl_enter();
    const int r = blockIdx.x, u = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int c0 = 256 * u + qtc_lane_col_a(lane), c1 = c0 + 32;
    float y[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const bool live = r < p.n_rows;
    float4 v[2], wv[2], av[2];
    double sum = 0.0;
    if (live) {
        float * xr = p.x + (int64_t) r * p.dim;
        v[0] = *reinterpret_cast<const float4 *>(xr + c0);
        v[1] = *reinterpret_cast<const float4 *>(xr + c1);
        // the norm weights (and time scale) are loaded with the row, before the reduction
        wv[0] = *reinterpret_cast<const float4 *>(p.w + c0);
        wv[1] = *reinterpret_cast<const float4 *>(p.w + c1);
        if (p.ada) {
            av[0] = *reinterpret_cast<const float4 *>(p.ada + c0);
            av[1] = *reinterpret_cast<const float4 *>(p.ada + c1);
        }
        if (p.add) {
            const float * ar = p.add + (int64_t) r * p.dim;
            float4 a[2] = {*reinterpret_cast<const float4 *>(ar + c0), *reinterpret_cast<const float4 *>(ar + c1)};
            if (p.add_bias) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 bb = *reinterpret_cast<const float4 *>(p.add_bias + (h ? c1 : c0));
                    a[h].x = __fadd_rn(a[h].x, bb.x);
                    a[h].y = __fadd_rn(a[h].y, bb.y);
                    a[h].z = __fadd_rn(a[h].z, bb.z);
                    a[h].w = __fadd_rn(a[h].w, bb.w);
                }
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                v[h].x = __fadd_rn(v[h].x, a[h].x);
                v[h].y = __fadd_rn(v[h].y, a[h].y);
                v[h].z = __fadd_rn(v[h].z, a[h].z);
                v[h].w = __fadd_rn(v[h].w, a[h].w);
            }
            *reinterpret_cast<float4 *>(xr + c0) = v[0];
            *reinterpret_cast<float4 *>(xr + c1) = v[1];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            sum += (double) __fmul_rn(v[h].x, v[h].x);
            sum += (double) __fmul_rn(v[h].y, v[h].y);
            sum += (double) __fmul_rn(v[h].z, v[h].z);
            sum += (double) __fmul_rn(v[h].w, v[h].w);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[u] = sum;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += red[w];
    if (live) {
        const float scale = rms_scale(t, p.dim, p.eps);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int c = h ? c1 : c0;
            float4 o;
            o.x = __fmul_rn(__fmul_rn(v[h].x, scale), wv[h].x);
            o.y = __fmul_rn(__fmul_rn(v[h].y, scale), wv[h].y);
            o.z = __fmul_rn(__fmul_rn(v[h].z, scale), wv[h].z);
            o.w = __fmul_rn(__fmul_rn(v[h].w, scale), wv[h].w);
            if (p.ada) {
                o.x = __fadd_rn(o.x, __fmul_rn(o.x, av[h].x));
                o.y = __fadd_rn(o.y, __fmul_rn(o.y, av[h].y));
                o.z = __fadd_rn(o.z, __fmul_rn(o.z, av[h].z));
                o.w = __fadd_rn(o.w, __fmul_rn(o.w, av[h].w));
            }
            if (p.out) *reinterpret_cast<float4 *>(p.out + (int64_t) r * p.dim + c) = o;
            y[4 * h + 0] = o.x;
            y[4 * h + 1] = o.y;
            y[4 * h + 2] = o.z;
            y[4 * h + 3] = o.w;
        }
    }
    const int np = p.q_npad, chunk = r / np, rr = r - chunk * np;
    const int64_t cu = (int64_t) chunk * nw + u;  // this chunk's unit
    qtc_quantize_unit(y, lane, rr, np, p.q_tiles ? p.q_tiles + cu * np * 512 : nullptr,
                      p.q_bmin ? p.q_bmin + cu * np * 32 : nullptr, p.q_tiles8 ? p.q_tiles8 + cu * np * 256 : nullptr,
                      p.q_dx + cu * np + rr);
}

__device__ __forceinline__ float gelu_erf(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}

__global__ void gelu_erf_kernel(float * x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        x[i] = gelu_erf(x[i]);
}

__global__ void adapter_gather_kernel(const float4 * enc, int32_t enc_cap, int32_t enc_dim4, const AdaptRow * rows,
                                      float4 * out) {
    const AdaptRow row = rows[blockIdx.x];
    const int64_t n = 4 * (int64_t) enc_dim4;
    const float4 * src = enc + ((int64_t) row.stream * enc_cap + row.enc_slot) * enc_dim4;
    float4 * dst = out + (int64_t) blockIdx.x * n;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];  // 4 consecutive slots, no wrap
}

__global__ void audio_scatter_kernel(const float4 * y, float4 * audio, int32_t audio_cap, int32_t dim4,
                                     const AdaptRow * rows) {
    const AdaptRow row = rows[blockIdx.x];
    const float4 * src = y + (int64_t) blockIdx.x * dim4;
    float4 * dst = audio + ((int64_t) row.stream * audio_cap + row.audio_slot) * dim4;
    for (int i = threadIdx.x; i < dim4; i += blockDim.x) dst[i] = src[i];
}

template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, unsigned block, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int grid_for(int64_t n, int threads) {
    const int64_t g = (n + threads - 1) / threads;
    return (int) (g < 148 * 16 ? (g > 0 ? g : 1) : 148 * 16);
}

}  // namespace

cudaError_t launch_embed_norm(const EmbedParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    embed_norm_kernel<<<p.n_rows, kNormThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_add_norm(const NormParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    if (p.dim % 4 || p.dim > 16 * 4 * kNormThreads) return cudaErrorInvalidValue;
    const int v = (p.dim / 4 + kNormThreads - 1) / kNormThreads;
    const dim3 grid((unsigned) p.n_rows);
    if (v <= 1) return launch_pdl(add_norm_kernel<1>, grid, kNormThreads, stream, p);
    if (v <= 2) return launch_pdl(add_norm_kernel<2>, grid, kNormThreads, stream, p);
    if (v <= 4) return launch_pdl(add_norm_kernel<4>, grid, kNormThreads, stream, p);
    if (v <= 8) return launch_pdl(add_norm_kernel<8>, grid, kNormThreads, stream, p);
    return launch_pdl(add_norm_kernel<16>, grid, kNormThreads, stream, p);
}

cudaError_t launch_add_norm_quant(const NormParams & p, cudaStream_t stream) {
    if (p.n_rows <= 0) return cudaSuccess;
    if (p.compact || (!p.q_tiles && !p.q_tiles8) || (p.q_tiles && !p.q_bmin) || !p.q_dx || p.dim % 256 ||
        p.dim / 256 > 32 ||
        (p.q_npad != 16 && p.q_npad != 32 && p.q_npad != 64) || p.q_rows_padded < p.n_rows ||
        p.q_rows_padded % p.q_npad || (p.q_npad != 64 && p.q_rows_padded != p.q_npad))
        return cudaErrorInvalidValue;
    for (const void * a : {(const void *) p.x, (const void *) p.add, (const void *) p.add_bias, (const void *) p.w,
                           (const void *) p.ada, (const void *) p.out})
        if (reinterpret_cast<uintptr_t>(a) & 15) return cudaErrorInvalidValue;
    return launch_pdl(add_norm_quant_kernel, dim3((unsigned) p.q_rows_padded), (unsigned) (p.dim / 256 * 32), stream, p);
}

cudaError_t launch_gelu_erf(float * x, int64_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    gelu_erf_kernel<<<grid_for(n, 256), 256, 0, stream>>>(x, n);
    return cudaGetLastError();
}

cudaError_t launch_adapter_gather(const float * enc, int32_t enc_cap, int32_t enc_dim, const AdaptRow * rows,
                                  int32_t n, float * out, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (enc_dim % 4) return cudaErrorInvalidValue;
    adapter_gather_kernel<<<n, 256, 0, stream>>>(reinterpret_cast<const float4 *>(enc), enc_cap, enc_dim / 4, rows,
                                                 reinterpret_cast<float4 *>(out));
    return cudaGetLastError();
}

cudaError_t launch_audio_scatter(const float * y, float * audio, int32_t audio_cap, int32_t dim,
                                 const AdaptRow * rows, int32_t n, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    if (dim % 4) return cudaErrorInvalidValue;
    audio_scatter_kernel<<<n, 256, 0, stream>>>(reinterpret_cast<const float4 *>(y), reinterpret_cast<float4 *>(audio),
                                                audio_cap, dim / 4, rows);
    return cudaGetLastError();
}

}  // namespace vxk
