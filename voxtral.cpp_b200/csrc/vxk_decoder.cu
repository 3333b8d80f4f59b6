// Row-wise kernels of the whole decoder step (voxtral.cpp's
// build_decoder_layer, src/voxtral.cpp:2630-2886, and the step graph around
// it, 3047-3104), and of the adapter ring (2589-2620).  The matrix products,
// the attention and the head run in their own kernels; these are the pieces
// between them, each one pass over a row that stays in L2:
//   embed_norm_kernel  x = tok_embeddings[token] + audio_emb[slot] (ggml_get_rows
//                      of the GGUF type, ggml_add), xn = rms_norm(x) * attn_norm
//   add_norm_kernel    x += proj (ggml_add), out = rms_norm(x) * w, optional
//                      out + out * ada (the time conditioning, 2862-2874)
//   swiglu_kernel      silu(gate) * up (2877-2880)
//   gelu_erf_kernel    the adapter's and time MLP's ggml_gelu_erf
//   adapter gather / audio scatter: 4 encoder frames per group, audio ring rows
//
// RMS norm follows ggml's CPU rms_norm: the squares are rounded in fp32 and
// summed in fp64, mean = (float) (sum / n), scale = 1 / sqrtf(mean + eps),
// y = x * scale, then * w; every product and sum is rounded separately.
#include "vxk_dequant.h"
#include "vxk_internal.h"

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

__global__ void __launch_bounds__(kNormThreads) add_norm_kernel(NormParams p) {
    __shared__ double red[kNormThreads / 32];
    const int r = blockIdx.x;
    int out_row = r;
    if (p.compact) {
        out_row = p.rows[r].out_index;
        if (out_row < 0) return;  // the last norm: only each stream's last row goes on
    }
    float * x = p.x + (int64_t) r * p.dim;
    const float * add = p.add ? p.add + (int64_t) r * p.dim : nullptr;
    double sum = 0.0;
    for (int i = threadIdx.x; i < p.dim; i += kNormThreads) {
        float v = x[i];
        if (add) {
            v = __fadd_rn(v, add[i]);
            x[i] = v;
        }
        sum += (double) __fmul_rn(v, v);
    }
    sum = block_sum(sum, red);
    const float scale = rms_scale(sum, p.dim, p.eps);
    float * out = p.out + (int64_t) out_row * p.dim;
    for (int i = threadIdx.x; i < p.dim; i += kNormThreads) {
        float y = __fmul_rn(__fmul_rn(x[i], scale), p.w[i]);
        if (p.ada) y = __fadd_rn(y, __fmul_rn(y, p.ada[i]));
        out[i] = y;
    }
}

__global__ void swiglu_kernel(const float4 * gate, const float4 * up, float4 * out, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n4; i += (int64_t) gridDim.x * blockDim.x) {
        const float4 g = gate[i];
        const float4 u = up[i];
        float4 o;
        o.x = __fmul_rn(__fdiv_rn(g.x, __fadd_rn(1.0f, expf(-g.x))), u.x);
        o.y = __fmul_rn(__fdiv_rn(g.y, __fadd_rn(1.0f, expf(-g.y))), u.y);
        o.z = __fmul_rn(__fdiv_rn(g.z, __fadd_rn(1.0f, expf(-g.z))), u.z);
        o.w = __fmul_rn(__fdiv_rn(g.w, __fadd_rn(1.0f, expf(-g.w))), u.w);
        out[i] = o;
    }
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
    add_norm_kernel<<<p.n_rows, kNormThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const float * gate, const float * up, float * out, int64_t n, cudaStream_t stream) {
    if (n <= 0 || n % 4) return n ? cudaErrorInvalidValue : cudaSuccess;
    const int64_t n4 = n / 4;
    swiglu_kernel<<<grid_for(n4, 256), 256, 0, stream>>>(reinterpret_cast<const float4 *>(gate),
                                                         reinterpret_cast<const float4 *>(up),
                                                         reinterpret_cast<float4 *>(out), n4);
    return cudaGetLastError();
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
