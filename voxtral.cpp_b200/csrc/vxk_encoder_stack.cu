// The streaming encoder's conv stem and bias adds (vxk_encoder_*, include/vxk.h),
// the parts of build_encoder_steady_graph (src/voxtral.cpp:2386-2420) that are
// not matrix products or the windowed attention:
//   conv0 = gelu_erf(conv1d(mel, k 3, stride 1, 2 causal zero pads) + b0)
//   conv1 = gelu_erf(conv1d(conv0, k 3, stride 2, 1 causal zero pad) + b1)
// over each stream's window of 2 n + 4 Mel frames (causal_conv1d_graph and
// compute_causal_conv1d_dims, src/voxtral.cpp:1670-1687, 1767-1814), of which
// conv1 positions 2 .. n + 1 are the stream's n new encoder frames.  ggml_conv_1d
// rounds its im2col input to f16 and its f16 dot product takes the weights as
// f16, so both operands are f16 here too, with fp32 sums.
//
// CUDA cores, one thread per output channel: the stem is ~50 MFLOP per stream and
// 80 ms chunk, against ~7.7 GFLOP in the encoder layers' products.
#include "vxk_internal.h"

#include <cuda_fp16.h>

namespace vxk {
namespace {

constexpr int kConvThreads = 128;
constexpr int kConv1Chunk = 8;  // conv1 outputs per pass (17 input rows staged)

__device__ __forceinline__ float gelu_erf_f(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752440f))));
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

// y0[t][c] for every local t of the stream's window.  Grid (channel tiles, streams).
__global__ void __launch_bounds__(kConvThreads) conv0_kernel(const ConvParams p) {
    extern __shared__ float sx[];  // [n_mel][win], f16-rounded
    const ConvStream cs = p.streams[blockIdx.y];
    const int win = cs.win;
    for (int i = threadIdx.x; i < p.n_mel * win; i += kConvThreads) sx[i] = f16r(p.mel[cs.mel_offset + i]);
    __syncthreads();
    const int c = blockIdx.x * kConvThreads + threadIdx.x;
    if (c >= p.dim) return;
    float * y0 = p.y0 + (int64_t) blockIdx.y * p.max_win * p.dim;
    const float bias = p.b0[c];
    for (int t0 = 0; t0 < win; t0 += 4) {
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int ci = 0; ci < p.n_mel; ++ci) {
            const float * xr = sx + ci * win;
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const float w = __half2float(p.w0[((int64_t) ci * 3 + k) * p.dim + c]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int idx = t0 + j + k - 2;  // two causal zero pads on the left
                    const float xv = (t0 + j < win && idx >= 0) ? xr[idx] : 0.0f;
                    acc[j] = fmaf(w, xv, acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (t0 + j < win) y0[(int64_t) (t0 + j) * p.dim + c] = gelu_erf_f(__fadd_rn(acc[j], bias));
    }
}

// x[row0 + t1 - 2][c] for t1 = 2 .. n_new + 1.  Grid (channel tiles, streams).
__global__ void __launch_bounds__(kConvThreads) conv1_kernel(const ConvParams p) {
    extern __shared__ __half sy[];  // [2 * kConv1Chunk + 1][dim], f16-rounded conv0 rows
    const ConvStream cs = p.streams[blockIdx.y];
    const float * y0 = p.y0 + (int64_t) blockIdx.y * p.max_win * p.dim;
    const int c = blockIdx.x * kConvThreads + threadIdx.x;
    const float bias = c < p.dim ? p.b1[c] : 0.0f;
    for (int t1 = 2; t1 < 2 + cs.n_new; t1 += kConv1Chunk) {
        const int nt = min(kConv1Chunk, 2 + cs.n_new - t1);
        const int first = 2 * t1 - 1;  // one causal zero pad: input position 2 t1 + k - 1
        const int nrows = 2 * nt + 1;
        __syncthreads();  // the previous pass has read sy
        for (int i = threadIdx.x; i < nrows * p.dim; i += kConvThreads) {
            const int rr = i / p.dim, ci = i - rr * p.dim;
            const int pos = first + rr;
            sy[i] = __float2half_rn(pos >= 0 && pos < cs.win ? y0[(int64_t) pos * p.dim + ci] : 0.0f);
        }
        __syncthreads();
        if (c < p.dim) {
            float acc[kConv1Chunk];
#pragma unroll
            for (int j = 0; j < kConv1Chunk; ++j) acc[j] = 0.0f;
            for (int ci = 0; ci < p.dim; ++ci) {
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const float w = __half2float(p.w1[((int64_t) ci * 3 + k) * p.dim + c]);
#pragma unroll
                    for (int j = 0; j < kConv1Chunk; ++j)
                        if (j < nt) acc[j] = fmaf(w, __half2float(sy[(2 * j + k) * p.dim + ci]), acc[j]);
                }
            }
            for (int j = 0; j < nt; ++j)
                p.x[(int64_t) (cs.row0 + t1 - 2 + j) * p.dim + c] = gelu_erf_f(__fadd_rn(acc[j], bias));
        }
    }
}

__global__ void bias2_kernel(float * y0, const float * b0, int32_t n0, float * y1, const float * b1, int32_t n1,
                             int32_t rows) {
    const int64_t total0 = (int64_t) rows * n0, total = total0 + (int64_t) rows * n1;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < total;
         i += (int64_t) gridDim.x * blockDim.x) {
        if (i < total0) {
            y0[i] = __fadd_rn(y0[i], b0[i % n0]);
        } else {
            const int64_t j = i - total0;
            y1[j] = __fadd_rn(y1[j], b1[j % n1]);
        }
    }
}

}  // namespace

cudaError_t launch_conv_stem(const ConvParams & p, cudaStream_t stream) {
    if (p.n_streams <= 0) return cudaSuccess;
    const dim3 grid((unsigned) ((p.dim + kConvThreads - 1) / kConvThreads), (unsigned) p.n_streams);
    const size_t smem0 = (size_t) p.n_mel * p.max_win * sizeof(float);
    const size_t smem1 = (size_t) (2 * kConv1Chunk + 1) * p.dim * sizeof(__half);
    if (smem0 > 227 * 1024 || smem1 > 227 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(conv0_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem0);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(conv1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem1);
    if (e != cudaSuccess) return e;
    conv0_kernel<<<grid, kConvThreads, smem0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    conv1_kernel<<<grid, kConvThreads, smem1, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_bias2(float * y0, const float * b0, int32_t n0, float * y1, const float * b1, int32_t n1,
                         int32_t rows, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int64_t total = (int64_t) rows * (n0 + n1);
    const int grid = (int) ((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    bias2_kernel<<<grid, 256, 0, stream>>>(y0, b0, n0, y1, b1, n1, rows);
    return cudaGetLastError();
}

}  // namespace vxk
