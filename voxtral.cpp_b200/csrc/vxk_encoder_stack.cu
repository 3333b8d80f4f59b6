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

#include <algorithm>

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

// Steady chunks (every stream n_new = 4, windows of 12 frames): a block computes
// 128 channels for kSteadyStreams streams, so each weight load feeds 4 streams,
// and a stream's inputs of one input channel are read from shared memory once
// for every tap and position.  conv0 is needed at local positions 3 .. 11 only
// (conv1's inputs), conv1 at 2 .. 5.
constexpr int kSteadyStreams = 4;
constexpr int kSteadyWin = 12;

// conv0: y0[s][t][c] for t = 3 .. 11.  Grid (channel tiles, stream groups).
__global__ void __launch_bounds__(kConvThreads) conv0_steady_kernel(const ConvParams p) {
    extern __shared__ float smel[];  // [kSteadyStreams][n_mel][12], f16-rounded
    const int s0 = blockIdx.y * kSteadyStreams;
    const int ns = min(kSteadyStreams, p.n_streams - s0);
    const int per = p.n_mel * kSteadyWin;
    for (int i = threadIdx.x; i < ns * per; i += kConvThreads) {
        const int ss = i / per, o = i - ss * per;
        smel[i] = f16r(p.mel[p.streams[s0 + ss].mel_offset + o]);
    }
    __syncthreads();
    const int c = blockIdx.x * kConvThreads + threadIdx.x;
    if (c >= p.dim) return;
    float acc[kSteadyStreams][9];
#pragma unroll
    for (int ss = 0; ss < kSteadyStreams; ++ss)
#pragma unroll
        for (int t = 0; t < 9; ++t) acc[ss][t] = 0.0f;
    for (int ci = 0; ci < p.n_mel; ++ci) {
        const float w0 = __half2float(p.w0[((int64_t) ci * 3 + 0) * p.dim + c]);
        const float w1 = __half2float(p.w0[((int64_t) ci * 3 + 1) * p.dim + c]);
        const float w2 = __half2float(p.w0[((int64_t) ci * 3 + 2) * p.dim + c]);
#pragma unroll
        for (int ss = 0; ss < kSteadyStreams; ++ss) {
            if (ss < ns) {
                const float * xr = smel + (ss * p.n_mel + ci) * kSteadyWin;
                float xv[11];  // mel local 1 .. 11
#pragma unroll
                for (int m = 0; m < 11; ++m) xv[m] = xr[m + 1];
#pragma unroll
                for (int t = 0; t < 9; ++t) {  // local position 3 + t reads mel local 1 + t + k
                    acc[ss][t] = fmaf(w0, xv[t], acc[ss][t]);
                    acc[ss][t] = fmaf(w1, xv[t + 1], acc[ss][t]);
                    acc[ss][t] = fmaf(w2, xv[t + 2], acc[ss][t]);
                }
            }
        }
    }
    const float bias = p.b0[c];
#pragma unroll
    for (int ss = 0; ss < kSteadyStreams; ++ss) {
        if (ss < ns) {
            float * y0 = p.y0 + (int64_t) (s0 + ss) * p.max_win * p.dim;
#pragma unroll
            for (int t = 0; t < 9; ++t) y0[(int64_t) (3 + t) * p.dim + c] = gelu_erf_f(__fadd_rn(acc[ss][t], bias));
        }
    }
}

// conv1: encoder rows 4 s .. 4 s + 3 (positions 2 .. 5) from y0 positions 3 .. 11.
// 256 threads: thread t computes channel blockIdx.x * 128 + t % 128 for two of
// the block's four streams (t / 128 picks which two).
constexpr int kConv1Threads = 256;

__global__ void __launch_bounds__(kConv1Threads) conv1_steady_kernel(const ConvParams p) {
    extern __shared__ __half sy2[];  // [kSteadyStreams][dim][10]: f16-rounded y0 positions 3 .. 11
    const int s0 = blockIdx.y * kSteadyStreams;
    const int ns = min(kSteadyStreams, p.n_streams - s0);
    for (int i = threadIdx.x; i < ns * p.dim * 9; i += kConv1Threads) {
        const int ss = i / (p.dim * 9), o = i - ss * p.dim * 9;
        const int ci = o / 9, rr = o - ci * 9;
        sy2[(ss * p.dim + ci) * 10 + rr] =
            __float2half_rn(p.y0[(int64_t) (s0 + ss) * p.max_win * p.dim + (int64_t) (3 + rr) * p.dim + ci]);
    }
    __syncthreads();
    // the two halves of the block take streams 0, 1 and 2, 3 of the group; each
    // thread sums its column over all input channels in order, as conv1_kernel does
    constexpr int kPer = kSteadyStreams / 2;
    const int sb = (threadIdx.x >> 7) * kPer;
    const int c = blockIdx.x * 128 + (threadIdx.x & 127);
    if (c >= p.dim || sb >= ns) return;
    float acc[kPer][4];
#pragma unroll
    for (int ss = 0; ss < kPer; ++ss)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[ss][j] = 0.0f;
    // weights of 8 input channels loaded before they are used: 24 independent
    // loads in flight per thread (dim is a multiple of 8)
    for (int ci0 = 0; ci0 < p.dim; ci0 += 8) {
        float w[8][3];
#pragma unroll
        for (int uu = 0; uu < 8; ++uu)
#pragma unroll
            for (int k = 0; k < 3; ++k) w[uu][k] = __half2float(p.w1[((int64_t) (ci0 + uu) * 3 + k) * p.dim + c]);
#pragma unroll
        for (int uu = 0; uu < 8; ++uu) {
#pragma unroll
            for (int ss = 0; ss < kPer; ++ss) {
                if (sb + ss < ns) {
                    const __half * yr = sy2 + ((sb + ss) * p.dim + ci0 + uu) * 10;
                    float yv[9];
#pragma unroll
                    for (int m = 0; m < 9; ++m) yv[m] = __half2float(yr[m]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {  // output 2 + j reads y0 positions 3 + 2j + k
                        acc[ss][j] = fmaf(w[uu][0], yv[2 * j], acc[ss][j]);
                        acc[ss][j] = fmaf(w[uu][1], yv[2 * j + 1], acc[ss][j]);
                        acc[ss][j] = fmaf(w[uu][2], yv[2 * j + 2], acc[ss][j]);
                    }
                }
            }
        }
    }
    const float bias = p.b1[c];
#pragma unroll
    for (int ss = 0; ss < kPer; ++ss)
        if (sb + ss < ns)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                p.x[(int64_t) (4 * (s0 + sb + ss) + j) * p.dim + c] = gelu_erf_f(__fadd_rn(acc[ss][j], bias));
}

// Grid (column tiles, rows, 2): z = 0 adds b0 to the rows of y0, z = 1 b1 to y1.
__global__ void bias2_kernel(float * y0, const float * b0, int32_t n0, float * y1, const float * b1, int32_t n1) {
    float * y = blockIdx.z == 0 ? y0 : y1;
    const float * b = blockIdx.z == 0 ? b0 : b1;
    const int n = blockIdx.z == 0 ? n0 : n1;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (!b || i >= n) return;
    float * row = y + (int64_t) blockIdx.y * n;
    row[i] = __fadd_rn(row[i], b[i]);
}

}  // namespace

cudaError_t launch_conv_stem(const ConvParams & p, cudaStream_t stream) {
    if (p.n_streams <= 0) return cudaSuccess;
    if (p.steady) {
        // every stream has n_new = 4 (rows 4 s .. 4 s + 3), windows of 12 frames
        const dim3 grid((unsigned) ((p.dim + kConvThreads - 1) / kConvThreads),
                        (unsigned) ((p.n_streams + kSteadyStreams - 1) / kSteadyStreams));
        const size_t smem0 = (size_t) kSteadyStreams * p.n_mel * kSteadyWin * sizeof(float);
        const size_t smem1 = (size_t) kSteadyStreams * p.dim * 10 * sizeof(__half);
        if (smem0 > 227 * 1024 || smem1 > 227 * 1024 || p.max_win < kSteadyWin || p.dim % 8)
            return cudaErrorInvalidValue;
        cudaError_t e = cudaFuncSetAttribute(conv0_steady_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int) smem0);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(conv1_steady_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem1);
        if (e != cudaSuccess) return e;
        conv0_steady_kernel<<<grid, kConvThreads, smem0, stream>>>(p);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        conv1_steady_kernel<<<grid, kConv1Threads, smem1, stream>>>(p);
        return cudaGetLastError();
    }
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
    if (rows <= 0 || (!b0 && !b1)) return cudaSuccess;
    const int n = std::max(b0 ? n0 : 0, b1 ? n1 : 0);
    bias2_kernel<<<dim3((unsigned) ((n + 255) / 256), (unsigned) rows, 2), 256, 0, stream>>>(y0, b0, n0, y1, b1, n1);
    return cudaGetLastError();
}

}  // namespace vxk
