// ebx_packed_op.cu -- drop-in kernel for the reference dispatcher op
// mlbricks_native::elastic_linear_packed (mlbricks/bolt/ops.cpp:1012-1043,
// kernel mlbricks/bolt/ops_cuda.cu:2708-2796).
//
// Format (the op's own, distinct from MLB4): LSB-first bitstream, flat index
// o * in_features + k, code uq in [0, 2^b), q = uq - 2^(b-1), b in [2, 8];
// weight = q * scales[flat / group_size]; fp32 accumulation; bias added before
// the final rounding to x's dtype.
//
// The reference runs one thread per output element over a scalar K loop, so each
// row of x re-reads the whole packed weight.  Here one warp owns one output
// feature for a block of up to kRowsPerBlock rows of x: lanes stride K
// (consecutive lanes touch consecutive codes of the bitstream), each decoded
// weight is used for kRowChunk rows at once (one fp32 sum per row in registers),
// and a shuffle tree sums the lane partials.  The warp walks its row block chunk
// by chunk while the feature's codes stay in L1, so the weight crosses HBM once
// per row block instead of once per row.
#include <cuda_bf16.h>

#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {
namespace {

template <class T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <class T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

constexpr int kRowChunk = 8;        // rows of x per decoded weight
constexpr int kRowsPerBlock = 64;    // rows of x per CTA (blockIdx.y)
constexpr int kWarpsPerBlock = 8;    // output features per CTA (blockIdx.x)

template <class XT, class ST>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) packed_linear_kernel(
    const XT* __restrict__ x, const uint8_t* __restrict__ packed, const ST* __restrict__ scales,
    const XT* __restrict__ bias, XT* __restrict__ out, int64_t rows, int64_t in_f, int64_t out_f,
    int bits, int64_t group) {
    const int64_t o = int64_t(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (o >= out_f) return;
    const uint32_t mask = (1u << bits) - 1u;
    const int qmin = -(1 << (bits - 1));
    const int64_t wbase = o * in_f;
    for (int64_t row_lo = int64_t(blockIdx.y) * kRowsPerBlock; row_lo < rows;
         row_lo += int64_t(gridDim.y) * kRowsPerBlock) {
        const int64_t row_hi = row_lo + kRowsPerBlock < rows ? row_lo + kRowsPerBlock : rows;
        for (int64_t m0 = row_lo; m0 < row_hi; m0 += kRowChunk) {
            const int nr = int(row_hi - m0 < kRowChunk ? row_hi - m0 : kRowChunk);
            float acc[kRowChunk];
#pragma unroll
            for (int j = 0; j < kRowChunk; ++j) acc[j] = 0.0f;
            // scale group of the current flat index, advanced without a division per code
            int64_t gi = -1, g_end = 0;
            for (int64_t k = lane; k < in_f; k += 32) {
                const int64_t wi = wbase + k;
                if (wi >= g_end || gi < 0) {
                    gi = wi / group;
                    g_end = (gi + 1) * group;
                }
                const int64_t bp = wi * bits;
                const int64_t by = bp >> 3;
                const int off = int(bp & 7);
                uint32_t word = __ldg(packed + by);
                if (off + bits > 8) word |= uint32_t(__ldg(packed + by + 1)) << 8;
                const int q = int((word >> off) & mask) + qmin;
                const float w = float(q) * to_f<ST>(scales[gi]);
                const XT* xk = x + m0 * in_f + k;
#pragma unroll
                for (int j = 0; j < kRowChunk; ++j)
                    if (j < nr) acc[j] = fmaf(to_f<XT>(xk[j * in_f]), w, acc[j]);
            }
#pragma unroll
            for (int j = 0; j < kRowChunk; ++j) {
#pragma unroll
                for (int d = 16; d > 0; d >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], d);
            }
            if (lane < nr) {
                float v = acc[0];
#pragma unroll
                for (int j = 1; j < kRowChunk; ++j)
                    if (lane == j) v = acc[j];
                if (bias) v += to_f<XT>(bias[o]);
                out[(m0 + lane) * out_f + o] = from_f<XT>(v);
            }
        }
    }
}

template <class XT, class ST>
cudaError_t launch_t(const void* x, int64_t rows, const uint8_t* packed, const void* scales,
                     const void* bias, int bits, int64_t group, int64_t out_f, int64_t in_f,
                     void* out, cudaStream_t s) {
    const int64_t bx = (out_f + kWarpsPerBlock - 1) / kWarpsPerBlock;
    int64_t by = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
    if (by > 65535) by = 65535;  // the kernel strides over the remaining row blocks
    if (bx > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    const dim3 blocks{unsigned(bx), unsigned(by), 1u};
    const int threads = kWarpsPerBlock * 32;
    packed_linear_kernel<XT, ST><<<blocks, threads, 0, s>>>(
        static_cast<const XT*>(x), packed, static_cast<const ST*>(scales),
        static_cast<const XT*>(bias), static_cast<XT*>(out), rows, in_f, out_f, bits, group);
    return cudaGetLastError();
}

template <class XT>
cudaError_t launch_s(int scale_dtype, const void* x, int64_t rows, const uint8_t* packed,
                     const void* scales, const void* bias, int bits, int64_t group, int64_t out_f,
                     int64_t in_f, void* out, cudaStream_t s) {
    switch (scale_dtype) {
        case 0: return launch_t<XT, float>(x, rows, packed, scales, bias, bits, group, out_f, in_f, out, s);
        case 1: return launch_t<XT, __half>(x, rows, packed, scales, bias, bits, group, out_f, in_f, out, s);
        default: return launch_t<XT, __nv_bfloat16>(x, rows, packed, scales, bias, bits, group, out_f, in_f, out, s);
    }
}

}  // namespace

cudaError_t launch_elastic_linear_packed(const void* x, int x_dtype, int64_t rows,
                                         const uint8_t* packed, const void* scales,
                                         int scale_dtype, const void* bias, int bits,
                                         int64_t group_size, int64_t out_features,
                                         int64_t in_features, void* out, cudaStream_t s) {
    switch (x_dtype) {
        case 0: return launch_s<float>(scale_dtype, x, rows, packed, scales, bias, bits, group_size, out_features, in_features, out, s);
        case 1: return launch_s<__half>(scale_dtype, x, rows, packed, scales, bias, bits, group_size, out_features, in_features, out, s);
        default: return launch_s<__nv_bfloat16>(scale_dtype, x, rows, packed, scales, bias, bits, group_size, out_features, in_features, out, s);
    }
}

}  // namespace ebx
