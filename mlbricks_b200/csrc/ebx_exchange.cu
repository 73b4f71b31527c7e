// ebx_exchange.cu -- finish kernel of the tensor-parallel exchange.
//
// Row-parallel sharding (Megatron): rank r holds the K slice K_r of a weight
// and all of its rows, computes p_r = x_r @ W_r^T in fp32, and every rank
// needs y = fp16(sum_r p_r + bias).  The decode kernel (ebx_decode.cu, with
// XchgArgs) stores p_r into every rank's region as {value, epoch} words
// (ebx_xchg.cuh).  When its grid could not be made co-resident it does not
// reduce; this kernel, next on the same stream, then polls each rank's word of
// every output, sums them in rank order 0..world-1 -- the same order on every
// rank, so all ranks produce bit-identical y -- adds the bias in fp32, rounds
// once, and advances the epoch.  It only waits for words written by decode
// kernels that themselves never wait, so it cannot deadlock.
#include <cuda_fp16.h>

#include "ebx_internal.h"
#include "ebx_xchg.cuh"

namespace ebx {
namespace {

__device__ int g_xchg_status = 0;

constexpr int kFinishThreads = 256;

__global__ void __launch_bounds__(kFinishThreads) xchg_finish_kernel(XchgArgs xa, int M, int N,
                                                                     const uint16_t* bias,
                                                                     uint16_t* y, float* y32) {
    const uint32_t e = xchg_epoch(xa) + 1u;
    const size_t total = size_t(M) * size_t(N);
    bool ok = true;
    for (size_t i = size_t(blockIdx.x) * kFinishThreads + threadIdx.x; i < total;
         i += size_t(gridDim.x) * kFinishThreads) {
        const int tok = int(i / size_t(N));
        const int row = int(i % size_t(N));
        float v;
        if (!xchg_gather(xa, e, M, N, tok, row, v)) {
            ok = false;
            break;
        }
        if (bias) v += __half2float(__ushort_as_half(bias[row]));
        y[i] = __half_as_ushort(__float2half_rn(v));
        if (y32) y32[i] = v;
    }
    if (!ok) atomicExch(&g_xchg_status, kXchgTimeout);
    xchg_advance(xa, e);
}

}  // namespace

cudaError_t launch_xchg_finish(const XchgArgs& xa, int M, int N, const uint16_t* bias,
                               uint16_t* y, float* y32, cudaStream_t s) {
    const size_t total = size_t(M) * size_t(N);
    size_t blocks = (total + kFinishThreads - 1) / kFinishThreads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    if (blocks < 1) blocks = 1;
    xchg_finish_kernel<<<unsigned(blocks), kFinishThreads, 0, s>>>(xa, M, N, bias, y, y32);
    return cudaGetLastError();
}

cudaError_t read_xchg_status(int* status, bool clear, cudaStream_t s) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_xchg_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_xchg_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

}  // namespace ebx
