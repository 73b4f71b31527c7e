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

// One-shot all-reduce of an fp32 partial [M, N] that this rank already holds (a
// row-parallel shard's y32 from the decode-GEMM): every CTA first stores all of its
// elements (into every rank's region, or in the two-phase form into each row's owner
// rank), then gathers them (or, two-phase, reduces its own rows and broadcasts them,
// waiting for the other owners' sums); the launch is cooperative, so every CTA of
// every rank gets to store before any of them can be waited on.
__global__ void __launch_bounds__(kFinishThreads) xchg_allreduce_kernel(XchgArgs xa, const float* part,
                                                                        int M, int N,
                                                                        const uint16_t* bias,
                                                                        uint16_t* y, float* y32) {
    const uint32_t e = xchg_epoch(xa) + 1u;
    const size_t total = size_t(M) * size_t(N);
    const size_t step = size_t(gridDim.x) * kFinishThreads;
    const size_t first = size_t(blockIdx.x) * kFinishThreads + threadIdx.x;
    for (size_t i = first; i < total; i += step) {
        const int tok = int(i / size_t(N)), row = int(i % size_t(N));
        if (xa.two_phase)
            xchg_push_owner(xa, e, xchg_owner(xa, row, N), N, tok, row, part[i]);
        else
            xchg_push(xa, e, M, N, tok, row, part[i]);
    }
    bool ok = true;
    for (size_t i = first; i < total; i += step) {
        const int tok = int(i / size_t(N)), row = int(i % size_t(N));
        float v;
        const bool got = xa.two_phase ? xchg_reduce_owner(xa, e, xchg_owner(xa, row, N), M, N, tok, row, v)
                                      : xchg_gather(xa, e, M, N, tok, row, v);
        if (!got) {
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

cudaError_t launch_xchg_allreduce(const XchgArgs& xa, const float* part, int M, int N,
                                  const uint16_t* bias, uint16_t* y, float* y32, cudaStream_t s) {
    int dev = 0, sms = 0, per_sm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, xchg_allreduce_kernel, kFinishThreads, 0);
    if (e != cudaSuccess) return e;
    const size_t total = size_t(M) * size_t(N);
    size_t blocks = (total + kFinishThreads - 1) / kFinishThreads;
    const size_t cap = size_t(sms) * size_t(per_sm < 4 ? per_sm : 4);
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    XchgArgs xa2 = xa;
    xa2.two_phase = xchg_two_phase(xa, M) ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(blocks));
    cfg.blockDim = dim3(kFinishThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, xchg_allreduce_kernel, xa2, part, M, N, bias, y, y32);
}

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
