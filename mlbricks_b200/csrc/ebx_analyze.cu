// ebx_analyze.cu -- matrix-path bit selection and quantisation on the device.
//
// Restates the reference host analyzer (elasticbit_runtime.cu:280-436) and the
// weight quantiser (cu:77-148) as kernels.  Per (calibration sample, row) the
// float sums run over k in order with explicitly rounded fp32 products and
// adds (__fmul_rn / __fadd_rn: no FMA contraction), exactly like the host
// loops, so every per-row output value is bit-identical to the reference.
// The reference then sums squared differences over all (sample, row) pairs in
// an 80-bit long double; here those sums are fp64 with a fixed reduction tree
// (warp shuffle over samples, then rows in index order), so the returned
// error values agree to ~1e-15 relative and the selected width only differs
// if an error lies within that distance of the threshold.
//
// Layout: one warp per (row, width); lane s handles calibration sample s
// (samples are processed 32 at a time).  The width-16 pass is the fp16
// reference itself (cu:280-309 equals the b = 16 branch of cu:339-344).
#include <mutex>
#include <string>

#include "../../include/ebx.h"
#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {
namespace {

__device__ __forceinline__ float round_fp16(float v) { return __half2float(__float2half_rn(v)); }

__device__ __forceinline__ int quantize_scalar(float v, float scale, int qmax) {
    const float r = rintf(__fdiv_rn(v, scale));  // nearbyint: round half to even
    int q = int(r);
    if (r > float(qmax)) q = qmax;
    if (r < -float(qmax)) q = -qmax;
    return q < -qmax ? -qmax : (q > qmax ? qmax : q);
}

// Per-row scale max|w| / qmax, or 1 for an all-zero row (cu:83-101).
__device__ float row_scale(const float* wr, int cols, int bits, int lane) {
    float m = 0.0f;
    for (int k = lane; k < cols; k += 32) m = fmaxf(m, fabsf(wr[k]));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    return m > 0.0f ? __fdiv_rn(m, float(qmax_for(bits))) : 1.0f;
}

// ref[s * rows + r] = sum_k fp16(w[r,k]) * fp16(x[s,k])  (cu:280-309)
__global__ void reference_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                 int rows, int cols, int samples, float* __restrict__ ref) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int chunks = (samples + 31) / 32;
    if (warp >= rows * chunks) return;
    const int r = warp / chunks;
    const int s = (warp % chunks) * 32 + lane;
    const float* wr = w + size_t(r) * cols;
    const float* xs = x + size_t(s < samples ? s : 0) * cols;
    float acc = 0.0f;
    for (int k = 0; k < cols; ++k)
        acc = __fadd_rn(acc, __fmul_rn(round_fp16(wr[k]), round_fp16(xs[k])));
    if (s < samples) ref[size_t(s) * rows + r] = acc;
}

// Squared error sums of one (row, width) pair (cu:311-376).  Writes
// part[(bits-3) * rows + r] = {hw_num, full_num, den} summed over samples.
__global__ void width_kernel(const float* __restrict__ w, const float* __restrict__ x,
                             const float* __restrict__ ref, int rows, int cols, int samples,
                             double* __restrict__ part) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows * 14) return;
    const int bits = 3 + warp / rows;
    const int r = warp % rows;
    const float* wr = w + size_t(r) * cols;
    const int qmax = qmax_for(bits);
    const float scale = bits == kFp16Bits ? 1.0f : row_scale(wr, cols, bits, lane);
    double hw_num = 0.0, full_num = 0.0, den = 0.0;
    for (int s0 = 0; s0 < samples; s0 += 32) {
        const int s = s0 + lane;
        const float* xs = x + size_t(s < samples ? s : 0) * cols;
        float hw = 0.0f, full = 0.0f;
        if (bits == kFp16Bits) {
            for (int k = 0; k < cols; ++k)
                hw = __fadd_rn(hw, __fmul_rn(round_fp16(wr[k]), round_fp16(xs[k])));
            full = hw;
        } else if (bits <= 8) {
            float idot = 0.0f;
            for (int k = 0; k < cols; ++k) {
                const float xh = round_fp16(xs[k]);
                const int q = quantize_scalar(wr[k], scale, qmax);
                idot = __fadd_rn(idot, __fmul_rn(float(q), xh));
                full = __fadd_rn(full, __fmul_rn(round_fp16(__fmul_rn(float(q), scale)), xh));
            }
            hw = __fmul_rn(idot, scale);
        } else {
            for (int k = 0; k < cols; ++k) {
                const float xh = round_fp16(xs[k]);
                const int q = quantize_scalar(wr[k], scale, qmax);
                hw = __fadd_rn(hw, __fmul_rn(round_fp16(__fmul_rn(float(q), scale)), xh));
            }
            full = hw;
        }
        if (s < samples) {
            const double rv = ref[size_t(s) * rows + r];
            const double dh = double(hw) - rv, df = double(full) - rv;
            hw_num += dh * dh;
            full_num += df * df;
            den += rv * rv;
        }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        hw_num += __shfl_xor_sync(0xffffffffu, hw_num, d);
        full_num += __shfl_xor_sync(0xffffffffu, full_num, d);
        den += __shfl_xor_sync(0xffffffffu, den, d);
    }
    if (lane == 0) {
        double* p = part + 3 * (size_t(bits - 3) * rows + r);
        p[0] = hw_num;
        p[1] = full_num;
        p[2] = den;
    }
}

// One block per width: fixed-order sum over rows, then sqrt(num / den).
__global__ void finish_kernel(const double* __restrict__ part, int rows, double* __restrict__ hw,
                              double* __restrict__ full) {
    __shared__ double sh[3][256];
    const int wi = blockIdx.x;
    double a = 0.0, b = 0.0, c = 0.0;
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
        const double* p = part + 3 * (size_t(wi) * rows + r);
        a += p[0];
        b += p[1];
        c += p[2];
    }
    sh[0][threadIdx.x] = a;
    sh[1][threadIdx.x] = b;
    sh[2][threadIdx.x] = c;
    __syncthreads();
    for (int d = blockDim.x / 2; d > 0; d >>= 1) {
        if (threadIdx.x < d)
            for (int j = 0; j < 3; ++j) sh[j][threadIdx.x] += sh[j][threadIdx.x + d];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const double den = sh[2][0] > 1.0e-30 ? sh[2][0] : 1.0e-30;
        hw[wi] = sqrt(sh[0][0] / den);
        full[wi] = sqrt(sh[1][0] / den);
    }
}

// Quantise float weights to int16 codes + scales for width `bits` (3..15)
// (cu:77-101, 126-146).  One warp per row.
__global__ void quantize_kernel(const float* __restrict__ w, int rows, int cols, int bits,
                                int16_t* __restrict__ codes, float* __restrict__ scales) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float* wr = w + size_t(warp) * cols;
    const float scale = row_scale(wr, cols, bits, lane);
    const int qmax = qmax_for(bits);
    for (int k = lane; k < cols; k += 32)
        codes[size_t(warp) * cols + k] = int16_t(quantize_scalar(wr[k], scale, qmax));
    if (lane == 0) scales[warp] = scale;
}

// fp32 weights to fp16 bit patterns (the 16-bit storage, cu:113-120).
__global__ void to_fp16_kernel(const float* __restrict__ w, int64_t n, uint16_t* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __half_as_ushort(__float2half_rn(w[i]));
}

}  // namespace

cudaError_t launch_analyze(const float* w, int rows, int cols, const float* x, int samples,
                           float* ref_scratch, double* part_scratch, double* hw, double* full,
                           cudaStream_t s) {
    const int chunks = (samples + 31) / 32;
    const int64_t ref_threads = int64_t(rows) * chunks * 32;
    reference_kernel<<<unsigned((ref_threads + 255) / 256), 256, 0, s>>>(w, x, rows, cols, samples,
                                                                        ref_scratch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t width_threads = int64_t(rows) * 14 * 32;
    width_kernel<<<unsigned((width_threads + 255) / 256), 256, 0, s>>>(w, x, ref_scratch, rows, cols,
                                                                      samples, part_scratch);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    finish_kernel<<<14, 256, 0, s>>>(part_scratch, rows, hw, full);
    return cudaGetLastError();
}

cudaError_t launch_quantize(const float* w, int rows, int cols, int bits, int16_t* codes,
                            float* scales, cudaStream_t s) {
    const int64_t threads = int64_t(rows) * 32;
    quantize_kernel<<<unsigned((threads + 255) / 256), 256, 0, s>>>(w, rows, cols, bits, codes, scales);
    return cudaGetLastError();
}

cudaError_t launch_to_fp16(const float* w, int64_t n, uint16_t* out, cudaStream_t s) {
    to_fp16_kernel<<<unsigned((n + 255) / 256), 256, 0, s>>>(w, n, out);
    return cudaGetLastError();
}

}  // namespace ebx

// ---------------------------------------------------------------------------
// Allocation-free analyzer: the same kernels, scratch in a fixed device array.
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory: code running inside a host
// framework whose device memory belongs to that framework's pooled allocator
// (with a fixed budget and no workspace handed to plugins), or latency-bound
// code that must never hit the implicit device synchronisation of
// cudaMalloc/cudaFree.  ebx_analyze_noalloc serves them from one static array
// that every GPU loading this library holds for the life of the process.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_analyze_scratch[kNoAllocScratchBytes];

// In host code `g_analyze_scratch` names a host-side stand-in, not device
// memory; the device address comes from cudaGetSymbolAddress, taken once per
// device with that device current and kept for the process (a cudaDeviceReset
// would free the array and leave the kept address stale; the header forbids
// calls after one).
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[64] = {};

cudaError_t noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_analyze_scratch);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" ebx_status ebx_analyze_noalloc(const float* weights, int32_t rows, int32_t cols,
                                          const float* calib, int32_t samples, double* hw_err,
                                          double* full_err, void* stream) {
    if (rows <= 0 || cols <= 0 || samples <= 0) {
        ebx::set_error("weights and calibration must be non-empty");
        return EBX_ERR_INVALID;
    }
    if (!weights || !calib || !hw_err || !full_err) {
        ebx::set_error("null argument");
        return EBX_ERR_INVALID;
    }
    // same layout as ebx_analyze's workspace: fp16 reference outputs, then the
    // per-(width, row) squared-error sums
    const uint64_t ref_bytes = ebx::round_up(uint64_t(rows) * uint64_t(samples) * 4, 256);
    const uint64_t need = ref_bytes + uint64_t(rows) * 14 * 3 * 8;
    if (need > kNoAllocScratchBytes) {
        ebx::set_error("ebx_analyze_noalloc: " + std::to_string(rows) + " rows x " +
                       std::to_string(samples) + " samples need " + std::to_string(need) +
                       " bytes of scratch, more than the built-in " +
                       std::to_string(kNoAllocScratchBytes) +
                       "; use ebx_analyze with a caller workspace");
        return EBX_ERR_INVALID;
    }
    void* base = nullptr;
    cudaError_t e = noalloc_scratch(&base);
    if (e == cudaSuccess) {
        // Nothing needs zeroing: every reference value and every partial sum the
        // finishing kernel reads is written earlier in this same call.
        float* ref = static_cast<float*>(base);
        double* part = reinterpret_cast<double*>(static_cast<unsigned char*>(base) + ref_bytes);
        e = ebx::launch_analyze(weights, rows, cols, calib, samples, ref, part, hw_err, full_err,
                                static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) {
        ebx::set_error(std::string("CUDA error: ") + cudaGetErrorString(e) +
                       " in ebx_analyze_noalloc");
        return EBX_ERR_CUDA;
    }
    return EBX_OK;
}
