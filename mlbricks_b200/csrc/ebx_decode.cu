// ebx_decode.cu -- small-M (decode, M <= 16) ElasticBit linear on B200.
//
// Replaces the reference's M=1 FastWarp GEMV (elasticbit_runtime.cu:508-648)
// and its M>1 "materialise to FP16 + cuBLAS" route (cu:982-1022, core.py:465-
// 471) for M <= 16.  The HBM stream is the exact-width code (b bits per
// weight), not an expanded FP16/INT8 copy.
//
// Work mapping.  One CTA = one 16-row group; its 8 warps split the k-tiles into
// contiguous runs.  Per warp, a D-stage cp.async ring in shared memory streams
// each 64-k supertile (b * 128 bytes, coalesced 16-byte vectors) plus the
// lane's 32-byte activation runs.  Each lane decodes its 32 codes exactly to
// fp16 A-fragments (fp16_rn(fp32_rn(q * s)), bit-identical to the reference's
// dequantised weight) and issues mma.m16n8k16 with the activations as the
// 8-token B operand (two of them for M > 8), accumulating in fp32 registers.
// The 8 warp partials are summed in a fixed order through shared memory, so
// the result is deterministic run to run.
//
// Semantics.
//   exec width 16 (fullPrecision, and hardwareNative for b >= 9):
//       y = fp16( sum_k x_k * fp16(q_k * s) + bias )        (cu:614-648)
//   exec width 8/4 (hardwareNative integer dot, b <= 8):
//       y = fp16( s * sum_k x_k * q_k + bias )              (cu:508-609)
// Bias is added in fp32 before the single fp16 rounding, as cuBLAS does for
// F.linear(x, W, b) on the reference's M>1 route.
#include <atomic>

#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct DecodeArgs {
    const uint8_t* tiles;
    const float* scales;
    const uint16_t* x;
    const uint16_t* bias;
    uint16_t* y;
    float* y32;
    int M, N, K;
    int kt;
};

template <int B, int NT, bool VECX>
struct StageLayout {
    static constexpr int kTileBytes = B * 128;
    static constexpr int kXBytes = VECX ? NT * 32 * 32 : 0;
    static constexpr int kStage = kTileBytes + kXBytes;
};

template <int B, bool HW, int NT, bool VECX, int D>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(DecodeArgs a) {
    using L = StageLayout<B, NT, VECX>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = blockIdx.x;
    const int t0 = (warp * a.kt) / kWarps;
    const int t1 = ((warp + 1) * a.kt) / kWarps;
    uint8_t* ring = smem + warp * D * L::kStage;
    const uint8_t* gtiles = a.tiles + size_t(g) * a.kt * L::kTileBytes;

    const int r0 = lane >> 2;
    const int c = lane & 3;
    const int row_lo = g * kRowGroup + r0;
    const int row_hi = row_lo + 8;

    uint64_t nb2 = 0, slo2 = 0, shi2 = 0;
    if constexpr (B != kFp16Bits) {
        const float nb = -(8388608.0f + float(qmax_for(B)));
        nb2 = pack2f(nb, nb);
        if constexpr (!HW) {
            const float sl = row_lo < a.N ? a.scales[row_lo] : 0.0f;
            const float sh = row_hi < a.N ? a.scales[row_hi] : 0.0f;
            slo2 = pack2f(sl, sl);
            shi2 = pack2f(sh, sh);
        }
    }

    auto issue = [&](int t, int stage) {
        uint8_t* dst = ring + stage * L::kStage;
        const uint8_t* src = gtiles + size_t(t) * L::kTileBytes;
#pragma unroll
        for (int q = 0; q < B / 4; ++q)
            cp_async16(smem_u32(dst + q * 512 + lane * 16), src + q * 512 + lane * 16, 16);
        if constexpr ((B & 2) != 0)
            cp_async8(smem_u32(dst + (B / 4) * 512 + lane * 8), src + (B / 4) * 512 + lane * 8);
        if constexpr ((B & 1) != 0) {
            const int off = (B / 4) * 512 + ((B & 2) ? 256 : 0) + lane * 4;
            cp_async4(smem_u32(dst + off), src + off);
        }
        if constexpr (VECX) {
#pragma unroll
            for (int nb = 0; nb < NT; ++nb) {
                const int n = r0 + 8 * nb;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int k = t * kKTile + 16 * c + 8 * h;
                    const bool ok = n < a.M && k < a.K;
                    const uint16_t* s = ok ? a.x + size_t(n) * a.K + k : a.x;
                    cp_async16(smem_u32(dst + L::kTileBytes + ((nb * 2 + h) * 32 + lane) * 16), s,
                               ok ? 16 : 0);
                }
            }
        }
    };

    float acc[NT][4];
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;

#pragma unroll
    for (int i = 0; i < D - 1; ++i) {
        if (t0 + i < t1) issue(t0 + i, i);
        cp_async_commit();
    }

    for (int t = t0; t < t1; ++t) {
        const int i = t - t0;
        cp_async_wait<D - 2>();
        const uint8_t* st = ring + (i % D) * L::kStage;
        uint32_t w[B];
#pragma unroll
        for (int q = 0; q < B / 4; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(st + q * 512 + lane * 16);
            w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
        }
        if constexpr ((B & 2) != 0) {
            const uint2 v = *reinterpret_cast<const uint2*>(st + (B / 4) * 512 + lane * 8);
            w[4 * (B / 4)] = v.x;
            w[4 * (B / 4) + 1] = v.y;
        }
        if constexpr ((B & 1) != 0) {
            w[B - 1] = *reinterpret_cast<const uint32_t*>(st + (B / 4) * 512 + ((B & 2) ? 256 : 0) +
                                                          lane * 4);
        }
        uint32_t xb[NT][8];
        if constexpr (VECX) {
#pragma unroll
            for (int nb = 0; nb < NT; ++nb)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 v = *reinterpret_cast<const uint4*>(
                        st + L::kTileBytes + ((nb * 2 + h) * 32 + lane) * 16);
                    xb[nb][4 * h] = v.x; xb[nb][4 * h + 1] = v.y;
                    xb[nb][4 * h + 2] = v.z; xb[nb][4 * h + 3] = v.w;
                }
        } else {
#pragma unroll
            for (int nb = 0; nb < NT; ++nb) {
                const int n = r0 + 8 * nb;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int k = t * kKTile + 16 * c + 2 * e;
                    uint32_t lo = 0, hi = 0;
                    if (n < a.M && k < a.K) lo = a.x[size_t(n) * a.K + k];
                    if (n < a.M && k + 1 < a.K) hi = a.x[size_t(n) * a.K + k + 1];
                    xb[nb][e] = lo | (hi << 16);
                }
            }
        }
        if (t + D - 1 < t1) issue(t + D - 1, (i + D - 1) % D);
        cp_async_commit();

#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t af[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int p = 4 * s + r;
                if constexpr (B == kFp16Bits) {
                    af[r] = w[p];
                } else if constexpr (HW) {
                    af[r] = codes2_to_half(code_magic<B>(w, 2 * p), code_magic<B>(w, 2 * p + 1), nb2);
                } else {
                    af[r] = dequant2(code_magic<B>(w, 2 * p), code_magic<B>(w, 2 * p + 1), nb2,
                                     (r & 1) ? shi2 : slo2);
                }
            }
#pragma unroll
            for (int nb = 0; nb < NT; ++nb)
                mma_16816(acc[nb], af, xb[nb][(s >> 1) * 4 + (s & 1) * 2],
                          xb[nb][(s >> 1) * 4 + (s & 1) * 2 + 1]);
        }
    }
    cp_async_wait<0>();

    // Fixed-order cross-warp reduction.
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((warp * NT + nb) * 32 + lane) * 4 + i] = acc[nb][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NT * 128; idx += kThreads) {
        const int nb = idx >> 7, l = (idx >> 2) & 31, i = idx & 3;
        float v = 0.0f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) v += red[((ww * NT + nb) * 32 + l) * 4 + i];
        const int row = g * kRowGroup + (l >> 2) + 8 * (i >> 1);
        const int tok = 8 * nb + (l & 3) * 2 + (i & 1);
        if (row < a.N && tok < a.M) {
            if constexpr (HW && B != kFp16Bits) v = v * a.scales[row];
            if (a.bias) v += __half2float(__ushort_as_half(a.bias[row]));
            a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(v));
            if (a.y32) a.y32[size_t(tok) * a.N + row] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// v2: TMA-staged weight stream (the fast path; K % 8 == 0, x 16-byte aligned)
// ---------------------------------------------------------------------------
// Same CTA/warp mapping and arithmetic as decode_kernel, but each warp streams
// its contiguous k-run of supertiles with cp.async.bulk (one instruction per
// stage of ST supertiles, completing on a per-stage mbarrier) into a D-deep
// shared-memory ring, and loads activations straight into registers one tile
// ahead.  Every mbarrier wait is bounded: after kWaitLimit probes the warp
// records EBX_DEVICE_TIMEOUT in g_device_status, drains its own copies (again
// bounded) and leaves the loop, so a stuck copy cannot hang the GPU.
__device__ int g_device_status = 0;
constexpr int kDeviceTimeout = 0x7101;
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < kWaitLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

template <int B, bool HW, int NT, int D, int ST>
__global__ void __launch_bounds__(kThreads, 2) decode_tma_kernel(DecodeArgs a) {
    constexpr int kTileBytes = B * 128;
    constexpr int kStageBytes = ST * kTileBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = blockIdx.x;
    const int t0 = (warp * a.kt) / kWarps;
    const int t1 = ((warp + 1) * a.kt) / kWarps;
    const int nchunks = (t1 - t0 + ST - 1) / ST;
    uint8_t* ring = smem + warp * D * kStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * D * kStageBytes) + warp * D;
    const uint8_t* gtiles = a.tiles + (size_t(g) * a.kt + t0) * kTileBytes;

    if (lane == 0) {
        for (int i = 0; i < D; ++i) mbar_init(smem_u32(&bars[i]), 1);
        fence_proxy_async_smem();
    }
    __syncwarp();

    auto issue = [&](int chunk) {  // lane 0 only
        const int stage = chunk % D;
        const int ntiles = min(ST, t1 - t0 - chunk * ST);
        const uint32_t bytes = uint32_t(ntiles * kTileBytes);
        const uint32_t bar = smem_u32(&bars[stage]);
        mbar_expect_tx(bar, bytes);
        bulk_g2s(smem_u32(ring + stage * kStageBytes), gtiles + size_t(chunk) * kStageBytes, bytes,
                 bar);
    };
    if (lane == 0)
        for (int c = 0; c < D && c < nchunks; ++c) issue(c);

    const int r0 = lane >> 2;
    const int c = lane & 3;
    const int row_lo = g * kRowGroup + r0;
    const int row_hi = row_lo + 8;
    const uint32_t mask = (1u << B) - 1u;
    const uint32_t magic = 0x4B000000u;
    uint64_t nb2 = 0, slo2 = 0, shi2 = 0;
    if constexpr (B != kFp16Bits) {
        const float nb = -(8388608.0f + float(qmax_for(B)));
        nb2 = pack2f(nb, nb);
        if constexpr (!HW) {
            const float sl = row_lo < a.N ? a.scales[row_lo] : 0.0f;
            const float sh = row_hi < a.N ? a.scales[row_hi] : 0.0f;
            slo2 = pack2f(sl, sl);
            shi2 = pack2f(sh, sh);
        }
    }

    // activation B-fragments: x[n][k0 + 16c .. +16) for n = r0 + 8nb
    bool tok_ok[NT];
    const uint16_t* xrow[NT];
#pragma unroll
    for (int nb = 0; nb < NT; ++nb) {
        const int n = r0 + 8 * nb;
        tok_ok[nb] = n < a.M;
        xrow[nb] = a.x + size_t(tok_ok[nb] ? n : 0) * a.K + 16 * c;
    }
    auto load_x = [&](int t, uint32_t (&xb)[NT][8]) {
#pragma unroll
        for (int nb = 0; nb < NT; ++nb)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int k = t * kKTile + 16 * c + 8 * h;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (tok_ok[nb] && k < a.K)
                    v = __ldg(reinterpret_cast<const uint4*>(xrow[nb] + t * kKTile + 8 * h));
                xb[nb][4 * h] = v.x; xb[nb][4 * h + 1] = v.y;
                xb[nb][4 * h + 2] = v.z; xb[nb][4 * h + 3] = v.w;
            }
    };

    float acc[NT][4];
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;

    uint32_t xcur[NT][8], xnext[NT][8];
    if (t0 < t1) load_x(t0, xcur);
    bool ok = true;
    for (int chunk = 0; chunk < nchunks && ok; ++chunk) {
        const int stage = chunk % D;
        if (!bounded_wait(smem_u32(&bars[stage]), uint32_t((chunk / D) & 1))) {
            ok = false;
            break;
        }
        const int ntiles = min(ST, t1 - t0 - chunk * ST);
        for (int tt = 0; tt < ntiles; ++tt) {
            const int t = t0 + chunk * ST + tt;
            const uint8_t* st = ring + stage * kStageBytes + tt * kTileBytes;
            uint32_t w[B];
#pragma unroll
            for (int q = 0; q < B / 4; ++q) {
                const uint4 v = *reinterpret_cast<const uint4*>(st + q * 512 + lane * 16);
                w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
            }
            if constexpr ((B & 2) != 0) {
                const uint2 v = *reinterpret_cast<const uint2*>(st + (B / 4) * 512 + lane * 8);
                w[4 * (B / 4)] = v.x;
                w[4 * (B / 4) + 1] = v.y;
            }
            if constexpr ((B & 1) != 0)
                w[B - 1] = *reinterpret_cast<const uint32_t*>(st + (B / 4) * 512 +
                                                              ((B & 2) ? 256 : 0) + lane * 4);
            if (t + 1 < t1) load_x(t + 1, xnext);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                uint32_t af[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int p = 4 * s + r;
                    if constexpr (B == kFp16Bits) {
                        af[r] = w[p];
                    } else if constexpr (HW) {
                        af[r] = codes2_lop(code_word<B>(w, 2 * p), code_word<B>(w, 2 * p + 1), mask,
                                           magic, nb2);
                    } else {
                        af[r] = dequant2_lop(code_word<B>(w, 2 * p), code_word<B>(w, 2 * p + 1),
                                             mask, magic, nb2, (r & 1) ? shi2 : slo2);
                    }
                }
#pragma unroll
                for (int nb = 0; nb < NT; ++nb)
                    mma_16816(acc[nb], af, xcur[nb][(s >> 1) * 4 + (s & 1) * 2],
                              xcur[nb][(s >> 1) * 4 + (s & 1) * 2 + 1]);
            }
#pragma unroll
            for (int nb = 0; nb < NT; ++nb)
#pragma unroll
                for (int i = 0; i < 8; ++i) xcur[nb][i] = xnext[nb][i];
        }
        // every lane has read this stage; refill it with chunk + D
        __syncwarp();
        if (lane == 0 && chunk + D < nchunks) {
            fence_proxy_async_smem();
            issue(chunk + D);
        }
    }
    if (!ok) {
        if (lane == 0) atomicExch(&g_device_status, kDeviceTimeout);
        // drain this warp's copies still in flight (bounded), then fall through
        for (int chunk = 0; chunk < nchunks; ++chunk)
            bounded_wait(smem_u32(&bars[chunk % D]), uint32_t((chunk / D) & 1));
    }

    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((warp * NT + nb) * 32 + lane) * 4 + i] = acc[nb][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NT * 128; idx += kThreads) {
        const int nb = idx >> 7, l = (idx >> 2) & 31, i = idx & 3;
        float v = 0.0f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) v += red[((ww * NT + nb) * 32 + l) * 4 + i];
        const int row = g * kRowGroup + (l >> 2) + 8 * (i >> 1);
        const int tok = 8 * nb + (l & 3) * 2 + (i & 1);
        if (row < a.N && tok < a.M) {
            if constexpr (HW && B != kFp16Bits) v = v * a.scales[row];
            if (a.bias) v += __half2float(__ushort_as_half(a.bias[row]));
            a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(v));
            if (a.y32) a.y32[size_t(tok) * a.N + row] = v;
        }
    }
}

constexpr int kStages = 4;

template <int B, bool HW, int NT, bool VECX>
cudaError_t launch_one(const DecodeArgs& a, int groups, cudaStream_t s) {
    using L = StageLayout<B, NT, VECX>;
    constexpr int ring = kWarps * kStages * L::kStage;
    constexpr int red = kWarps * NT * 128 * 4;
    constexpr int smem = ring > red ? ring : red;
    auto kern = decode_kernel<B, HW, NT, VECX, kStages>;
    // The dynamic shared-memory opt-in is per function and per device.
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    kern<<<groups, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <int B, bool HW, int NT>
cudaError_t launch_tma(const DecodeArgs& a, int groups, cudaStream_t s) {
    constexpr int ST = B <= 12 ? 2 : 1;
    constexpr int D = 4;
    constexpr int ring = kWarps * D * ST * B * 128 + kWarps * D * 8;
    constexpr int red = kWarps * NT * 128 * 4;
    constexpr int smem = ring > red ? ring : red;
    auto kern = decode_tma_kernel<B, HW, NT, D, ST>;
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    kern<<<groups, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

template <int B, bool HW>
cudaError_t dispatch_nt(const DecodeArgs& a, int groups, bool vecx, cudaStream_t s) {
    if (vecx)
        return a.M <= 8 ? launch_tma<B, HW, 1>(a, groups, s) : launch_tma<B, HW, 2>(a, groups, s);
    return a.M <= 8 ? launch_one<B, HW, 1, false>(a, groups, s) : launch_one<B, HW, 2, false>(a, groups, s);
}

}  // namespace

cudaError_t read_device_status(int* status, bool clear, cudaStream_t s) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_device_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

cudaError_t launch_decode(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                          uint16_t* y, float* y32, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const bool vecx = (m.cols % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const bool hw = m.exec_width < 16 && m.bits <= 8;
    for (int64_t m0 = 0; m0 < M; m0 += 16) {
        DecodeArgs a;
        a.tiles = m.tiles;
        a.scales = m.scales;
        a.x = x + m0 * m.cols;
        a.bias = bias;
        a.y = y + m0 * m.rows;
        a.y32 = y32 ? y32 + m0 * m.rows : nullptr;
        a.M = int(M - m0 < 16 ? M - m0 : 16);
        a.N = m.rows;
        a.K = m.cols;
        a.kt = int(m.kt);
        const int groups = int(m.groups);
        cudaError_t e = cudaErrorInvalidValue;
        const bool v = vecx && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
        switch (m.bits) {
#define EBX_DEC_CASE(BB)                                                                \
    case BB:                                                                            \
        e = hw ? dispatch_nt<BB, true>(a, groups, v, s) : dispatch_nt<BB, false>(a, groups, v, s); \
        break;
            EBX_DEC_CASE(3) EBX_DEC_CASE(4) EBX_DEC_CASE(5) EBX_DEC_CASE(6) EBX_DEC_CASE(7)
            EBX_DEC_CASE(8)
#undef EBX_DEC_CASE
#define EBX_DEC_CASE_FULL(BB) \
    case BB:                  \
        e = dispatch_nt<BB, false>(a, groups, v, s); \
        break;
            EBX_DEC_CASE_FULL(9) EBX_DEC_CASE_FULL(10) EBX_DEC_CASE_FULL(11)
            EBX_DEC_CASE_FULL(12) EBX_DEC_CASE_FULL(13) EBX_DEC_CASE_FULL(14)
            EBX_DEC_CASE_FULL(15) EBX_DEC_CASE_FULL(16)
#undef EBX_DEC_CASE_FULL
            default:
                break;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace ebx
