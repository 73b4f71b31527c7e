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
#include <cstdlib>
#include <cstring>

#include "ebx_common.cuh"
#include "ebx_internal.h"
#include "ebx_xchg.cuh"

namespace ebx {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Device health word: bounded waits that give up record their code here.
__device__ int g_device_status = 0;
constexpr int kDeviceTimeout = 0x7101;

struct DecodeArgs {
    const uint8_t* tiles;
    const float* scales;
    const uint16_t* x;
    const uint16_t* bias;
    uint16_t* y;
    float* y32;
    int M, N, K;
    int kt;
    int groups;       // row groups (N padded to 16) / 16
    uint32_t magic;   // 0x4B000000 (2^23), passed in so the compiler keeps it in a register
    uint32_t magic_plane;  // 0x64646464 (fp16 upper bytes of 1024), likewise
    int stages;       // pipe kernel: ring depth (runtime, <= kMaxStages)
    int stage_bytes;  // pipe kernel: RG weight rounds + (min(M, 8 NT) + 1) activation rows
    XchgArgs xa;      // world > 0: fp32 partials go to the tensor-parallel exchange
    int act;          // 1: SwiGLU over interleaved gate/up rows (y has N / 2 columns)
    int code;         // multi launch: 2 * bits + (integer semantics), selects the decode
    int pdl_early;    // pipe kernel: signal dependents at the start instead of the end
};

// SwiGLU epilogue.  The matrix holds gate and up rows interleaved in blocks of 8
// (rows 16j..16j+7 = gate rows 8j..8j+7, rows 16j+8..16j+15 = the matching up
// rows), so the two sums of one output sit in fragment elements i and i + 2 of
// the same lane: y[tok, 8j + r] = fp16(silu(g) * u) from the fp32 sums (bias, if
// any, added to each first; integer-path scales applied per row).
template <int B, bool HW>
__device__ __forceinline__ void store_swiglu(const DecodeArgs& a, int g, int l, int tok, float vg,
                                             float vu) {
    const int grow = g * kRowGroup + (l >> 2);
    const int urow = grow + 8;
    if (urow >= a.N || tok >= a.M) return;
    if constexpr (HW && B != kFp16Bits) {
        vg *= a.scales[grow];
        vu *= a.scales[urow];
    }
    if (a.bias) {
        vg += __half2float(__ushort_as_half(a.bias[grow]));
        vu += __half2float(__ushort_as_half(a.bias[urow]));
    }
    const float v = vg / (1.0f + __expf(-vg)) * vu;
    const int nout = a.N >> 1;
    const int col = g * 8 + (l >> 2);
    a.y[size_t(tok) * nout + col] = __half_as_ushort(__float2half_rn(v));
    if (a.y32) a.y32[size_t(tok) * nout + col] = v;
}

// Fused exchange: all ranks' partials of (tok, row) -> bias -> one fp16 rounding.
// owner >= 0: the two-phase form (the owner rank reduces, the others wait for its sum).
__device__ __forceinline__ void xchg_finish_one(const DecodeArgs& a, uint32_t e, int tok, int row,
                                                int owner = -1) {
    float v;
    const bool ok = owner >= 0 ? xchg_reduce_owner(a.xa, e, owner, a.M, a.N, tok, row, v)
                               : xchg_gather(a.xa, e, a.M, a.N, tok, row, v);
    if (!ok) {
        atomicExch(&g_device_status, kXchgTimeout);
        return;
    }
    if (a.bias) v += __half2float(__ushort_as_half(a.bias[row]));
    a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(v));
    if (a.y32) a.y32[size_t(tok) * a.N + row] = v;
}

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
    const uint32_t xe = a.xa.world ? xchg_epoch(a.xa) + 1u : 0u;  // epoch this call publishes

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

        if constexpr (plane_layout(B)) {
            // plane layout: exact q pairs, then (fullPrecision) fp16_rn(fp32_rn(q * s))
            uint32_t q16[16];
            PlaneConsts pk;
            pk.init(a.magic_plane);
            plane_q16_all<B>(w, pk, q16);
            if constexpr (!HW) {
#pragma unroll
                for (int p = 0; p < 16; ++p) q16[p] = q16_to_w16(q16[p], (p & 1) ? shi2 : slo2);
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                const uint32_t af[4] = {q16[4 * s], q16[4 * s + 1], q16[4 * s + 2], q16[4 * s + 3]};
#pragma unroll
                for (int nb = 0; nb < NT; ++nb)
                    mma_16816(acc[nb], af, xb[nb][(s >> 1) * 4 + (s & 1) * 2],
                              xb[nb][(s >> 1) * 4 + (s & 1) * 2 + 1]);
            }
            continue;
        }
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
        if (a.act) {
            if ((i >> 1) == 0) {
                float vu = 0.0f;
#pragma unroll
                for (int ww = 0; ww < kWarps; ++ww) vu += red[((ww * NT + nb) * 32 + l) * 4 + i + 2];
                store_swiglu<B, HW>(a, g, l, tok, v, vu);
            }
            continue;
        }
        if (row < a.N && tok < a.M) {
            if constexpr (HW && B != kFp16Bits) v = v * a.scales[row];
            if (a.xa.world) {
                xchg_push(a.xa, xe, a.M, a.N, tok, row, v);
            } else {
                if (a.bias) v += __half2float(__ushort_as_half(a.bias[row]));
                a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(v));
                if (a.y32) a.y32[size_t(tok) * a.N + row] = v;
            }
        }
    }
    if (a.xa.world && a.xa.fused) {
        for (int idx = threadIdx.x; idx < NT * 128; idx += kThreads) {
            const int l = (idx >> 2) & 31, i = idx & 3;
            const int row = g * kRowGroup + (l >> 2) + 8 * (i >> 1);
            const int tok = 8 * (idx >> 7) + (l & 3) * 2 + (i & 1);
            if (row < a.N && tok < a.M) xchg_finish_one(a, xe, tok, row);
        }
        xchg_advance(a.xa, xe);
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

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity) {
    return mbar_wait_bounded(bar, parity);  // wall-clock bound (ebx_common.cuh)
}

// ---------------------------------------------------------------------------
// v4: CTA-wide TMA pipeline (the fast path)
// ---------------------------------------------------------------------------
// One CTA = one 16-row group over the full K.  Warps 0..7 consume; warp 8
// produces.  The k-tiles are processed in rounds of 8 (one per consumer warp:
// warp w takes tile 8r + w), so a round's 8 supertiles form one contiguous
// byte range -> ONE bulk copy, and the round's activation slice is one bulk
// copy of up to 512 halves per token row (lanes < M of the producer warp).  A
// D-deep ring of rounds is guarded by per-stage full (TMA transaction count)
// and empty (8 consumer-warp arrivals) mbarriers; every wait is bounded.
constexpr int kMaxStages = 16;

// TPW: supertiles each consumer warp takes per round (one barrier wait, one
// release and one loop trip per TPW tiles instead of per tile).
template <int B, int NT, int RG, int TPW>
struct PipeStage {
    static constexpr int kTileBytes = B * 128;
    static constexpr int kRound = kWarps * TPW;                // supertiles per round and row group
    static constexpr int kWBytes = kRound * kTileBytes;        // one row group's round
    static constexpr int kXStride = kRound * kKTile * 2 + 16;  // bank-shifted activation rows
    // the consumers' fragment sums, written over the (drained) ring after the main loop
    static constexpr int kRedBytes = RG * kWarps * NT * 128 * 4;
    // stage = RG weight rounds + activation rows of tokens 0..m-1, and one zero row read
    // by the lanes whose token is >= m when m < 8 NT
    static int bytes(int m) { return RG * kWBytes + (m + (m < NT * 8 ? 1 : 0)) * kXStride; }
};

// Barrier 1 over the `warps` consumer warps (the producer warp does not take part).
__device__ __forceinline__ void consumers_sync(int warps) {
    asm volatile("bar.sync 1, %0;" ::"r"(warps * 32) : "memory");
}

// Programmatic dependent launch (no-ops when the launch did not ask for it):
// griddepcontrol.wait blocks until the previous kernel in the stream has
// completed and its writes are visible; launch_dependents lets the next
// kernel's CTAs be scheduled once every CTA of this grid has signalled it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// One ring round of a plane-decode consumer warp: TPW consecutive supertiles of the
// round (those with index < rem), their codes decoded to exact fp16 q pairs with byte
// permutes (plane_q16_all) and multiplied by mma.m16n8k16 against the staged
// activations into acc.  The warp releases the stage (empty barrier) once every
// shared-memory load of it has been issued.
//   HW:   integer codes as operands, row scale applied after accumulation
//         (the epilogue multiplies); fp16 holds every |q| <= 2047 exactly.
//   !HW:  fp16_rn(fp32_rn(q * s)) operands (W16A16 semantics), from the same q;
//         s2 = (s, s) of the lane's two rows.
template <int B, bool HW, int NT, int TPW, class S>
__device__ __forceinline__ void plane_round(const uint8_t* smem, int so, int rem, int w16, int w8,
                                            int w4, const int (&xa)[NT], const PlaneConsts& pk,
                                            const uint64_t (&s2)[2], float (&acc)[NT][4],
                                            uint32_t empty_bar, int lane) {
#pragma unroll
    for (int j = 0; j < TPW; ++j) {
        const bool have = rem > j;
        uint32_t w[B];
        uint32_t xb[NT][8];
        if (have) {
            const int T0 = so + j * S::kTileBytes;
#pragma unroll
            for (int q = 0; q < B / 4; ++q) {
                const uint4 v = *reinterpret_cast<const uint4*>(smem + w16 + T0 + q * 512);
                w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
            }
            if constexpr ((B & 2) != 0) {
                const uint2 v = *reinterpret_cast<const uint2*>(smem + w8 + T0 + (B / 4) * 512);
                w[4 * (B / 4)] = v.x;
                w[4 * (B / 4) + 1] = v.y;
            }
            if constexpr ((B & 1) != 0)
                w[B - 1] = *reinterpret_cast<const uint32_t*>(smem + w4 + T0 + (B / 4) * 512 +
                                                              ((B & 2) ? 256 : 0));
#pragma unroll
            for (int nb = 0; nb < NT; ++nb)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 v = *reinterpret_cast<const uint4*>(smem + xa[nb] + so +
                                                                    j * kKTile * 2 + 16 * h);
                    xb[nb][4 * h] = v.x; xb[nb][4 * h + 1] = v.y;
                    xb[nb][4 * h + 2] = v.z; xb[nb][4 * h + 3] = v.w;
                }
        }
        if (j == TPW - 1) {  // every load of this stage has been issued
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar);
        }
        if (!have) continue;
        uint32_t af[16];
        plane_q16_all<B>(w, pk, af);
        if constexpr (!HW) {
#pragma unroll
            for (int p = 0; p < 16; ++p) af[p] = q16_to_w16(af[p], s2[p & 1]);
        }
#pragma unroll
        for (int s4 = 0; s4 < 4; ++s4) {
            const uint32_t f[4] = {af[4 * s4], af[4 * s4 + 1], af[4 * s4 + 2], af[4 * s4 + 3]};
#pragma unroll
            for (int nb = 0; nb < NT; ++nb)
                mma_16816(acc[nb], f, xb[nb][(s4 >> 1) * 4 + (s4 & 1) * 2],
                          xb[nb][(s4 >> 1) * 4 + (s4 & 1) * 2 + 1]);
        }
    }
}

// (s, s) of the two rows lane `lane` holds in row group g (zero past N); only the
// fullPrecision (!HW) decode multiplies by them.
__device__ __forceinline__ void plane_row_scales(const DecodeArgs& a, int g, int lane,
                                                 uint64_t (&s2)[2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int row = g * kRowGroup + (lane >> 2) + 8 * h;
        const float sv = (g < a.groups && row < a.N) ? a.scales[row] : 0.0f;
        s2[h] = pack2f(sv, sv);
    }
}

// Consumer warp of the plane-layout decode (b = 8..12): per ring round it takes TPW
// consecutive supertiles of the round's 8 * TPW (plane_round).  Leaves the fp32
// fragment sums of this warp in red[] for the CTA reduction.
template <int B, bool HW, int NT, int TPW, int RG, class S>
__device__ __forceinline__ void plane_consume(const DecodeArgs& a, uint8_t* smem, uint32_t full0,
                                              uint32_t empty0, int rounds, int mrows, int warp,
                                              int lane, float* red, int cta) {
    const int rgl = warp / kWarps;  // local row group (RG > 1: the groups share each activation stage)
    const int wt = warp % kWarps;   // tile slot within the round
    const int g = cta * RG + rgl;
    const bool grp_ok = g < a.groups;
    const int r0 = lane >> 2;
    const int c = lane & 3;
    PlaneConsts pk;
    pk.init(a.magic_plane);
    uint64_t s2[2] = {0, 0};
    if constexpr (!HW) plane_row_scales(a, g, lane, s2);
    float acc[NT][4];
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;
    // this lane's operands in stage 0 (a round adds the stage offset `so`)
    const int wb = rgl * S::kWBytes + wt * TPW * S::kTileBytes;
    const int w16 = wb + lane * 16, w8 = wb + lane * 8, w4 = wb + lane * 4;
    int xa[NT];
#pragma unroll
    for (int nb = 0; nb < NT; ++nb) {
        const int tok = r0 + 8 * nb;
        xa[nb] = RG * S::kWBytes + (tok < mrows ? tok : mrows) * S::kXStride + wt * TPW * kKTile * 2 +
                 32 * c;
    }
    int rem = grp_ok ? a.kt - wt * TPW : 0;  // tiles of this warp's slot still ahead
    int so = 0, st = 0;
    uint32_t ph = 0;
    for (int r = 0; r < rounds; ++r) {
        if (!mbar_wait_bounded(full0 + 8u * uint32_t(st), ph)) {
            if (lane == 0) atomicExch(&g_device_status, kDeviceTimeout);
            break;
        }
        plane_round<B, HW, NT, TPW, S>(smem, so, rem, w16, w8, w4, xa, pk, s2, acc,
                                       empty0 + 8u * uint32_t(st), lane);
        rem -= S::kRound;
        so += a.stage_bytes;
        if (++st == a.stages) {
            st = 0;
            so = 0;
            ph ^= 1u;
        }
    }
    consumers_sync(RG * kWarps);  // red[] lies over the ring: every consumer is done with it
#pragma unroll
    for (int nb = 0; nb < NT; ++nb)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[(((rgl * kWarps + wt) * NT + nb) * 32 + lane) * 4 + i] = acc[nb][i];
}

// RG row groups per CTA (consumer warp w: row group w / 8, tile 8r + w % 8);
// every consumer of a round reads the same activation slice, so activation
// traffic per weight falls by RG.  Requires K % 64 == 0 (the generic kernel
// covers the rest); activation rows of tokens >= M are zeroed once and never
// written by the copy engine, so the fragment loads need no predicates.
// The pipe decode of CTA `cta` of a launch over one matrix (decode_pipe_kernel: cta =
// blockIdx.x; decode_multi_kernel: the CTA's index within its matrix's row groups).
template <int B, bool HW, int NT, bool DIRECT, int RG, int TPW>
__device__ __forceinline__ void decode_pipe_body(const DecodeArgs& a, const int cta) {
    using S = PipeStage<B, NT, RG, TPW>;
    constexpr int kConsumers = kWarps * RG;
    // plane layout (b = 9..12), and b = 8's byte codes under integer semantics
    constexpr bool kPlane = plane_layout(B) || (B == 8 && HW);
    extern __shared__ __align__(128) uint8_t smem[];
    const int D = a.stages;
    const int SB = a.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + D * SB);
    uint64_t* empty = full + kMaxStages;
    float* red = reinterpret_cast<float*>(smem);  // over the ring once every consumer is done
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rounds = (a.kt + S::kRound - 1) / S::kRound;
    const int mrows = a.M < NT * 8 ? a.M : NT * 8;

    if (threadIdx.x == 0) {
        for (int i = 0; i < D; ++i) {
            mbar_init(smem_u32(&full[i]), 1);
            mbar_init(smem_u32(&empty[i]), kConsumers);
        }
    }
    // zero row (index mrows) of every stage, never written by the copy engine:
    // lanes whose token is >= M read it
    if (mrows < NT * 8)
        for (int i = threadIdx.x; i < D * (S::kXStride / 16); i += blockDim.x)
            *reinterpret_cast<uint4*>(smem + (i / (S::kXStride / 16)) * SB + RG * S::kWBytes +
                                      mrows * S::kXStride + (i % (S::kXStride / 16)) * 16) =
                make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    __syncthreads();

    if (a.pdl_early) pdl_trigger();
    if (warp == kConsumers) {
        // ---------------- producer warp ----------------
        // The weight bytes of the first D rounds are requested before
        // griddepcontrol.wait (weights never depend on the previous kernel), their
        // activation slices after it.
        int ngroups = 0;
#pragma unroll
        for (int rg = 0; rg < RG; ++rg) ngroups += (cta * RG + rg) < a.groups ? 1 : 0;
        auto weights = [&](int r, int st) {
            const int ntile = min(S::kRound, a.kt - r * S::kRound);
            const uint32_t xbytes = uint32_t(ntile * kKTile * 2);
            uint8_t* dst = smem + st * SB;
            const uint32_t bar = smem_u32(&full[st]);
            if (lane == 0) {
                mbar_expect_tx(bar, uint32_t(ngroups * ntile * S::kTileBytes) + xbytes * uint32_t(mrows));
#pragma unroll
                for (int rg = 0; rg < RG; ++rg) {
                    const int g = cta * RG + rg;
                    if (g < a.groups)
                        bulk_g2s(smem_u32(dst + rg * S::kWBytes),
                                 a.tiles + (size_t(g) * a.kt + size_t(r) * S::kRound) * S::kTileBytes,
                                 uint32_t(ntile * S::kTileBytes), bar);
                }
            }
        };
        auto acts = [&](int r, int st) {
            const int ntile = min(S::kRound, a.kt - r * S::kRound);
            if (lane < mrows)
                bulk_g2s(smem_u32(smem + st * SB + RG * S::kWBytes + lane * S::kXStride),
                         a.x + size_t(lane) * a.K + size_t(r) * S::kRound * kKTile,
                         uint32_t(ntile * kKTile * 2), smem_u32(&full[st]));
        };
        const int pre = rounds < D ? rounds : D;
        for (int r = 0; r < pre; ++r) weights(r, r);
        pdl_wait();
        __syncwarp();
        for (int r = 0; r < pre; ++r) acts(r, r);
        for (int r = pre; r < rounds; ++r) {
            const int st = r % D;
            const uint32_t ph = uint32_t(r / D) & 1u;
            if (!bounded_wait(smem_u32(&empty[st]), ph ^ 1u)) {
                if (lane == 0) atomicExch(&g_device_status, kDeviceTimeout);
                break;
            }
            weights(r, st);
            __syncwarp();
            acts(r, st);
        }
        if (!a.pdl_early) pdl_trigger();
    } else {
        // ---------------- consumer warps ----------------
      if constexpr (kPlane) {
        plane_consume<B, HW, NT, TPW, RG, S>(a, smem, smem_u32(&full[0]), smem_u32(&empty[0]),
                                             rounds, mrows, warp, lane, red, cta);
        if (!a.pdl_early) pdl_trigger();
      } else {
        const int rgl = warp / kWarps;   // local row group
        const int wt = warp % kWarps;    // tile slot within the round
        const int g = cta * RG + rgl;
        const bool grp_ok = g < a.groups;
        const int r0 = lane >> 2;
        const int c = lane & 3;
        const int row_lo = g * kRowGroup + r0;
        const uint32_t magic = a.magic;  // opaque: kept in a register, never re-materialised
        // b = 8..12 (fullPrecision): paired f32x2 decode with the row scale itself
        constexpr bool kPaired = !HW && B == 8;
        constexpr int kPB = kPaired ? B : 8;
        PairConsts<kPB> pk;
        uint64_t s2[2] = {0, 0};
        if constexpr (kPaired) {
            pk.init(magic);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = row_lo + 8 * h;
                const float sv = (grp_ok && row < a.N) ? a.scales[row] : 0.0f;
                s2[h] = pack2f(sv, sv);
            }
        }
        float sc[2][kMaxSlots];
        if constexpr (B != kFp16Bits && !HW && !kPaired) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = row_lo + 8 * h;
                const float s = (grp_ok && row < a.N) ? a.scales[row] : 0.0f;
                // s * 2^-o for each in-place offset (exact power-of-two scaling)
                sc[h][0] = s * SlotScale<B, 0>::kFactor;
                sc[h][1] = s * SlotScale<B, 1>::kFactor;
                sc[h][2] = s * SlotScale<B, 2>::kFactor;
                sc[h][3] = s * SlotScale<B, 3>::kFactor;
                sc[h][4] = s * SlotScale<B, 4>::kFactor;
                sc[h][5] = s * SlotScale<B, 5>::kFactor;
                sc[h][6] = s * SlotScale<B, 6>::kFactor;
                sc[h][7] = s * SlotScale<B, 7>::kFactor;
            }
        }
        float acc[NT][4];
#pragma unroll
        for (int nb = 0; nb < NT; ++nb)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;
        // Byte offsets (in the dynamic shared array) of this lane's operands in
        // stage 0; a round adds the stage offset `so`.  Weight words sit at
        // q*512 + lane*16 (16-byte segments), then lane*8 and lane*4 (see
        // ebx_common.cuh).
        const int wb = rgl * S::kWBytes + wt * TPW * S::kTileBytes;
        const int w16 = wb + lane * 16, w8 = wb + lane * 8, w4 = wb + lane * 4;
        // activation row of token r0 + 8 nb, or the zero row when that token >= M
        int xa[NT];
#pragma unroll
        for (int nb = 0; nb < NT; ++nb) {
            const int tok = r0 + 8 * nb;
            xa[nb] = RG * S::kWBytes + (tok < mrows ? tok : mrows) * S::kXStride + wt * TPW * kKTile * 2 +
                     32 * c;
        }
        const uint32_t full0 = smem_u32(&full[0]), empty0 = smem_u32(&empty[0]);
        // tiles of this warp's slot still ahead of the current round
        int rem = grp_ok ? a.kt - wt * TPW : 0;
        int so = 0;
        int st = 0;
        uint32_t ph = 0;
        for (int r = 0; r < rounds; ++r) {
            if (!bounded_wait(full0 + 8u * uint32_t(st), ph)) {
                if (lane == 0) atomicExch(&g_device_status, kDeviceTimeout);
                break;
            }
#pragma unroll
          for (int j = 0; j < TPW; ++j) {
            const bool have = rem > j;
            uint32_t w[B];
            uint32_t xb[NT][8];
            if (have) {
                const int T0 = j * S::kTileBytes;
#pragma unroll
                for (int q = 0; q < B / 4; ++q) {
                    const uint4 v = *reinterpret_cast<const uint4*>(smem + w16 + so + T0 + q * 512);
                    w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
                }
                if constexpr ((B & 2) != 0) {
                    const uint2 v = *reinterpret_cast<const uint2*>(smem + w8 + so + T0 + (B / 4) * 512);
                    w[4 * (B / 4)] = v.x;
                    w[4 * (B / 4) + 1] = v.y;
                }
                if constexpr ((B & 1) != 0)
                    w[B - 1] = *reinterpret_cast<const uint32_t*>(smem + w4 + so + T0 + (B / 4) * 512 +
                                                                  ((B & 2) ? 256 : 0));
#pragma unroll
                for (int nb = 0; nb < NT; ++nb)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint4 v = *reinterpret_cast<const uint4*>(smem + xa[nb] + so + j * kKTile * 2 +
                                                                        16 * h);
                        xb[nb][4 * h] = v.x; xb[nb][4 * h + 1] = v.y;
                        xb[nb][4 * h + 2] = v.z; xb[nb][4 * h + 3] = v.w;
                    }
            }
            if (j == TPW - 1) {  // every load of this stage has been issued
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8u * uint32_t(st));
            }
            if (!have) continue;
            if constexpr (kPaired) {
                // k-steps 0 and 2, then 1 and 3, share their decode pairs
#pragma unroll
                for (int sp = 0; sp < 2; ++sp) {
                    uint32_t af_lo[4], af_hi[4];
                    if (sp == 0)
                        dequant_steps<kPB, 0>(reinterpret_cast<const uint32_t(&)[kPB]>(w), pk, s2, af_lo, af_hi);
                    else
                        dequant_steps<kPB, 1>(reinterpret_cast<const uint32_t(&)[kPB]>(w), pk, s2, af_lo, af_hi);
#pragma unroll
                    for (int nb = 0; nb < NT; ++nb) {
                        mma_16816(acc[nb], af_lo, xb[nb][sp * 2], xb[nb][sp * 2 + 1]);
                        mma_16816(acc[nb], af_hi, xb[nb][4 + sp * 2], xb[nb][4 + sp * 2 + 1]);
                    }
                }
            } else {
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    uint32_t af[4];
                    if constexpr (B == kFp16Bits) {
#pragma unroll
                        for (int rr = 0; rr < 4; ++rr) af[rr] = w[4 * s + rr];
                    } else {
                        // pair p = 4s + rr holds codes 2p, 2p+1; rr odd -> row r0+8
#define EBX_PAIR(RR)                                                                               \
        do {                                                                                           \
            constexpr int J = 2 * (4 * S_ + RR);                                                       \
            float lo, hi;                                                                              \
            if constexpr (HW) {                                                                        \
                lo = decode_code_int<B, J>(w, magic);                                                  \
                hi = decode_code_int<B, J + 1>(w, magic);                                              \
            } else {                                                                                   \
                lo = decode_code<B, J, DIRECT>(w, sc[RR & 1], magic);                                  \
                hi = decode_code<B, J + 1, DIRECT>(w, sc[RR & 1], magic);                              \
            }                                                                                          \
            af[RR] = pack_half2(lo, hi);                                                               \
        } while (0)
                        switch (s) {
#define EBX_STEP(SS)                    \
        case SS: {                          \
            constexpr int S_ = SS;          \
            EBX_PAIR(0);                    \
            EBX_PAIR(1);                    \
            EBX_PAIR(2);                    \
            EBX_PAIR(3);                    \
            break;                          \
        }
                            EBX_STEP(0) EBX_STEP(1) EBX_STEP(2) EBX_STEP(3)
#undef EBX_STEP
#undef EBX_PAIR
                        }
                    }
#pragma unroll
                    for (int nb = 0; nb < NT; ++nb)
                        mma_16816(acc[nb], af, xb[nb][(s >> 1) * 4 + (s & 1) * 2],
                                  xb[nb][(s >> 1) * 4 + (s & 1) * 2 + 1]);
                }
            }
          }
            rem -= S::kRound;
            so += SB;
            if (++st == D) {
                st = 0;
                so = 0;
                ph ^= 1u;
            }
        }
        consumers_sync(kConsumers);  // red[] lies over the ring: every consumer is done with it
#pragma unroll
        for (int nb = 0; nb < NT; ++nb)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                red[(((rgl * kWarps + wt) * NT + nb) * 32 + lane) * 4 + i] = acc[nb][i];
        if (!a.pdl_early) pdl_trigger();
      }
    }
    pdl_wait();  // outputs may alias the previous kernel's buffers
    __syncthreads();
    // epoch this call publishes: read after griddepcontrol.wait, so a previous exchange
    // call on the same stream has completed and advanced it
    const uint32_t xe = a.xa.world ? xchg_epoch(a.xa) + 1u : 0u;
    constexpr int kOut = RG * NT * 128;  // fragment elements of this CTA's sums
    // sum over the consumer warps of fragment element idx
    auto cta_sum = [&](int idx) {
        const int rgl = idx / (NT * 128);
        const int rem = idx % (NT * 128);
        float v = 0.0f;
#pragma unroll
        for (int ww = 0; ww < kWarps; ++ww) v += red[(rgl * kWarps + ww) * NT * 128 + rem];
        return v;
    };
    for (int idx = threadIdx.x; idx < kOut; idx += blockDim.x) {
        const int rgl = idx / (NT * 128);
        const int rem = idx % (NT * 128);
        const int nb = rem >> 7, l = (rem >> 2) & 31, i = rem & 3;
        const int g = cta * RG + rgl;
        float v = cta_sum(idx);
        const int row = g * kRowGroup + (l >> 2) + 8 * (i >> 1);
        const int tok = 8 * nb + (l & 3) * 2 + (i & 1);
        if (a.act) {
            if ((i >> 1) == 0 && g < a.groups) store_swiglu<B, HW>(a, g, l, tok, v, cta_sum(idx + 2));
            continue;
        }
        if (g < a.groups && row < a.N && tok < a.M) {
            if constexpr (HW && B != kFp16Bits) v = v * a.scales[row];
            if (a.xa.two_phase) {
                xchg_push_owner(a.xa, xe, xchg_owner(a.xa, g, a.groups), a.N, tok, row, v);
            } else if (a.xa.world) {
                xchg_push(a.xa, xe, a.M, a.N, tok, row, v);
            } else {
                if (a.bias) v += __half2float(__ushort_as_half(a.bias[row]));
                a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(v));
                if (a.y32) a.y32[size_t(tok) * a.N + row] = v;
            }
        }
    }
    if (a.xa.world && a.xa.fused) {
        // every CTA of the grid is resident (cooperative launch) and has pushed
        // before it waits, so each rank's CTAs eventually deliver
        for (int idx = threadIdx.x; idx < RG * NT * 128; idx += blockDim.x) {
            const int rgl = idx / (NT * 128);
            const int rem = idx % (NT * 128);
            const int nb = rem >> 7, l = (rem >> 2) & 31, i = rem & 3;
            const int g = cta * RG + rgl;
            const int row = g * kRowGroup + (l >> 2) + 8 * (i >> 1);
            const int tok = 8 * nb + (l & 3) * 2 + (i & 1);
            if (g < a.groups && row < a.N && tok < a.M)
                xchg_finish_one(a, xe, tok, row, a.xa.two_phase ? xchg_owner(a.xa, g, a.groups) : -1);
        }
        xchg_advance(a.xa, xe);
    }
}

template <int B, bool HW, int NT, bool DIRECT, int RG, int MINB, int TPW>
__global__ void __launch_bounds__(kThreads * RG + 32, MINB) decode_pipe_kernel(DecodeArgs a) {
    decode_pipe_body<B, HW, NT, DIRECT, RG, TPW>(a, int(blockIdx.x));
}

constexpr int kStages = 4;

// Dynamic shared memory of one pipe-kernel CTA when MINB of them share an SM: the SM's
// 228 KB less 1 KB reserved per CTA, split evenly (227 KB for one CTA).
constexpr int pipe_smem_budget(int minb) {
    return minb >= 4 ? 56 * 1024 : minb == 3 ? 75 * 1024 : minb == 2 ? 113 * 1024 : 227 * 1024;
}

// Multiprocessors of the current device (cached per device).
int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    int n = cache[dev & 63].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
        cache[dev & 63].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Exchange launches: fused (reduce inside the decode kernel) only when the whole
// grid fits on the GPU at once; the launch is then cooperative, which makes the
// runtime guarantee that co-residency, so CTAs that wait for peers' partials can
// never hold back CTAs of their own grid that those peers wait for in turn.
template <typename Kern>
cudaError_t launch_maybe_xchg(Kern kern, DecodeArgs& a, unsigned grid, unsigned threads, int smem,
                              cudaStream_t s, bool pdl = false, bool two_phase_ok = false) {
    if (!a.xa.world) {
        // pdl: the kernel waits (griddepcontrol.wait) before it reads anything the
        // previous kernel may write, so it may be launched before that one completes
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = size_t(smem);
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        // measured: overlapping helps when a CTA's run is short (K <= 8192) and costs
        // 5-8 % when it is long (K = 14336: next grid's CTAs land unevenly)
        cfg.numAttrs = pdl && a.kt <= 128 ? 1 : 0;
        a.pdl_early = 0;
        return cudaLaunchKernelEx(&cfg, kern, a);
    }
    int dev = 0, sms = 0, per_sm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, int(threads), size_t(smem));
    if (e != cudaSuccess) return e;
    a.xa.fused = int64_t(grid) <= int64_t(per_sm) * sms ? 1 : 0;
    // owner reduce + owner broadcast (fused launches of the pipe kernel only)
    a.xa.two_phase = a.xa.fused && two_phase_ok && xchg_two_phase(a.xa, a.M) ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = s;
    // pdl (pipe kernel): the next kernel's weight prefetch may overlap this one's
    // exchange, and this one's the previous kernel's tail (it reads the exchange epoch,
    // the activations and its outputs' memory only after griddepcontrol.wait)
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.xa.fused ? (pdl ? 2 : 1) : 0;
    a.pdl_early = 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int B, bool HW, int NT, bool VECX>
cudaError_t launch_one(DecodeArgs& a, int groups, cudaStream_t s) {
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
    return launch_maybe_xchg(kern, a, unsigned(groups), kThreads, smem, s);
}

template <int B, bool HW, int NT, bool DIRECT, int RG, int TPW, int MINB = (RG == 1 ? 3 : 1)>
cudaError_t launch_pipe(DecodeArgs& a, int groups, cudaStream_t s, int max_stages = kMaxStages) {
    using S = PipeStage<B, NT, RG, TPW>;
    // MINB CTAs per SM share its shared memory (three: 27 warps; two: 18; RG == 2:
    // one CTA of 17 warps).  The ring is as deep as that budget allows for this M
    // (2..kMaxStages stages).
    constexpr int kBudget = pipe_smem_budget(MINB);
    constexpr int kFixed = 2 * kMaxStages * 8 + 16;  // barriers; red[] reuses the ring
    const int mrows = a.M < NT * 8 ? a.M : NT * 8;
    a.stage_bytes = S::bytes(mrows);
    int D = (kBudget - kFixed) / a.stage_bytes;
    D = D > max_stages ? max_stages : D;
    if (D < 2 || D * a.stage_bytes < S::kRedBytes)  // dispatch keeps every case >= 2 stages
        return cudaErrorInvalidConfiguration;
    a.stages = D;
    const int smem = D * a.stage_bytes + kFixed;
    auto kern = decode_pipe_kernel<B, HW, NT, DIRECT, RG, MINB, TPW>;
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBudget);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    return launch_maybe_xchg(kern, a, unsigned((groups + RG - 1) / RG), kThreads * RG + 32, smem, s,
                             true, true);
}

// ---------------------------------------------------------------------------
// Several matrices over the same activations in one launch
// ---------------------------------------------------------------------------
// The grid is the concatenation of every matrix's row-group CTAs; a CTA finds its
// matrix from the prefix of CTA counts and runs that matrix's pipe decode (its own
// width, scales, semantics, ring depth and outputs).  Widths 8..12 (the plane
// decode, and b = 8's byte codes) are compiled in; anything else takes separate
// launches.
constexpr int kMaxMulti = 8;

struct MultiArgs {
    DecodeArgs m[kMaxMulti];
    int first_cta[kMaxMulti + 1];
    int count;
};

template <int NT, int TPW>
__device__ __forceinline__ void multi_body(const DecodeArgs& a, int cta) {
    switch (a.code) {
#define EBX_MULTI_CASE(BB)                                                     \
    case 2 * BB:                                                               \
        decode_pipe_body<BB, false, NT, false, 1, TPW>(a, cta);                \
        break;                                                                 \
    case 2 * BB + 1:                                                           \
        decode_pipe_body<BB, true, NT, false, 1, TPW>(a, cta);                 \
        break;
        EBX_MULTI_CASE(8) EBX_MULTI_CASE(9) EBX_MULTI_CASE(10) EBX_MULTI_CASE(11) EBX_MULTI_CASE(12)
#undef EBX_MULTI_CASE
        default:
            break;
    }
}

template <int NT, int TPW, int MINB>
__global__ void __launch_bounds__(kThreads + 32, MINB) decode_multi_kernel(const __grid_constant__ MultiArgs ma) {
    int j = 0;
    while (j + 1 < ma.count && int(blockIdx.x) >= ma.first_cta[j + 1]) ++j;
    multi_body<NT, TPW>(ma.m[j], int(blockIdx.x) - ma.first_cta[j]);
}

template <int NT, int TPW, int MINB>
cudaError_t launch_multi(MultiArgs& ma, int total_ctas, int max_kt, cudaStream_t s) {
    constexpr int kBudget = pipe_smem_budget(MINB);
    constexpr int kFixed = 2 * kMaxStages * 8 + 16;  // barriers; red[] reuses the ring
    int smem = 0;
    for (int i = 0; i < ma.count; ++i) {
        DecodeArgs& a = ma.m[i];
        const int bits = a.code / 2;
        const int mrows = a.M < NT * 8 ? a.M : NT * 8;
        const int wbytes = kWarps * TPW * bits * 128;
        const int xstride = kWarps * TPW * kKTile * 2 + 16;
        a.stage_bytes = wbytes + (mrows + (mrows < NT * 8 ? 1 : 0)) * xstride;
        int D = (kBudget - kFixed) / a.stage_bytes;
        D = D > kMaxStages ? kMaxStages : D;
        if (D < 2 || D * a.stage_bytes < kWarps * NT * 128 * 4) return cudaErrorInvalidConfiguration;
        a.stages = D;
        const int need = D * a.stage_bytes + kFixed;
        smem = need > smem ? need : smem;
    }
    auto kern = decode_multi_kernel<NT, TPW, MINB>;
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBudget);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(total_ctas));
    cfg.blockDim = dim3(kThreads + 32);
    cfg.dynamicSmemBytes = size_t(smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = max_kt <= 128 ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, ma);
}

template <int B, bool HW>
cudaError_t dispatch_nt(DecodeArgs& a, int groups, bool pipe, bool direct, cudaStream_t s) {
    constexpr bool kPlane = plane_layout(B) || (B == 8 && HW);
    if constexpr (kPlane) {
        if (pipe) {
            // Launch shapes of the plane decode, measured on the BASELINE decode shapes
            // (b = 10, 11; GB/s of the sweep's graph replay):
            //  * grids that fit two CTAs per SM in one wave with K <= 8192 (4096 x 4096):
            //    two CTAs per SM, two supertiles per warp and round, up to M = 8;
            //  * 896-row-group grids (N = 14336): three CTAs per SM with two supertiles
            //    per warp and round at M = 1, four CTAs with one supertile for 1 < M <= 8
            //    (4.41 vs 4.26 TB/s at M = 2, 3.98 vs 3.60 at M = 8);
            //  * K = 14336 (few, long CTAs): three CTAs per SM at M <= 4, two at M <= 8;
            //  * 8 < M <= 16: integer codes, one row group per CTA and two CTAs per SM;
            //    fullPrecision, two row groups per CTA sharing each activation stage
            //    (halves the activation bytes staged per weight byte).
            // The consumers' sums go over the drained ring (no separate buffer) and the
            // zero activation row exists only when M < 8 NT, which buys a stage at M = 16.
            const bool two_per_sm = groups <= 2 * sm_count() && a.kt <= 128;
            if (a.M <= 8) {
                if (two_per_sm) return launch_pipe<B, HW, 1, false, 1, 2, 2>(a, groups, s);
                if (a.kt > 128)
                    return a.M <= 4 ? launch_pipe<B, HW, 1, false, 1, 2, 3>(a, groups, s)
                                    : launch_pipe<B, HW, 1, false, 1, 2, 2>(a, groups, s);
                // (a two-stage ring: three stages measured 13 % slower on 4096 x 14336)
                if (a.M == 1) return launch_pipe<B, HW, 1, false, 1, 2, 3>(a, groups, s, 2);
                // (the fullPrecision operands need more registers than four CTAs per SM leave)
                if (!HW)
                    return a.M <= 4 ? launch_pipe<B, HW, 1, false, 1, 2, 3>(a, groups, s)
                                    : launch_pipe<B, HW, 1, false, 1, 2, 2>(a, groups, s);
                return launch_pipe<B, HW, 1, false, 1, 1, 4>(a, groups, s);
            }
            // 8 < M <= 16, integer codes: one row group per CTA, two supertiles per warp and
            // round, two CTAs per SM (measured against two row groups sharing activation
            // stages: 6.8 -> 6.4, 24.4 -> 23.5, 23.2 -> 22.6 us on the three shapes)
            if (HW) return launch_pipe<B, HW, 2, false, 1, 2, 2>(a, groups, s);
            return launch_pipe<B, HW, 2, false, 2, 2, 1>(a, groups, s);
        }
    }
    if (pipe) {
        // M <= 4 and b <= 12: two supertiles per warp per round (a stage of 16 supertiles
        // and up to 5 activation rows still leaves >= 2 stages in the 74 KB budget);
        // M <= 8: one per warp; M <= 16: one row group per CTA with 16 activation rows
        // (two stages; measured faster than two row groups per CTA at one CTA per SM,
        // whose 448-CTA grid for N = 14336 runs in 3.03 waves).
        // (8..12-bit full semantics decode in pairs and ignore `direct`)
        constexpr bool kCanDirect = !HW && B != kFp16Bits && !(B >= 8 && B <= 12);
        // Two CTAs per SM (a deeper ring, up to 113 registers) pay off when the grid
        // is then still one wave and each CTA's run is short (measured on the
        // BASELINE shapes: 4096x4096 12 % faster; 14336-row and 14336-column
        // matrices slower), else three CTAs per SM.
        const bool two_per_sm = groups <= 2 * sm_count() && a.kt <= 128;
        if (B <= 12 && a.M <= 4) {
            if (two_per_sm)
                return launch_pipe<B, HW, 1, false, 1, 2, 2>(a, groups, s);
            if constexpr (kCanDirect)
                if (direct) return launch_pipe<B, HW, 1, true, 1, 2>(a, groups, s);
            return launch_pipe<B, HW, 1, false, 1, 2>(a, groups, s);
        }
        if (a.M <= 8) {
            // two CTAs per SM with two supertiles per warp and round (measured 13-22 %
            // faster than three CTAs with one supertile on the BASELINE decode shapes)
            if constexpr (B <= 12) return launch_pipe<B, HW, 1, false, 1, 2, 2>(a, groups, s);
            if constexpr (kCanDirect)
                if (direct) return launch_pipe<B, HW, 1, true, 1, 1>(a, groups, s);
            return launch_pipe<B, HW, 1, false, 1, 1>(a, groups, s);
        }
        if constexpr (B == kFp16Bits)  // 16-bit weights: two stages need the larger budget
            return launch_pipe<B, HW, 2, false, 2, 1>(a, groups, s);
        // 16 activation rows: two CTAs per SM (a three-stage ring) under the same
        // rule, else three CTAs per SM (two stages)
        if (two_per_sm)
            return launch_pipe<B, HW, 2, false, 1, 1, 2>(a, groups, s);
        if constexpr (kCanDirect)
            if (direct) return launch_pipe<B, HW, 2, true, 1, 1>(a, groups, s);
        return launch_pipe<B, HW, 2, false, 1, 1>(a, groups, s);
    }
    return a.M <= 8 ? launch_one<B, HW, 1, false>(a, groups, s) : launch_one<B, HW, 2, false>(a, groups, s);
}

}  // namespace

bool multi_supported(const Matrix& m) {
    return m.bits >= 8 && m.bits <= 12 && (m.cols % 64) == 0;
}

cudaError_t launch_decode_multi(const Matrix* const* ms, int count, const uint16_t* x, int64_t M,
                                const uint16_t* const* bias, uint16_t* const* y,
                                float* const* y32, cudaStream_t s) {
    if (count < 1 || count > kMaxMulti || M < 1 || M > 16) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return cudaErrorInvalidValue;
    MultiArgs ma = {};
    ma.count = count;
    int total = 0, max_kt = 0;
    for (int i = 0; i < count; ++i) {
        const Matrix& m = *ms[i];
        if (!multi_supported(m) || m.cols != ms[0]->cols) return cudaErrorInvalidValue;
        DecodeArgs& a = ma.m[i];
        a.tiles = m.tiles;
        a.scales = m.scales;
        a.x = x;
        a.bias = bias ? bias[i] : nullptr;
        a.y = y[i];
        a.y32 = y32 ? y32[i] : nullptr;
        a.M = int(M);
        a.N = m.rows;
        a.K = m.cols;
        a.kt = int(m.kt);
        a.groups = int(m.groups);
        a.magic = 0x4B000000u;
        a.magic_plane = 0x64646464u;
        a.code = 2 * m.bits + ((m.exec_width < 16 && m.bits <= 12) ? 1 : 0);
        ma.first_cta[i] = total;
        total += int(m.groups);
        max_kt = int(m.kt) > max_kt ? int(m.kt) : max_kt;
    }
    ma.first_cta[count] = total;
    return M <= 8 ? launch_multi<1, 2, 2>(ma, total, max_kt, s)
                  : launch_multi<2, 1, 2>(ma, total, max_kt, s);
}

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
                          uint16_t* y, float* y32, cudaStream_t s, XchgArgs* xa, int act) {
    if (M <= 0) return cudaSuccess;
    if (act && (xa || (m.rows % 16) != 0)) return cudaErrorInvalidValue;
    if (xa && M > 16) return cudaErrorInvalidValue;  // one launch = one exchange epoch
    const bool vecx = (m.cols % 64) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    // integer-code semantics: exec width 4 / 8 (b <= 8, the reference's W4A16 / W8A16) and
    // 12 (b <= 12: every |q| <= 2047 is an exact fp16 operand)
    const bool hw = m.exec_width < 16 && m.bits <= 12;
    for (int64_t m0 = 0; m0 < M; m0 += 16) {
        DecodeArgs a;
        a.tiles = m.tiles;
        a.scales = m.scales;
        a.x = x + m0 * m.cols;
        a.bias = bias;
        const int64_t ycols = act ? m.rows / 2 : m.rows;
        a.y = y ? y + m0 * ycols : nullptr;
        a.y32 = y32 ? y32 + m0 * ycols : nullptr;
        a.act = act;
        if (xa) a.xa = *xa;
        a.M = int(M - m0 < 16 ? M - m0 : 16);
        a.N = m.rows;
        a.K = m.cols;
        a.kt = int(m.kt);
        a.groups = int(m.groups);
        a.magic = 0x4B000000u;
        a.magic_plane = 0x64646464u;
        const int groups = int(m.groups);
        cudaError_t e = cudaErrorInvalidValue;
        const bool v = vecx && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
        a.pdl_early = 0;
        switch (m.bits) {
#define EBX_DEC_CASE(BB)                                                                \
    case BB:                                                                            \
        e = hw ? dispatch_nt<BB, true>(a, groups, v, m.direct_ok, s) : dispatch_nt<BB, false>(a, groups, v, m.direct_ok, s); \
        break;
            EBX_DEC_CASE(3) EBX_DEC_CASE(4) EBX_DEC_CASE(5) EBX_DEC_CASE(6) EBX_DEC_CASE(7)
            EBX_DEC_CASE(8) EBX_DEC_CASE(9) EBX_DEC_CASE(10) EBX_DEC_CASE(11) EBX_DEC_CASE(12)
#undef EBX_DEC_CASE
#define EBX_DEC_CASE_FULL(BB) \
    case BB:                  \
        e = dispatch_nt<BB, false>(a, groups, v, m.direct_ok, s); \
        break;
            EBX_DEC_CASE_FULL(13) EBX_DEC_CASE_FULL(14)
            EBX_DEC_CASE_FULL(15) EBX_DEC_CASE_FULL(16)
#undef EBX_DEC_CASE_FULL
            default:
                break;
        }
        if (e != cudaSuccess) return e;
        if (xa) xa->fused = a.xa.fused;
    }
    return cudaSuccess;
}

}  // namespace ebx
