// ebx_gemm.cu -- prefill (M > 64) ElasticBit linear on B200 tensor cores.
//
// Replaces the reference's prefill route, materialise + cuBLAS F.linear
// (core.py:465-471, elasticbit_runtime.cu:982-1022): the exactly dequantised
// FP16 weight W16[n,k] = fp16(q * s) (the same bits the reference's
// RuntimeMatrix holds for its W16 path) is written to the caller's workspace by
// ebx_pack.cu's materialize kernel, then this kernel computes
//     y[m, n] = fp16( sum_k x[m,k] * W16[n,k] + bias[n] )
// with 5th-generation tensor cores, as a persistent kernel (one CTA per SM):
//   * output tiles 128 (tokens, MMA M) x 256 (weight rows, MMA N), K step 64,
//     visited in groups of kGroupM token tiles per weight tile so that the
//     tiles in flight on the whole GPU share an L2-resident slice of x and W16;
//   * warp 0: TMA producer (cp.async.bulk.tensor, 128-byte swizzle, no
//     multicast) into a 4-stage shared-memory ring, running ahead across tiles;
//   * warp 1: one thread issues tcgen05.mma (kind::f16, fp32 accumulate) into
//     one of two 128 x 256 fp32 accumulators in tensor memory (512 columns)
//     and tcgen05.commit frees each ring stage, then marks the accumulator full;
//   * warps 2-5: epilogue -- tcgen05.ld of TMEM lanes 32(w%4)..+31 (tokens),
//     bias in fp32, fp16 (+fp32) stores, then the accumulator is released --
//     while the MMAs of the next tile run into the other accumulator.
// Every mbarrier wait is bounded in time; a timeout sets the device status word
// and the roles leave their loops.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kABytes = BM * BK * 2;
constexpr int kGemmThreads = 192;        // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kGroupM = 8;               // token tiles per raster group

// Per weight-tile width BN (256, 128 or 64 rows): the ring, the TMEM
// accumulators (two of BN fp32 columns) and the MMA instruction descriptor
// (D fp32, A/B fp16, both K-major, M = 128, N = BN).
template <int BN>
struct GemmCfg {
    static constexpr int kBBytes = BN * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = 4 * (kABytes + 256 * BK * 2) / kStageBytes < 8
                                       ? 4 * (kABytes + 256 * BK * 2) / kStageBytes
                                       : 8;  // same ring bytes as BN = 256, at most 8 stages
    static constexpr int kAccCols = BN;
    static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr uint32_t kIdesc =
        (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
    static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

__device__ int g_gemm_status = 0;

struct GemmArgs {
    const uint16_t* bias;
    uint16_t* y;
    float* y32;
    int M, N, K;
    int full_tiles;  // output tiles computed whole (the first full waves)
    int tail_split;  // K splits of each remaining tile (1: none)
    float* part;     // tail_split > 1: fp32 partial tiles [tail_split][tail tiles][BM][BN]
};

// Work unit u: tiles [0, full_tiles) whole, one unit each; every tile after them
// (the last, partial wave) as tail_split units over consecutive k-block ranges, so the
// last wave takes 1 / tail_split of a tile's time.  tail = tile index among the split
// tiles, s = its split (-1: a whole tile).
__device__ __forceinline__ void gemm_unit(const GemmArgs& a, int u, int tiles, int kblocks, int& t,
                                          int& s, int& kb0, int& kb1) {
    if (u < a.full_tiles) {
        t = u;
        s = -1;
        kb0 = 0;
        kb1 = kblocks;
        return;
    }
    const int v = u - a.full_tiles, tail_tiles = tiles - a.full_tiles;
    t = a.full_tiles + v % tail_tiles;
    s = v / tail_tiles;
    kb0 = kblocks * s / a.tail_split;
    kb1 = kblocks * (s + 1) / a.tail_split;
}

// Shared-memory matrix descriptor: K-major tile with 128-byte swizzle, rows of
// 128 bytes, 8-row core groups 1024 bytes apart (SBO), sm_100 version field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);
    d |= uint64_t(1) << 16;            // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;    // stride byte offset
    d |= uint64_t(1) << 46;            // descriptor version
    d |= uint64_t(2) << 61;            // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ bool gemm_wait(uint32_t bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_gemm_status, 0x7103);
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// 4-d tensor load (the code tiles of several row groups at one k-block; see make_code_map).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            int c3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
}

// Output tile t -> (token tile, weight tile): groups of kGroupM token tiles walk
// the weight tiles together, so concurrently resident CTAs share operands in L2.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
    const int per_group = kGroupM * n_tiles;
    const int grp = t / per_group;
    const int first = grp * kGroupM;
    const int gm = m_tiles - first < kGroupM ? m_tiles - first : kGroupM;
    const int idx = t - grp * per_group;
    mt = first + idx % gm;
    nt = idx / gm;
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                    GemmArgs a) {
    using G = GemmCfg<BN>;
    constexpr int kStagesG = G::kStages;
    constexpr int kStageBytesG = G::kStageBytes;
    constexpr int kAccCols = G::kAccCols;
    constexpr int kTmemCols = G::kTmemCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStagesG * kStageBytesG);
    uint64_t* empty = full + kStagesG;
    uint64_t* acc_full = empty + kStagesG;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int kblocks = (a.K + BK - 1) / BK;
    const int m_tiles = (a.M + BM - 1) / BM;
    const int n_tiles = (a.N + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int units = a.full_tiles + (tiles - a.full_tiles) * a.tail_split;

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < kStagesG; ++i) {
                mbar_init(smem_u32(&full[i]), 1);
                mbar_init(smem_u32(&empty[i]), 1);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(smem_u32(&acc_full[i]), 1);
                mbar_init(smem_u32(&acc_empty[i]), 4);  // one arrival per epilogue warp
            }
            fence_proxy_async_smem();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: runs ahead across tiles
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                int t, sp, kb0, kb1, mt, nt;
                gemm_unit(a, u, tiles, kblocks, t, sp, kb0, kb1);
                tile_coords(t, m_tiles, n_tiles, mt, nt);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int st = it % kStagesG;
                    if (it >= kStagesG &&
                        !gemm_wait(smem_u32(&empty[st]), uint32_t(((it / kStagesG) - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    const uint32_t bar = smem_u32(&full[st]);
                    mbar_expect_tx(bar, kStageBytesG);
                    uint8_t* stage = smem + st * kStageBytesG;
                    tma_load_2d(smem_u32(stage), &tma_x, kb * BK, mt * BM, bar);
                    tma_load_2d(smem_u32(stage + kABytes), &tma_w, kb * BK, nt * BN, bar);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            int it = 0, i = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
                int t, sp, kb0, kb1;
                gemm_unit(a, u, tiles, kblocks, t, sp, kb0, kb1);
                const int acc = i & 1;
                if (i >= 2 && !gemm_wait(smem_u32(&acc_empty[acc]), uint32_t(((i >> 1) - 1) & 1))) break;
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t d = tmem + uint32_t(acc * kAccCols);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int st = it % kStagesG;
                    if (!gemm_wait(smem_u32(&full[st]), uint32_t((it / kStagesG) & 1))) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                    const uint32_t abase = smem_u32(smem + st * kStageBytesG);
                    const uint32_t bbase = abase + kABytes;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_f16(d, sw128_desc(abase + k * 32), sw128_desc(bbase + k * 32), G::kIdesc,
                                 (kb != kb0 || k != 0) ? 1u : 0u);
                    umma_commit(smem_u32(&empty[st]));
                }
                umma_commit(smem_u32(&acc_full[acc]));  // fires when this tile's MMAs are done
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: TMEM -> registers -> global ----------------
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const bool vec = (a.N % 8) == 0;
        int i = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
            const int acc = i & 1;
            if (!gemm_wait(smem_u32(&acc_full[acc]), uint32_t((i >> 1) & 1))) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            int t, sp, kb0, kb1, mt, nt;
            gemm_unit(a, u, tiles, kblocks, t, sp, kb0, kb1);
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            const int m = mt * BM + quarter * 32 + lane;
            const int n0 = nt * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                const uint32_t taddr =
                    tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * kAccCols + c * 32);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                      "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
                      "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]),
                      "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                      "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
                      "=r"(v[30]), "=r"(v[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
                const int nb = n0 + c * 32;
                if (m >= a.M || nb >= a.N) continue;
                if (sp >= 0) {  // fp32 partial tile of split sp; gemm_tail_reduce adds splits and bias
                    float* prow = a.part +
                                  (size_t(sp) * (tiles - a.full_tiles) + (t - a.full_tiles)) * (BM * BN) +
                                  size_t(quarter * 32 + lane) * BN + c * 32;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        reinterpret_cast<float4*>(prow)[q] =
                            make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                        __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
                    continue;
                }
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    f[j] = __uint_as_float(v[j]);
                    if (a.bias && nb + j < a.N) f[j] += __half2float(__ushort_as_half(a.bias[nb + j]));
                }
                uint16_t* yrow = a.y + size_t(m) * a.N + nb;
                if (vec && nb + 32 <= a.N) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 pk;
                        pk.x = pack_half2(f[8 * q + 0], f[8 * q + 1]);
                        pk.y = pack_half2(f[8 * q + 2], f[8 * q + 3]);
                        pk.z = pack_half2(f[8 * q + 4], f[8 * q + 5]);
                        pk.w = pack_half2(f[8 * q + 6], f[8 * q + 7]);
                        reinterpret_cast<uint4*>(yrow)[q] = pk;
                    }
                    if (a.y32) {
                        float* y32row = a.y32 + size_t(m) * a.N + nb;
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            reinterpret_cast<float4*>(y32row)[q] =
                                make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (nb + j < a.N) {
                            yrow[j] = __half_as_ushort(__float2half_rn(f[j]));
                            if (a.y32) a.y32[size_t(m) * a.N + nb + j] = f[j];
                        }
                    }
                }
            }
            // this accumulator may be overwritten by the MMAs of tile i + 2
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// The tile layout of a matrix's codes as a 4-d uint8 tensor [groups][kt][b rows][128 B]
// (dims innermost first: 128 bytes, b, kt, groups), with a box of `box_groups` row groups
// at one k-tile: ONE TMA request brings the supertiles of that many row groups for one
// k-block, landing contiguously (group after group) -- instead of one bulk copy per
// row group.  Row groups past the matrix read as zeros (the box is always full).
bool make_code_map(CUtensorMap* map, const Matrix& m, int box_groups) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t tb = cuuint64_t(tile_bytes(m.bits));
    const cuuint64_t dims[4] = {128, cuuint64_t(m.bits), cuuint64_t(m.kt), cuuint64_t(m.groups)};
    const cuuint64_t strides[3] = {128, tb, tb * cuuint64_t(m.kt)};
    const cuuint32_t box[4] = {128, cuuint32_t(m.bits), 1, cuuint32_t(box_groups)};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(m.tiles), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major fp16 [rows, K] tensor map with a (64 x box_rows) box, 128 B swizzle.
bool make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
    const cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


// ---------------------------------------------------------------------------
// Decode-GEMM for 16 < M <= 256 activation rows
// ---------------------------------------------------------------------------
// The weights are the 128-row side of tcgen05.mma (A operand) and the tokens
// the N side (B operand, N = M rounded up to 16): a CTA owns 128 weight rows (8
// row groups) and a contiguous range of k-blocks; the weights stream from HBM
// once, as exact-width codes.  Per 64-k block:
//   * warp 0 (one thread): one bulk copy per row group's supertile (b x 128
//     bytes) and one TMA load of the activations' 64-k slice (M rows, 128-byte
//     swizzle, rows past M filled with zeros) into a D-stage ring;
//   * warps 2-9: decode one supertile each to exact fp16 (the decode kernel's
//     arithmetic) and store it, K-major with the 128-byte swizzle
//     (16-byte chunk j of row n at n*128 + (j ^ (n & 7))*16), as the A tile;
//     fence.proxy.async makes the stores visible to the tensor core;
//   * warp 1 (one thread): four tcgen05.mma (K = 16) into a 128 x N fp32
//     accumulator in TMEM, then tcgen05.commit frees the stage.
// After the last k-block warps 2-9 read TMEM lanes 32(w % 4).. (one weight row
// per thread; two warps per lane quarter take alternate 16-token chunks) and write either y = fp16(acc (* s for integer codes) + bias)
// directly, or, when K is split over S CTAs to fill the GPU, an fp32 partial
// that dgemm_reduce_kernel adds in split order (deterministic).
constexpr int kDgRows = 128;
constexpr int kDgGroups = kDgRows / kRowGroup;  // 8 row groups per CTA
constexpr int kDgDecoders = 8;                   // one decoding warp per row group
constexpr int kDgThreads = 64 + 32 * kDgDecoders;  // producer, MMA issuer, decoders
constexpr int kDgABytes = kDgRows * BK * 2;     // 16 KB decoded weight tile
constexpr int kDgMaxTokens = 256;

__device__ int g_dgemm_status = 0;

struct DgArgs {
    const uint8_t* tiles;
    const float* scales;
    const uint16_t* bias;
    uint16_t* y;
    float* y32;
    float* part;  // [S][M][N] fp32 partials when S > 1
    int M, N, kt, groups;
    int S, kb_per;     // K splits and k-blocks per split
    int stages, stage_bytes, mp, tmem_cols;
    int b_off, c_off;  // byte offsets of the activation and code tiles in a stage
};

__device__ __forceinline__ bool dg_wait(uint32_t bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_dgemm_status, 0x7104);
    return false;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// A-fragment registers of one lane's 32 codes (register 4s + rr: codes 2(4s+rr),
// +1; rr odd -> row r0 + 8) -> exact fp16 pairs.
// Paired-decode constants of a b = 8..12 code (a placeholder width otherwise).
template <int B>
using DgConsts = PairConsts<8>;

template <int B, bool HW>
__device__ __forceinline__ void dg_decode(const uint32_t (&w)[B], const uint64_t (&s2)[2],
                                          const DgConsts<B>& pk, uint32_t (&af)[16]) {
    if constexpr (B == kFp16Bits) {
#pragma unroll
        for (int p = 0; p < 16; ++p) af[p] = w[p];
    } else if constexpr (plane_layout(B) || (B == 8 && HW)) {
        // plane layout (and b = 8's byte codes): exact q pairs by byte permutes;
        // fullPrecision then rounds fp32_rn(q * s) once to fp16
        PlaneConsts k;
        k.init(0x64646464u);
        plane_q16_all<B>(w, k, af);
        if constexpr (!HW) {
#pragma unroll
            for (int p = 0; p < 16; ++p) af[p] = q16_to_w16(af[p], s2[p & 1]);
        }
    } else if constexpr (HW) {
        const float nb = -(8388608.0f + float(qmax_for(B)));
        const uint64_t nb2 = pack2f(nb, nb);
#pragma unroll
        for (int p = 0; p < 16; ++p) af[p] = codes2_to_half(code_magic<B>(w, 2 * p), code_magic<B>(w, 2 * p + 1), nb2);
    } else if constexpr (B == 8) {
        uint32_t lo[4], hi[4];
        dequant_steps<B, 0>(w, pk, s2, lo, hi);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            af[r] = lo[r];
            af[8 + r] = hi[r];
        }
        dequant_steps<B, 1>(w, pk, s2, lo, hi);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            af[4 + r] = lo[r];
            af[12 + r] = hi[r];
        }
    } else {
        const float nb = -(8388608.0f + float(qmax_for(B)));
        const uint64_t nb2 = pack2f(nb, nb);
#pragma unroll
        for (int p = 0; p < 16; ++p)
            af[p] = dequant2(code_magic<B>(w, 2 * p), code_magic<B>(w, 2 * p + 1), nb2, s2[p & 1]);
    }
}

template <int B, bool HW>
__global__ void __launch_bounds__(kDgThreads, 2)
    dgemm_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_c,
                 DgArgs a) {
    constexpr int kCodeBytes = B * 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const int D = a.stages;
    const int SB = a.stage_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + D * SB);
    uint64_t* ready = full + D;
    uint64_t* empty = ready + D;
    uint64_t* acc_full = empty + D;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rb = blockIdx.x / a.S;
    const int split = blockIdx.x % a.S;
    const int kb0 = split * a.kb_per;
    const int kb1 = min(a.kt, kb0 + a.kb_per);
    const int nkb = kb1 - kb0;
    const int g0 = rb * kDgGroups;
    const int ngroups = min(kDgGroups, a.groups - g0);

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < D; ++i) {
                mbar_init(smem_u32(&full[i]), 1);
                mbar_init(smem_u32(&ready[i]), kDgDecoders);  // one arrival per decoding warp
                mbar_init(smem_u32(&empty[i]), 1);
            }
            mbar_init(smem_u32(acc_full), 1);
            fence_proxy_async_smem();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // producer: lane 0 arms the stage and loads the activations, lanes r < ngroups
        // copy row group r's supertile (the copies are issued in parallel)
        for (int i = 0; i < nkb; ++i) {
            const int st = i % D;
            bool ok = true;
            if (lane == 0 && i >= D) ok = dg_wait(smem_u32(&empty[st]), uint32_t(((i / D) - 1) & 1));
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
            const int kb = kb0 + i;
            const uint32_t bar = smem_u32(&full[st]);
            uint8_t* stage = smem + st * SB;
            if (lane == 0) {
                // one request for all 8 row groups' supertiles (full box: groups past
                // the matrix read as zeros)
                mbar_expect_tx(bar, uint32_t(kDgGroups * kCodeBytes + a.mp * BK * 2));
                tma_load_2d(smem_u32(stage + a.b_off), &tma_x, kb * BK, 0, bar);
                tma_load_4d(smem_u32(stage + a.c_off), &tma_c, 0, 0, kb, g0, bar);
            }
            __syncwarp();
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = (1u << 4) | (uint32_t(a.mp >> 3) << 17) | (uint32_t(kDgRows >> 4) << 24);
            bool ok = true;
            for (int i = 0; i < nkb && ok; ++i) {
                const int st = i % D;
                const uint32_t ph = uint32_t(i / D) & 1u;
                if (!dg_wait(smem_u32(&full[st]), ph) || !dg_wait(smem_u32(&ready[st]), ph)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t abase = smem_u32(smem + st * SB);
                const uint32_t bbase = abase + uint32_t(a.b_off);
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    umma_f16(tmem, sw128_desc(abase + k * 32), sw128_desc(bbase + k * 32), idesc,
                             (i | k) != 0 ? 1u : 0u);
                umma_commit(smem_u32(&empty[st]));
            }
            umma_commit(smem_u32(acc_full));  // fires when every MMA above has completed
        }
        __syncwarp();
    } else {
        // ---------------- decode (warps 2-9), then the epilogue ----------------
        const int r = warp - 2;  // this warp's row group within the CTA
        const int r0 = lane >> 2;
        const int c = lane & 3;
        uint64_t s2[2] = {0, 0};
        if constexpr (B != kFp16Bits && !HW) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = (g0 + r) * kRowGroup + r0 + 8 * h;
                const float sv = (r < ngroups && row < a.N) ? a.scales[row] : 0.0f;
                s2[h] = pack2f(sv, sv);
            }
        }
        DgConsts<B> pk;  // built once: they depend on the width only
        pk.init(0x4B000000u);
        // byte offsets in the A tile of this lane's four 16-byte chunks: rows 16r + r0 (+8),
        // k = 16c..16c+15 = chunks 2c, 2c+1, 128-byte swizzle
        const int nlo = 16 * r + r0, nhi = nlo + 8;
        const uint32_t o_lo0 = uint32_t(nlo * 128 + (((2 * c) ^ (nlo & 7)) << 4));
        const uint32_t o_lo1 = uint32_t(nlo * 128 + (((2 * c + 1) ^ (nlo & 7)) << 4));
        const uint32_t o_hi0 = uint32_t(nhi * 128 + (((2 * c) ^ (nhi & 7)) << 4));
        const uint32_t o_hi1 = uint32_t(nhi * 128 + (((2 * c + 1) ^ (nhi & 7)) << 4));
        for (int i = 0; i < nkb; ++i) {
            const int st = i % D;
            if (!dg_wait(smem_u32(&full[st]), uint32_t(i / D) & 1u)) break;
            const uint8_t* stage = smem + st * SB;
            if (r < ngroups) {  // rows past N: never read back
                const uint8_t* cb = stage + a.c_off + r * kCodeBytes;
                uint32_t w[B];
#pragma unroll
                for (int q = 0; q < B / 4; ++q) {
                    const uint4 v = *reinterpret_cast<const uint4*>(cb + q * 512 + lane * 16);
                    w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
                }
                if constexpr ((B & 2) != 0) {
                    const uint2 v = *reinterpret_cast<const uint2*>(cb + (B / 4) * 512 + lane * 8);
                    w[4 * (B / 4)] = v.x;
                    w[4 * (B / 4) + 1] = v.y;
                }
                if constexpr ((B & 1) != 0)
                    w[B - 1] = *reinterpret_cast<const uint32_t*>(cb + (B / 4) * 512 + ((B & 2) ? 256 : 0) +
                                                                  lane * 4);
                uint32_t af[16];
                dg_decode<B, HW>(w, s2, pk, af);
                const uint32_t abase = smem_u32(stage);
                sts128(abase + o_lo0, af[0], af[2], af[4], af[6]);
                sts128(abase + o_lo1, af[8], af[10], af[12], af[14]);
                sts128(abase + o_hi0, af[1], af[3], af[5], af[7]);
                sts128(abase + o_hi1, af[9], af[11], af[13], af[15]);
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ready[st]));
        }
        // the split-K reduction (or the next layer) may be scheduled now; it waits for
        // this grid to complete before it reads anything this grid writes
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        // epilogue: TMEM lane = weight row, column = token
        if (dg_wait(smem_u32(acc_full), 0u)) {
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const int quarter = warp & 3;
            const int row = rb * kDgRows + quarter * 32 + lane;
            float sc = 1.0f, bv = 0.0f;
            if (row < a.N) {
                if constexpr (HW && B != kFp16Bits) sc = a.scales[row];
                if (a.bias && a.S == 1) bv = __half2float(__ushort_as_half(a.bias[row]));
            }
            const int half = (warp - 2) >> 2;  // two warps per lane quarter: alternate chunks
#pragma unroll 1
            for (int t0 = 16 * half; t0 < a.mp; t0 += 32) {
                uint32_t v[16];
                const uint32_t taddr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(t0);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                      "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
                      "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
                if (row >= a.N) continue;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int tok = t0 + j;
                    if (tok >= a.M) break;
                    float f = __uint_as_float(v[j]);
                    if (a.S == 1) {
                        f = f * sc + bv;
                        a.y[size_t(tok) * a.N + row] = __half_as_ushort(__float2half_rn(f));
                        if (a.y32) a.y32[size_t(tok) * a.N + row] = f;
                    } else {
                        a.part[(size_t(split) * a.M + tok) * a.N + row] = f;
                    }
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(a.tmem_cols)
                     : "memory");
    }
}

// y = fp16(sum over splits in order (* s for integer codes) + bias); four outputs per
// thread (N % 4 == 0) or one.
template <bool HW>
__global__ void dgemm_reduce_kernel(const float* part, int S, int M, int N, const float* scales,
                                    const uint16_t* bias, uint16_t* y, float* y32) {
    // launched with programmatic dependent launch: the partials are read only once the
    // decode-GEMM grid has completed (a no-op wait when launched without it)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const size_t total = size_t(M) * size_t(N);
    const bool vec = (N & 3) == 0;
    const size_t i0 = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) * (vec ? 4 : 1);
    if (i0 >= total) return;
    const int row0 = int(i0 % uint32_t(N));
    if (vec) {
        float4 v = *reinterpret_cast<const float4*>(part + i0);
        for (int s = 1; s < S; ++s) {
            const float4 u = *reinterpret_cast<const float4*>(part + size_t(s) * total + i0);
            v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
        }
        float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if constexpr (HW) f[j] *= scales[row0 + j];
            if (bias) f[j] += __half2float(__ushort_as_half(bias[row0 + j]));
        }
        uint2 h;
        h.x = pack_half2(f[0], f[1]);
        h.y = pack_half2(f[2], f[3]);
        *reinterpret_cast<uint2*>(y + i0) = h;
        if (y32) *reinterpret_cast<float4*>(y32 + i0) = make_float4(f[0], f[1], f[2], f[3]);
        return;
    }
    float v = part[i0];
    for (int s = 1; s < S; ++s) v += part[size_t(s) * total + i0];
    if constexpr (HW) v *= scales[row0];
    if (bias) v += __half2float(__ushort_as_half(bias[row0]));
    y[i0] = __half_as_ushort(__float2half_rn(v));
    if (y32) y32[i0] = v;
}

// ---------------------------------------------------------------------------
// Prefill decode-GEMM (larger M): the codes decoded straight into the B tile
// ---------------------------------------------------------------------------
// The persistent structure of gemm_f16_kernel (output tiles of 128 tokens x 256
// weight rows, two TMEM accumulators so the epilogue of one tile runs under the
// MMAs of the next), but the weight operand never exists in HBM as FP16: per
// 64-k block the producer copies the 16 row groups' exact-width supertiles
// (b x 128 bytes each, one 4-d TMA request) next to the TMA-loaded x tile (a
// D-stage load ring); sixteen decoding warps, one row group each, turn them into
// the K-major, 128-byte-swizzled fp16 B tile in one of two B buffers, one
// k-block ahead of the MMAs (the decode kernel's
// arithmetic: integer codes under integer-code semantics -- the row scale is
// applied in the epilogue -- or fp16_rn(fp32_rn(q * s)) under fullPrecision)
// and the MMA thread consumes it.  No workspace, one HBM pass over the codes per
// concurrently resident token-tile row; the x and code tiles of a raster group
// of token tiles stay L2-resident.
constexpr int kPgBN = 256;                                 // weight rows per tile (MMA N)
constexpr int kPgGroups = kPgBN / kRowGroup;               // 16 row groups
constexpr int kPgDecoders = 16;                            // one row group each
constexpr int kPgThreads = 32 * (2 + 4 + kPgDecoders);     // producer, MMA, epilogue x4, decoders
constexpr int kPgBBytes = kPgBN * BK * 2;                  // 32 KB decoded tile
constexpr uint32_t kPgIdesc = (1u << 4) | (uint32_t(kPgBN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

struct PgArgs {
    const uint8_t* tiles;
    const float* scales;
    const uint16_t* bias;
    uint16_t* y;
    float* y32;
    int M, N, kt, groups;
    int stages, stage_bytes;  // load-ring stage: [x tile | codes]; two B tiles follow the ring
};

__device__ __forceinline__ bool pg_wait(uint32_t bar, uint32_t parity) {
    if (mbar_wait_bounded(bar, parity)) return true;
    atomicExch(&g_gemm_status, 0x7105);
    return false;
}

template <int B, bool HW>
__global__ void __launch_bounds__(kPgThreads, 1)
    pgemm_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_c,
                 PgArgs a) {
    constexpr int kCodeBytes = B * 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const int D = a.stages;
    const int SB = a.stage_bytes;
    uint8_t* btile = smem + D * SB;  // two decoded B tiles, 1024-aligned
    uint64_t* full = reinterpret_cast<uint64_t*>(btile + 2 * kPgBBytes);
    uint64_t* empty = full + D;
    uint64_t* bready = empty + D;  // [2]: decoders -> MMA
    uint64_t* bempty = bready + 2; // [2]: MMA -> decoders
    uint64_t* acc_full = bempty + 2;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (a.M + BM - 1) / BM;
    const int n_tiles = (a.groups + kPgGroups - 1) / kPgGroups;
    const int tiles = m_tiles * n_tiles;
    const int kblocks = a.kt;

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < D; ++i) {
                mbar_init(smem_u32(&full[i]), 1);
                mbar_init(smem_u32(&empty[i]), 1);
            }
            for (int i = 0; i < 2; ++i) {
                mbar_init(smem_u32(&bready[i]), kPgDecoders);
                mbar_init(smem_u32(&bempty[i]), 1);
                mbar_init(smem_u32(&acc_full[i]), 1);
                mbar_init(smem_u32(&acc_empty[i]), 4);
            }
            fence_proxy_async_smem();
        }
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(2 * kPgBN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer: x tile (TMA) + the 16 row groups' supertiles ----------------
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            const int g0 = nt * kPgGroups;
            const int ng = min(kPgGroups, a.groups - g0);
            for (int kb = 0; kb < kblocks; ++kb, ++it) {
                const int st = it % D;
                bool w_ok = true;
                if (lane == 0 && it >= D) w_ok = pg_wait(smem_u32(&empty[st]), uint32_t(((it / D) - 1) & 1));
                if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) {
                    ok = false;
                    break;
                }
                uint8_t* stage = smem + st * SB;
                const uint32_t bar = smem_u32(&full[st]);
                if (lane == 0) {
                    // the code box is always full (row groups past the matrix read as zeros)
                    mbar_expect_tx(bar, uint32_t(kABytes + kPgGroups * kCodeBytes));
                    tma_load_2d(smem_u32(stage), &tma_x, kb * BK, mt * BM, bar);
                    tma_load_4d(smem_u32(stage + kABytes), &tma_c, 0, 0, kb, g0, bar);
                }
                __syncwarp();
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int it = 0, i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++i) {
                const int acc = i & 1;
                if (i >= 2 && !pg_wait(smem_u32(&acc_empty[acc]), uint32_t(((i >> 1) - 1) & 1))) break;
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t d = tmem + uint32_t(acc * kPgBN);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int st = it % D;
                    const int bb = it & 1;
                    // x tile landed (the decoders also waited for it) and the B tile is decoded
                    if (!pg_wait(smem_u32(&full[st]), uint32_t(it / D) & 1u) ||
                        !pg_wait(smem_u32(&bready[bb]), uint32_t(it >> 1) & 1u)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                    const uint32_t abase = smem_u32(smem + st * SB);
                    const uint32_t bbase = smem_u32(btile + bb * kPgBBytes);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        umma_f16(d, sw128_desc(abase + k * 32), sw128_desc(bbase + k * 32), kPgIdesc,
                                 (kb | k) != 0 ? 1u : 0u);
                    umma_commit(smem_u32(&empty[st]));
                    umma_commit(smem_u32(&bempty[bb]));
                }
                umma_commit(smem_u32(&acc_full[acc]));
            }
        }
        __syncwarp();
    } else if (warp < 6) {
        // ---------------- epilogue: TMEM lanes = tokens, columns = weight rows ----------------
        const int quarter = warp & 3;
        const bool vec = (a.N % 8) == 0;
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const int acc = i & 1;
            if (!pg_wait(smem_u32(&acc_full[acc]), uint32_t((i >> 1) & 1))) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            const int m = mt * BM + quarter * 32 + lane;
            const int n0 = nt * kPgBN;
#pragma unroll 1
            for (int c = 0; c < kPgBN / 32; ++c) {
                uint32_t v[32];
                const uint32_t taddr =
                    tmem + (uint32_t(quarter * 32) << 16) + uint32_t(acc * kPgBN + c * 32);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                      "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
                      "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]),
                      "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
                      "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
                      "=r"(v[30]), "=r"(v[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
                const int nb = n0 + c * 32;
                if (m >= a.M || nb >= a.N) continue;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    f[j] = __uint_as_float(v[j]);
                    if (nb + j < a.N) {
                        if constexpr (HW && B != kFp16Bits) f[j] *= a.scales[nb + j];
                        if (a.bias) f[j] += __half2float(__ushort_as_half(a.bias[nb + j]));
                    }
                }
                uint16_t* yrow = a.y + size_t(m) * a.N + nb;
                if (vec && nb + 32 <= a.N) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint4 pk;
                        pk.x = pack_half2(f[8 * q + 0], f[8 * q + 1]);
                        pk.y = pack_half2(f[8 * q + 2], f[8 * q + 3]);
                        pk.z = pack_half2(f[8 * q + 4], f[8 * q + 5]);
                        pk.w = pack_half2(f[8 * q + 6], f[8 * q + 7]);
                        reinterpret_cast<uint4*>(yrow)[q] = pk;
                    }
                    if (a.y32) {
                        float* y32row = a.y32 + size_t(m) * a.N + nb;
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            reinterpret_cast<float4*>(y32row)[q] =
                                make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (nb + j < a.N) {
                            yrow[j] = __half_as_ushort(__float2half_rn(f[j]));
                            if (a.y32) a.y32[size_t(m) * a.N + nb + j] = f[j];
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty[acc]));
        }
    } else {
        // ---------------- decoders: row groups dw and dw + 8 of the tile ----------------
        const int dw = warp - 6;
        const int r0 = lane >> 2;
        const int c = lane & 3;
        DgConsts<B> pk;
        pk.init(0x4B000000u);
        constexpr int kPer = kPgGroups / kPgDecoders;  // row groups per decoding warp
        uint32_t off[kPer][4];  // swizzled 16-byte chunk offsets of this lane's rows, per group
#pragma unroll
        for (int h = 0; h < kPer; ++h) {
            const int nlo = 16 * (dw + kPgDecoders * h) + r0, nhi = nlo + 8;
            off[h][0] = uint32_t(nlo * 128 + (((2 * c) ^ (nlo & 7)) << 4));
            off[h][1] = uint32_t(nlo * 128 + (((2 * c + 1) ^ (nlo & 7)) << 4));
            off[h][2] = uint32_t(nhi * 128 + (((2 * c) ^ (nhi & 7)) << 4));
            off[h][3] = uint32_t(nhi * 128 + (((2 * c + 1) ^ (nhi & 7)) << 4));
        }
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            const int g0 = nt * kPgGroups;
            const int ng = min(kPgGroups, a.groups - g0);
            uint64_t s2[kPer][2] = {};
            if constexpr (B != kFp16Bits && !HW) {
#pragma unroll
                for (int h = 0; h < kPer; ++h)
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int gr = dw + kPgDecoders * h;
                        const int row = (g0 + gr) * kRowGroup + r0 + 8 * q;
                        const float sv = (gr < ng && row < a.N) ? a.scales[row] : 0.0f;
                        s2[h][q] = pack2f(sv, sv);
                    }
            }
            for (int kb = 0; kb < kblocks; ++kb, ++it) {
                const int st = it % D;
                const int bb = it & 1;
                if (!pg_wait(smem_u32(&full[st]), uint32_t(it / D) & 1u) ||
                    (it >= 2 && !pg_wait(smem_u32(&bempty[bb]), uint32_t((it >> 1) - 1) & 1u))) {
                    ok = false;
                    break;
                }
                uint8_t* stage = smem + st * SB;
                const uint32_t bbase = smem_u32(btile + bb * kPgBBytes);
#pragma unroll
                for (int h = 0; h < kPer; ++h) {
                    const int r = dw + kPgDecoders * h;
                    if (r >= ng) continue;  // rows past N: their columns are never stored
                    const uint8_t* cb = stage + kABytes + r * kCodeBytes;
                    uint32_t w[B];
#pragma unroll
                    for (int q = 0; q < B / 4; ++q) {
                        const uint4 v = *reinterpret_cast<const uint4*>(cb + q * 512 + lane * 16);
                        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
                    }
                    if constexpr ((B & 2) != 0) {
                        const uint2 v = *reinterpret_cast<const uint2*>(cb + (B / 4) * 512 + lane * 8);
                        w[4 * (B / 4)] = v.x;
                        w[4 * (B / 4) + 1] = v.y;
                    }
                    if constexpr ((B & 1) != 0)
                        w[B - 1] = *reinterpret_cast<const uint32_t*>(cb + (B / 4) * 512 +
                                                                      ((B & 2) ? 256 : 0) + lane * 4);
                    uint32_t af[16];
                    dg_decode<B, HW>(w, s2[h], pk, af);
                    sts128(bbase + off[h][0], af[0], af[2], af[4], af[6]);
                    sts128(bbase + off[h][1], af[8], af[10], af[12], af[14]);
                    sts128(bbase + off[h][2], af[1], af[3], af[5], af[7]);
                    sts128(bbase + off[h][3], af[9], af[11], af[13], af[15]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bready[bb]));
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(2 * kPgBN)
                     : "memory");
    }
}

template <int B, bool HW>
cudaError_t launch_pgemm_b(const CUtensorMap& tx, const CUtensorMap& tc, const PgArgs& a, unsigned grid,
                           int smem, int dev, cudaStream_t s) {
    auto kern = pgemm_kernel<B, HW>;
    static std::atomic<uint64_t> configured{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    kern<<<grid, kPgThreads, smem, s>>>(tx, tc, a);
    return cudaGetLastError();
}

struct DgPlan {
    int S, kb_per, mp, tmem_cols, stages, stage_bytes, b_off, c_off, smem;
};

DgPlan dg_plan(const Matrix& m, int64_t M, int sms) {
    DgPlan p{};
    p.mp = int(round_up(M, 16));
    p.tmem_cols = p.mp <= 32 ? 32 : (p.mp <= 64 ? 64 : (p.mp <= 128 ? 128 : 256));
    const int kt = int(m.kt);
    const int rbs = int((m.groups + kDgGroups - 1) / kDgGroups);
    const int bbytes = p.mp * BK * 2;
    const int cbytes = kDgGroups * (m.bits == 16 ? 2048 : m.bits * 128);
    p.b_off = kDgABytes;
    p.c_off = p.b_off + bbytes;
    p.stage_bytes = int(round_up(p.c_off + cbytes, 1024));
    // Two CTAs per SM when each can still hold a ring of two or three stages
    // (measured: more stages at one CTA per SM do not help), else one CTA with up to six.
    constexpr int kOverhead = 1024 + 256;
    int per_sm = 1;
    int D = (227 * 1024 - kOverhead) / p.stage_bytes;
    D = D > 6 ? 6 : D;
    const int D2 = (227 * 1024 / 2 - kOverhead) / p.stage_bytes;
    if (D2 >= 2) {
        per_sm = 2;
        D = D2 > 3 ? 3 : D2;
    }
    p.stages = D;
    p.smem = D * p.stage_bytes + kOverhead;
    // K split: minimise (waves x k-blocks per split) x ~0.5 us + the fp32 partials'
    // write and read (S * M * N * 8 bytes at ~5 TB/s); at least 4 k-blocks per split
    const double slots = double(per_sm) * sms;
    double best = 1e30;
    int bestS = 1;
    for (int S = 1; S <= 16 && (S == 1 || kt / S >= 4); S *= 2) {
        const int kb_per = (kt + S - 1) / S;
        const int splits = (kt + kb_per - 1) / kb_per;
        const double waves = std::ceil(double(rbs) * splits / slots);
        const double t = waves * kb_per * 0.5 +
                         (splits > 1 ? double(splits) * double(M) * m.rows * 8.0 / 5.0e6 : 0.0);
        if (t < best - 1e-9) {
            best = t;
            bestS = splits;
        }
    }
    p.kb_per = (kt + bestS - 1) / bestS;
    p.S = (kt + p.kb_per - 1) / p.kb_per;  // no empty split
    return p;
}

template <int B, bool HW>
cudaError_t launch_dgemm_b(const Matrix& m, const CUtensorMap& tx, const CUtensorMap& tc, const DgArgs& a,
                           unsigned grid, int smem, int dev, cudaStream_t s) {
    auto kern = dgemm_kernel<B, HW>;
    static std::atomic<uint64_t> configured{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    kern<<<grid, kDgThreads, smem, s>>>(tx, tc, a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.S == 1) return e;
    const int64_t total = int64_t(a.M) * a.N;
    const int64_t threads = (a.N % 4) == 0 ? total / 4 : total;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dgemm_reduce_kernel<HW && B != kFp16Bits>, a.part, a.S, a.M, a.N,
                              m.scales, a.bias, a.y, a.y32);
}
}  // namespace

bool pgemm_supported(const Matrix& m, const void* x) {
    return (m.cols % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t launch_pgemm(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                         uint16_t* y, float* y32, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    CUtensorMap tx, tc;
    if (M > INT32_MAX || !make_map(&tx, x, int(M), m.cols, BM) || !make_code_map(&tc, m, kPgGroups))
        return cudaErrorInvalidValue;
    PgArgs a{};
    a.tiles = m.tiles;
    a.scales = m.scales;
    a.bias = bias;
    a.y = y;
    a.y32 = y32;
    a.M = int(M);
    a.N = m.rows;
    a.kt = int(m.kt);
    a.groups = int(m.groups);
    a.stage_bytes = int(round_up(kABytes + kPgGroups * tile_bytes(m.bits), 1024));
    constexpr int kOverhead = 1024 + 512;
    int D = (227 * 1024 - kOverhead - 2 * kPgBBytes) / a.stage_bytes;
    D = D > 8 ? 8 : D;
    if (D < 2) return cudaErrorInvalidConfiguration;
    a.stages = D;
    const int smem = D * a.stage_bytes + 2 * kPgBBytes + kOverhead;
    const int64_t tiles = ((M + BM - 1) / BM) * ((m.groups + kPgGroups - 1) / kPgGroups);
    const unsigned grid = unsigned(tiles < sms ? tiles : sms);
    const bool hw = m.exec_width < 16 && m.bits <= 12;
    switch (m.bits) {
#define EBX_PG_CASE(BB)                                                       \
    case BB:                                                                  \
        return hw ? launch_pgemm_b<BB, true>(tx, tc, a, grid, smem, dev, s)   \
                  : launch_pgemm_b<BB, false>(tx, tc, a, grid, smem, dev, s);
        EBX_PG_CASE(3) EBX_PG_CASE(4) EBX_PG_CASE(5) EBX_PG_CASE(6) EBX_PG_CASE(7) EBX_PG_CASE(8)
        EBX_PG_CASE(9) EBX_PG_CASE(10) EBX_PG_CASE(11) EBX_PG_CASE(12)
#undef EBX_PG_CASE
#define EBX_PG_CASE(BB) \
    case BB:            \
        return launch_pgemm_b<BB, false>(tx, tc, a, grid, smem, dev, s);
        EBX_PG_CASE(13) EBX_PG_CASE(14) EBX_PG_CASE(15) EBX_PG_CASE(16)
#undef EBX_PG_CASE
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t read_gemm_status(int* status, bool clear, cudaStream_t s) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_gemm_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

bool gemm_supported(int K, const void* x, const void* w16) {
    return (K % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(w16) & 15) == 0 && encode_fn() != nullptr;
}

int gemm_sm_count(int dev) {
    static std::atomic<int> cache[64];
    int sms = cache[dev & 63].load(std::memory_order_relaxed);
    if (sms == 0) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
        cache[dev & 63].store(sms, std::memory_order_relaxed);
    }
    return sms;
}

// The split tiles of the last wave: y = fp16(sum of the splits in order + bias).  A
// block covers 1024 consecutive elements of one tile (4 per thread: one float4 of each
// split's partial), so the tile's coordinates are computed once per thread
// (programmatic dependent launch: waits for the GEMM grid).
template <int BN>
__global__ void __launch_bounds__(256) gemm_tail_reduce_kernel(const float* part, int S, int full_tiles,
                                                               int tail_tiles, int M, int N,
                                                               const uint16_t* bias, uint16_t* y,
                                                               float* y32) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    constexpr int kPerTile = BM * BN;
    constexpr int kBlocksPerTile = kPerTile / 1024;
    const int r = int(blockIdx.x) / kBlocksPerTile;
    const int off = (int(blockIdx.x) % kBlocksPerTile) * 1024 + int(threadIdx.x) * 4;
    int mt, nt;
    tile_coords(full_tiles + r, (M + BM - 1) / BM, (N + BN - 1) / BN, mt, nt);
    const int m = mt * BM + off / BN, n = nt * BN + off % BN;
    if (m >= M || n >= N) return;
    const size_t base = size_t(r) * kPerTile + off;
    float4 v = *reinterpret_cast<const float4*>(part + base);
    for (int sp = 1; sp < S; ++sp) {
        const float4 u = *reinterpret_cast<const float4*>(part + size_t(sp) * tail_tiles * kPerTile + base);
        v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
    }
    float f[4] = {v.x, v.y, v.z, v.w};
    const size_t o = size_t(m) * N + n;
    if ((N & 3) == 0 && n + 4 <= N) {
        if (bias) {
#pragma unroll
            for (int j = 0; j < 4; ++j) f[j] += __half2float(__ushort_as_half(bias[n + j]));
        }
        uint2 h;
        h.x = pack_half2(f[0], f[1]);
        h.y = pack_half2(f[2], f[3]);
        *reinterpret_cast<uint2*>(y + o) = h;
        if (y32) *reinterpret_cast<float4*>(y32 + o) = make_float4(f[0], f[1], f[2], f[3]);
        return;
    }
    for (int j = 0; j < 4 && n + j < N; ++j) {
        float w = f[j];
        if (bias) w += __half2float(__ushort_as_half(bias[n + j]));
        y[o + j] = __half_as_ushort(__float2half_rn(w));
        if (y32) y32[o + j] = w;
    }
}

// Weight-tile width (256 columns: measured fastest at every config-3 size, against 128
// and 64) and the tail split: whole waves of output tiles stay whole, the tiles of a
// last, partial wave are split over K so that they occupy up to every SM (at most 8 ways,
// at least 4 k-blocks each).  Measured per call, materialise included (B200, graph
// replay): 4096 x 4096 at M = 512 40.9 -> 34.6 us, 14336 x 4096 at M = 512 129 -> 96 us
// and at M = 4096 420 -> 400 us, 4096 x 14336 at M = 1024 140 -> 133 us; no shape slower.
// Splitting every tile instead (partials of the whole output through HBM) was slower at
// every M >= 1024.
struct GemmPlan {
    int bn = 256;
    int full_tiles = 0;
    int tail_split = 1;
};

GemmPlan gemm_plan(int64_t M, int N, int K, int sms) {
    GemmPlan p;
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn);
    const int64_t kblocks = (K + BK - 1) / BK;
    const int64_t tail = tiles % sms;
    p.full_tiles = int(tiles - tail);
    if (tail == 0) return p;
    int S = int(sms / tail);
    if (S > 8) S = 8;
    while (S > 1 && kblocks < 4 * S) --S;
    p.tail_split = S;
    if (S == 1) p.full_tiles = int(tiles);
    return p;
}

uint64_t gemm_part_bytes(int64_t M, int N, int K) {
    if (M <= 0) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const GemmPlan p = gemm_plan(M, N, K, gemm_sm_count(dev));
    if (p.tail_split == 1) return 0;
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn);
    return uint64_t(round_up((tiles - p.full_tiles) * p.tail_split * int64_t(BM) * p.bn * 4, 256));
}

template <int BN>
cudaError_t launch_gemm_bn(const uint16_t* x, const uint16_t* w16, int64_t M, int N, int K,
                           const uint16_t* bias, uint16_t* y, float* y32, GemmPlan p, float* part,
                           int sms, int dev, cudaStream_t s) {
    using G = GemmCfg<BN>;
    CUtensorMap tx, tw;
    if (!make_map(&tx, x, int(M), K, BM) || !make_map(&tw, w16, N, K, BN)) return cudaErrorInvalidValue;
    auto kern = gemm_f16_kernel<BN>;
    static std::atomic<uint64_t> configured{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(configured.load(std::memory_order_relaxed) & bit)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit);
    }
    const int64_t tiles = ((M + BM - 1) / BM) * int64_t((N + BN - 1) / BN);
    if (tiles > INT32_MAX / 8) return cudaErrorInvalidValue;
    GemmArgs a{bias, y, y32, int(M), N, K, p.full_tiles, p.tail_split, part};
    const int64_t units = p.full_tiles + (tiles - p.full_tiles) * p.tail_split;
    const unsigned grid = unsigned(units < sms ? units : sms);  // persistent: one CTA per SM
    kern<<<grid, kGemmThreads, G::kSmem, s>>>(tx, tw, a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || p.tail_split == 1) return e;
    const int tail_tiles = int(tiles - p.full_tiles);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(tail_tiles * (BM * BN / 1024)));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_tail_reduce_kernel<BN>, static_cast<const float*>(part),
                              p.tail_split, p.full_tiles, tail_tiles, int(M), N, bias, y, y32);
}

cudaError_t launch_gemm_f16(const uint16_t* x, const uint16_t* w16, int64_t M, int N, int K,
                            const uint16_t* bias, uint16_t* y, float* y32, float* part,
                            uint64_t part_bytes, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int sms = gemm_sm_count(dev);
    GemmPlan p = gemm_plan(M, N, K, sms);
    if (p.tail_split > 1 && (!part || part_bytes < gemm_part_bytes(M, N, K))) {
        p.full_tiles = int(((M + BM - 1) / BM) * ((N + p.bn - 1) / p.bn));  // no room: no split
        p.tail_split = 1;
    }
    return launch_gemm_bn<256>(x, w16, M, N, K, bias, y, y32, p, part, sms, dev, s);
}

// Measured on the BASELINE shapes: the decode-GEMM beats chunked decode for every
// 16 < M <= 128 and materialise + GEMM for M <= 128 and, up to 256 rows, when K >= 8192
// (14336x4096 at M = 256: 64 vs 104 us); with K = 4096 and 128 < M <= 256 the separate
// materialise + GEMM is as fast or faster.
bool dgemm_supported(const Matrix& m, int64_t M, const void* x) {
    return dgemm_route(m, M) && M <= kDgMaxTokens && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           encode_fn() != nullptr;
}

uint64_t dgemm_workspace_bytes(const Matrix& m, int64_t M) {
    const DgPlan p = dg_plan(m, M, gemm_sm_count(m.device));
    return p.S > 1 ? uint64_t(round_up(int64_t(p.S) * M * m.rows * 4, 256)) : 0;
}

cudaError_t launch_dgemm(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                         uint16_t* y, float* y32, void* ws, uint64_t ws_bytes, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const DgPlan p = dg_plan(m, M, gemm_sm_count(dev));
    if (p.stages < 2) return cudaErrorInvalidConfiguration;
    if (p.S > 1 && (ws == nullptr || ws_bytes < dgemm_workspace_bytes(m, M))) return cudaErrorInvalidValue;
    CUtensorMap tx;
    CUtensorMap tc;
    if (!make_map(&tx, x, int(M), m.cols, p.mp) || !make_code_map(&tc, m, kDgGroups))
        return cudaErrorInvalidValue;
    DgArgs a{};
    a.tiles = m.tiles;
    a.scales = m.scales;
    a.bias = bias;
    a.y = y;
    a.y32 = y32;
    a.part = static_cast<float*>(ws);
    a.M = int(M);
    a.N = m.rows;
    a.kt = int(m.kt);
    a.groups = int(m.groups);
    a.S = p.S;
    a.kb_per = p.kb_per;
    a.stages = p.stages;
    a.stage_bytes = p.stage_bytes;
    a.mp = p.mp;
    a.tmem_cols = p.tmem_cols;
    a.b_off = p.b_off;
    a.c_off = p.c_off;
    const unsigned grid = unsigned(((m.groups + kDgGroups - 1) / kDgGroups) * p.S);
    const bool hw = m.exec_width < 16 && m.bits <= 12;
    switch (m.bits) {
#define EBX_DG_CASE(BB)                                                                  \
    case BB:                                                                             \
        return hw ? launch_dgemm_b<BB, true>(m, tx, tc, a, grid, p.smem, dev, s)         \
                  : launch_dgemm_b<BB, false>(m, tx, tc, a, grid, p.smem, dev, s);
        EBX_DG_CASE(3) EBX_DG_CASE(4) EBX_DG_CASE(5) EBX_DG_CASE(6) EBX_DG_CASE(7) EBX_DG_CASE(8)
        EBX_DG_CASE(9) EBX_DG_CASE(10) EBX_DG_CASE(11) EBX_DG_CASE(12)
#undef EBX_DG_CASE
#define EBX_DG_CASE(BB) \
    case BB:            \
        return launch_dgemm_b<BB, false>(m, tx, tc, a, grid, p.smem, dev, s);
        EBX_DG_CASE(13) EBX_DG_CASE(14) EBX_DG_CASE(15) EBX_DG_CASE(16)
#undef EBX_DG_CASE
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t read_dgemm_status(int* status, bool clear, cudaStream_t s) {
    cudaError_t e = cudaMemcpyFromSymbolAsync(status, g_dgemm_status, sizeof(int), 0,
                                              cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_dgemm_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    return e;
}

}  // namespace ebx
