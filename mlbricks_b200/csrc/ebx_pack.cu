// ebx_pack.cu -- device-side conversion between the reference's storage code
// and the B200 tile layout (see ebx_common.cuh), plus exact materialisation.
//
// The reference packs and unpacks on the host, single-threaded
// (elasticbit_runtime.cu:150-238, 1180-1239).  Here every conversion is a
// kernel: one thread owns one lane-slice (32 codes) of one supertile, or one
// 32-bit word of the MLB4 bitstream.
#include "ebx_common.cuh"
#include "ebx_internal.h"

namespace ebx {
namespace {

// Storage code of weight (row, k): q + qmax, or qmax (q = 0) for padding.
struct CodeFromInt16 {
    const int16_t* codes;
    int rows, cols, qmax;
    int* bad;
    __device__ uint32_t operator()(int row, int k) const {
        if (row >= rows || k >= cols) return uint32_t(qmax);
        const int q = codes[int64_t(row) * cols + k];
        if (q < -qmax || q > qmax) {
            atomicOr(bad, 1);
            return uint32_t(qmax);
        }
        return uint32_t(q + qmax);
    }
};

// Code read from the MLB4 LSB-first bitstream (cu:188-206 semantics).
struct CodeFromPayload {
    const uint8_t* payload;
    uint64_t nbytes;
    int rows, cols, bits, qmax;
    __device__ uint32_t operator()(int row, int k) const {
        if (row >= rows || k >= cols) return uint32_t(qmax);
        const uint64_t bit = (uint64_t(row) * cols + k) * uint64_t(bits);
        const uint64_t b0 = bit >> 3;
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 3; ++j)
            if (b0 + j < nbytes) word |= uint32_t(payload[b0 + j]) << (8 * j);
        return (word >> (bit & 7)) & ((1u << bits) - 1u);
    }
};

struct CodeFromFp16 {
    const uint16_t* w;
    int rows, cols;
    __device__ uint32_t operator()(int row, int k) const {
        if (row >= rows || k >= cols) return 0u;
        return w[int64_t(row) * cols + k];
    }
};

// One thread = one lane-slice of one supertile: gather 32 codes, pack them
// LSB-first into `bits` words, scatter the words to their vector segments.
template <class Src>
__global__ void to_tiles_kernel(Src src, uint8_t* tiles, int bits, int64_t kt,
                                int64_t total_slices) {
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= total_slices) return;
    const int lane = int(id & 31);
    const int64_t tile = id >> 5;
    const int64_t g = tile / kt;
    const int64_t t = tile - g * kt;
    uint32_t words[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) words[i] = 0;
    const bool plane = plane_layout(bits);
    for (int j = 0; j < 32; ++j) {
        int r, k;
        code_position(lane, j, &r, &k);
        const uint32_t code = src(int(g * kRowGroup + r), int(t * kKTile + k));
        if (plane) {
            words[j >> 2] |= (code & 0xFFu) << (8 * (j & 3));
            for (int hb = 0; hb < bits - 8; ++hb) {
                int wi, bi;
                plane_hi_bit(bits, j, hb, &wi, &bi);
                words[wi] |= ((code >> (8 + hb)) & 1u) << bi;
            }
            continue;
        }
        const int bit = j * bits;
        const int wi = bit >> 5, o = bit & 31;
        words[wi] |= code << o;
        if (o + bits > 32) words[wi + 1] |= code >> (32 - o);
    }
    uint8_t* base = tiles + tile * tile_bytes(bits);
    for (int i = 0; i < bits; ++i)
        *reinterpret_cast<uint32_t*>(base + word_offset(bits, lane, i)) = words[i];
}

// Code of (row, k) read back from the tile layout.
__device__ __forceinline__ uint32_t tile_code(const uint8_t* tiles, int bits, int64_t kt, int row,
                                              int k) {
    const int64_t g = row / kRowGroup, t = k / kKTile;
    const int rin = row % kRowGroup, kin = k % kKTile;
    const int c = kin >> 4, kk = kin & 15, s = kk >> 2, u = kk & 3;
    const int e = ((u >> 1) << 2) | ((rin >> 3) << 1) | (u & 1);
    const int lane = (rin & 7) * 4 + c;
    const int j = 8 * s + e;
    const uint8_t* base = tiles + (g * kt + t) * tile_bytes(bits);
    if (plane_layout(bits)) {
        uint32_t code =
            (*reinterpret_cast<const uint32_t*>(base + word_offset(bits, lane, j >> 2)) >> (8 * (j & 3))) &
            0xFFu;
        for (int hb = 0; hb < bits - 8; ++hb) {
            int wi, bi;
            plane_hi_bit(bits, j, hb, &wi, &bi);
            code |= ((*reinterpret_cast<const uint32_t*>(base + word_offset(bits, lane, wi)) >> bi) & 1u)
                    << (8 + hb);
        }
        return code;
    }
    const int bit = j * bits, wi = bit >> 5, o = bit & 31;
    uint64_t v = *reinterpret_cast<const uint32_t*>(base + word_offset(bits, lane, wi));
    if (o + bits > 32)
        v |= uint64_t(*reinterpret_cast<const uint32_t*>(base + word_offset(bits, lane, wi + 1)))
             << 32;
    return uint32_t(v >> o) & ((1u << bits) - 1u);
}

// One thread = one 32-bit word of the MLB4 bitstream (the trailing partial
// word is written bytewise).  Bits beyond rows*cols*bits are zero, like the
// reference's zero-initialised payload (cu:163).
__global__ void to_payload_kernel(const uint8_t* tiles, int bits, int64_t kt, int rows, int cols,
                                  uint8_t* payload, uint64_t nbytes) {
    const uint64_t w = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t nwords = (nbytes + 3) / 4;
    if (w >= nwords) return;
    const uint64_t count = uint64_t(rows) * cols;
    const uint64_t bit0 = w * 32;
    uint64_t i = bit0 / bits;
    uint32_t out = 0;
    for (; i < count; ++i) {
        const uint64_t b = i * bits;
        if (b >= bit0 + 32) break;
        const int row = int(i / cols), k = int(i % cols);
        const uint64_t code = tile_code(tiles, bits, kt, row, k);
        const int64_t sh = int64_t(b) - int64_t(bit0);
        out |= sh >= 0 ? uint32_t(code << sh) : uint32_t(code >> (-sh));
    }
    if (w * 4 + 4 <= nbytes) {
        *reinterpret_cast<uint32_t*>(payload + w * 4) = out;
    } else {
        for (uint64_t j = 0; w * 4 + j < nbytes; ++j) payload[w * 4 + j] = uint8_t(out >> (8 * j));
    }
}

// Exact dequantisation to row-major fp16: W[n,k] = fp16_rn(fp32_rn(q * s_n))
// (cu:208-238; core.py:156).  One thread decodes one lane-slice with the same
// dequant2 helper the GEMV kernel uses, so both paths give identical weights.
template <int B>
__global__ void materialize_kernel(const uint8_t* tiles, const float* scales, int rows, int cols,
                                   int64_t kt, int64_t total_slices, uint16_t* out, bool vec) {
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= total_slices) return;
    const int lane = int(id & 31);
    const int64_t tile = id >> 5;
    const int64_t g = tile / kt, t = tile - (tile / kt) * kt;
    const uint8_t* base = tiles + tile * tile_bytes(B);
    // the lane's words: 16-byte segments, then an 8- and a 4-byte one (word_offset)
    uint32_t w[B];
#pragma unroll
    for (int q = 0; q < B / 4; ++q) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + q * 512 + lane * 16));
        w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
    }
    if constexpr ((B & 2) != 0) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(base + (B / 4) * 512 + lane * 8));
        w[4 * (B / 4)] = v.x;
        w[4 * (B / 4) + 1] = v.y;
    }
    if constexpr ((B & 1) != 0)
        w[B - 1] = __ldg(reinterpret_cast<const uint32_t*>(base + (B / 4) * 512 + ((B & 2) ? 256 : 0) +
                                                           lane * 4));
    const int r0 = int(g * kRowGroup) + (lane >> 2);
    const int kb = int(t * kKTile) + 16 * (lane & 3);
    uint32_t h[16];
    if constexpr (B == kFp16Bits) {
#pragma unroll
        for (int p = 0; p < 16; ++p) h[p] = w[p];
    } else if constexpr (plane_layout(B)) {
        // plane layout: exact q pairs, then fp16_rn(fp32_rn(q * s)) (the decode kernel's
        // arithmetic for the fullPrecision semantics)
        const float sl = r0 < rows ? scales[r0] : 0.0f;
        const float sh = r0 + 8 < rows ? scales[r0 + 8] : 0.0f;
        PlaneConsts pk;
        pk.init(0x64646464u);
        uint32_t q16[16];
        plane_q16_all<B>(w, pk, q16);
        const uint64_t s2[2] = {pack2f(sl, sl), pack2f(sh, sh)};
#pragma unroll
        for (int p = 0; p < 16; ++p) h[p] = q16_to_w16(q16[p], s2[p & 1]);
    } else if constexpr (B == 8) {
        // paired f32x2 decode (the decode kernel's arithmetic)
        const float sl = r0 < rows ? scales[r0] : 0.0f;
        const float sh = r0 + 8 < rows ? scales[r0 + 8] : 0.0f;
        PairConsts<B> pk;
        pk.init(0x4B000000u);
        const uint64_t s2[2] = {pack2f(sl, sl), pack2f(sh, sh)};
        uint32_t lo[4], hi[4];
        dequant_steps<B, 0>(w, pk, s2, lo, hi);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            h[r] = lo[r];
            h[8 + r] = hi[r];
        }
        dequant_steps<B, 1>(w, pk, s2, lo, hi);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            h[4 + r] = lo[r];
            h[12 + r] = hi[r];
        }
    } else {
        const float sl = r0 < rows ? scales[r0] : 0.0f;
        const float sh = r0 + 8 < rows ? scales[r0 + 8] : 0.0f;
        const float nb = -(8388608.0f + float(qmax_for(B)));
        const uint64_t nb2 = pack2f(nb, nb), sl2 = pack2f(sl, sl), sh2 = pack2f(sh, sh);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            const int j = 2 * p;
            h[p] = dequant2(code_magic<B>(w, j), code_magic<B>(w, j + 1), nb2, (p & 1) ? sh2 : sl2);
        }
    }
    // h[4s + r]: r = 0 -> row r0, k = kb+4s+{0,1}; r = 1 -> row r0+8, same k;
    //            r = 2 -> row r0, k = kb+4s+{2,3}; r = 3 -> row r0+8, k+{2,3}.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int row = r0 + 8 * half;
        if (row >= rows) continue;
        uint32_t v[8];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            v[2 * s] = h[4 * s + half];
            v[2 * s + 1] = h[4 * s + 2 + half];
        }
        uint16_t* dst = out + int64_t(row) * cols + kb;
        if (vec && kb + 16 <= cols) {
            reinterpret_cast<uint4*>(dst)[0] = make_uint4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<uint4*>(dst)[1] = make_uint4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e)
                if (kb + e < cols) dst[e] = uint16_t(v[e >> 1] >> (16 * (e & 1)));
        }
    }
}

inline unsigned blocks_for(int64_t n, int threads) { return unsigned((n + threads - 1) / threads); }

}  // namespace

cudaError_t launch_codes_to_tiles(const Matrix& m, const int16_t* codes, int* bad, cudaStream_t s) {
    const int64_t slices = m.groups * m.kt * 32;
    CodeFromInt16 src{codes, m.rows, m.cols, qmax_for(m.bits), bad};
    to_tiles_kernel<<<blocks_for(slices, 256), 256, 0, s>>>(src, m.tiles, m.bits, m.kt, slices);
    return cudaGetLastError();
}

cudaError_t launch_payload_to_tiles(const Matrix& m, const uint8_t* payload, uint64_t nbytes,
                                    cudaStream_t s) {
    const int64_t slices = m.groups * m.kt * 32;
    CodeFromPayload src{payload, nbytes, m.rows, m.cols, m.bits, qmax_for(m.bits)};
    to_tiles_kernel<<<blocks_for(slices, 256), 256, 0, s>>>(src, m.tiles, m.bits, m.kt, slices);
    return cudaGetLastError();
}

cudaError_t launch_fp16_to_tiles(const Matrix& m, const uint16_t* w, cudaStream_t s) {
    const int64_t slices = m.groups * m.kt * 32;
    CodeFromFp16 src{w, m.rows, m.cols};
    to_tiles_kernel<<<blocks_for(slices, 256), 256, 0, s>>>(src, m.tiles, 16, m.kt, slices);
    return cudaGetLastError();
}

cudaError_t launch_tiles_to_payload(const Matrix& m, uint8_t* payload, uint64_t nbytes,
                                    cudaStream_t s) {
    const uint64_t nwords = (nbytes + 3) / 4;
    to_payload_kernel<<<blocks_for(int64_t(nwords), 256), 256, 0, s>>>(
        m.tiles, m.bits, m.kt, m.rows, m.cols, payload, nbytes);
    return cudaGetLastError();
}

cudaError_t launch_materialize(const Matrix& m, uint16_t* out, cudaStream_t s) {
    const int64_t slices = m.groups * m.kt * 32;
    const unsigned grid = blocks_for(slices, 256);
    const bool vec = (m.cols & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    switch (m.bits) {
#define EBX_MAT_CASE(B) \
    case B:             \
        materialize_kernel<B><<<grid, 256, 0, s>>>(m.tiles, m.scales, m.rows, m.cols, m.kt, slices, out, vec); \
        break;
        EBX_MAT_CASE(3) EBX_MAT_CASE(4) EBX_MAT_CASE(5) EBX_MAT_CASE(6) EBX_MAT_CASE(7)
        EBX_MAT_CASE(8) EBX_MAT_CASE(9) EBX_MAT_CASE(10) EBX_MAT_CASE(11) EBX_MAT_CASE(12)
        EBX_MAT_CASE(13) EBX_MAT_CASE(14) EBX_MAT_CASE(15) EBX_MAT_CASE(16)
#undef EBX_MAT_CASE
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace ebx
