// ebx_common.cuh -- shared definitions for the B200 ElasticBit runtime (libebx).
//
// Device execution layout ("tile layout")
// ---------------------------------------
// Storage stays the reference's MLB4 code: b-bit codes q+qmax (b = 3..15) or
// raw fp16 (b = 16), one fp32 scale per row (elasticbit_runtime.cu:83-238).
// On the device the same codes are kept at exactly b bits per weight, but
// permuted so that one warp can stream them with 128-bit loads and decode them
// straight into mma.m16n8k16 A-fragments:
//
//   * rows are grouped by 16 ("row group" g), K by 64 ("k-tile" t);
//     N and K are padded up to 16 and 64 with q = 0 (decodes to +0.0);
//   * one (g, t) supertile = 16 rows x 64 k = 1024 codes = b x 128 bytes,
//     stored at ((g * KT) + t) * b * 128 (KT = Kp / 64): a row group's whole
//     K-run is one contiguous byte range;
//   * inside a supertile lane l owns 32 codes = b 32-bit words, packed LSB-first
//     (code j at bits [j*b, j*b+b) of the lane's 32*b-bit little-endian word
//     string).  The words are interleaved across lanes in vector segments so a
//     warp loads them with coalesced 16-byte (then 8-, then 4-byte) accesses:
//     seg s < b/4 holds words 4s..4s+3 at s*512 + l*16; if b%4 has bit 1, words
//     4(b/4), +1 sit at (b/4)*512 + l*8; if b%4 has bit 0, the last word sits at
//     (b/4)*512 + (b%4 >= 2 ? 256 : 0) + l*4;
//   * code j = 8*s + e (s = MMA k-step 0..3, e = A-fragment element 0..7) holds
//     the weight at  row = l/4 + 8*((e>>1)&1),
//                    k   = 16*(l%4) + 4*s + 2*(e>>2) + (e&1).
//     Matching B fragments then come from x[n][16*(l%4) .. 16*(l%4)+16), one
//     32-byte run per token, because the same k permutation is applied to the
//     activations (a dot product is invariant under a shared permutation of k).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ebx {

constexpr int kRowGroup = 16;  // rows per supertile
constexpr int kKTile = 64;     // k per supertile
constexpr int kMinBits = 3;
constexpr int kMaxBits = 15;
constexpr int kFp16Bits = 16;

__host__ __device__ constexpr int qmax_for(int bits) { return (1 << (bits - 1)) - 1; }
__host__ __device__ constexpr int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
__host__ __device__ constexpr int64_t tile_bytes(int bits) { return int64_t(bits) * 128; }

// Byte offset of word i of lane l inside one supertile of width `bits`.
__host__ __device__ inline int word_offset(int bits, int lane, int i) {
    const int nq = bits >> 2;
    const int r = bits & 3;
    if (i < 4 * nq) return (i >> 2) * 512 + lane * 16 + (i & 3) * 4;
    int base = nq * 512;
    if (r & 2) {
        if (i < 4 * nq + 2) return base + lane * 8 + (i - 4 * nq) * 4;
        base += 256;
    }
    return base + lane * 4;
}

// (row, k) inside the supertile of code j owned by lane l.
__host__ __device__ inline void code_position(int lane, int j, int* row, int* k) {
    const int s = j >> 3, e = j & 7;
    *row = (lane >> 2) + 8 * ((e >> 1) & 1);
    *k = 16 * (lane & 3) + 4 * s + 2 * (e >> 2) + (e & 1);
}

// ---------------------------------------------------------------------------
// PTX helpers (sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
    return (uint64_t(__float_as_uint(hi)) << 32) | uint64_t(__float_as_uint(lo));
}

// Exact decode of two codes to fp16: fp16_rn(fp32_rn((c - qmax) * s)).
// `m0`, `m1` are the codes OR-ed into the mantissa of 2^23 (float 2^23 + c);
// `neg_bias2` = (-(2^23 + qmax), same), `scale2` = (s, s).  The add is exact
// (integers below 2^24), the multiply is one RN fp32 product like the
// reference's `static_cast<float>(q) * scale`, and cvt.rn.f16x2 is the RN fp16
// rounding of __float2half_rn.  Result: low half = first code.
__device__ __forceinline__ uint32_t dequant2(uint32_t m0, uint32_t m1, uint64_t neg_bias2,
                                             uint64_t scale2) {
    uint32_t h;
    asm("{\n\t.reg .b64 a, r;\n\t.reg .f32 lo, hi;\n\t"
        "mov.b64 a, {%1, %2};\n\t"
        "add.rn.f32x2 r, a, %3;\n\t"
        "mul.rn.f32x2 r, r, %4;\n\t"
        "mov.b64 {lo, hi}, r;\n\t"
        "cvt.rn.f16x2.f32 %0, hi, lo;\n\t}"
        : "=r"(h)
        : "r"(m0), "r"(m1), "l"(neg_bias2), "l"(scale2));
    return h;
}

// Integer codes as fp16 (no scale): used by the hardwareNative integer-dot
// semantics, where the row scale is applied after accumulation.
__device__ __forceinline__ uint32_t codes2_to_half(uint32_t m0, uint32_t m1, uint64_t neg_bias2) {
    uint32_t h;
    asm("{\n\t.reg .b64 a, r;\n\t.reg .f32 lo, hi;\n\t"
        "mov.b64 a, {%1, %2};\n\t"
        "add.rn.f32x2 r, a, %3;\n\t"
        "mov.b64 {lo, hi}, r;\n\t"
        "cvt.rn.f16x2.f32 %0, hi, lo;\n\t}"
        : "=r"(h)
        : "r"(m0), "r"(m1), "l"(neg_bias2));
    return h;
}

// Code j of a lane-slice held in registers w[0..B-1], OR-ed into the mantissa
// of 2^23 (the float 2^23 + code).  With B a compile-time constant and j an
// unrolled index, the word index and shift fold to constants: one funnel or
// plain shift (none when the code sits at bit 0) plus one LOP3.
template <int B>
__device__ __forceinline__ uint32_t code_magic(const uint32_t (&w)[B], int j) {
    const int bit = j * B, wi = bit >> 5, o = bit & 31;
    uint32_t v;
    if (o == 0) v = w[wi];
    else if (o + B <= 32) v = w[wi] >> o;
    else v = __funnelshift_r(w[wi], w[wi + 1], o);
    return (v & ((1u << B) - 1u)) | 0x4B000000u;
}

// Shifted code word: code j moved to bit 0 (upper bits still hold the next
// codes; the LOP3 in dequant2_lop masks them).  No shift for a code at bit 0.
template <int B>
__device__ __forceinline__ uint32_t code_word(const uint32_t (&w)[B], int j) {
    const int bit = j * B, wi = bit >> 5, o = bit & 31;
    if (o == 0) return w[wi];
    if (o + B <= 32) return w[wi] >> o;
    return __funnelshift_r(w[wi], w[wi + 1], o);
}

// Exact decode of two shifted code words to fp16x2 in one asm block: LOP3
// ((v & mask) | 2^23 magic, register operands), f32x2 add of -(2^23 + qmax),
// f32x2 RN multiply by the row scale, cvt.rn.f16x2.  Same arithmetic as
// dequant2; written as one block so the pair lives in one register pair.
__device__ __forceinline__ uint32_t dequant2_lop(uint32_t v0, uint32_t v1, uint32_t mask,
                                                 uint32_t magic, uint64_t neg_bias2,
                                                 uint64_t scale2) {
    uint32_t h;
    asm("{\n\t.reg .b32 c0, c1;\n\t.reg .b64 a;\n\t"
        "lop3.b32 c0, %1, %3, %4, 0xEA;\n\t"
        "lop3.b32 c1, %2, %3, %4, 0xEA;\n\t"
        "mov.b64 a, {c0, c1};\n\t"
        "add.rn.f32x2 a, a, %5;\n\t"
        "mul.rn.f32x2 a, a, %6;\n\t"
        "mov.b64 {c0, c1}, a;\n\t"
        "cvt.rn.f16x2.f32 %0, c1, c0;\n\t}"
        : "=r"(h)
        : "r"(v0), "r"(v1), "r"(mask), "r"(magic), "l"(neg_bias2), "l"(scale2));
    return h;
}

// Scalar formulation of dequant2_lop (two LOP3, two FADD, two FMUL, one cvt):
// identical results, no register-pair packing.
__device__ __forceinline__ uint32_t dequant2_scalar(uint32_t v0, uint32_t v1, uint32_t mask,
                                                    uint32_t magic, float neg_bias, float scale) {
    uint32_t h;
    asm("{\n\t.reg .b32 c0, c1;\n\t"
        "lop3.b32 c0, %1, %3, %4, 0xEA;\n\t"
        "lop3.b32 c1, %2, %3, %4, 0xEA;\n\t"
        "add.rn.f32 c0, c0, %5;\n\t"
        "add.rn.f32 c1, c1, %5;\n\t"
        "mul.rn.f32 c0, c0, %6;\n\t"
        "mul.rn.f32 c1, c1, %6;\n\t"
        "cvt.rn.f16x2.f32 %0, c1, c0;\n\t}"
        : "=r"(h)
        : "r"(v0), "r"(v1), "r"(mask), "r"(magic), "f"(neg_bias), "f"(scale));
    return h;
}

// Integer codes to fp16x2 (no scale), for the scale-after-accumulation path.
__device__ __forceinline__ uint32_t codes2_lop(uint32_t v0, uint32_t v1, uint32_t mask,
                                               uint32_t magic, uint64_t neg_bias2) {
    uint32_t h;
    asm("{\n\t.reg .b32 c0, c1;\n\t.reg .b64 a;\n\t"
        "lop3.b32 c0, %1, %3, %4, 0xEA;\n\t"
        "lop3.b32 c1, %2, %3, %4, 0xEA;\n\t"
        "mov.b64 a, {c0, c1};\n\t"
        "add.rn.f32x2 a, a, %5;\n\t"
        "mov.b64 {c0, c1}, a;\n\t"
        "cvt.rn.f16x2.f32 %0, c1, c0;\n\t}"
        : "=r"(h)
        : "r"(v0), "r"(v1), "r"(mask), "r"(magic), "l"(neg_bias2));
    return h;
}

// --- mbarrier + TMA bulk copy (non-tensor, no multicast) -------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
                 : "memory");
}
// One bounded probe; returns true once the phase with parity `parity` completed.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every mbarrier wait in libebx is bounded in wall-clock time (a try_wait probe
// may itself suspend the thread for a while, so a probe count alone is not a
// bound): after kMbarWaitNs the caller gets false and must record an error,
// skip the work that depended on the barrier and leave.
constexpr uint64_t kMbarWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < 64; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kMbarWaitNs) return false;
    }
}

// Global -> shared bulk copy completing on an mbarrier.  src/dst 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// D += A(16x16 fp16, row) * B(16x8 fp16, col), fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16/8/4-byte async global->shared copies; src_bytes < size zero-fills.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

}  // namespace ebx

namespace ebx {

// ---------------------------------------------------------------------------
// Compile-time decode plan for a lane's 32 codes of width B (3..15).
// Code j occupies bits [o, o+B) of word j*B/32 at o = (j*B) % 32.  When
// o + B <= 23 the code can be decoded *in place*: (w & (mask << o)) | 2^23 is
// the float 2^23 + code * 2^o, so subtracting 2^23 + qmax * 2^o gives q * 2^o
// exactly and multiplying by s * 2^-o gives fp32_rn(q * s) (a power-of-two
// factor moves between the operands without changing the exact product).  Up
// to kMaxSlots distinct in-place offsets get their own scale register; every
// other code is first shifted down to bit 0.
// ---------------------------------------------------------------------------
constexpr int kMaxSlots = 8;

struct CodePlan {
    int shift_word;  // -1: in place; else word index to shift from
    int o;           // bit offset within the word
    int slot;        // scale slot (in place only), 0 = offset 0
};

constexpr CodePlan plan_code(int B, int j) {
    const int bit = j * B, wi = bit >> 5, o = bit & 31;
    if (o + B <= 23) {
        // slot = rank of o among the distinct in-place offsets of codes 0..j
        int offs[kMaxSlots] = {0, 0, 0, 0, 0, 0, 0, 0};
        int n = 0;
        for (int jj = 0; jj <= j; ++jj) {
            const int oo = (jj * B) & 31;
            if (oo + B > 23) continue;
            bool seen = false;
            for (int k = 0; k < n; ++k) seen = seen || offs[k] == oo;
            if (!seen) {
                if (n == kMaxSlots) {
                    if (oo == o) return CodePlan{wi, o, -1};
                    continue;
                }
                offs[n++] = oo;
            }
        }
        for (int k = 0; k < n; ++k)
            if (offs[k] == o) return CodePlan{-1, o, k};
        return CodePlan{wi, o, -1};
    }
    return CodePlan{wi, o, -1};
}

constexpr int slot_offset(int B, int slot) {
    int offs[kMaxSlots] = {0, 0, 0, 0, 0, 0, 0, 0};
    int n = 0;
    for (int j = 0; j < 32; ++j) {
        const int o = (j * B) & 31;
        if (o + B > 23) continue;
        bool seen = false;
        for (int k = 0; k < n; ++k) seen = seen || offs[k] == o;
        if (!seen && n < kMaxSlots) offs[n++] = o;
    }
    return slot < n ? offs[slot] : -1;
}

constexpr int slot_count(int B) {
    int n = 0;
    for (int k = 0; k < kMaxSlots; ++k) n += slot_offset(B, k) >= 0 ? 1 : 0;
    return n;
}

// s * 2^-offset factor per slot, as compile-time float constants.
template <int B, int K>
struct SlotScale {
    static constexpr int kOff = slot_offset(B, K) < 0 ? 0 : slot_offset(B, K);
    static constexpr float kFactor = 1.0f / float(1u << kOff);
};

// q*2^o as float from a code word (in place) or a shifted word (o = 0).
template <int B, int O>
__device__ __forceinline__ float code_to_float(uint32_t word, uint32_t magic) {
    constexpr uint32_t kMask = ((1u << B) - 1u) << O;
    constexpr float kBias = -(8388608.0f + float(qmax_for(B)) * float(1u << O));
    uint32_t v;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(v) : "r"(word), "n"(kMask), "r"(magic));
    return __fadd_rn(__uint_as_float(v), kBias);
}

// Code j of the lane slice -> fp32 q*s exactly rounded (before the fp16 cvt).
// `sc` holds s * 2^-offset for each slot; sc[0] = s.
template <int B, int J, bool DIRECT>
__device__ __forceinline__ float decode_code(const uint32_t (&w)[B], const float (&sc)[kMaxSlots],
                                             uint32_t magic) {
    constexpr CodePlan p = plan_code(B, J);
    if constexpr (DIRECT && p.shift_word < 0) {
        return __fmul_rn(code_to_float<B, p.o>(w[(J * B) >> 5], magic), sc[p.slot]);
    } else {
        constexpr int bit = J * B, wi = bit >> 5, o = bit & 31;
        uint32_t v;
        if constexpr (o == 0) v = w[wi];
        else if constexpr (o + B <= 32) v = w[wi] >> o;
        else v = __funnelshift_r(w[wi], w[wi + 1], o);
        return __fmul_rn(code_to_float<B, 0>(v, magic), sc[0]);
    }
}

// Integer-code variant (scale applied after accumulation): exact q as float.
template <int B, int J>
__device__ __forceinline__ float decode_code_int(const uint32_t (&w)[B], uint32_t magic) {
    constexpr int bit = J * B, wi = bit >> 5, o = bit & 31;
    uint32_t v;
    if constexpr (o == 0) v = w[wi];
    else if constexpr (o + B <= 32) v = w[wi] >> o;
    else v = __funnelshift_r(w[wi], w[wi + 1], o);
    return code_to_float<B, 0>(v, magic);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    uint32_t h;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
    return h;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------------------
// Paired exact dequantisation (b = 8..12, fullPrecision semantics)
// ---------------------------------------------------------------------------
// A lane's codes j and j + 16 feed the same row (fragment element e = j mod 8).
// Each code is read from a "view" of the lane's word string: its own word, or a
// funnel shift of its word pair, placed so that the code sits at an offset o
// with o + b <= 23 and so that codes j and j + 16 sit at the same o:
//   b <= 11: views start at codes 0, 2, 4, ...; code j at o = (j & 1) * b, so
//            one shift serves two codes;
//   b = 12:  a code at bit 0, 4 or 8 of its word is used in place, any other
//            code is shifted to bit 0 (16 * 12 is a multiple of 32, so codes j
//            and j + 16 have the same position within their words).
// With the float of exponent 23 - o, (view & mask << o) | exponent is exactly
// 2^(23-o) + code.  One f32x2 add of -(2^(23-o) + qmax) gives both codes' q
// exactly; one f32x2 RN multiply by (s, s) gives fp32_rn(q * s) for both, the
// reference's static_cast<float>(q) * scale; cvt.rn.f16x2 then rounds once to
// fp16 as __float2half_rn does.
template <int B>
struct PairPlan {
    static_assert(B >= 8 && B <= 12, "paired plan covers 8..12-bit codes");
    static constexpr int kOffsets = B <= 11 ? 2 : 3;
    static constexpr int off(int j) {
        return B <= 11 ? (j & 1) * B : (((j * B) & 31) + B <= 23 ? ((j * B) & 31) : 0);
    }
    static constexpr int view(int j) { return j * B - off(j); }  // first bit of the view
    static constexpr int off_index(int o) { return B <= 11 ? (o == 0 ? 0 : 1) : o / 4; }
    static constexpr int offset_at(int i) { return B <= 11 ? i * B : i * 4; }
};

// The 32 bits of the lane's word string starting at bit V (zeros past the end).
template <int B, int V>
__device__ __forceinline__ uint32_t view_word(const uint32_t (&w)[B]) {
    constexpr int wi = V >> 5, sh = V & 31;
    if constexpr (sh == 0) return w[wi];
    else if constexpr (wi + 1 >= B) return w[wi] >> sh;
    else return __funnelshift_r(w[wi], w[wi + 1], sh);
}

// Constants of the paired decode, built once per thread: magic[i] is the float
// 2^(23 - o_i) as bits, nbias[i] the pair (-(2^(23 - o_i) + qmax), same).
template <int B>
struct PairConsts {
    uint32_t magic[3];
    uint64_t nbias[3];
    // magic23: the bits of 2^23 (0x4B000000), passed in at run time so that
    // the compiler keeps the constants in registers
    __device__ __forceinline__ void init(uint32_t magic23) {
#pragma unroll
        for (int i = 0; i < PairPlan<B>::kOffsets; ++i) {
            const int o = PairPlan<B>::offset_at(i);
            magic[i] = magic23 - (uint32_t(o) << 23);
            const float nb = -(float(1u << (23 - o)) + float(qmax_for(B)));
            nbias[i] = pack2f(nb, nb);
        }
    }
};

// fp32_rn(q * s) of codes J and J + 16 (scale pair s2 = (s, s) of their row).
template <int B, int J>
__device__ __forceinline__ void dequant_pair(const uint32_t (&w)[B], const PairConsts<B>& k,
                                             uint64_t s2, float& lo, float& hi) {
    using PP = PairPlan<B>;
    constexpr int O = PP::off(J);
    static_assert(PP::off(J + 16) == O, "paired codes share their in-view offset");
    constexpr int I = PP::off_index(O);
    constexpr uint32_t kMask = ((1u << B) - 1u) << O;
    const uint32_t va = view_word<B, PP::view(J)>(w);
    const uint32_t vb = view_word<B, PP::view(J + 16)>(w);
    uint32_t ra, rb;
    asm("{\n\t.reg .b32 c0, c1;\n\t.reg .b64 a;\n\t"
        "lop3.b32 c0, %2, %4, %5, 0xEA;\n\t"
        "lop3.b32 c1, %3, %4, %5, 0xEA;\n\t"
        "mov.b64 a, {c0, c1};\n\t"
        "add.rn.f32x2 a, a, %6;\n\t"
        "mul.rn.f32x2 a, a, %7;\n\t"
        "mov.b64 {%0, %1}, a;\n\t}"
        : "=r"(ra), "=r"(rb)
        : "r"(va), "r"(vb), "n"(kMask), "r"(k.magic[I]), "l"(k.nbias[I]), "l"(s2));
    lo = __uint_as_float(ra);
    hi = __uint_as_float(rb);
}

// A-fragments of k-steps S and S + 2 (codes 8S..8S+7 and 8S+16..8S+23):
// register rr of a step holds codes 2rr, 2rr + 1 of that step (row r0 + 8 for rr odd).
template <int B, int S>
__device__ __forceinline__ void dequant_steps(const uint32_t (&w)[B], const PairConsts<B>& k,
                                              const uint64_t (&s2)[2], uint32_t (&af_lo)[4],
                                              uint32_t (&af_hi)[4]) {
    // register rr = codes 2rr, 2rr + 1: packed as soon as its two pairs are done
    // (keeps at most four unpacked floats live)
    float l0, l1, h0, h1;
    dequant_pair<B, 8 * S + 0>(w, k, s2[0], l0, h0);
    dequant_pair<B, 8 * S + 1>(w, k, s2[0], l1, h1);
    af_lo[0] = pack_half2(l0, l1);
    af_hi[0] = pack_half2(h0, h1);
    dequant_pair<B, 8 * S + 2>(w, k, s2[1], l0, h0);
    dequant_pair<B, 8 * S + 3>(w, k, s2[1], l1, h1);
    af_lo[1] = pack_half2(l0, l1);
    af_hi[1] = pack_half2(h0, h1);
    dequant_pair<B, 8 * S + 4>(w, k, s2[0], l0, h0);
    dequant_pair<B, 8 * S + 5>(w, k, s2[0], l1, h1);
    af_lo[2] = pack_half2(l0, l1);
    af_hi[2] = pack_half2(h0, h1);
    dequant_pair<B, 8 * S + 6>(w, k, s2[1], l0, h0);
    dequant_pair<B, 8 * S + 7>(w, k, s2[1], l1, h1);
    af_lo[3] = pack_half2(l0, l1);
    af_hi[3] = pack_half2(h0, h1);
}

}  // namespace ebx

namespace ebx {

// ---------------------------------------------------------------------------
// Plane layout (b = 9..12)
// ---------------------------------------------------------------------------
// Same supertiles, same 32 codes per lane, same b words per lane in the same
// vector segments as the bitstream layout above (so every size and offset is
// unchanged), but the bits of code j are split into planes so that the decode
// can build fp16 operands with byte permutes instead of per-code shifts:
//   low plane, words 0..7:  byte (j & 3) of word (j >> 2) = low 8 bits of code j;
//   high plane, words 8..b-1 = the remaining b - 8 bits of code j (bit k = bit 8+k):
//     b = 9:  bit 8*(j & 3) + (j >> 2) of word 8;
//     b = 10: bits 8*(j & 3) + 2*((j >> 2) & 3) + k of word 8 + (j >> 4);
//     b = 11: pair p = j >> 1 (codes 2p, 2p+1 share an A-fragment register),
//             side = j & 1: p < 15 -> bit 16*side + 3*(p % 5) + k of word 8 + p / 5;
//             p = 15 -> bit 15 + 16*side of word 8 + k;
//     b = 12: bit 16*side + 4*(p % 4) + k of word 8 + p / 4.
// For b = 9, 10 the high bits of codes 4i..4i+3 sit one per byte after one
// shift, so (shifted & mask) | 0x64646464 gives each code its fp16 upper byte
// (exponent of 1024 plus the top mantissa bits): one byte permute per pair then
// yields fp16(1024 + code) exactly.  For b = 11, 12 (codes up to 2046 / 4094
// do not fit one fp16 binade) the high part of a pair is one LOP3 away from
// fp16x2(1024 + hi) and q = 256 * (hi - h0) + (lo - l0) is one fp16 FMA, exact
// because every intermediate is an integer of magnitude below 2048.
// b = 8's bitstream layout already is the low plane alone.
__host__ __device__ constexpr bool plane_layout(int bits) { return bits >= 9 && bits <= 12; }

// Word and bit of high bit k (0 .. bits-9) of code j in the plane layout.
__host__ __device__ inline void plane_hi_bit(int bits, int j, int k, int* word, int* bit) {
    const int p = j >> 1, side = j & 1;
    if (bits == 9) {
        *word = 8;
        *bit = 8 * (j & 3) + (j >> 2);
    } else if (bits == 10) {
        *word = 8 + (j >> 4);
        *bit = 8 * (j & 3) + 2 * ((j >> 2) & 3) + k;
    } else if (bits == 11) {
        if (p < 15) {
            *word = 8 + p / 5;
            *bit = 16 * side + 3 * (p % 5) + k;
        } else {
            *word = 8 + k;
            *bit = 15 + 16 * side;
        }
    } else {
        *word = 8 + p / 4;
        *bit = 16 * side + 4 * (p % 4) + k;
    }
}

// fp16 bit pattern of a small integer (|n| < 2048, exactly representable).
__host__ __device__ constexpr uint32_t half_bits_int(int n) {
    const uint32_t sign = n < 0 ? 0x8000u : 0u;
    const uint32_t a = uint32_t(n < 0 ? -n : n);
    if (a == 0) return sign;
    int e = 0;
    while ((a >> (e + 1)) != 0) ++e;
    const uint32_t mant = ((a << (10 - e)) - 1024u) & 0x3FFu;
    return sign | (uint32_t(e + 15) << 10) | mant;
}
__host__ __device__ constexpr uint32_t half2_bits_int(int n) {
    return half_bits_int(n) | (half_bits_int(n) << 16);
}

template <uint32_t MASK>
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "n"(MASK), "r"(c));  // (a & MASK) | c
    return d;
}
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Constants of the plane decode, built once per thread from the run-time word
// 0x64646464 (kept in registers instead of being re-materialised per use).
struct PlaneConsts {
    uint32_t k64;    // 0x64646464: fp16 upper byte of 1024 in every byte
    uint32_t k6400;  // 0x64006400: fp16x2 (1024, 1024)
    __device__ __forceinline__ void init(uint32_t k64_word) {
        k64 = k64_word;
        k6400 = k64_word & 0xFF00FF00u;
    }
};

// Upper bytes (0x64 | high bits) of codes 4I .. 4I+3 (b = 9, 10); 0x64 bytes for b = 8.
template <int B, int I>
__device__ __forceinline__ uint32_t plane_hb(const uint32_t (&w)[B], const PlaneConsts& k) {
    if constexpr (B == 8) {
        return k.k64;
    } else if constexpr (B == 9) {
        return lop3_and_or<0x01010101u>(I == 0 ? w[8] : (w[8] >> I), k.k64);
    } else {
        static_assert(B == 10, "byte-plane high bits cover b = 9, 10");
        constexpr int sh = 2 * (I & 3);
        const uint32_t h = w[8 + (I >> 2)];
        return lop3_and_or<0x03030303u>(sh == 0 ? h : (h >> sh), k.k64);
    }
}

// fp16x2 (1024 + hi) of the high parts of pair P (b = 11, 12).
template <int B, int P>
__device__ __forceinline__ uint32_t plane_hi_pair(const uint32_t (&w)[B], const PlaneConsts& k) {
    if constexpr (B == 12) {
        constexpr int sh = 4 * (P % 4);
        const uint32_t h = w[8 + P / 4];
        return lop3_and_or<0x000F000Fu>(sh == 0 ? h : (h >> sh), k.k6400);
    } else {
        static_assert(B == 11, "pair high parts cover b = 11, 12");
        if constexpr (P < 15) {
            constexpr int sh = 3 * (P % 5);
            const uint32_t h = w[8 + P / 5];
            return lop3_and_or<0x00070007u>(sh == 0 ? h : (h >> sh), k.k6400);
        } else {
            uint32_t t = lop3_and_or<0x00010001u>(w[8] >> 15, k.k6400);
            t = lop3_and_or<0x00020002u>(w[9] >> 14, t);
            return lop3_and_or<0x00040004u>(w[10] >> 13, t);
        }
    }
}

// q = code - qmax of codes 2P, 2P+1 as exact fp16x2 (low half = code 2P), b = 8..12.
template <int B, int P>
__device__ __forceinline__ uint32_t plane_q16(const uint32_t (&w)[B], const PlaneConsts& k,
                                              uint32_t hb) {
    constexpr uint32_t kSel = (P & 1) ? 0x7362u : 0x5140u;
    if constexpr (B <= 10) {
        // (1024 + code) - (1024 + qmax)
        const uint32_t v = __byte_perm(w[P >> 1], hb, kSel);
        return hsub2_u(v, half2_bits_int(1024 + qmax_for(B)));
    } else {
        // qmax = 256 * h0 + l0 with h0 = 2^(B-9), l0 = -1
        constexpr int h0 = 1 << (B - 9);
        const uint32_t lo = hsub2_u(__byte_perm(w[P >> 1], k.k64, kSel), half2_bits_int(1023));
        const uint32_t hi = hsub2_u(plane_hi_pair<B, P>(w, k), half2_bits_int(1024 + h0));
        return hfma2_u(hi, half2_bits_int(256), lo);
    }
}

// Pairs 2I, 2I+1 (codes 4I .. 4I+3) of a lane's slice, exact fp16x2 q.
template <int B, int I>
__device__ __forceinline__ void plane_quad(const uint32_t (&w)[B], const PlaneConsts& k,
                                           uint32_t (&q16)[16]) {
    uint32_t hb = 0;
    if constexpr (B <= 10) hb = plane_hb<B, I>(w, k);
    q16[2 * I] = plane_q16<B, 2 * I>(w, k, hb);
    q16[2 * I + 1] = plane_q16<B, 2 * I + 1>(w, k, hb);
}

// All 16 pairs of a lane's slice: q16[p] = fp16x2 q of codes 2p, 2p+1
// (A-fragment register p: k-step p / 4, register p % 4).
template <int B>
__device__ __forceinline__ void plane_q16_all(const uint32_t (&w)[B], const PlaneConsts& k,
                                              uint32_t (&q16)[16]) {
    plane_quad<B, 0>(w, k, q16);
    plane_quad<B, 1>(w, k, q16);
    plane_quad<B, 2>(w, k, q16);
    plane_quad<B, 3>(w, k, q16);
    plane_quad<B, 4>(w, k, q16);
    plane_quad<B, 5>(w, k, q16);
    plane_quad<B, 6>(w, k, q16);
    plane_quad<B, 7>(w, k, q16);
}

// Exact W16 operand from an exact q pair: fp16_rn(fp32_rn(float(q) * s)) for
// both halves (the reference's static_cast<float>(q) * scale, then
// __float2half_rn); s2 = (s, s) of the pair's row.
__device__ __forceinline__ uint32_t q16_to_w16(uint32_t q16, uint64_t s2) {
    uint32_t h;
    asm("{\n\t.reg .b16 l, u;\n\t.reg .f32 fl, fu;\n\t.reg .b64 a;\n\t"
        "mov.b32 {l, u}, %1;\n\t"
        "cvt.f32.f16 fl, l;\n\t"
        "cvt.f32.f16 fu, u;\n\t"
        "mov.b64 a, {fl, fu};\n\t"
        "mul.rn.f32x2 a, a, %2;\n\t"
        "mov.b64 {fl, fu}, a;\n\t"
        "cvt.rn.f16x2.f32 %0, fu, fl;\n\t}"
        : "=r"(h)
        : "r"(q16), "l"(s2));
    return h;
}

}  // namespace ebx
