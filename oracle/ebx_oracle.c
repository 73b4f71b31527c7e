/*
 * ebx_oracle.c -- CPU restatement of MLBricks ElasticBit storage arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in mlbricks_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference leg of bench.py may load it.  The product
 * path never calls it and never falls back to it.
 *
 * Every function restates one piece of the reference runtime
 * (mlbricks/elasticbit/csrc/elasticbit_runtime.cu, cited as "cu:<line>") in
 * plain C.  Floating-point order of operations is kept identical to the
 * reference host code (float products and sums in index order, long double
 * error norms) so the analyzer reproduces the reference's selected bits and
 * error values exactly when compiled with -ffp-contract=off on x86-64.
 *
 * Parity pins: tests/golden/ holds outputs of the reference's own compiled
 * host analyzer (_C.analyze) produced by tests/golden/make_golden.py; the
 * oracle's analyzer is checked against them bit-for-bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EBO_MIN_BITS 3
#define EBO_MAX_BITS 15
#define EBO_FP16_BITS 16

/* qmax = 2^(b-1) - 1  (cu:64-67) */
uint32_t ebo_qmax(int bits) {
    if (bits >= 32) return 0x7fffffffu;
    return (1u << (bits - 1)) - 1u;
}

/* ceil(count * b / 8)  (cu:69-71) */
uint64_t ebo_packed_bytes(uint64_t count, int bits) {
    return (count * (uint64_t)bits + 7u) / 8u;
}

/* float -> fp16 (round to nearest even, IEEE subnormals) -> float  (cu:73-75).
 * gcc's _Float16 conversion on x86-64 is correctly rounded RN-even. */
float ebo_round_fp16(float v) {
    return (float)(_Float16)v;
}

uint16_t ebo_fp16_bits(float v) {
    _Float16 h = (_Float16)v;
    uint16_t b;
    memcpy(&b, &h, 2);
    return b;
}

float ebo_fp16_to_float(uint16_t b) {
    _Float16 h;
    memcpy(&h, &b, 2);
    return (float)h;
}

/* q = clamp(nearbyint(v / s), -qmax, qmax)  (cu:77-81; core.py:153-155) */
int32_t ebo_quantize_scalar(float value, float scale, int bits) {
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    const float ratio = value / scale;
    int32_t q = (int32_t)nearbyintf(ratio);
    if (q < -qmax) q = -qmax;
    if (q > qmax) q = qmax;
    return q;
}

/* per-row scale = max|w| / qmax, or 1.0 for an all-zero row  (cu:83-101;
 * core.py:143-151).  Returns 0 on success. */
int ebo_row_scales(const float* w, int rows, int cols, int bits, float* out) {
    if (bits == EBO_FP16_BITS) return 0;
    const float qmax = (float)ebo_qmax(bits);
    for (int r = 0; r < rows; ++r) {
        const float* p = w + (size_t)r * cols;
        float m = 0.0f;
        for (int c = 0; c < cols; ++c) {
            const float a = fabsf(p[c]);
            if (a > m) m = a;
        }
        out[r] = m > 0.0f ? m / qmax : 1.0f;
    }
    return 0;
}

/* OR one b-bit code into the LSB-first little-endian bitstream at element
 * index i (bit offset i*b).  Shared by both packers. */
static void put_code(uint8_t* payload, uint64_t nbytes, uint64_t i, int bits, uint32_t code) {
    const uint64_t bit = i * (uint64_t)bits;
    const uint64_t byte0 = bit >> 3;
    const uint64_t v = (uint64_t)code << (bit & 7u);
    for (int j = 0; j < 3; ++j) {
        if (byte0 + (uint64_t)j < nbytes) payload[byte0 + j] |= (uint8_t)(v >> (8 * j));
    }
}

/* Pack signed codes q (|q| <= qmax) as q + qmax.  (cu:150-186)
 * payload must hold ebo_packed_bytes(rows*cols, bits) zeroed bytes.
 * Returns 0, or 1 if a code is out of range, or 2 for an invalid width. */
int ebo_pack_codes(const int16_t* codes, int rows, int cols, int bits, uint8_t* payload) {
    if (bits < EBO_MIN_BITS || bits > EBO_MAX_BITS) return 2;
    const uint64_t count = (uint64_t)rows * (uint64_t)cols;
    const uint64_t nbytes = ebo_packed_bytes(count, bits);
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    memset(payload, 0, nbytes);
    for (uint64_t i = 0; i < count; ++i) {
        const int32_t q = codes[i];
        if (q < -qmax || q > qmax) return 1;
        put_code(payload, nbytes, i, bits, (uint32_t)(q + qmax));
    }
    return 0;
}

/* Quantize-and-pack float weights with given row scales; 16 bits stores raw
 * fp16.  (cu:103-148)  payload must be sized for the width. */
int ebo_pack_weights(const float* w, int rows, int cols, int bits, const float* scales,
                     uint8_t* payload) {
    if (bits < EBO_MIN_BITS || bits > EBO_FP16_BITS) return 2;
    const uint64_t count = (uint64_t)rows * (uint64_t)cols;
    if (bits == EBO_FP16_BITS) {
        for (uint64_t i = 0; i < count; ++i) {
            const uint16_t h = ebo_fp16_bits(w[i]);
            memcpy(payload + 2 * i, &h, 2);
        }
        return 0;
    }
    const uint64_t nbytes = ebo_packed_bytes(count, bits);
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    memset(payload, 0, nbytes);
    for (int r = 0; r < rows; ++r) {
        for (int c = 0; c < cols; ++c) {
            const uint64_t i = (uint64_t)r * cols + c;
            const int32_t q = ebo_quantize_scalar(w[i], scales[r], bits);
            put_code(payload, nbytes, i, bits, (uint32_t)(q + qmax));
        }
    }
    return 0;
}

/* Read the b-bit code of element i.  (cu:188-206) */
uint32_t ebo_extract_code(const uint8_t* payload, uint64_t nbytes, uint64_t i, int bits) {
    const uint64_t bit = i * (uint64_t)bits;
    const uint64_t byte0 = bit >> 3;
    uint32_t word = 0;
    for (int j = 0; j < 3; ++j) {
        if (byte0 + (uint64_t)j < nbytes) word |= (uint32_t)payload[byte0 + j] << (8 * j);
    }
    return (word >> (bit & 7u)) & ((1u << bits) - 1u);
}

/* Unpack signed codes (q = code - qmax) into int16.  Inverse of ebo_pack_codes. */
int ebo_unpack_codes(const uint8_t* payload, uint64_t nbytes, int rows, int cols, int bits,
                     int16_t* out) {
    if (bits < EBO_MIN_BITS || bits > EBO_MAX_BITS) return 2;
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    const uint64_t count = (uint64_t)rows * (uint64_t)cols;
    for (uint64_t i = 0; i < count; ++i) {
        out[i] = (int16_t)((int32_t)ebo_extract_code(payload, nbytes, i, bits) - qmax);
    }
    return 0;
}

/* W16[n,k] = fp16(fp32(q) * s_n) as float; raw fp16 for 16-bit storage.
 * (cu:208-238; core.py:156) */
int ebo_dequantize(const uint8_t* payload, uint64_t nbytes, const float* scales, int rows,
                   int cols, int bits, float* out) {
    const uint64_t count = (uint64_t)rows * (uint64_t)cols;
    if (bits == EBO_FP16_BITS) {
        for (uint64_t i = 0; i < count; ++i) {
            uint16_t h;
            memcpy(&h, payload + 2 * i, 2);
            out[i] = ebo_fp16_to_float(h);
        }
        return 0;
    }
    if (bits < EBO_MIN_BITS || bits > EBO_MAX_BITS) return 2;
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    for (int r = 0; r < rows; ++r) {
        const float s = scales[r];
        for (int c = 0; c < cols; ++c) {
            const uint64_t i = (uint64_t)r * cols + c;
            const int32_t q = (int32_t)ebo_extract_code(payload, nbytes, i, bits) - qmax;
            out[i] = ebo_round_fp16((float)q * s);
        }
    }
    return 0;
}

/* Same as ebo_dequantize, but emits the fp16 bit patterns. */
int ebo_dequantize_fp16(const uint8_t* payload, uint64_t nbytes, const float* scales, int rows,
                        int cols, int bits, uint16_t* out) {
    const uint64_t count = (uint64_t)rows * (uint64_t)cols;
    if (bits == EBO_FP16_BITS) {
        memcpy(out, payload, 2 * count);
        return 0;
    }
    if (bits < EBO_MIN_BITS || bits > EBO_MAX_BITS) return 2;
    const int32_t qmax = (int32_t)ebo_qmax(bits);
    for (int r = 0; r < rows; ++r) {
        const float s = scales[r];
        for (int c = 0; c < cols; ++c) {
            const uint64_t i = (uint64_t)r * cols + c;
            const int32_t q = (int32_t)ebo_extract_code(payload, nbytes, i, bits) - qmax;
            out[i] = ebo_fp16_bits((float)q * s);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------
 * Host analyzer: error of every width 3..16 against the fp16 reference.
 * (cu:280-436)  Outputs arrays of 14 entries indexed by bits-3.
 * ---------------------------------------------------------------------- */

/* Reference outputs ref[s*rows + r] = sum_c fp16(w) * fp16(x), float sum in
 * column order.  (cu:280-309) */
static void fp16_reference(const float* w, int rows, int cols, const float* calib, int samples,
                           float* ref, float* wh, float* xh) {
    const uint64_t count = (uint64_t)rows * cols;
    for (uint64_t i = 0; i < count; ++i) wh[i] = ebo_round_fp16(w[i]);
    for (int s = 0; s < samples; ++s) {
        const float* in = calib + (size_t)s * cols;
        for (int c = 0; c < cols; ++c) xh[c] = ebo_round_fp16(in[c]);
        for (int r = 0; r < rows; ++r) {
            const float* p = wh + (size_t)r * cols;
            float acc = 0.0f;
            for (int c = 0; c < cols; ++c) acc += p[c] * xh[c];
            ref[(size_t)s * rows + r] = acc;
        }
    }
}

/* One width.  (cu:311-392) */
static void analyze_width(const float* w, int rows, int cols, const float* calib, int samples,
                          const float* ref, int bits, float* scales, float* xh, double* hw_err,
                          double* full_err, uint64_t* storage) {
    if (bits != EBO_FP16_BITS) ebo_row_scales(w, rows, cols, bits, scales);
    long double hw_num = 0.0L, full_num = 0.0L, den = 0.0L;
    for (int s = 0; s < samples; ++s) {
        const float* in = calib + (size_t)s * cols;
        for (int c = 0; c < cols; ++c) xh[c] = ebo_round_fp16(in[c]);
        for (int r = 0; r < rows; ++r) {
            const float* p = w + (size_t)r * cols;
            float hw = 0.0f, full = 0.0f;
            if (bits == EBO_FP16_BITS) {
                for (int c = 0; c < cols; ++c) hw += ebo_round_fp16(p[c]) * xh[c];
                full = hw;
            } else if (bits <= 8) {
                const float sc = scales[r];
                float idot = 0.0f;
                for (int c = 0; c < cols; ++c) {
                    const int32_t q = ebo_quantize_scalar(p[c], sc, bits);
                    idot += (float)q * xh[c];
                    full += ebo_round_fp16((float)q * sc) * xh[c];
                }
                hw = idot * sc;
            } else {
                const float sc = scales[r];
                for (int c = 0; c < cols; ++c) {
                    const int32_t q = ebo_quantize_scalar(p[c], sc, bits);
                    hw += ebo_round_fp16((float)q * sc) * xh[c];
                }
                full = hw;
            }
            const double rv = ref[(size_t)s * rows + r];
            const double dh = (double)hw - rv;
            const double df = (double)full - rv;
            hw_num += (long double)dh * dh;
            full_num += (long double)df * df;
            den += (long double)rv * rv;
        }
    }
    const long double safe = den > 1.0e-30L ? den : 1.0e-30L;
    *hw_err = sqrt((double)(hw_num / safe));
    *full_err = sqrt((double)(full_num / safe));
    const uint64_t count = (uint64_t)rows * cols;
    *storage = bits == EBO_FP16_BITS ? count * 2u
                                     : ebo_packed_bytes(count, bits) + (uint64_t)rows * 4u;
}

/* Analyze widths 3..16.  Arrays hold 14 entries (index bits-3).
 * Returns 0, or 1 for empty inputs.  (cu:394-415) */
int ebo_analyze(const float* w, int rows, int cols, const float* calib, int samples,
                double* hw_err, double* full_err, double* err, uint64_t* storage) {
    if (rows <= 0 || cols <= 0 || samples <= 0) return 1;
    float* ref = (float*)malloc(sizeof(float) * (size_t)samples * rows);
    float* wh = (float*)malloc(sizeof(float) * (size_t)rows * cols);
    float* xh = (float*)malloc(sizeof(float) * (size_t)cols);
    float* sc = (float*)malloc(sizeof(float) * (size_t)rows);
    if (!ref || !wh || !xh || !sc) {
        free(ref); free(wh); free(xh); free(sc);
        return 3;
    }
    fp16_reference(w, rows, cols, calib, samples, ref, wh, xh);
    for (int bits = EBO_MIN_BITS; bits <= EBO_FP16_BITS; ++bits) {
        const int i = bits - EBO_MIN_BITS;
        analyze_width(w, rows, cols, calib, samples, ref, bits, sc, xh, &hw_err[i], &full_err[i],
                      &storage[i]);
        err[i] = hw_err[i] > full_err[i] ? hw_err[i] : full_err[i];
    }
    free(ref); free(wh); free(xh); free(sc);
    return 0;
}

/* First width 3..15 whose error is within the threshold, else 16.
 * Returns -1 for an invalid threshold.  (cu:417-436) */
int ebo_select(const double* err, double threshold) {
    if (!isfinite(threshold) || threshold < 0.0) return -1;
    for (int bits = EBO_MIN_BITS; bits <= EBO_MAX_BITS; ++bits) {
        if (err[bits - EBO_MIN_BITS] <= threshold) return bits;
    }
    return EBO_FP16_BITS;
}

/* ------------------------------------------------------------------------
 * Forward semantics (the quantities the CUDA kernels must reproduce).
 * ---------------------------------------------------------------------- */

/* fullPrecision / W16A16: y[m,n] = sum_k fp32(x16[m,k]) * W16[n,k], summed in
 * double so it serves as the tolerance reference for any fp32 summation order.
 * (cu:614-648 per row; core.py:471 F.linear on the materialised weight) */
void ebo_linear_full(const uint16_t* x16, int64_t M, const float* w16f, int N, int K,
                     const float* bias, double* y) {
    for (int64_t m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            const float* wr = w16f + (size_t)n * K;
            const uint16_t* xr = x16 + (size_t)m * K;
            for (int k = 0; k < K; ++k) acc += (double)ebo_fp16_to_float(xr[k]) * (double)wr[k];
            if (bias) acc += (double)bias[n];
            y[(size_t)m * N + n] = acc;
        }
    }
}

/* hardwareNative low-bit (W8A16/W4A16): y = s_n * sum_k x * q, integer codes
 * accumulated first, scale after.  (cu:508-609; core.py:166-170) */
void ebo_linear_hw(const uint16_t* x16, int64_t M, const int16_t* q, const float* scales, int N,
                   int K, const float* bias, double* y) {
    for (int64_t m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            double acc = 0.0;
            const int16_t* qr = q + (size_t)n * K;
            const uint16_t* xr = x16 + (size_t)m * K;
            for (int k = 0; k < K; ++k) acc += (double)ebo_fp16_to_float(xr[k]) * (double)qr[k];
            acc *= (double)scales[n];
            if (bias) acc += (double)bias[n];
            y[(size_t)m * N + n] = acc;
        }
    }
}

/* The registered-but-unused reference operator mlbricks_native::
 * elastic_linear_packed: q = uq - 2^(b-1), scale index = flat / group_size,
 * float accumulation in k order, bias added before the final rounding.
 * (mlbricks/bolt/ops_cuda.cu:2708-2750)  x and out are float here. */
void ebo_elastic_linear_packed(const float* x, int64_t rows, const uint8_t* packed,
                               const float* scales, const float* bias, int bits,
                               int64_t group_size, int64_t out_features, int64_t in_features,
                               float* out) {
    const int mask = (1 << bits) - 1;
    const int qmin = -(1 << (bits - 1));
    for (int64_t m = 0; m < rows; ++m) {
        for (int64_t o = 0; o < out_features; ++o) {
            float acc = 0.0f;
            for (int64_t k = 0; k < in_features; ++k) {
                const int64_t wi = o * in_features + k;
                const int64_t bp = wi * bits;
                const int64_t by = bp >> 3;
                const int off = (int)(bp & 7);
                uint32_t word = packed[by];
                if (off + bits > 8) word |= (uint32_t)packed[by + 1] << 8;
                const int q = (int)((word >> off) & (uint32_t)mask) + qmin;
                const float wv = (float)q * scales[wi / group_size];
                acc += x[m * in_features + k] * wv;
            }
            if (bias) acc += bias[o];
            out[m * out_features + o] = acc;
        }
    }
}

/* FNV-1a 64 over a byte range.  (cu:682-690) */
uint64_t ebo_fnv1a64(const uint8_t* data, uint64_t size) {
    uint64_t h = 1469598103934665603ull;
    for (uint64_t i = 0; i < size; ++i) {
        h ^= (uint64_t)data[i];
        h *= 1099511628211ull;
    }
    return h;
}
