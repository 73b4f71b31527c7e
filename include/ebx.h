/*
 * ebx.h -- C ABI of libebx, the B200-native ElasticBit compressed-linear runtime.
 *
 * Plain C: opaque handles, raw pointers, sizes and integer status codes; no
 * C++ exceptions or torch types cross this boundary.  `stream` arguments are
 * cudaStream_t values passed as void* (NULL = legacy default stream).  Every
 * device-side entry point is stream-ordered.  Calls on one matrix handle from
 * several host threads are safe as long as each call uses its own output
 * buffers; creation/destruction of a handle must not race with its use.
 *
 * Reference interfaces replaced (paths inside the MLBricks tree):
 *   mlbricks/elasticbit/csrc/elasticbit_runtime.cu  -- pybind module _C,
 *       class RuntimeMatrix (cu:714-1384, bindings cu:1411-1469)
 *   mlbricks/bolt/ops.cpp:1012-1043,1132  -- op mlbricks_native::
 *       elastic_linear_packed, kernel mlbricks/bolt/ops_cuda.cu:2708-2796
 */
#ifndef EBX_H_
#define EBX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define EBX_API __attribute__((visibility("default")))
#else
#define EBX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  ebx_last_error() gives the message of the calling thread's
 * most recent failure. */
typedef enum {
    EBX_OK = 0,
    EBX_ERR_INVALID = 1,     /* bad argument (reference: std::invalid_argument -> ValueError) */
    EBX_ERR_CUDA = 2,        /* CUDA runtime failure (reference: CUDA_CHECK -> RuntimeError)  */
    EBX_ERR_UNSUPPORTED = 3, /* shape/width this build does not execute                        */
    EBX_ERR_WORKSPACE = 4,   /* caller workspace missing or too small                          */
    EBX_ERR_CODE_RANGE = 5   /* a prequantized code lies outside [-qmax, qmax]                 */
} ebx_status;

typedef struct ebx_matrix ebx_matrix;

/* Matrix description returned by ebx_matrix_query. */
typedef struct {
    int32_t rows;              /* N (out_features)                                  */
    int32_t cols;              /* K (in_features)                                   */
    int32_t storage_bits;      /* 3..15, or 16 for the FP16 fallback                */
    int32_t execution_width;   /* 16, 8 or 4 (see ebx_matrix_set_execution_width)   */
    int32_t device;            /* CUDA ordinal that owns the buffers                */
    int32_t reserved;
    uint64_t payload_bytes;    /* MLB4 payload size: ceil(N*K*b/8), or 2*N*K for b=16 */
    uint64_t device_bytes;     /* resident device bytes (tile codes + scales)       */
} ebx_matrix_info;

/* Library version string, e.g. "ebx 0.1.0 sm_100a". */
EBX_API const char* ebx_version(void);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len-1) and returns the full message length. */
EBX_API size_t ebx_last_error(char* buf, size_t len);

/* Create from the analyzer's selected signed codes q (int16, row-major
 * [rows, cols], DEVICE pointer) and per-row fp32 scales (DEVICE pointer),
 * 3 <= bits <= 15.  Packing runs on the device.
 * Replaces RuntimeMatrix._compressSelectedCodes -> pack_exact_codes
 * (elasticbit_runtime.cu:778-808, 150-186).  Returns EBX_ERR_CODE_RANGE when
 * any |q| > qmax (cu:168-170).  Synchronizes `stream`. */
EBX_API ebx_status ebx_matrix_create_from_codes(const int16_t* codes, const float* scales, int32_t rows,
                                        int32_t cols, int32_t bits, int32_t device, void* stream,
                                        ebx_matrix** out);

/* Create from an MLB4 payload (LSB-first bitstream of q+qmax codes, or raw
 * fp16 for bits == 16) and per-row scales (ignored for bits == 16).
 * `on_device` = 1: both pointers are device memory; 0: host memory.
 * Replaces the RuntimeMatrix(rows, cols, bits, ..., scales, payload)
 * constructor behind RuntimeMatrix.load (cu:810-871, 1143-1157). */
EBX_API ebx_status ebx_matrix_create_from_payload(const void* payload, uint64_t payload_bytes,
                                          const float* scales, int32_t rows, int32_t cols,
                                          int32_t bits, int32_t on_device, int32_t device,
                                          void* stream, ebx_matrix** out);

/* Create a 16-bit (FP16 fallback) matrix from row-major fp16 weights (DEVICE).
 * Replaces RuntimeMatrix._compressSelected with selectedBits = 16
 * (cu:748-776, pack_exact_weights cu:113-120). */
EBX_API ebx_status ebx_matrix_create_from_fp16(const void* weights, int32_t rows, int32_t cols,
                                       int32_t device, void* stream, ebx_matrix** out);

/* Release the handle and its device buffers (cu:716, 1370-1383). */
EBX_API ebx_status ebx_matrix_destroy(ebx_matrix* m);

EBX_API ebx_status ebx_matrix_query(const ebx_matrix* m, ebx_matrix_info* info);

/* Select execution semantics (cu:240-244, 1174-1178, 1315-1334):
 * 16 = fp16(q*s) operands (W16A16 / fullPrecision), 8 or 4 = integer codes with
 * the row scale applied after accumulation (W8A16 / W4A16).  8 requires
 * bits <= 8, 4 requires bits <= 4.  The stored code is the same either way. */
EBX_API ebx_status ebx_matrix_set_execution_width(ebx_matrix* m, int32_t width);

/* Write the MLB4 payload bitstream (payload_bytes bytes) to `dst` (DEVICE).
 * Replaces the payload half of RuntimeMatrix.save (cu:1024-1049). */
EBX_API ebx_status ebx_matrix_export_payload(const ebx_matrix* m, void* dst, uint64_t dst_bytes,
                                     void* stream);

/* Copy the rows fp32 scales to `dst` (DEVICE).  No-op for bits == 16. */
EBX_API ebx_status ebx_matrix_export_scales(const ebx_matrix* m, float* dst, void* stream);

/* Exact dequantised weight, row-major fp16 [rows, cols] into `dst` (DEVICE):
 * W[n,k] = fp16_rn(fp32(q) * s_n).  Replaces RuntimeMatrix._materializeTorch
 * (cu:982-1022) and the values of RuntimeMatrix.dequantize (cu:208-238). */
EBX_API ebx_status ebx_matrix_materialize(const ebx_matrix* m, void* dst, void* stream);

/* Workspace bytes ebx_linear asks for with M activation rows (0 when none):
 * the decode-GEMM's fp32 split-K partials for 16 < M <= 256 (required when
 * nonzero), and for larger M room for the exactly dequantised fp16 weight
 * followed by the fp32 partial tiles of the GEMM's split last wave --
 * optional: with it the prefill takes materialise + tcgen05 GEMM (the faster
 * route; fp16(q*s) operands, the reference's prefill arithmetic, whatever the
 * execution width; given only the fp16 weight's rows*cols*2 bytes, rounded up to
 * 256, the GEMM runs without the split), without it (NULL or smaller) the
 * prefill decode-GEMM, which decodes the codes into shared memory per k-block,
 * needs no memory at all and keeps the execution width's semantics.  The
 * workspace_bytes passed to ebx_linear must not exceed the buffer's size. */
EBX_API uint64_t ebx_linear_workspace_bytes(const ebx_matrix* m, int64_t M);

/* y[M, rows] = x[M, cols] * W^T (+ bias), all fp16 DEVICE pointers, row-major,
 * contiguous; bias may be NULL; y32 (fp32 [M, rows]) may be NULL and receives
 * the fp32 value that was rounded into y.  Replaces _ElasticLinear.forward's
 * two routes (core.py:446-471): RuntimeMatrix.forwardTorch (cu:902-931) for
 * M = 1 and materialise + F.linear for M > 1.  Routes by M: the decode kernel
 * (M <= 16, in 16-row launches where the decode-GEMM does not apply), the
 * decode-GEMM (16 < M <= 256: codes decoded into tcgen05 tiles), and for larger
 * M materialise + tcgen05 GEMM (given the optional workspace) or the prefill
 * decode-GEMM; workspace as ebx_linear_workspace_bytes says. */
EBX_API ebx_status ebx_linear(const ebx_matrix* m, const void* x, int64_t M, const void* bias, void* y,
                      float* y32, void* workspace, uint64_t workspace_bytes, void* stream);

/* Workspace bytes for ebx_analyze (fp16 reference outputs + per-row partial
 * sums). */
EBX_API uint64_t ebx_analyze_workspace_bytes(int32_t rows, int32_t samples);

/* Matrix-path width analysis on the device: for every width 3..16 the
 * hardwareNative and fullPrecision relative-L2 errors against the fp16
 * reference, written to hw_err[14] / full_err[14] (DEVICE, index bits-3).
 * weights fp32 [rows, cols], calib fp32 [samples, cols] (DEVICE).
 * Replaces the host analyzer analyze_all_bits (elasticbit_runtime.cu:280-415)
 * behind _C.analyze and RuntimeMatrix.compress (cu:438-483, 720-746). */
EBX_API ebx_status ebx_analyze(const float* weights, int32_t rows, int32_t cols, const float* calib,
                       int32_t samples, double* hw_err, double* full_err, void* workspace,
                       uint64_t workspace_bytes, void* stream);

/* Allocation-free form of ebx_analyze, for callers that cannot allocate
 * device memory (their memory belongs to a host framework's fixed pool with no
 * workspace to hand out, or they must avoid the device synchronisation that
 * cudaMalloc/cudaFree can cause).  No counterpart in the reference: its
 * analyzer runs on the host.  Same inputs, outputs and results as
 * ebx_analyze; the scratch is a fixed 8 MiB array inside the library that
 * every GPU loading it keeps until the process exits, so the call needs
 * 256-byte-rounded 4*rows*samples + 336*rows bytes <= 8 MiB (e.g. 8192 rows x
 * 32 samples) and returns EBX_ERR_INVALID with a message beyond that (an
 * argument-size error, unlike ebx_analyze's EBX_ERR_WORKSPACE, which reports a
 * caller workspace that is too small).  The first call on a device looks up
 * the array's device address (with that device current) and keeps it for the
 * life of the process; make that first call before any stream capture, and
 * make no call after a cudaDeviceReset of that device (the reset frees the
 * array and the kept address goes stale, like every other device object of
 * this library).  All
 * calls on a device share the array: calls whose kernels overlap on the GPU
 * (different streams without ordering) race and give wrong results. */
EBX_API ebx_status ebx_analyze_noalloc(const float* weights, int32_t rows, int32_t cols,
                                       const float* calib, int32_t samples, double* hw_err,
                                       double* full_err, void* stream);

/* Quantise fp32 weights [rows, cols] (DEVICE) for width 3..15: per-row scale
 * max|w|/qmax (1 for a zero row) and codes clamp(rint(w/s), +-qmax), written
 * to codes (int16 DEVICE) and scales (fp32 DEVICE).  Replaces make_row_scales +
 * quantize_scalar (cu:77-101) inside RuntimeMatrix._compressSelected. */
EBX_API ebx_status ebx_quantize(const float* weights, int32_t rows, int32_t cols, int32_t bits,
                        int16_t* codes, float* scales, void* stream);

/* fp32 -> fp16 (round to nearest even) of n values, DEVICE to DEVICE
 * (the 16-bit storage of pack_exact_weights, cu:113-120). */
EBX_API ebx_status ebx_weights_to_fp16(const float* weights, int64_t n, void* out, void* stream);

/* Device health word of `device`: 0 = healthy, nonzero = a kernel's bounded
 * wait (on a TMA copy, or on a peer's exchange flag) gave up (the kernel then
 * returned early; its outputs are unspecified).  `clear` = 1 resets it.
 * Synchronizes the device's legacy stream.  No reference counterpart: the
 * reference kernels never wait. */
EBX_API ebx_status ebx_device_status(int32_t device, int32_t* status, int32_t clear);

/* FNV-1a 64 of a HOST byte range: the MLB4 scale/payload checksum
 * (elasticbit_runtime.cu:682-690, written at cu:1036-1037, checked at
 * cu:857-863). */
EBX_API uint64_t ebx_fnv1a64(const void* data, uint64_t size);

/* Drop-in for the dispatcher op mlbricks_native::elastic_linear_packed
 * (ops.cpp:1012-1043; ops_cuda.cu:2708-2796): packed LSB-first codes with
 * q = uq - 2^(bits-1), 2 <= bits <= 8, scale index = flat_index / group_size.
 * dtype codes: 0 = fp32, 1 = fp16, 2 = bf16.  x, bias and out share x_dtype;
 * bias may be NULL.  rows = x.numel / in_features. */
EBX_API ebx_status ebx_elastic_linear_packed(const void* x, int32_t x_dtype, int64_t rows,
                                     const uint8_t* packed, const void* scales,
                                     int32_t scale_dtype, const void* bias, int32_t bits,
                                     int64_t group_size, int64_t out_features,
                                     int64_t in_features, void* out, void* stream);

/* SwiGLU projection for decode batches: m holds a gate and an up projection
 * with their rows interleaved in blocks of 8 (rows 16j..16j+7 = gate rows
 * 8j..8j+7, rows 16j+8..16j+15 = up rows 8j..8j+7; rows % 16 == 0), and
 * y[M, rows/2] = fp16( silu(g) * u ) with g, u the fp32 sums x @ W^T (+ bias,
 * in the same interleaved order, may be NULL) before any rounding.  One launch
 * replaces "gate/up GEMV, silu, multiply".  1 <= M <= 16; y32 (fp32 copy, may be
 * NULL).  No reference counterpart (the reference computes gate and up as two
 * linears and the activation in PyTorch). */
EBX_API ebx_status ebx_linear_swiglu(const ebx_matrix* m, const void* x, int64_t M, const void* bias,
                                     void* y, float* y32, void* stream);

/* Several matrices that read the same activations -- Q, K and V projections,
 * or gate and up -- each with its own storage width, scales, execution
 * semantics and bias, in ONE decode launch: ys[i][M, rows_i] = x[M, cols] *
 * W_i^T (+ biases[i]), i < count.  Replaces the reference's fused multi-matrix
 * execution, which concatenates the dequantised FP16 weights of such a group
 * into one matrix for a single GEMM (mlbricks/elasticbit/stage2f.py:382-420);
 * here the codes stay at their own widths.  1 <= count <= 8, 0 <= M <= 16,
 * every matrix on one device with the same cols; biases, y32s (and their
 * entries) may be NULL.  EBX_ERR_UNSUPPORTED (nothing launched) unless every
 * storage width is 8..12, cols % 64 == 0 and x is 16-byte aligned: run such
 * matrices with ebx_linear. */
EBX_API ebx_status ebx_linear_multi(const ebx_matrix* const* mats, int32_t count, const void* x,
                                    int64_t M, const void* const* biases, void* const* ys,
                                    float* const* y32s, void* stream);

/* ---- Tensor-parallel exchange (row-parallel linear + all-reduce) ----------
 * No reference counterpart: the reference has no distributed code.  These
 * replace "row-parallel shard GEMV, then an NCCL all-reduce of the fp32
 * partials, then bias and one fp16 rounding" for decode-sized M (<= 16) with
 * a one-shot exchange over NVLink peer memory, one process per GPU:
 *
 *   1. every rank: ebx_exchange_create -> a device region (flags + two slots
 *      of world * max_m * max_n fp32 partials) and an opaque handle blob of
 *      EBX_EXCHANGE_HANDLE_BYTES (CUDA IPC handle, GPU UUID, shape);
 *   2. the caller all-gathers the blobs (any host transport) and passes all
 *      of them, in rank order, to ebx_exchange_connect, which maps every
 *      peer's region (cudaIpcOpenMemHandle);
 *   3. ebx_linear_allreduce: the shard's decode kernel stores each fp32
 *      partial sum, tagged with the exchange's epoch in the same 8-byte word,
 *      into the regions of the ranks that need it; readers poll the words
 *      themselves (bounded, ~2 s), sum all ranks' partials in rank order
 *      0..world-1, add bias in fp32 and round once to fp16.  Every rank gets
 *      bit-identical outputs.  When the grid fits on the GPU this all happens
 *      inside the decode launch (cooperative); otherwise a finish kernel sums.
 *      Two protocols (ebx_exchange_set_protocol): broadcast -- every partial
 *      into every rank's region, one hop, world x M x N words per rank -- and
 *      two-phase -- each output's partials to one owner rank, which sums them
 *      and stores the sum into every other rank's region, about 2 x M x N words
 *      per rank for a second hop.  Both give the same bits.
 *
 * All ranks must issue the same sequence of ebx_linear_allreduce calls, each
 * call with the same M and shard shape on every rank; M and the shard's rows
 * may change from one call to the next (up to max_m and max_n), because the
 * two partial slots are laid out with the exchange's fixed max_m * max_n
 * stride.  The epoch lives in device memory, so the calls may be captured in a
 * CUDA graph.  Ranks must be on distinct GPUs (connect
 * refuses otherwise).  A wait that gives up sets the device status word
 * (ebx_device_status) and leaves y unwritten; the exchange is then out of
 * step and must be destroyed. */
#define EBX_EXCHANGE_HANDLE_BYTES 128

typedef struct ebx_exchange ebx_exchange;

/* Allocate this rank's region on `device`; 1 <= world <= 8, 1 <= max_m <= 256
 * (ebx_linear_allreduce itself takes M <= 16).  handle_out receives
 * EBX_EXCHANGE_HANDLE_BYTES bytes. */
EBX_API ebx_status ebx_exchange_create(int32_t world, int32_t rank, int32_t device, int64_t max_m,
                                       int64_t max_n, void* handle_out, ebx_exchange** out);
/* Map the regions of all ranks: `handles` = world blobs in rank order. */
EBX_API ebx_status ebx_exchange_connect(ebx_exchange* ex, const void* handles);
EBX_API ebx_status ebx_exchange_destroy(ebx_exchange* ex);
/* y[M, rows] (fp16, DEVICE) = fp16( sum over ranks of x_r @ W_r^T + bias ), where
 * this rank holds W_r (its K slice of the weight, all rows) and x_r [M, cols]
 * (its slice of the activations).  bias (fp16, may be NULL) and y32 (fp32
 * copy before rounding, may be NULL) as in ebx_linear. */
EBX_API ebx_status ebx_linear_allreduce(const ebx_matrix* m, const void* x, int64_t M,
                                        const void* bias, void* y, float* y32, ebx_exchange* ex,
                                        void* stream);

/* Exchange protocol for this rank's later calls (every rank must choose the same):
 * EBX_EXCHANGE_AUTO (the default: two-phase once world * M >= 48, broadcast
 * below), EBX_EXCHANGE_BROADCAST or EBX_EXCHANGE_TWO_PHASE.  The two-phase form
 * applies to ebx_exchange_allreduce and to ebx_linear_allreduce launches whose
 * grid fits on the GPU; the others broadcast.  No reference counterpart. */
#define EBX_EXCHANGE_AUTO 0
#define EBX_EXCHANGE_BROADCAST 1
#define EBX_EXCHANGE_TWO_PHASE 2
EBX_API ebx_status ebx_exchange_set_protocol(ebx_exchange* ex, int32_t protocol);

/* y[M, N] (fp16) = fp16( sum over ranks of partial_r + bias ) for an fp32 partial
 * [M, N] this rank already holds -- a row-parallel shard's fp32 output from
 * ebx_linear (y32) at batch sizes above ebx_linear_allreduce's 16 rows -- over the
 * same exchange: one cooperative launch exchanges the elements (broadcast or
 * two-phase, as above) and sums all ranks' words in rank order (bit-identical on
 * every rank), replacing an NCCL all-reduce of the partials.  M <= max_m, N <= max_n; bias (fp16,
 * may be NULL), y32 (fp32 copy before rounding, may be NULL).  The same call-order
 * rules as ebx_linear_allreduce; no reference counterpart. */
EBX_API ebx_status ebx_exchange_allreduce(ebx_exchange* ex, const float* partial, int64_t M,
                                          int64_t N, const void* bias, void* y, float* y32,
                                          void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EBX_H_ */
