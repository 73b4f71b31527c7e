// ebx_internal.h -- launchers shared between the libebx translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace ebx {

struct Matrix {
    int rows = 0;
    int cols = 0;
    int bits = 16;
    int device = 0;
    int exec_width = 16;       // 16: fp16(q*s) operands; 8/4: integer codes, scale after
    int64_t kt = 0;            // k-tiles (Kp / 64)
    int64_t groups = 0;        // row groups (Np / 16)
    uint8_t* tiles = nullptr;  // groups * kt * bits * 128 bytes
    size_t tiles_bytes = 0;
    float* scales = nullptr;   // rows fp32 (null for 16-bit storage)
    // Every scale is a finite normal >= 2^-100, so the decode kernel may use
    // exactly rescaled copies s * 2^-o (in-place code extraction).
    bool direct_ok = false;
};

void set_error(const std::string& msg);

// ebx_pack.cu ---------------------------------------------------------------
// All return cudaError_t of the launch; `bad` (device int, may be null)
// receives 1 if a code is outside [-qmax, qmax].
cudaError_t launch_codes_to_tiles(const Matrix& m, const int16_t* codes, int* bad,
                                  cudaStream_t s);
cudaError_t launch_payload_to_tiles(const Matrix& m, const uint8_t* payload,
                                    uint64_t payload_bytes, cudaStream_t s);
cudaError_t launch_fp16_to_tiles(const Matrix& m, const uint16_t* w, cudaStream_t s);
cudaError_t launch_tiles_to_payload(const Matrix& m, uint8_t* payload, uint64_t payload_bytes,
                                    cudaStream_t s);
cudaError_t launch_materialize(const Matrix& m, uint16_t* out, cudaStream_t s);

// Tensor-parallel exchange region (one per rank, mapped by every rank):
//   [kXchgCounterOff] uint32: CTAs of the running exchange kernel that are done (local)
//   [kXchgEpochOff]   uint32: epoch of the last completed exchange (local)
//   [kXchgDataOff]    uint64 word[2][world][M][N]: partial of source rank r for epoch E
//                     in slot (E & 1), stored as one 8-byte word {fp32 bits, E}
// A reader polls a word until its upper half equals the epoch it expects: data
// and flag arrive in one single-copy-atomic store, so no fence or separate flag
// is needed (the low-latency protocol of NCCL's LL transport, restated).
constexpr int kMaxWorld = 8;
constexpr size_t kXchgCounterOff = 0;
constexpr size_t kXchgEpochOff = 128;
constexpr size_t kXchgDataOff = 256;

struct XchgArgs {
    uint8_t* peer[kMaxWorld];  // every rank's region as mapped here; peer[rank] is our own
    int world = 0;             // 0: no exchange (plain y / y32 output)
    int rank = 0;
    int fused = 0;             // set by the launcher: the decode kernel also reduces (grid co-resident)
    int protocol = 0;          // 0: automatic, 1: broadcast, 2: two-phase (ebx_exchange_set_protocol)
    int two_phase = 0;         // set by the launcher: owner reduce + owner broadcast (ebx_xchg.cuh)
    int64_t slot_words = 0;    // words per (slot, source rank): max_m * max_n of the exchange
};

// Two-phase exchange for this call?  Automatic: once world x M reaches 48, where
// storing every partial into every rank's region costs more than a second hop.
inline bool xchg_two_phase(const XchgArgs& xa, int64_t M) {
    return xa.protocol == 2 || (xa.protocol == 0 && int64_t(xa.world) * M >= 48);
}

// ebx_decode.cu -------------------------------------------------------------
// With xa (world > 0, M <= 16) the kernel stores its fp32 partials (before
// bias) into every rank's region for epoch + 1.  If its whole grid can be
// co-resident it is launched cooperatively with xa->fused = 1 and also waits
// for all ranks' partials of its own outputs, reduces them, writes y / y32 and
// advances the epoch; otherwise xa->fused = 0 and launch_xchg_finish must follow.
// act = 1: SwiGLU over gate/up rows interleaved in blocks of 8 (y has rows / 2 columns).
cudaError_t launch_decode(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                          uint16_t* y, float* y32, cudaStream_t s, XchgArgs* xa = nullptr,
                          int act = 0);
// Several matrices reading the same x [M, cols] (M <= 16) in one launch; each keeps
// its own width (8..12), scales, semantics, bias and outputs (bias / y32 entries may
// be null, bias and y32 arrays themselves may be null).
bool multi_supported(const Matrix& m);
cudaError_t launch_decode_multi(const Matrix* const* ms, int count, const uint16_t* x, int64_t M,
                                const uint16_t* const* bias, uint16_t* const* y,
                                float* const* y32, cudaStream_t s);
// Reads (and optionally clears) the device-side status word that bounded
// waits set on timeout (0 = healthy).  Synchronizes `s`.
cudaError_t read_device_status(int* status, bool clear, cudaStream_t s);

// ebx_exchange.cu -----------------------------------------------------------
// Waits for every rank's partials of epoch + 1, y = fp16(sum_r partial_r + bias), advances the epoch.
cudaError_t launch_xchg_finish(const XchgArgs& xa, int M, int N, const uint16_t* bias,
                               uint16_t* y, float* y32, cudaStream_t s);
cudaError_t read_xchg_status(int* status, bool clear, cudaStream_t s);
// The same exchange for an fp32 partial the caller already holds (M up to the exchange's
// max_m): push to every rank, gather in rank order, bias, one rounding, advance the epoch.
cudaError_t launch_xchg_allreduce(const XchgArgs& xa, const float* part, int M, int N,
                                  const uint16_t* bias, uint16_t* y, float* y32, cudaStream_t s);

// ebx_gemm.cu ---------------------------------------------------------------
// Rows above which ebx_linear takes the materialise + tcgen05 GEMM route.
constexpr int64_t kGemmMinRows = 64;
bool gemm_supported(int K, const void* x, const void* w16);
// part (may be null): room for fp32 split-K partials; the GEMM splits K over CTAs only when
// part_bytes covers what gemm_part_bytes(M, N, K) asks for, and adds the splits in order.
cudaError_t launch_gemm_f16(const uint16_t* x, const uint16_t* w16, int64_t M, int N, int K,
                            const uint16_t* bias, uint16_t* y, float* y32, float* part,
                            uint64_t part_bytes, cudaStream_t s);
uint64_t gemm_part_bytes(int64_t M, int N, int K);
cudaError_t read_gemm_status(int* status, bool clear, cudaStream_t s);
// Decode-GEMM for 16 < M <= 256: codes decoded straight into tcgen05 tiles (weights as the
// 128-row MMA side, tokens as N); K split over CTAs when needed, with an fp32 partial
// workspace of dgemm_workspace_bytes() reduced in split order.
constexpr int64_t kDgemmMinRows = 16;
constexpr int64_t kDgemmMaxRows = 256;
// dgemm_route: the shape rule alone (16 < M <= 256), which
// also decides ebx_linear_workspace_bytes; dgemm_supported adds the activation checks.
inline bool dgemm_route(const Matrix& m, int64_t M) {
    return M > kDgemmMinRows && M <= kDgemmMaxRows && (m.cols % 8) == 0;
}
bool dgemm_supported(const Matrix& m, int64_t M, const void* x);
uint64_t dgemm_workspace_bytes(const Matrix& m, int64_t M);
cudaError_t launch_dgemm(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                         uint16_t* y, float* y32, void* ws, uint64_t ws_bytes, cudaStream_t s);
cudaError_t read_dgemm_status(int* status, bool clear, cudaStream_t s);
// Prefill decode-GEMM (larger M): persistent tcgen05 GEMM whose weight operand is
// decoded from the codes into shared memory per 64-k block; no workspace.
bool pgemm_supported(const Matrix& m, const void* x);
cudaError_t launch_pgemm(const Matrix& m, const uint16_t* x, int64_t M, const uint16_t* bias,
                         uint16_t* y, float* y32, cudaStream_t s);

// ebx_analyze.cu ------------------------------------------------------------
cudaError_t launch_analyze(const float* w, int rows, int cols, const float* x, int samples,
                           float* ref_scratch, double* part_scratch, double* hw, double* full,
                           cudaStream_t s);
cudaError_t launch_quantize(const float* w, int rows, int cols, int bits, int16_t* codes,
                            float* scales, cudaStream_t s);
cudaError_t launch_to_fp16(const float* w, int64_t n, uint16_t* out, cudaStream_t s);

// ebx_packed_op.cu -----------------------------------------------------------
cudaError_t launch_elastic_linear_packed(const void* x, int x_dtype, int64_t rows,
                                         const uint8_t* packed, const void* scales,
                                         int scale_dtype, const void* bias, int bits,
                                         int64_t group_size, int64_t out_features,
                                         int64_t in_features, void* out, cudaStream_t s);

}  // namespace ebx
