// ebx_capi.cu -- the extern "C" boundary of libebx (declared in include/ebx.h).
//
// Ownership mirrors the reference RuntimeMatrix (elasticbit_runtime.cu:714-
// 1384): the handle owns its device buffers and frees them on destroy.  Unlike
// the reference, no host copy of the payload is kept and nothing is unpacked on
// the host: the device holds only the exact-width tile codes and fp32 scales.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/ebx.h"
#include "ebx_common.cuh"
#include "ebx_internal.h"

struct ebx_matrix {
    ebx::Matrix m;
};

// Handle blob exchanged between ranks (EBX_EXCHANGE_HANDLE_BYTES).
struct ExchangeBlob {
    cudaIpcMemHandle_t ipc;   // 64 bytes: this rank's region
    unsigned char uuid[16];   // GPU identity: ranks must be on distinct GPUs
    int32_t world, rank;
    int64_t max_m, max_n;
    uint64_t bytes;
    unsigned char pad[EBX_EXCHANGE_HANDLE_BYTES - 64 - 16 - 8 - 24];
};
static_assert(sizeof(ExchangeBlob) == EBX_EXCHANGE_HANDLE_BYTES, "exchange blob size");

struct ebx_exchange {
    ebx::XchgArgs xa;          // peer pointers (valid after connect)
    int device = 0;
    int64_t max_m = 0, max_n = 0;
    uint8_t* own = nullptr;    // cudaMalloc'd region of this rank
    uint64_t bytes = 0;
    bool connected = false;
    bool mapped[ebx::kMaxWorld] = {};
    ExchangeBlob blob;
};

namespace ebx {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

}  // namespace ebx

namespace {

using ebx::set_error;

ebx_status cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " in " + what);
    return EBX_ERR_CUDA;
}

#define EBX_CUDA(call)                                 \
    do {                                               \
        cudaError_t e__ = (call);                      \
        if (e__ != cudaSuccess) return cuda_fail(e__, #call); \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && (prev == dev || cudaSetDevice(dev) == cudaSuccess))
            ok = true;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

uint64_t payload_bytes_for(int rows, int cols, int bits) {
    const uint64_t count = uint64_t(rows) * uint64_t(cols);
    return bits == 16 ? count * 2 : (count * uint64_t(bits) + 7) / 8;
}

ebx_status validate_shape(int rows, int cols, int bits, bool allow16) {
    if (rows <= 0 || cols <= 0) {
        set_error("invalid ElasticBit matrix dimensions");
        return EBX_ERR_INVALID;
    }
    if (bits < ebx::kMinBits || bits > (allow16 ? 16 : ebx::kMaxBits)) {
        set_error(allow16 ? "ElasticBit storage bits must be between 3 and 16"
                          : "prequantized codes require 3..15-bit storage");
        return EBX_ERR_INVALID;
    }
    return EBX_OK;
}

// Allocates the handle and its tile/scale buffers (zeroed).
ebx_status alloc_matrix(int rows, int cols, int bits, int device, ebx_matrix** out) {
    ebx_matrix* h = new (std::nothrow) ebx_matrix();
    if (!h) {
        set_error("out of host memory");
        return EBX_ERR_INVALID;
    }
    ebx::Matrix& m = h->m;
    m.rows = rows;
    m.cols = cols;
    m.bits = bits;
    m.device = device;
    m.exec_width = 16;
    m.kt = ebx::round_up(cols, ebx::kKTile) / ebx::kKTile;
    m.groups = ebx::round_up(rows, ebx::kRowGroup) / ebx::kRowGroup;
    m.tiles_bytes = size_t(m.groups * m.kt * ebx::tile_bytes(bits));
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&m.tiles), m.tiles_bytes);
    if (e == cudaSuccess && bits != 16)
        e = cudaMalloc(reinterpret_cast<void**>(&m.scales), sizeof(float) * size_t(rows));
    if (e != cudaSuccess) {
        if (m.tiles) cudaFree(m.tiles);
        if (m.scales) cudaFree(m.scales);
        delete h;
        return cuda_fail(e, "cudaMalloc(matrix buffers)");
    }
    *out = h;
    return EBX_OK;
}

// Host check of the scales for the in-place decode path (see Matrix::direct_ok).
cudaError_t check_scales(ebx::Matrix& m, cudaStream_t s) {
    m.direct_ok = false;
    if (!m.scales) return cudaSuccess;
    std::vector<float> host(size_t(m.rows));
    cudaError_t e = cudaMemcpyAsync(host.data(), m.scales, sizeof(float) * host.size(),
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return e;
    bool ok = true;
    for (float v : host) ok = ok && std::isfinite(v) && std::fabs(v) >= 0x1p-100f;
    m.direct_ok = ok;
    return cudaSuccess;
}

void free_matrix(ebx_matrix* h) {
    if (!h) return;
    DeviceGuard g(h->m.device);
    if (h->m.tiles) cudaFree(h->m.tiles);
    if (h->m.scales) cudaFree(h->m.scales);
    delete h;
}

}  // namespace

extern "C" {

const char* ebx_version(void) { return "ebx 0.1.0 sm_100a"; }

size_t ebx_last_error(char* buf, size_t len) {
    const std::string& s = ebx::g_last_error;
    if (buf && len) {
        const size_t n = s.size() < len - 1 ? s.size() : len - 1;
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return s.size();
}

ebx_status ebx_matrix_create_from_codes(const int16_t* codes, const float* scales, int32_t rows,
                                        int32_t cols, int32_t bits, int32_t device, void* stream,
                                        ebx_matrix** out) {
    if (!out || !codes || !scales) {
        set_error("codes, scales and out must be non-null");
        return EBX_ERR_INVALID;
    }
    *out = nullptr;
    ebx_status st = validate_shape(rows, cols, bits, false);
    if (st != EBX_OK) return st;
    DeviceGuard g(device);
    if (!g.ok) return cuda_fail(cudaErrorInvalidDevice, "cudaSetDevice");
    ebx_matrix* h = nullptr;
    st = alloc_matrix(rows, cols, bits, device, &h);
    if (st != EBX_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* bad = nullptr;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&bad), sizeof(int));
    if (e == cudaSuccess) e = cudaMemsetAsync(bad, 0, sizeof(int), s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(h->m.scales, scales, sizeof(float) * size_t(rows),
                            cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = ebx::launch_codes_to_tiles(h->m, codes, bad, s);
    int bad_host = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bad_host, bad, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (bad) cudaFree(bad);
    if (e == cudaSuccess) e = check_scales(h->m, s);
    if (e != cudaSuccess) {
        free_matrix(h);
        return cuda_fail(e, "ebx_matrix_create_from_codes");
    }
    if (bad_host) {
        free_matrix(h);
        set_error("prequantized ElasticBit code exceeds selected bit range");
        return EBX_ERR_CODE_RANGE;
    }
    *out = h;
    return EBX_OK;
}

ebx_status ebx_matrix_create_from_payload(const void* payload, uint64_t payload_bytes,
                                          const float* scales, int32_t rows, int32_t cols,
                                          int32_t bits, int32_t on_device, int32_t device,
                                          void* stream, ebx_matrix** out) {
    if (!out || !payload || (bits != 16 && !scales)) {
        set_error("payload, scales and out must be non-null");
        return EBX_ERR_INVALID;
    }
    *out = nullptr;
    ebx_status st = validate_shape(rows, cols, bits, true);
    if (st != EBX_OK) return st;
    if (payload_bytes != payload_bytes_for(rows, cols, bits)) {
        set_error("invalid ElasticBit MLB4 metadata");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(device);
    if (!g.ok) return cuda_fail(cudaErrorInvalidDevice, "cudaSetDevice");
    ebx_matrix* h = nullptr;
    st = alloc_matrix(rows, cols, bits, device, &h);
    if (st != EBX_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint8_t* dpay = static_cast<const uint8_t*>(payload);
    uint8_t* staged = nullptr;
    cudaError_t e = cudaSuccess;
    if (!on_device) {
        e = cudaMalloc(reinterpret_cast<void**>(&staged), payload_bytes);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(staged, payload, payload_bytes, cudaMemcpyHostToDevice, s);
        dpay = staged;
    }
    if (e == cudaSuccess && bits != 16)
        e = cudaMemcpyAsync(h->m.scales, scales, sizeof(float) * size_t(rows),
                            on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        e = bits == 16 ? ebx::launch_fp16_to_tiles(h->m, reinterpret_cast<const uint16_t*>(dpay), s)
                       : ebx::launch_payload_to_tiles(h->m, dpay, payload_bytes, s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = check_scales(h->m, s);
    if (staged) cudaFree(staged);
    if (e != cudaSuccess) {
        free_matrix(h);
        return cuda_fail(e, "ebx_matrix_create_from_payload");
    }
    *out = h;
    return EBX_OK;
}

ebx_status ebx_matrix_create_from_fp16(const void* weights, int32_t rows, int32_t cols,
                                       int32_t device, void* stream, ebx_matrix** out) {
    return ebx_matrix_create_from_payload(weights, payload_bytes_for(rows, cols, 16), nullptr,
                                          rows, cols, 16, 1, device, stream, out);
}

ebx_status ebx_matrix_destroy(ebx_matrix* m) {
    free_matrix(m);
    return EBX_OK;
}

ebx_status ebx_matrix_query(const ebx_matrix* h, ebx_matrix_info* info) {
    if (!h || !info) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    const ebx::Matrix& m = h->m;
    info->rows = m.rows;
    info->cols = m.cols;
    info->storage_bits = m.bits;
    info->execution_width = m.exec_width;
    info->device = m.device;
    info->reserved = 0;
    info->payload_bytes = payload_bytes_for(m.rows, m.cols, m.bits);
    info->device_bytes = m.tiles_bytes + (m.scales ? sizeof(float) * size_t(m.rows) : 0);
    return EBX_OK;
}

ebx_status ebx_matrix_set_execution_width(ebx_matrix* h, int32_t width) {
    if (!h) {
        set_error("null matrix");
        return EBX_ERR_INVALID;
    }
    if (width != 4 && width != 8 && width != 12 && width != 16) {
        set_error("ElasticBit execution width must be 4, 8, 12, or 16");
        return EBX_ERR_INVALID;
    }
    if (width == 12 && h->m.bits > 12) {
        set_error("W12A16 cannot represent this ElasticBit storage width");
        return EBX_ERR_INVALID;
    }
    if (width == 4 && h->m.bits > 4) {
        set_error("W4A16 cannot represent this ElasticBit storage width");
        return EBX_ERR_INVALID;
    }
    if (width == 8 && h->m.bits > 8) {
        set_error("W8A16 cannot represent this ElasticBit storage width");
        return EBX_ERR_INVALID;
    }
    h->m.exec_width = width;
    return EBX_OK;
}

ebx_status ebx_matrix_export_payload(const ebx_matrix* h, void* dst, uint64_t dst_bytes,
                                     void* stream) {
    if (!h || !dst) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    const ebx::Matrix& m = h->m;
    const uint64_t need = payload_bytes_for(m.rows, m.cols, m.bits);
    if (dst_bytes < need) {
        set_error("payload destination too small");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(m.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m.bits == 16) {
        EBX_CUDA(ebx::launch_materialize(m, static_cast<uint16_t*>(dst), s));
    } else {
        EBX_CUDA(ebx::launch_tiles_to_payload(m, static_cast<uint8_t*>(dst), need, s));
    }
    return EBX_OK;
}

ebx_status ebx_matrix_export_scales(const ebx_matrix* h, float* dst, void* stream) {
    if (!h || !dst) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (!h->m.scales) return EBX_OK;
    DeviceGuard g(h->m.device);
    EBX_CUDA(cudaMemcpyAsync(dst, h->m.scales, sizeof(float) * size_t(h->m.rows),
                             cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

ebx_status ebx_matrix_materialize(const ebx_matrix* h, void* dst, void* stream) {
    if (!h || !dst) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(h->m.device);
    EBX_CUDA(ebx::launch_materialize(h->m, static_cast<uint16_t*>(dst),
                                     static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

uint64_t ebx_linear_workspace_bytes(const ebx_matrix* h, int64_t M) {
    // 16 < M <= 256: the decode-GEMM's fp32 split-K partials (when K is split);
    // M <= 16: nothing (decode kernel).
    if (!h || M <= ebx::kDgemmMinRows || (h->m.cols % 8) != 0) return 0;
    if (M <= ebx::kDgemmMaxRows && ebx::dgemm_route(h->m, M)) return ebx::dgemm_workspace_bytes(h->m, M);
    // larger M: optional room for the exactly dequantised fp16 weight, which takes the
    // materialise + tcgen05 GEMM route (faster); without it the prefill decode-GEMM runs
    if (M <= ebx::kGemmMinRows) return 0;
    DeviceGuard g(h->m.device);
    return uint64_t(ebx::round_up(int64_t(h->m.rows) * h->m.cols * 2, 256)) +
           ebx::gemm_part_bytes(M, h->m.rows, h->m.cols);
}

ebx_status ebx_linear(const ebx_matrix* h, const void* x, int64_t M, const void* bias, void* y,
                      float* y32, void* workspace, uint64_t workspace_bytes, void* stream) {
    if (!h || (M > 0 && (!x || !y))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (M < 0) {
        set_error("M must be non-negative");
        return EBX_ERR_INVALID;
    }
    if (M == 0) return EBX_OK;
    DeviceGuard g(h->m.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint64_t need = ebx_linear_workspace_bytes(h, M);
    if (M > ebx::kDgemmMinRows && M <= ebx::kDgemmMaxRows && ebx::dgemm_route(h->m, M) &&
        ebx::dgemm_supported(h->m, M, x)) {
        // weights decoded straight into tensor-core tiles (fp32 partials in the workspace
        // when K is split over CTAs)
        if (workspace_bytes < need || (need > 0 && !workspace)) {
            set_error("ebx_linear: workspace missing or smaller than ebx_linear_workspace_bytes()");
            return EBX_ERR_WORKSPACE;
        }
        EBX_CUDA(ebx::launch_dgemm(h->m, static_cast<const uint16_t*>(x), M,
                                   static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), y32,
                                   workspace, workspace_bytes, s));
        return EBX_OK;
    }
    const uint64_t w16_bytes = uint64_t(ebx::round_up(int64_t(h->m.rows) * h->m.cols * 2, 256));
    if (M > ebx::kGemmMinRows && need > 0 && workspace && workspace_bytes >= w16_bytes &&
        ebx::gemm_supported(h->m.cols, x, workspace)) {
        // prefill with the optional workspace: exact fp16 weight into it, then the tcgen05 GEMM
        // (and, after it, room for fp32 split-K partials when the GEMM splits K)
        uint16_t* w16 = static_cast<uint16_t*>(workspace);
        float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + w16_bytes);
        EBX_CUDA(ebx::launch_materialize(h->m, w16, s));
        EBX_CUDA(ebx::launch_gemm_f16(static_cast<const uint16_t*>(x), w16, M, h->m.rows,
                                      h->m.cols, static_cast<const uint16_t*>(bias),
                                      static_cast<uint16_t*>(y), y32, part,
                                      workspace_bytes - w16_bytes, s));
        return EBX_OK;
    }
    if (M > ebx::kGemmMinRows && ebx::pgemm_supported(h->m, x)) {
        // prefill without a workspace: tcgen05 GEMM with the codes decoded into shared
        // memory per k-block
        EBX_CUDA(ebx::launch_pgemm(h->m, static_cast<const uint16_t*>(x), M,
                                   static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), y32,
                                   s));
        return EBX_OK;
    }
    EBX_CUDA(ebx::launch_decode(h->m, static_cast<const uint16_t*>(x), M,
                                static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), y32,
                                s));
    return EBX_OK;
}

ebx_status ebx_linear_swiglu(const ebx_matrix* h, const void* x, int64_t M, const void* bias,
                             void* y, float* y32, void* stream) {
    if (!h || (M > 0 && (!x || !y))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (M < 0 || M > 16) {
        set_error("ebx_linear_swiglu: need 0 <= M <= 16 (decode batches)");
        return EBX_ERR_INVALID;
    }
    if (h->m.rows % 16 != 0) {
        set_error("ebx_linear_swiglu: rows must be a multiple of 16 (gate/up interleaved by 8)");
        return EBX_ERR_INVALID;
    }
    if (M == 0) return EBX_OK;
    DeviceGuard g(h->m.device);
    EBX_CUDA(ebx::launch_decode(h->m, static_cast<const uint16_t*>(x), M,
                                static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), y32,
                                static_cast<cudaStream_t>(stream), nullptr, 1));
    return EBX_OK;
}

ebx_status ebx_linear_multi(const ebx_matrix* const* mats, int32_t count, const void* x, int64_t M,
                            const void* const* biases, void* const* ys, float* const* y32s,
                            void* stream) {
    if (!mats || !ys || count < 1 || (M > 0 && !x)) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (count > 8) {
        set_error("ebx_linear_multi: at most 8 matrices per launch");
        return EBX_ERR_INVALID;
    }
    if (M < 0 || M > 16) {
        set_error("ebx_linear_multi: need 0 <= M <= 16 (decode batches)");
        return EBX_ERR_INVALID;
    }
    const ebx::Matrix* ms[8];
    for (int i = 0; i < count; ++i) {
        if (!mats[i] || !ys[i]) {
            set_error("null argument");
            return EBX_ERR_INVALID;
        }
        ms[i] = &mats[i]->m;
        if (ms[i]->cols != ms[0]->cols || ms[i]->device != ms[0]->device) {
            set_error("ebx_linear_multi: every matrix must have the same cols and device");
            return EBX_ERR_INVALID;
        }
    }
    if (M == 0) return EBX_OK;
    for (int i = 0; i < count; ++i) {
        if (!ebx::multi_supported(*ms[i]) || (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
            set_error("ebx_linear_multi: one launch needs storage widths 8..12, cols % 64 == 0 and "
                      "16-byte aligned x; run these matrices with ebx_linear");
            return EBX_ERR_UNSUPPORTED;
        }
    }
    DeviceGuard g(ms[0]->device);
    EBX_CUDA(ebx::launch_decode_multi(ms, count, static_cast<const uint16_t*>(x), M,
                                      reinterpret_cast<const uint16_t* const*>(biases),
                                      reinterpret_cast<uint16_t* const*>(ys), y32s,
                                      static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

ebx_status ebx_device_status(int32_t device, int32_t* status, int32_t clear) {
    if (!status) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(device);
    if (!g.ok) return cuda_fail(cudaErrorInvalidDevice, "cudaSetDevice");
    int v = 0, vg = 0, vd = 0, vx = 0;
    EBX_CUDA(ebx::read_device_status(&v, clear != 0, nullptr));
    EBX_CUDA(ebx::read_gemm_status(&vg, clear != 0, nullptr));
    EBX_CUDA(ebx::read_dgemm_status(&vd, clear != 0, nullptr));
    EBX_CUDA(ebx::read_xchg_status(&vx, clear != 0, nullptr));
    *status = v ? v : (vg ? vg : (vd ? vd : vx));
    return EBX_OK;
}

// ---- tensor-parallel exchange ----------------------------------------------

ebx_status ebx_exchange_create(int32_t world, int32_t rank, int32_t device, int64_t max_m,
                               int64_t max_n, void* handle_out, ebx_exchange** out) {
    if (!handle_out || !out) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    *out = nullptr;
    if (world < 1 || world > ebx::kMaxWorld || rank < 0 || rank >= world) {
        set_error("exchange: need 1 <= world <= 8 and 0 <= rank < world");
        return EBX_ERR_INVALID;
    }
    if (max_m < 1 || max_m > 256 || max_n < 1 || max_n > (int64_t(1) << 24)) {
        set_error("exchange: need 1 <= max_m <= 256 and 1 <= max_n <= 2^24");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(device);
    if (!g.ok) return cuda_fail(cudaErrorInvalidDevice, "cudaSetDevice");
    cudaDeviceProp prop;
    EBX_CUDA(cudaGetDeviceProperties(&prop, device));
    ebx_exchange* ex = new (std::nothrow) ebx_exchange();
    if (!ex) {
        set_error("out of host memory");
        return EBX_ERR_INVALID;
    }
    ex->device = device;
    ex->max_m = max_m;
    ex->max_n = max_n;
    ex->xa.world = world;
    ex->xa.rank = rank;
    ex->xa.slot_words = max_m * max_n;
    ex->bytes = ebx::kXchgDataOff + 2ull * uint64_t(world) * uint64_t(max_m) * uint64_t(max_n) * 8ull;
    cudaError_t e = cudaMalloc(&ex->own, ex->bytes);
    if (e == cudaSuccess) e = cudaMemset(ex->own, 0, ex->bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ex->blob.ipc, ex->own);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (ex->own) cudaFree(ex->own);
        delete ex;
        return cuda_fail(e, "ebx_exchange_create");
    }
    std::memcpy(ex->blob.uuid, &prop.uuid, 16);
    ex->blob.world = world;
    ex->blob.rank = rank;
    ex->blob.max_m = max_m;
    ex->blob.max_n = max_n;
    ex->blob.bytes = ex->bytes;
    std::memset(ex->blob.pad, 0, sizeof(ex->blob.pad));
    std::memcpy(handle_out, &ex->blob, sizeof(ExchangeBlob));
    *out = ex;
    return EBX_OK;
}

ebx_status ebx_exchange_connect(ebx_exchange* ex, const void* handles) {
    if (!ex || !handles) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (ex->connected) {
        set_error("exchange already connected");
        return EBX_ERR_INVALID;
    }
    const int world = ex->xa.world, rank = ex->xa.rank;
    std::vector<ExchangeBlob> b(world);
    std::memcpy(b.data(), handles, sizeof(ExchangeBlob) * size_t(world));
    for (int r = 0; r < world; ++r) {
        if (b[r].world != world || b[r].rank != r || b[r].max_m != ex->max_m ||
            b[r].max_n != ex->max_n || b[r].bytes != ex->bytes) {
            set_error("exchange: handle " + std::to_string(r) +
                      " does not match (world, rank order, max_m, max_n)");
            return EBX_ERR_INVALID;
        }
        for (int q = 0; q < r; ++q)
            if (std::memcmp(b[q].uuid, b[r].uuid, 16) == 0) {
                set_error("exchange: ranks " + std::to_string(q) + " and " + std::to_string(r) +
                          " share one GPU; the exchange needs one GPU per rank");
                return EBX_ERR_UNSUPPORTED;
            }
    }
    if (std::memcmp(&b[rank], &ex->blob, sizeof(ExchangeBlob)) != 0) {
        set_error("exchange: handle of this rank is not the one ebx_exchange_create returned");
        return EBX_ERR_INVALID;
    }
    DeviceGuard g(ex->device);
    if (!g.ok) return cuda_fail(cudaErrorInvalidDevice, "cudaSetDevice");
    for (int r = 0; r < world; ++r) {
        if (r == rank) {
            ex->xa.peer[r] = ex->own;
            continue;
        }
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, b[r].ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (ex->mapped[q]) {
                    cudaIpcCloseMemHandle(ex->xa.peer[q]);
                    ex->mapped[q] = false;
                }
            return cuda_fail(e, "cudaIpcOpenMemHandle");
        }
        ex->xa.peer[r] = static_cast<uint8_t*>(p);
        ex->mapped[r] = true;
    }
    ex->connected = true;
    return EBX_OK;
}

ebx_status ebx_exchange_destroy(ebx_exchange* ex) {
    if (!ex) return EBX_OK;
    DeviceGuard g(ex->device);
    cudaError_t first = cudaSuccess;
    for (int r = 0; r < ebx::kMaxWorld; ++r)
        if (ex->mapped[r]) {
            const cudaError_t e = cudaIpcCloseMemHandle(ex->xa.peer[r]);
            if (first == cudaSuccess) first = e;
        }
    if (ex->own) {
        const cudaError_t e = cudaFree(ex->own);
        if (first == cudaSuccess) first = e;
    }
    delete ex;
    if (first != cudaSuccess) return cuda_fail(first, "ebx_exchange_destroy");
    return EBX_OK;
}

ebx_status ebx_linear_allreduce(const ebx_matrix* h, const void* x, int64_t M, const void* bias,
                                void* y, float* y32, ebx_exchange* ex, void* stream) {
    if (!h || !ex || (M > 0 && (!x || !y))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (!ex->connected) {
        set_error("exchange not connected (ebx_exchange_connect)");
        return EBX_ERR_INVALID;
    }
    if (M < 0 || M > ex->max_m || M > 16 || int64_t(h->m.rows) > ex->max_n) {
        set_error("ebx_linear_allreduce: need 0 <= M <= min(16, max_m) and rows <= max_n of the "
                  "exchange (larger M: ebx_linear's fp32 output, then ebx_exchange_allreduce)");
        return EBX_ERR_INVALID;
    }
    if (h->m.device != ex->device) {
        set_error("matrix and exchange live on different devices");
        return EBX_ERR_INVALID;
    }
    if (M == 0) return EBX_OK;
    DeviceGuard g(h->m.device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ebx::XchgArgs xa = ex->xa;
    // fused: the decode kernel reduces and writes y itself; else the finish kernel does
    EBX_CUDA(ebx::launch_decode(h->m, static_cast<const uint16_t*>(x), M,
                                static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y), y32,
                                s, &xa));
    if (!xa.fused)
        EBX_CUDA(ebx::launch_xchg_finish(xa, int(M), h->m.rows, static_cast<const uint16_t*>(bias),
                                         static_cast<uint16_t*>(y), y32, s));
    return EBX_OK;
}

ebx_status ebx_exchange_set_protocol(ebx_exchange* ex, int32_t protocol) {
    if (!ex) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (protocol < EBX_EXCHANGE_AUTO || protocol > EBX_EXCHANGE_TWO_PHASE) {
        set_error("ebx_exchange_set_protocol: protocol must be EBX_EXCHANGE_AUTO, "
                  "EBX_EXCHANGE_BROADCAST or EBX_EXCHANGE_TWO_PHASE");
        return EBX_ERR_INVALID;
    }
    ex->xa.protocol = protocol;
    return EBX_OK;
}

ebx_status ebx_exchange_allreduce(ebx_exchange* ex, const float* partial, int64_t M, int64_t N,
                                  const void* bias, void* y, float* y32, void* stream) {
    if (!ex || (M > 0 && N > 0 && (!partial || !y))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (!ex->connected) {
        set_error("exchange not connected (ebx_exchange_connect)");
        return EBX_ERR_INVALID;
    }
    if (M < 0 || N < 0 || M > ex->max_m || N > ex->max_n) {
        set_error("ebx_exchange_allreduce: need 0 <= M <= max_m and 0 <= N <= max_n");
        return EBX_ERR_INVALID;
    }
    if (M == 0 || N == 0) return EBX_OK;
    DeviceGuard g(ex->device);
    EBX_CUDA(ebx::launch_xchg_allreduce(ex->xa, partial, int(M), int(N),
                                        static_cast<const uint16_t*>(bias), static_cast<uint16_t*>(y),
                                        y32, static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

uint64_t ebx_fnv1a64(const void* data, uint64_t size) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    uint64_t h = 1469598103934665603ull;
    for (uint64_t i = 0; i < size; ++i) {
        h ^= uint64_t(p[i]);
        h *= 1099511628211ull;
    }
    return h;
}

uint64_t ebx_analyze_workspace_bytes(int32_t rows, int32_t samples) {
    if (rows <= 0 || samples <= 0) return 0;
    const uint64_t ref = ebx::round_up(uint64_t(rows) * uint64_t(samples) * 4, 256);
    return ref + uint64_t(rows) * 14 * 3 * 8;
}

ebx_status ebx_analyze(const float* weights, int32_t rows, int32_t cols, const float* calib,
                       int32_t samples, double* hw_err, double* full_err, void* workspace,
                       uint64_t workspace_bytes, void* stream) {
    if (rows <= 0 || cols <= 0 || samples <= 0) {
        set_error("weights and calibration must be non-empty");
        return EBX_ERR_INVALID;
    }
    if (!weights || !calib || !hw_err || !full_err) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    const uint64_t need = ebx_analyze_workspace_bytes(rows, samples);
    if (!workspace || workspace_bytes < need) {
        set_error("analyzer workspace missing or too small");
        return EBX_ERR_WORKSPACE;
    }
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* ref = reinterpret_cast<float*>(ws);
    double* part = reinterpret_cast<double*>(
        ws + ebx::round_up(uint64_t(rows) * uint64_t(samples) * 4, 256));
    EBX_CUDA(ebx::launch_analyze(weights, rows, cols, calib, samples, ref, part, hw_err, full_err,
                                 static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

ebx_status ebx_quantize(const float* weights, int32_t rows, int32_t cols, int32_t bits,
                        int16_t* codes, float* scales, void* stream) {
    ebx_status st = validate_shape(rows, cols, bits, false);
    if (st != EBX_OK) return st;
    if (!weights || !codes || !scales) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    EBX_CUDA(ebx::launch_quantize(weights, rows, cols, bits, codes, scales,
                                  static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

ebx_status ebx_weights_to_fp16(const float* weights, int64_t n, void* out, void* stream) {
    if (n < 0 || (n > 0 && (!weights || !out))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (n == 0) return EBX_OK;
    EBX_CUDA(ebx::launch_to_fp16(weights, n, static_cast<uint16_t*>(out),
                                 static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

ebx_status ebx_elastic_linear_packed(const void* x, int32_t x_dtype, int64_t rows,
                                     const uint8_t* packed, const void* scales,
                                     int32_t scale_dtype, const void* bias, int32_t bits,
                                     int64_t group_size, int64_t out_features,
                                     int64_t in_features, void* out, void* stream) {
    if (bits < 2 || bits > 8) {
        set_error("bits must be in [2,8]");
        return EBX_ERR_INVALID;
    }
    if (group_size <= 0 || out_features <= 0 || in_features <= 0) {
        set_error("invalid ElasticBit dimensions");
        return EBX_ERR_INVALID;
    }
    if (x_dtype < 0 || x_dtype > 2 || scale_dtype < 0 || scale_dtype > 2) {
        set_error("unsupported dtype code");
        return EBX_ERR_INVALID;
    }
    if (rows < 0 || (rows > 0 && (!x || !packed || !scales || !out))) {
        set_error("null argument");
        return EBX_ERR_INVALID;
    }
    if (rows == 0) return EBX_OK;
    EBX_CUDA(ebx::launch_elastic_linear_packed(x, x_dtype, rows, packed, scales, scale_dtype, bias,
                                               bits, group_size, out_features, in_features, out,
                                               static_cast<cudaStream_t>(stream)));
    return EBX_OK;
}

}  // extern "C"
