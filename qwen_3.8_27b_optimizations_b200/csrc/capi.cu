// capi.cu -- the C ABI (include/iq4xs.h): argument validation, workspace handling, launches.
//
// Argument checks and status mapping follow the reference launchers
// (kernels/matmul_iq4xs/impl_gemv_dp4a_gfx1100.hip:291-329, real_stock_dp4a_comparator.hip:266-315,
// patches/0001-gfx1100-mul-mat-custom.patch:148-154,261-280): null pointers, K % 256, non-positive
// sizes are rejected before any launch; nothing aborts; errors come back as status codes.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "../../include/iq4xs.h"
#include "../../include/iq4xs_decoder.h"
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

namespace {
__device__ uint32_t g_device_error;

constexpr int kMaxDevices = 64;
// Device address of g_device_error per device, filled on first use; several host threads may
// launch on one device at once, so the slots are atomics.
std::atomic<uint32_t*> g_err_ptr[kMaxDevices];
std::mutex g_mu;

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int status_from(cudaError_t e) { return e == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA; }
}  // namespace

uint32_t* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    uint32_t* cur = g_err_ptr[dev].load(std::memory_order_acquire);
    if (!cur) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        cur = static_cast<uint32_t*>(p);  // the same address whichever thread stores it
        g_err_ptr[dev].store(cur, std::memory_order_release);
    }
    return cur;
}

namespace {
// ------------------------------------------------------------------------------ validation
int check_matrix(const void* W, int64_t K, int64_t N) {
    if (!W) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K <= 0 || N <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % kQK != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (K > (int64_t)1 << 30 || N > ((int64_t)1 << 31) - 1) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(W, 8)) return IQ4XS_ERR_MISALIGNED;
    return IQ4XS_OK;
}

int check_batch(int64_t B) { return (B < 1 || B > IQ4XS_MAX_GEMV_BATCH) ? IQ4XS_ERR_UNSUPPORTED_SHAPE : IQ4XS_OK; }

GemvArgs make_gemv_args(const void* W, const void* q8, float* Y, int64_t K, int64_t N) {
    GemvArgs a;
    std::memset(&a, 0, sizeof a);
    a.W = static_cast<const uint8_t*>(W);
    a.q8 = static_cast<const uint8_t*>(q8);
    a.y = Y;
    a.err = device_error_word();
    a.N = N;
    a.K = (int)K;
    a.kb = (int)(K / kQK);
    a.rb = (int64_t)a.kb * kBlockBytes;
    a.lut[0] = kNegLo0;
    a.lut[1] = kNegLo1;
    a.lut[2] = kPosHi0;
    a.lut[3] = kPosHi1;
    return a;
}

// ------------------------------------------------------------------------------ internal workspace
// Library-owned workspace for the reference-named entry points that have no workspace argument.
struct Ws {
    void* ptr = nullptr;
    size_t bytes = 0;
};
// One buffer per (device, stream, kind): a GEMV and a GEMM queued on one stream use different
// layouts of their workspace, so the two kinds never share a buffer.
enum WsKind { kWsGemv = 0, kWsGemm = 1 };
std::map<std::tuple<int, cudaStream_t, int>, Ws> g_ws;

cudaError_t internal_workspace(cudaStream_t stream, size_t bytes, void** out, WsKind kind = kWsGemv) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_mu);
    Ws& w = g_ws[std::make_tuple(dev, stream, (int)kind)];
    if (w.bytes >= bytes) {
        *out = w.ptr;
        return cudaSuccess;
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cap);
    if (e != cudaSuccess) return e;
    if (cap != cudaStreamCaptureStatusNone) return cudaErrorNotSupported;  // never allocate while capturing
    if (w.ptr) {
        e = cudaStreamSynchronize(stream);  // the old buffer may still be read by queued work
        if (e != cudaSuccess) return e;
        cudaFree(w.ptr);
        w.ptr = nullptr;
        w.bytes = 0;
    }
    size_t want = 1 << 20;
    while (want < bytes) want <<= 1;
    e = cudaMalloc(&w.ptr, want);
    if (e != cudaSuccess) return e;
    w.bytes = want;
    *out = w.ptr;
    return cudaSuccess;
}

// GEMV workspace: [Q8_1 activations, f32 entry points only][partial sums of the K parts]; nothing in
// it carries over from one call to the next.
size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

size_t gemv_partials(int64_t K, int64_t N, int64_t B) {
    return gemv_mma_partial_bytes(K, N, (int)B);
}

void attach_workspace(GemvArgs& a, void* ws, size_t q8_bytes, int64_t K, int64_t N, int64_t B) {
    uint8_t* base = static_cast<uint8_t*>(ws);
    a.partials = reinterpret_cast<float*>(base + align256(q8_bytes));
    a.partial_bytes = gemv_partials(K, N, B);
}

cudaError_t to_cuda_error(int status) {
    switch (status) {
        case IQ4XS_OK: return cudaSuccess;
        case IQ4XS_ERR_CUDA: {
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? cudaErrorUnknown : e;
        }
        case IQ4XS_ERR_NOT_SUPPORTED: return cudaErrorNotSupported;
        case IQ4XS_ERR_MISALIGNED: return cudaErrorMisalignedAddress;
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace
}  // namespace iq4xs

using namespace iq4xs;

extern "C" {

const char* iq4xs_status_string(int s) {
    switch (s) {
        case IQ4XS_OK: return "ok";
        case IQ4XS_ERR_INVALID_ARGUMENT: return "invalid argument";
        case IQ4XS_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
        case IQ4XS_ERR_MISALIGNED: return "misaligned pointer";
        case IQ4XS_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
        case IQ4XS_ERR_CUDA: return "CUDA error";
        case IQ4XS_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case IQ4XS_ERR_NOT_SUPPORTED: return "not supported";
        default: return "unknown status";
    }
}

int iq4xs_version(void) { return 100; }

int iq4xs_device_error(uint32_t* code) {
    if (!code) return IQ4XS_ERR_INVALID_ARGUMENT;
    uint32_t* p = device_error_word();
    if (!p) return IQ4XS_ERR_CUDA;
    uint32_t v = 0;
    if (cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return IQ4XS_ERR_CUDA;
    const uint32_t zero = 0;
    if (cudaMemcpy(p, &zero, sizeof zero, cudaMemcpyHostToDevice) != cudaSuccess) return IQ4XS_ERR_CUDA;
    *code = v;
    return IQ4XS_OK;
}

size_t iq4xs_q8_1_bytes(int64_t K, int64_t M) {
    if (K <= 0 || M <= 0 || K % kQK8 != 0) return 0;
    return (size_t)(K / kQK8) * (size_t)M * kQ8Bytes;
}

int iq4xs_q8_1_quantize(const float* X, void* q8, int64_t K, int64_t M, cudaStream_t stream) {
    if (!X || !q8 || K <= 0 || M <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % kQK8 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(X, 4) || !aligned(q8, 4)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_q8_1_quantize(X, static_cast<uint8_t*>(q8), K, M, K, 1, stream, false));
}

size_t iq4xs_gemv_q8_workspace_bytes(int64_t K, int64_t N, int64_t B) {
    if (K <= 0 || N <= 0 || B <= 0) return 0;
    return gemv_partials(K, N, B);
}

size_t iq4xs_gemv_workspace_bytes(int64_t K, int64_t N, int64_t B) {
    if (K <= 0 || N <= 0 || B <= 0) return 0;
    return align256(iq4xs_q8_1_bytes(K, B)) + gemv_partials(K, N, B);
}

int iq4xs_gemv_q8(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream) {
    return iq4xs_gemv_q8_ex(W, q8, Y, K, N, B, workspace, workspace_bytes, 0u, stream);
}

int iq4xs_gemv_q8_ex(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B, void* workspace,
                     size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if ((s = check_batch(B))) return s;
    const size_t need = iq4xs_gemv_q8_workspace_bytes(K, N, B);
    if (!q8 || !Y || (need && !workspace)) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < need) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(q8, 4) || !aligned(Y, 4) || !aligned(workspace, 256)) return IQ4XS_ERR_MISALIGNED;
    GemvArgs a = make_gemv_args(W, q8, Y, K, N);
    attach_workspace(a, workspace, 0, K, N, B);
    return status_from(launch_gemv_q8(a, (int)B, stream, (flags & IQ4XS_FLAG_OVERLAP_PRECEDING) != 0));
}

int iq4xs_gemv_q8_generic(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B,
                          cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if ((s = check_batch(B))) return s;
    if (!q8 || !Y) return IQ4XS_ERR_INVALID_ARGUMENT;
    GemvArgs a = make_gemv_args(W, q8, Y, K, N);
    a.force_generic = 1;
    return status_from(launch_gemv_q8(a, (int)B, stream, false));
}

int iq4xs_gemv_f32(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B, void* workspace,
                   size_t workspace_bytes, cudaStream_t stream) {
    return iq4xs_gemv_f32_ex(W, X, Y, K, N, B, workspace, workspace_bytes, 0u, stream);
}

int iq4xs_gemv_f32_ex(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B, void* workspace,
                      size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if ((s = check_batch(B))) return s;
    if (!X || !Y || !workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < iq4xs_gemv_workspace_bytes(K, N, B)) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(X, 4) || !aligned(Y, 4) || !aligned(workspace, 256)) return IQ4XS_ERR_MISALIGNED;
    uint8_t* q8 = static_cast<uint8_t*>(workspace);
    const bool overlap = (flags & IQ4XS_FLAG_OVERLAP_PRECEDING) != 0;
    GemvArgs a = make_gemv_args(W, q8, Y, K, N);
    attach_workspace(a, workspace, iq4xs_q8_1_bytes(K, B), K, N, B);
    if (aligned(X, 16) && gemv_bulk_path(static_cast<const uint8_t*>(W), K)) {
        // The kernel launchers quantise X inside the GEMV (every CTA into its shared memory, while
        // its weight copies fly) when the per-CTA share is small, and otherwise launch the standalone
        // quantizer into the workspace's Q8_1 area first (see launch_rows / launch_gemv_mma).
        a.act.mode = kActF32;
        a.act.x = X;
        return status_from(launch_gemv_q8(a, (int)B, stream, overlap));
    }
    cudaError_t e = launch_q8_1_quantize(X, q8, K, B, K, 1, stream, true, overlap);
    if (e != cudaSuccess) return IQ4XS_ERR_CUDA;
    return status_from(launch_gemv_q8(a, (int)B, stream, true));
}

int iq4xs_debug_subblock_dots(const void* W, const void* q8, int32_t* S, int64_t K, int64_t N, int64_t B,
                              cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if ((s = check_batch(B))) return s;
    if (!q8 || !S) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (!aligned(q8, 4) || !aligned(S, 4)) return IQ4XS_ERR_MISALIGNED;
    GemvArgs a = make_gemv_args(W, q8, nullptr, K, N);  // sums only, no y
    a.sumi = S;
    return status_from(launch_gemv_q8_debug(a, (int)B, stream));
}

int iq4xs_fill_normal(float* dst, int64_t n, uint64_t seed, float mean, float stddev, cudaStream_t stream) {
    if (!dst || n <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    return status_from(launch_fill_normal(dst, n, seed, mean, stddev, stream));
}

int iq4xs_quantize_weights(const float* src, void* W, int64_t N, int64_t K, cudaStream_t stream) {
    if (!src || !W || N <= 0 || K <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % kQK != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(W, 8) || !aligned(src, 4)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_quantize_iq4_xs(src, static_cast<uint8_t*>(W), N, K, stream));
}

int iq4xs_dequantize(const void* W, float* out, int64_t K, int64_t N, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!out) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (!aligned(out, 4)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_dequantize(static_cast<const uint8_t*>(W), out, K, N, stream));
}

// ------------------------------------------------------------------------------ GEMM
// K/256 odd: the rows are 8 mod 16 bytes long, which no tensor map can address, so the tensor-core
// GEMM does not take them (the ggml hook accepts them all the same, patch:148-151).
static bool gemm_odd_superblocks(int64_t K) { return (K / kQK) % 2 != 0; }

static int check_gemm(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!X || !Y) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (M <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (M > ((int64_t)1 << 30) || N > ((int64_t)1 << 30) || K > ((int64_t)1 << 24)) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(X, 4) || !aligned(Y, 4)) return IQ4XS_ERR_MISALIGNED;
    if (!gemm_odd_superblocks(K) && !aligned(W, 16)) return IQ4XS_ERR_MISALIGNED;
    return IQ4XS_OK;
}

// Odd super-block count (ggml output layout only, Y [M][N]): the call's tokens are quantised to Q8_1
// into the workspace (the same bytes as the GEMM's own quantiser), then the direct-load GEMV kernel
// runs on them 8 tokens at a time -- the same per-sub-block arithmetic, the same fp32 term.
static int gemm_odd_k(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M, int64_t xsm,
                      int64_t xsk, void* workspace, cudaStream_t stream) {
    uint8_t* q8 = static_cast<uint8_t*>(workspace);
    cudaError_t e = launch_q8_1_quantize(X, q8, K, M, xsm, xsk, stream, true, false);
    if (e != cudaSuccess) return IQ4XS_ERR_CUDA;
    const int64_t blk = (K / kQK8) * kQ8Bytes;  // Q8_1 bytes of one token
    for (int64_t m0 = 0; m0 < M; m0 += IQ4XS_MAX_GEMV_BATCH) {
        const int64_t B = std::min<int64_t>(IQ4XS_MAX_GEMV_BATCH, M - m0);
        GemvArgs a = make_gemv_args(W, q8 + m0 * blk, Y + m0 * N, K, N);
        e = launch_gemv_q8(a, (int)B, stream, m0 == 0);  // the first waits for the quantiser (PDL)
        if (e != cudaSuccess) return IQ4XS_ERR_CUDA;
    }
    return IQ4XS_OK;
}

// Operand kind of the tensor-core GEMM when the call does not name one: fp16, measured 2-3% faster
// than int8 on B200 at the layer shapes (both kernels are bound by the TMEM accumulator round trip
// between the MMA issue and the drain, not by MMA throughput or operand bytes).
static constexpr uint32_t kGemmDefaultKind = IQ4XS_GEMM_KIND_F16;

static int gemm_strided(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M, int64_t xsm,
                        int64_t xsk, int64_t ysm, int64_t ysn, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream, uint32_t flags = 0) {
    if (flags & ~(IQ4XS_GEMM_KIND_F16 | IQ4XS_GEMM_KIND_I8)) return IQ4XS_ERR_INVALID_ARGUMENT;
    uint32_t kind = flags & (IQ4XS_GEMM_KIND_F16 | IQ4XS_GEMM_KIND_I8);
    if (kind == (IQ4XS_GEMM_KIND_F16 | IQ4XS_GEMM_KIND_I8)) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (!kind) kind = kGemmDefaultKind;
    int s = check_gemm(W, X, Y, K, N, M);
    if (s) return s;
    if (!workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < gemm_workspace_bytes(K, M)) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(workspace, 256)) return IQ4XS_ERR_MISALIGNED;
    if (gemm_odd_superblocks(K)) {
        if (ysm != N || ysn != 1) return IQ4XS_ERR_UNSUPPORTED_SHAPE;  // only the ggml output layout
        return gemm_odd_k(W, X, Y, K, N, M, xsm, xsk, workspace, stream);
    }
    const uint32_t lut[4] = {kNegLo0, kNegLo1, kPosHi0, kPosHi1};
    if (kind == IQ4XS_GEMM_KIND_I8)
        return status_from(launch_gemm_i8(static_cast<const uint8_t*>(W), X, Y, K, N, M, xsm, xsk, ysm, ysn, workspace,
                                          stream, device_error_word(), lut));
    return status_from(launch_gemm(static_cast<const uint8_t*>(W), X, Y, K, N, M, xsm, xsk, ysm, ysn, workspace, stream,
                                   device_error_word(), lut));
}

static cudaError_t gemm_internal_ws(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                                    int64_t xsm, int64_t xsk, int64_t ysm, int64_t ysn, cudaStream_t stream) {
    int s = check_gemm(W, X, Y, K, N, M);
    if (s) return to_cuda_error(s);
    const size_t need = gemm_workspace_bytes(K, M);
    void* ws = nullptr;
    cudaError_t e = internal_workspace(stream, need, &ws, kWsGemm);
    if (e != cudaSuccess) return e;
    return to_cuda_error(gemm_strided(W, X, Y, K, N, M, xsm, xsk, ysm, ysn, ws, need, stream));
}

size_t iq4xs_gemm_workspace_bytes(int64_t K, int64_t M) {
    if (K <= 0 || M <= 0 || K % kQK8 != 0) return 0;
    return gemm_workspace_bytes(K, M);
}

int iq4xs_gemm(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M, void* workspace,
               size_t workspace_bytes, cudaStream_t stream) {
    return gemm_strided(W, X, Y, K, N, M, K, 1, N, 1, workspace, workspace_bytes, stream);
}

int iq4xs_gemm_strided(const void* W, const float* X, int64_t ldx_m, int64_t ldx_k, float* Y, int64_t ldy_m,
                       int64_t ldy_n, int64_t K, int64_t N, int64_t M, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream) {
    if (ldx_m <= 0 || ldx_k <= 0 || ldy_m <= 0 || ldy_n <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    return gemm_strided(W, X, Y, K, N, M, ldx_m, ldx_k, ldy_m, ldy_n, workspace, workspace_bytes, stream);
}

int iq4xs_gemm_ex(const void* W, const float* X, int64_t ldx_m, int64_t ldx_k, float* Y, int64_t ldy_m, int64_t ldy_n,
                  int64_t K, int64_t N, int64_t M, void* workspace, size_t workspace_bytes, uint32_t flags,
                  cudaStream_t stream) {
    if (ldx_m <= 0 || ldx_k <= 0 || ldy_m <= 0 || ldy_n <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    return gemm_strided(W, X, Y, K, N, M, ldx_m, ldx_k, ldy_m, ldy_n, workspace, workspace_bytes, stream, flags);
}

int iq4xs_debug_gemm_quantize(const float* X, void* workspace, int64_t K, int64_t M, cudaStream_t stream) {
    if (!X || !workspace || K <= 0 || M <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % kQK8 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(X, 4) || !aligned(workspace, 256)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_gemm_quantize(X, workspace, K, M, K, 1, stream));
}

int iq4xs_debug_gemm_i8_quantize(const float* X, void* workspace, int64_t K, int64_t M, cudaStream_t stream) {
    if (!X || !workspace || K <= 0 || M <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % 128 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(X, 4) || !aligned(workspace, 256)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_gemm_i8_quantize(X, workspace, K, M, K, 1, stream));
}

// ------------------------------------------------------------------------------ reference-named
static cudaError_t gemv_f32_internal_ws(const void* W, const float* x, float* y, int64_t K, int64_t N, int64_t B,
                                        cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return to_cuda_error(s);
    if ((s = check_batch(B))) return cudaErrorInvalidValue;
    if (!x || !y) return cudaErrorInvalidValue;
    const size_t need = iq4xs_gemv_workspace_bytes(K, N, B);
    void* ws = nullptr;
    cudaError_t e = internal_workspace(stream, need, &ws);
    if (e != cudaSuccess) return e;
    return to_cuda_error(iq4xs_gemv_f32_ex(W, x, y, K, N, B, ws, need, IQ4XS_FLAG_OVERLAP_PRECEDING, stream));
}

cudaError_t gemv_iq4xs_dp4a_coop_gpu(const void* W, const float* x, float* y, int64_t K, int64_t N, cudaStream_t stream) {
    return gemv_f32_internal_ws(W, x, y, K, N, 1, stream);
}

cudaError_t gemv_iq4xs_stock_dp4a_gpu(const void* W, const float* x, float* y, int64_t K, int64_t N, cudaStream_t stream) {
    return gemv_f32_internal_ws(W, x, y, K, N, 1, stream);
}

cudaError_t quantize_row_q8_1_gpu(const float* x, void* y, int64_t K, cudaStream_t stream) {
    if (!x || !y || K <= 0 || K % kQK8 != 0) return cudaErrorInvalidValue;
    return launch_q8_1_quantize(x, static_cast<uint8_t*>(y), K, 1, K, 1, stream, false);
}

cudaError_t quantize_row_q8_1_batched_gpu(const float* X, void* Y, int64_t K, int64_t M, cudaStream_t stream) {
    if (!X || !Y || K <= 0 || M <= 0 || K % kQK8 != 0) return cudaErrorInvalidValue;
    return launch_q8_1_quantize(X, static_cast<uint8_t*>(Y), K, M, 1, M, stream, false);
}

bool custom_gemv_iq4xs_can_handle(int64_t K, int64_t N, int64_t M, int type) {
    if (type != IQ4XS_GGML_TYPE_IQ4_XS) return false;
    if (M < 1 || M > IQ4XS_MAX_GEMV_BATCH) return false;
    if (K <= 0 || N <= 0 || K % kQK != 0) return false;
    return true;
}

cudaError_t custom_gemv_iq4xs_dispatch(const void* W, const float* x, float* y, int64_t K, int64_t N, cudaStream_t stream) {
    return gemv_f32_internal_ws(W, x, y, K, N, 1, stream);
}

cudaError_t custom_gemv_iq4xs_dispatch_batched(const void* W, const float* x, float* y, int64_t K, int64_t N, int64_t M,
                                               cudaStream_t stream) {
    return gemv_f32_internal_ws(W, x, y, K, N, M, stream);
}

bool custom_gemm_iq4xs_can_handle(int64_t K, int64_t N, int64_t M, int type) {
    if (type != IQ4XS_GGML_TYPE_IQ4_XS) return false;
    if (M < 16) return false;  // patch:149: smaller batches stay on the GEMV path
    if (K <= 0 || N <= 0 || K % kQK != 0) return false;  // patch:150 (the N % 16 gate is not needed)
    return true;
}

cudaError_t custom_gemm_iq4xs_dispatch(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                                       cudaStream_t stream) {
    return gemm_internal_ws(W, X, Y, K, N, M, K, 1, N, 1, stream);
}

cudaError_t gemm_iq4xs_stock_dp4a_gpu(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                                      cudaStream_t stream) {
    return gemm_internal_ws(W, X, Y, K, N, M, 1, M, 1, M, stream);
}

cudaError_t gemm_iq4xs_wmma_stream_gpu(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                                       cudaStream_t stream) {
    return gemm_internal_ws(W, X, Y, K, N, M, 1, M, 1, M, stream);
}

// ------------------------------------------------------------------------------ decoder step
int iq4xs_dec_residual_rmsnorm_q8(float* x, const float* delta, const float* w, int64_t D, int64_t T, float eps,
                                  void* q8, float* h_out, unsigned flags, cudaStream_t stream) {
    if (!x || !w || (!q8 && !h_out) || D <= 0 || T <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (D % kQK8 != 0 || D > 8192 || T > 65535) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(x, 4) || !aligned(w, 4) || (delta && !aligned(delta, 4)) || (q8 && !aligned(q8, 4)) ||
        (h_out && !aligned(h_out, 4)))
        return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_residual_rmsnorm_q8(x, delta, w, (int)D, (int)T, eps, static_cast<uint8_t*>(q8), h_out,
                                                  stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_attention_decode_q8(const float* qkv, void* k_cache, void* v_cache, const float* cos_table,
                                  const float* sin_table, const int64_t* pos, int64_t q_heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t max_seq, void* q8, float* o_out, unsigned flags,
                                  cudaStream_t stream) {
    if (!qkv || !k_cache || !v_cache || !cos_table || !sin_table || !pos || !q8) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (q_heads <= 0 || kv_heads <= 0 || max_seq <= 0 || head_dim <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (head_dim != 128 || q_heads % kv_heads != 0 || q_heads > 65535 || max_seq > 8192)
        return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(qkv, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(cos_table, 4) ||
        !aligned(sin_table, 4) || !aligned(pos, 8) || !aligned(q8, 4) || (o_out && !aligned(o_out, 4)))
        return IQ4XS_ERR_MISALIGNED;
    uint32_t* err = device_error_word();
    if (!err) return IQ4XS_ERR_CUDA;
    return status_from(launch_attention_decode_q8(qkv, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
                                                  cos_table, sin_table, pos, (int)q_heads, (int)kv_heads,
                                                  (int)max_seq, static_cast<uint8_t*>(q8), o_out, err, stream,
                                                  (flags & IQ4XS_FLAG_PDL) != 0,
                                                  (flags & IQ4XS_FLAG_ATTN_EARLY_STATE) != 0));
}

int iq4xs_dec_rmsnorm_gemv(const void* W, const float* x, const float* delta, const float* w, float eps, float* x_out,
                           float* Y, int64_t K, int64_t N, void* workspace, size_t workspace_bytes, unsigned flags,
                           cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!x || !w || !Y || !workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (x_out && (x_out == x || x_out == delta)) return IQ4XS_ERR_INVALID_ARGUMENT;  // read by every CTA
    if (workspace_bytes < iq4xs_gemv_q8_workspace_bytes(K, N, 1)) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(Y, 4) || (delta && !aligned(delta, 16)) ||
        (x_out && !aligned(x_out, 16)) || !aligned(workspace, 256))
        return IQ4XS_ERR_MISALIGNED;
    if (!gemv_bulk_path(static_cast<const uint8_t*>(W), K) || gemv_takes_mma(static_cast<const uint8_t*>(W), K, 1))
        return IQ4XS_ERR_NOT_SUPPORTED;  // the row kernel's K range: the fused norm prologue lives there
    GemvArgs a = make_gemv_args(W, nullptr, Y, K, N);
    attach_workspace(a, workspace, 0, K, N, 1);
    a.act.mode = kActNorm;
    a.act.x = x;
    a.act.delta = delta;
    a.act.w = w;
    a.act.x_out = x_out;
    a.act.eps = eps;
    return status_from(launch_gemv_q8(a, 1, stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_gemv_q8_push(const void* W, const void* q8, int64_t K, int64_t N, const iq4xs_peer_slots* slots,
                           void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!q8 || !slots) return IQ4XS_ERR_INVALID_ARGUMENT;
    const size_t need = iq4xs_gemv_q8_workspace_bytes(K, N, 1);
    if (need && !workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < need) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(q8, 4) || !aligned(slots, 8) || (workspace && !aligned(workspace, 256))) return IQ4XS_ERR_MISALIGNED;
    if (!gemv_bulk_path(static_cast<const uint8_t*>(W), K) || gemv_takes_mma(static_cast<const uint8_t*>(W), K, 1))
        return IQ4XS_ERR_NOT_SUPPORTED;  // the row kernel carries the push epilogue
    GemvArgs a = make_gemv_args(W, q8, nullptr, K, N);
    attach_workspace(a, workspace, 0, K, N, 1);
    a.push = slots;
    return status_from(launch_gemv_q8(a, 1, stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

// The SwiGLU GEMV of both entry points below (push: outputs to the peers' slots instead of Y).
static int swiglu_gemv(const void* W, const float* gu, int64_t K, int64_t N, float* Y, const iq4xs_peer_slots* push,
                void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!gu || !workspace || (!Y && !push)) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < iq4xs_gemv_workspace_bytes(K, N, 1)) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(gu, 16) || (Y && !aligned(Y, 4)) || (push && !aligned(push, 8)) || !aligned(workspace, 256))
        return IQ4XS_ERR_MISALIGNED;
    if (!gemv_bulk_path(static_cast<const uint8_t*>(W), K) || gemv_takes_mma(static_cast<const uint8_t*>(W), K, 1))
        return IQ4XS_ERR_NOT_SUPPORTED;  // the row kernel's K range
    GemvArgs a = make_gemv_args(W, workspace, push ? nullptr : Y, K, N);
    attach_workspace(a, workspace, iq4xs_q8_1_bytes(K, 1), K, N, 1);
    a.act.mode = kActSwiGLU;
    a.act.x = gu;
    a.push = push;
    return status_from(launch_gemv_q8(a, 1, stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_swiglu_gemv(const void* W, const float* gu, int64_t K, int64_t N, float* Y, void* workspace,
                          size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    if (!Y) return IQ4XS_ERR_INVALID_ARGUMENT;
    return swiglu_gemv(W, gu, K, N, Y, nullptr, workspace, workspace_bytes, flags, stream);
}

int iq4xs_dec_swiglu_gemv_push(const void* W, const float* gu, int64_t K, int64_t N, const iq4xs_peer_slots* slots,
                               void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    if (!slots) return IQ4XS_ERR_INVALID_ARGUMENT;
    return swiglu_gemv(W, gu, K, N, nullptr, slots, workspace, workspace_bytes, flags, stream);
}

int iq4xs_dec_rmsnorm_gemv_peer(const void* W, const float* x, const iq4xs_peer_slots* slots, const float* w, float eps,
                                float* x_out, float* Y, int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                                unsigned flags, cudaStream_t stream) {
    int s = check_matrix(W, K, N);
    if (s) return s;
    if (!x || !slots || !w || !Y || !workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (x_out && x_out == x) return IQ4XS_ERR_INVALID_ARGUMENT;  // x is read by every CTA
    if (workspace_bytes < iq4xs_gemv_q8_workspace_bytes(K, N, 1)) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(Y, 4) || !aligned(slots, 8) || (x_out && !aligned(x_out, 16)) ||
        !aligned(workspace, 256))
        return IQ4XS_ERR_MISALIGNED;
    if (!gemv_bulk_path(static_cast<const uint8_t*>(W), K) || gemv_takes_mma(static_cast<const uint8_t*>(W), K, 1))
        return IQ4XS_ERR_NOT_SUPPORTED;
    GemvArgs a = make_gemv_args(W, nullptr, Y, K, N);
    attach_workspace(a, workspace, 0, K, N, 1);
    a.act.mode = kActNormPeer;
    a.act.x = x;
    a.act.peer = slots;
    a.act.w = w;
    a.act.x_out = x_out;
    a.act.eps = eps;
    return status_from(launch_gemv_q8(a, 1, stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_residual_rmsnorm_q8_peer(float* x, const iq4xs_peer_slots* slots, const float* w, int64_t D, float eps,
                                       void* q8, float* h_out, unsigned flags, cudaStream_t stream) {
    if (!x || !slots || !w || (!q8 && !h_out) || D <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (D % kQK8 != 0 || D > 8192) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(x, 4) || !aligned(w, 4) || !aligned(slots, 8) || (q8 && !aligned(q8, 4)) || (h_out && !aligned(h_out, 4)))
        return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_residual_rmsnorm_q8(x, nullptr, w, (int)D, 1, eps, static_cast<uint8_t*>(q8), h_out,
                                                  stream, (flags & IQ4XS_FLAG_PDL) != 0, slots));
}

int iq4xs_dec_embed(const void* emb, const int64_t* tok, int64_t vocab, int64_t D, float* x, unsigned flags,
                    cudaStream_t stream) {
    if (!emb || !tok || !x || vocab <= 0 || D <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (D % 8 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(emb, 16) || !aligned(tok, 8) || !aligned(x, 16)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_embed_f16(static_cast<const __half*>(emb), tok, vocab, D, x, stream,
                                        (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_argmax(const float* logits, int64_t n, int64_t* tok, int64_t* pos, unsigned flags, cudaStream_t stream) {
    if (!logits || !tok || n <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (!aligned(logits, 4) || !aligned(tok, 8) || (pos && !aligned(pos, 8))) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_argmax(logits, n, tok, pos, stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

int iq4xs_dec_swiglu_q8(const float* gu, int64_t F, int64_t T, void* q8, unsigned flags, cudaStream_t stream) {
    if (!gu || !q8 || F <= 0 || T <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (F % kQK8 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(gu, 4) || !aligned(q8, 4)) return IQ4XS_ERR_MISALIGNED;
    return status_from(launch_swiglu_q8(gu, F, T, static_cast<uint8_t*>(q8), stream, (flags & IQ4XS_FLAG_PDL) != 0));
}

}  // extern "C"
