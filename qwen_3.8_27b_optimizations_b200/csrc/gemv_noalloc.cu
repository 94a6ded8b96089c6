// gemv_noalloc.cu -- iq4xs_gemv_f32_noalloc: the fp32 decode GEMV without any caller workspace.
//
// Who needs this: callers that cannot allocate device memory at the point where they run the
// matmul -- a ggml backend hook called from inside a graph whose memory plan is fixed up front, a
// runtime that forbids cudaMalloc after start-up because it synchronises the device, or code that
// owns no allocator at all.  They pass only inputs and outputs; the Q8_1 activations and the
// partial sums of the K parts live in one file-scope static device array instead.
//
// Limits and rules:
//  * the array is kNoAllocScratchBytes (4 MiB) on every GPU that loads the library, held until the
//    process exits;
//  * a shape whose scratch need exceeds it is rejected with IQ4XS_ERR_WORKSPACE_TOO_SMALL before
//    anything is launched;
//  * every call uses the same array: calls that overlap on the GPU (other streams, other host
//    threads) race and give wrong results -- serialise them on one stream;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress); make
//    that first call before any stream capture;
//  * nothing here calls cudaMalloc, cudaFree, a memset or an allocating library routine: the array
//    needs no initialisation, each call writes what it reads.
#include <mutex>

#include "../../include/iq4xs.h"
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;

// In host code this name is only a host-side stand-in; kernels get the address from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDev = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDev];

cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // once per device, with that device current
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

size_t align_up256(size_t v) { return (v + 255) & ~(size_t)255; }
}  // namespace

}  // namespace iq4xs

using namespace iq4xs;

extern "C" int iq4xs_gemv_f32_noalloc(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B,
                                      cudaStream_t stream) {
    if (!W || !X || !Y || K <= 0 || N <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (K % kQK != 0 || B < 1 || B > IQ4XS_MAX_GEMV_BATCH) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (K > (int64_t)1 << 30 || N > ((int64_t)1 << 31) - 1) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(W) & 7u) || (reinterpret_cast<uintptr_t>(X) & 3u) ||
        (reinterpret_cast<uintptr_t>(Y) & 3u))
        return IQ4XS_ERR_MISALIGNED;

    // Scratch layout: [Q8_1 activations][partial sums], as the workspace of iq4xs_gemv_f32.
    // Partial sums exist only on the tensor-core path, with the part count its launcher picks for
    // this device (the same SM count and shared-memory limit the launch below looks up).
    const size_t q8_bytes = (size_t)(K / kQK8) * (size_t)B * kQ8Bytes;
    const size_t partials = gemv_takes_mma(static_cast<const uint8_t*>(W), K, (int)B)
                                ? gemv_mma_partial_bytes_for(K, N, (int)B, device_sm_count(), device_smem_optin())
                                : 0;
    const size_t need = align_up256(q8_bytes) + partials;
    if (need > kNoAllocScratchBytes) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;

    void* scratch = nullptr;
    if (scratch_address(&scratch) != cudaSuccess) return IQ4XS_ERR_CUDA;
    uint8_t* base = static_cast<uint8_t*>(scratch);
    uint8_t* q8 = base;
    float* part = reinterpret_cast<float*>(base + align_up256(q8_bytes));

    GemvArgs a = {};
    a.W = static_cast<const uint8_t*>(W);
    a.q8 = q8;
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
    a.partials = part;
    a.partial_bytes = partials;  // the size checked above: a launcher that wanted more fails loudly
    // The same activation policy as iq4xs_gemv_f32: from a 16-byte aligned X the GEMV launchers
    // quantise inside the kernel where that pays and otherwise run the standalone quantizer into q8.
    if ((reinterpret_cast<uintptr_t>(X) & 15u) == 0 && gemv_bulk_path(a.W, K)) {
        a.act.mode = kActF32;
        a.act.x = X;
        return launch_gemv_q8(a, (int)B, stream, false) == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
    }
    if (launch_q8_1_quantize(X, q8, K, B, K, 1, stream, true, false) != cudaSuccess) return IQ4XS_ERR_CUDA;
    return launch_gemv_q8(a, (int)B, stream, true) == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
}
