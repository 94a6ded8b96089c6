// q8_1.cu -- on-the-fly Q8_1 activation quantizer (sm_100a).
//
// Replaces quantize_row_q8_1_kernel / quantize_row_q8_1_batched_kernel
// (kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:230-315) and the coop variant
// (kernels/matmul_iq4xs/impl_gemv_dp4a_gfx1100.hip:138-160).  Same per-block semantics, bit for bit:
//   amax, sum: 32-lane xor butterfly (offsets 16..1); d = amax/127 (IEEE); q = (int8)roundf(x/d),
//   q = 0 when amax == 0; ds = {trunc_fp16(d), trunc_fp16(sum)} with the reference's truncating
//   conversion.  Output is the reference's 36-byte block_q8_1 layout.
// One warp per block, grid-stride; the 32 q bytes leave as eight 4-byte stores.
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

__global__ void __launch_bounds__(256) q8_1_quantize_kernel(const float* __restrict__ X, uint8_t* __restrict__ q8,
                                                            int64_t K, int64_t M, int64_t stride_m,
                                                            int64_t stride_k, int signal_dependents) {
    if (signal_dependents) grid_launch_dependents();
    grid_dependency_wait();  // X may be the output of the preceding kernel (no-op without PDL)
    const int lane = threadIdx.x & 31;
    const int64_t nb = K / kQK8;
    const int64_t total = nb * M;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total; blk += nwarps) {
        const int64_t m = blk / nb;
        const int64_t ib = blk - m * nb;
        const float x = X[m * stride_m + (ib * kQK8 + lane) * stride_k];
        q8_1_block_store(x, q8 + blk * kQ8Bytes, lane);
    }
}

cudaError_t launch_q8_1_quantize(const float* X, uint8_t* q8, int64_t K, int64_t M, int64_t stride_m,
                                 int64_t stride_k, cudaStream_t stream, bool signal_dependents, bool pdl) {
    const int64_t total = (K / kQK8) * M;
    const int sms = device_sm_count();
    const int64_t grid = std::min<int64_t>((total + 7) / 8, (int64_t)sms * 16);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q8_1_quantize_kernel, X, q8, K, M, stride_m, stride_k, signal_dependents ? 1 : 0);
}

}  // namespace iq4xs
