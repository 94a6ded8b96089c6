// iq4xs_kernels.h -- internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace iq4xs {

struct GemvArgs {
    const uint8_t* W;    // IQ4_XS rows [N][K/256][136]
    const uint8_t* q8;   // Q8_1 blocks [B][K/32][36]
    float* y;            // [B][N]
    int32_t* sumi;       // debug only: raw sub-block dots [B][N][K/32]
    uint32_t* err;       // device error word
    int64_t N;
    int K;
    int kb;              // K/256
    int64_t rb;          // bytes per weight row (kb*136)
    int kparts;          // set by the launcher
    int kb_per_part;     // set by the launcher
    int stages;          // set by the launcher
    int force_generic;   // test hook: take the direct-load kernel
};

// Q8_1 quantizer.  Element (m, k) of X is at X[m*stride_m + k*stride_k]; output blocks [M][K/32].
cudaError_t launch_q8_1_quantize(const float* X, uint8_t* q8, int64_t K, int64_t M, int64_t stride_m,
                                 int64_t stride_k, cudaStream_t stream, bool signal_dependents);

cudaError_t launch_gemv_q8(GemvArgs a, int B, cudaStream_t stream, bool pdl);
cudaError_t launch_gemv_q8_debug(GemvArgs a, int B, cudaStream_t stream);

// Synthetic data and the IQ4_XS weight quantizer.
cudaError_t launch_fill_normal(float* dst, int64_t n, uint64_t seed, float mean, float stddev, cudaStream_t stream);
cudaError_t launch_quantize_iq4_xs(const float* src, uint8_t* dst, int64_t nrows, int64_t n_per_row, cudaStream_t stream);
cudaError_t launch_dequantize(const uint8_t* W, float* out, int64_t K, int64_t N, cudaStream_t stream);

uint32_t* device_error_word();  // per-device error word (current device)

}  // namespace iq4xs
