// ref_capi.cpp -- C-linkage wrappers around the reference's own CPU oracle.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile together with the UNCHANGED reference
// source kernels/matmul_iq4xs/ref_cpu.cpp (read from the reference tree, never copied) into
// oracle/_ref/libref_cpu.so, so Python tests, golden-vector generation and bench.py's
// reference arm can call the reference's code through ctypes.
#include "ref_cpu.h"

extern "C" {

// ref_cpu.h:29-35 -- FP64 GEMV on unquantised x.
void ref_gemv_iq4xs_cpu_ref(const void* W, const float* x, float* y, int64_t K, int64_t N) {
    gemv_iq4xs_cpu_ref(static_cast<const block_iq4_xs*>(W), x, y, K, N);
}

// ref_cpu.h:40-47 -- FP64 GEMM, X [K][M], Y [N][M].
void ref_gemm_iq4xs_cpu_ref(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M) {
    gemm_iq4xs_cpu_ref(static_cast<const block_iq4_xs*>(W), X, Y, K, N, M);
}

// ref_cpu.h:50-55 -- fp32 dequantisation of a whole matrix.
void ref_dequant_mat_iq4xs_cpu(const void* W, float* out, int64_t K, int64_t N) {
    dequant_mat_iq4xs_cpu(static_cast<const block_iq4_xs*>(W), out, K, N);
}

// block_iq4_xs.h:34-68 and :71-86 -- the reference's fp16 helpers.
float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }
uint16_t ref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }

}  // extern "C"
