// iq4xs_kernels.h -- internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/iq4xs_peer.h"

namespace iq4xs {

// Where a GEMV's Q8_1 activations come from.  The fp32 sources are quantised (and, for kActNorm,
// normalised) by every CTA into its own shared memory at kernel start, while the weight copies
// are already in flight; the bytes equal those of the standalone quantizer on the same fp32 values.
enum ActMode : int {
    kActQ8 = 0,    // q8: Q8_1 blocks [B][K/32] in global memory
    kActF32 = 1,   // x: fp32 [B][K]
    kActNorm = 2,  // batch 1: h = rmsnorm(x + delta) * w, from fp32 x [K] (+ delta [K]), weight w [K]
    kActNormPeer = 3,  // kActNorm with delta = the fused all-reduce of `peer` (its own kernel instance)
    kActSwiGLU = 4,    // batch 1: h = silu(gate) * up from fp32 x = gu [2K] (gate [0, K), up [K, 2K))
};
struct ActSource {
    int mode;
    const float* x;
    const float* delta;  // kActNorm: may be null
    const float* w;      // kActNorm
    float* x_out;        // kActNorm: x + delta is written here by CTA 0 (may be null; must not alias x)
    float eps;
    const iq4xs_peer_slots* peer;  // kActNormPeer: delta = the fused all-reduce of these slots (device memory)
};

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
    int kw;              // row kernel: warps per row (set by the launcher)
    int rows_per_stage;  // row kernel: rows per stage (set by the launcher)
    uint32_t lut[4];     // codebook prmt tables {neg_lo0, neg_lo1, pos_hi0, pos_hi1} (read from the param bank)
    float* partials;     // tensor-core kernel: cross-CTA partial sums
    size_t partial_bytes;
    ActSource act;       // activation source (kActQ8: `q8` above)
    const iq4xs_peer_slots* push;  // batch 1: outputs go to slot `rank` of every rank's area, then the signal
};

struct GemvMmaArgs {
    const uint8_t* q8;   // Q8_1 blocks [B][K/32][36]
    float* y;            // [B][N]; nullptr: debug sums only
    float* partial;      // [parts][B][N] when parts > 1
    int32_t* sumi;       // debug only
    uint32_t* err;
    int64_t N;
    int K;
    int pairs;           // K/512 super-block pairs per row
    int pk;              // pairs per part (odd)
    int parts;
    int stages;
    uint32_t lut[4];
    ActSource act;       // kActQ8 or kActF32
};


// Tensor-core GEMV (batch 1..8).  Workspace = the partial sums of the K parts (none with one part).
size_t gemv_mma_partial_bytes(int64_t K, int64_t N, int B);
size_t gemv_mma_partial_bytes_for(int64_t K, int64_t N, int B, int sms, int smem_optin);
int device_smem_optin();
cudaError_t launch_gemv_mma(const uint8_t* W, const uint8_t* q8, float* y, int32_t* sumi, float* partials,
                            size_t partial_bytes, int64_t K, int64_t N, int B, cudaStream_t stream, bool pdl, int sms, int smem_optin, uint32_t* err, const uint32_t lut[4],
                            const ActSource* act = nullptr);
int device_sm_count();
// True when launch_gemv_q8 runs the bulk-copy kernels for this matrix (the fused fp32 activation
// sources need them; the generic kernel reads Q8_1 from global memory).
bool gemv_bulk_path(const uint8_t* W, int64_t K);
// True when launch_gemv_q8 runs the tensor-core kernel (the only one that may write partial sums of
// K parts): bulk path and batch 2..8, or batch 1 with K too long for the row kernel.
bool gemv_takes_mma(const uint8_t* W, int64_t K, int B);
// Row kernel: warps per row (kw) and sub-block slots per lane (spl) for K at batch B; false when K is
// too long for register-resident activations.
bool row_split(int64_t K, int B, int* kw_out, int* spl_out);
// Rows per stage of the batch-1 row kernel at this K.
int gemv_rows_per_stage(int64_t K);

// Grouped GEMV: several independent matrices of one batch size in one launch, each served by its own
// slice of the grid (`ctas` CTAs, contiguous block indices), so the launch, ramp and tail are paid once
// for the group.  Q8_1 activations are already in `q8`.
constexpr int kMaxGroup = 8;
struct GroupedProblem {
    const uint8_t* W;   // IQ4_XS [N][K/256], 16-byte aligned, K % 512 == 0
    const uint8_t* q8;  // Q8_1 [B][K/32]
    float* y;           // [B][N]
    float* partials;    // tensor-core kernel with more than one K part: [parts][B][N]
    int64_t K, N;
    int ctas;           // CTAs given to this matrix (the launchers may trim or raise it, see below)
};
// Batch 1 on the row kernel; cudaErrorNotSupported when a matrix's K is too long for it.
cudaError_t launch_gemv_rows_grouped(const GroupedProblem* p, int count, cudaStream_t stream, bool pdl, uint32_t* err,
                                     const uint32_t lut[4]);
// K parts the grouped tensor-core launch uses for one matrix given `ctas` CTAs (partial sums when > 1).
int gemv_mma_grouped_parts(int64_t K, int64_t N, int ctas, int smem_optin);
// The busiest CTA's estimated time when the tensor-core GEMV runs (K, N) on `ctas` CTAs, in units of
// one warp pair's super-block pair (choose_pk's cost model: rounds of units per pair x (pk + per-unit
// overhead)); the grouped planner balances the matrices with it.
double gemv_mma_cta_cost(int64_t K, int64_t N, int ctas, int smem_optin);
// Batch 2..8 on the tensor-core kernel (partial sums left in `partials`; the caller adds the parts).
cudaError_t launch_gemv_mma_grouped(const GroupedProblem* p, int count, int B, cudaStream_t stream, bool pdl,
                                    uint32_t* err, const uint32_t lut[4]);
void device_limits_current(int* sms, int* smem_optin);

// Tensor-core prefill GEMM (gemm.cu).  Y[m][n] at y + m*ldy_m + n*ldy_n.
struct GemmArgs {
    const uint8_t* act;  // quantised activations in stage blocks (gemm.cu)
    float* y;
    uint32_t* err;
    int64_t N, M;
    int K;
    int64_t ldy_m, ldy_n;
    int tiles_n, tiles_m;  // 128-row weight tiles, 128-token tiles
    uint32_t lut[4];
};
// Workspace: quantised activations as stage blocks of 17,408 bytes, [ceil(M/128)][K/64].
size_t gemm_workspace_bytes(int64_t K, int64_t M);
cudaError_t launch_gemm_quantize(const float* X, void* workspace, int64_t K, int64_t M, int64_t stride_m,
                                 int64_t stride_k, cudaStream_t stream);
// Element (m, k) of X at X[m*x_stride_m + k*x_stride_k].  K % 512 == 0.
cudaError_t launch_gemm(const uint8_t* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M, int64_t x_stride_m,
                        int64_t x_stride_k, int64_t y_stride_m, int64_t y_stride_n, void* workspace, cudaStream_t stream,
                        uint32_t* err, const uint32_t lut[4]);
// The int8 (kind::i8) GEMM (gemm_i8.cu): same arguments; workspace = stage blocks of 18,432 bytes,
// [ceil(M/128)][K/128].
size_t gemm_i8_workspace_bytes(int64_t K, int64_t M);
cudaError_t launch_gemm_i8_quantize(const float* X, void* workspace, int64_t K, int64_t M, int64_t stride_m,
                                    int64_t stride_k, cudaStream_t stream);
cudaError_t launch_gemm_i8(const uint8_t* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                           int64_t x_stride_m, int64_t x_stride_k, int64_t y_stride_m, int64_t y_stride_n,
                           void* workspace, cudaStream_t stream, uint32_t* err, const uint32_t lut[4]);

// Q8_1 quantizer.  Element (m, k) of X is at X[m*stride_m + k*stride_k]; output blocks [M][K/32].
// pdl: launch with programmatic stream serialization (the kernel waits on griddepcontrol before
// reading X, so it may overlap the tail of the preceding kernel).
cudaError_t launch_q8_1_quantize(const float* X, uint8_t* q8, int64_t K, int64_t M, int64_t stride_m,
                                 int64_t stride_k, cudaStream_t stream, bool signal_dependents, bool pdl = false);

cudaError_t launch_gemv_q8(GemvArgs a, int B, cudaStream_t stream, bool pdl);
cudaError_t launch_gemv_q8_debug(GemvArgs a, int B, cudaStream_t stream);

// Synthetic data and the IQ4_XS weight quantizer.
cudaError_t launch_fill_normal(float* dst, int64_t n, uint64_t seed, float mean, float stddev, cudaStream_t stream);
cudaError_t launch_quantize_iq4_xs(const float* src, uint8_t* dst, int64_t nrows, int64_t n_per_row, cudaStream_t stream);
cudaError_t launch_dequantize(const uint8_t* W, float* out, int64_t K, int64_t N, cudaStream_t stream);

uint32_t* device_error_word();  // per-device error word (current device)

// cudaFuncAttributeMaxDynamicSharedMemorySize for `kern` on the current device, set at most once per
// (device, kernel) to the device's opt-in maximum: a launch does not pay a runtime call for it.
cudaError_t ensure_dynamic_smem(const void* kern, int bytes);

// Decoder step operations (decode_ops.cu).
cudaError_t launch_residual_rmsnorm_q8(float* x, const float* delta, const float* w, int D, int T, float eps,
                                       uint8_t* q8, float* h_out, cudaStream_t stream, bool pdl,
                                       const iq4xs_peer_slots* peer = nullptr);
cudaError_t launch_attention_decode_q8(const float* qkv, __half* kc, __half* vc, const float* cosb,
                                       const float* sinb, const int64_t* pos, int hq, int hkv, int max_seq,
                                       uint8_t* q8, float* o_out, uint32_t* err, cudaStream_t stream, bool pdl,
                                       bool early_state = false);
cudaError_t launch_swiglu_q8(const float* gu, int64_t F, int64_t T, uint8_t* q8, cudaStream_t stream, bool pdl);
cudaError_t launch_embed_f16(const __half* emb, const int64_t* tok, int64_t vocab, int64_t D, float* x,
                             cudaStream_t stream, bool pdl);
cudaError_t launch_argmax(const float* v, int64_t n, int64_t* tok, int64_t* pos, cudaStream_t stream, bool pdl);

}  // namespace iq4xs
