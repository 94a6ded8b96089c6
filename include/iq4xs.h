/*
 * iq4xs.h -- C ABI of the B200 (sm_100a) IQ4_XS x Q8_1 matmul library (libiq4xs_b200.so).
 *
 * Drop-in boundary for the reference's matmul_iq4xs harness and its ggml MUL_MAT hook.  Every
 * entry point takes plain device pointers, sizes and a CUDA stream; nothing allocates on the
 * hot path (the caller passes the workspace), nothing synchronises, nothing aborts.  Status
 * codes instead of exceptions.  Citations are file:line in the reference project.
 *
 * Formats (bit-compatible with the reference / ggml):
 *   IQ4_XS  weight row n of a K-column matrix: K/256 super-blocks of 136 bytes
 *           {fp16 d, u16 scales_h, u8 scales_l[4], u8 qs[128]}   (kernels/common/block_iq4_xs.h:10-19)
 *   Q8_1    activation block of 32 values: 36 bytes {fp16 d, fp16 sum, int8 q[32]}
 *           (kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:22-26), fp16 by truncation.
 *   Activations X are token-major fp32 [M][K] (ggml src1), outputs Y are [M][N] (ggml dst),
 *   except where an entry point says it keeps the reference playground's [K][M] / [N][M].
 *
 * Constraints: K > 0, K % 256 == 0; N > 0; 1 <= B <= 8 for the GEMV entry points; pointers to
 * device memory (W 8-byte aligned; 16-byte alignment and K % 512 == 0 select the bulk-copy path).
 */
#ifndef IQ4XS_H
#define IQ4XS_H

#include <cuda_runtime_api.h>
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ */
/* Status codes (0 = success).  Argument checks mirror impl_gemv_dp4a_gfx1100.hip:299-300
 * (null pointers, K % 256, non-positive sizes -> invalid value) and :305 (grid overflow). */
typedef enum {
    IQ4XS_OK = 0,
    IQ4XS_ERR_INVALID_ARGUMENT = 1,   /* null pointer or non-positive size */
    IQ4XS_ERR_UNSUPPORTED_SHAPE = 2,  /* K % 256 != 0, batch outside 1..8, ... */
    IQ4XS_ERR_MISALIGNED = 3,         /* pointer alignment below what the format needs */
    IQ4XS_ERR_WORKSPACE_TOO_SMALL = 4,
    IQ4XS_ERR_CUDA = 5,               /* launch or runtime error (cudaGetLastError) */
    IQ4XS_ERR_DEVICE_TIMEOUT = 6,     /* a bounded device-side wait gave up (see iq4xs_device_error) */
    IQ4XS_ERR_NOT_SUPPORTED = 7       /* operation unavailable in this configuration */
} iq4xs_status;

#define IQ4XS_QK_K 256
#define IQ4XS_QK8_1 32
#define IQ4XS_BLOCK_BYTES 136
#define IQ4XS_Q8_1_BYTES 36
#define IQ4XS_MAX_GEMV_BATCH 8
#define IQ4XS_GGML_TYPE_IQ4_XS 23 /* ggml_type value of GGML_TYPE_IQ4_XS */

const char* iq4xs_status_string(int status);
int iq4xs_version(void); /* major*10000 + minor*100 + patch */

/* Reads the current device's error word set by bounded device waits and clears it.
 * *code = 0 when no kernel gave up since the last call; otherwise the first code recorded:
 * 1-4 a copy or tensor-core pipeline wait gave up, 5 a decode position outside the KV cache,
 * 6 a peer's data or flag did not arrive (multi-GPU), 7 a decode token id outside the vocabulary
 * (iq4xs_decoder.h, iq4xs_peer.h).  The read and the clear are two
 * synchronous copies, not one atomic exchange: call it between steps, with no kernel of this
 * library running on the device, or an error recorded between the two copies is lost. */
int iq4xs_device_error(uint32_t* code);

/* ------------------------------------------------------------------------------------------ */
/* Q8_1 activation quantizer.
 * Replaces quantize_row_q8_1_gpu (real_stock_dp4a_comparator.hip:266-273; kernel :230-264) and the
 * coop quantizer (impl_gemv_dp4a_gfx1100.hip:138-168).  X fp32 [M][K] -> q8 [M][K/32] blocks.
 * d = amax/127 (IEEE), q = roundf(x/d), ds = {trunc16(d), trunc16(sum)}; bit-exact. */
int iq4xs_q8_1_quantize(const float* X, void* q8, int64_t K, int64_t M, cudaStream_t stream);

/* Bytes of Q8_1 blocks for M tokens of K values. */
size_t iq4xs_q8_1_bytes(int64_t K, int64_t M);

/* ------------------------------------------------------------------------------------------ */
/* Workspace of the GEMV entry points: the call's quantised activations and the partial sums of
 * long rows split over CTAs.  It needs no initialisation and carries nothing from one call to the
 * next.  Calls that may overlap on the GPU must use separate workspaces.  256-byte aligned; may be
 * NULL when the matching *_workspace_bytes function returns 0. */

/* Decode GEMV on pre-quantised activations, batch B = 1..8:
 *   Y[b][n] = sum_k W[n][k] * x_b[k]  with the reference's per-sub-block integer pipeline.
 * Replaces gemv_iq4xs_dp4a_gfx1100_prequantized_gpu (impl_gemv_dp4a_gfx1100.hip:291-308) and the
 * patch's gemv_prequantized_cuh (patches/0001-gfx1100-mul-mat-custom.patch:261-266), both batch 1;
 * batch 2..8 is new (the reference routes it to stock MMVQ, patch:275).
 * q8: [B][K/32] Q8_1 blocks (iq4xs_q8_1_quantize output).  Y: fp32 [B][N].
 * workspace >= iq4xs_gemv_q8_workspace_bytes(K, N, B) (cross-CTA partial sums of long rows). */
int iq4xs_gemv_q8(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B,
                  void* workspace, size_t workspace_bytes, cudaStream_t stream);
size_t iq4xs_gemv_q8_workspace_bytes(int64_t K, int64_t N, int64_t B);

/* Decode GEMV on fp32 activations X [B][K]: quantise into the workspace, then GEMV (the GEMV is
 * launched with programmatic dependent launch so its weight stream overlaps the quantizer).
 * Replaces gemv_iq4xs_dp4a_gfx1100_gpu (impl_gemv_dp4a_gfx1100.hip:310-329) and
 * gemv_iq4xs_stock_dp4a_gpu (real_stock_dp4a_comparator.hip:480-503) without their per-call
 * hipMalloc/hipFree: workspace >= iq4xs_gemv_workspace_bytes(K, N, B). */
int iq4xs_gemv_f32(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B,
                   void* workspace, size_t workspace_bytes, cudaStream_t stream);
size_t iq4xs_gemv_workspace_bytes(int64_t K, int64_t N, int64_t B);

/* Flags of iq4xs_gemv_f32_ex. */
#define IQ4XS_FLAG_OVERLAP_PRECEDING 1u /* W is not written by the kernel that precedes this call on
                                          the stream: the quantizer is launched as a programmatic
                                          dependent (it still waits for X) and the GEMV's prologue and
                                          weight prefetch overlap the preceding kernel's tail */
/* iq4xs_gemv_q8 with flags (iq4xs_gemv_q8 == flags 0).  IQ4XS_FLAG_OVERLAP_PRECEDING: the GEMV is
 * launched as a programmatic dependent of the preceding kernel (the producer of q8, which must not
 * write W); its weight stream starts before that kernel ends and it waits for q8 before reading it.
 * The library's own q8 producers (the decoder-step operations of iq4xs_decoder.h) are written for
 * this.  No counterpart in the reference, whose prequantized GEMV takes no flags. */
int iq4xs_gemv_q8_ex(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B,
                     void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream);

/* iq4xs_gemv_f32 with flags (iq4xs_gemv_f32 == flags 0). */
int iq4xs_gemv_f32_ex(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B,
                      void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream);

/* iq4xs_gemv_f32 for callers that cannot allocate device memory where they call it (a ggml hook
 * inside a graph with a fixed memory plan, a runtime that forbids cudaMalloc after start-up because
 * it synchronises the device): no workspace argument, nothing allocated.  Its scratch (Q8_1
 * activations, partial sums) is one static 4 MiB device array per GPU, kept until the
 * process exits; shapes needing more are rejected with IQ4XS_ERR_WORKSPACE_TOO_SMALL.  All calls
 * share that array, so calls that overlap on the GPU race: serialise them on one stream.  The first
 * call on a device looks up the array's address; make it before any stream capture.
 * No counterpart in the reference (its launchers hipMalloc a scratch buffer on every call). */
int iq4xs_gemv_f32_noalloc(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t B,
                           cudaStream_t stream);

/* Grouped decode GEMV: `count` (1..IQ4XS_MAX_GROUP) independent GEMVs of one batch size B in one
 * launch sequence -- one Q8_1 quantiser for all activations, one GEMV grid whose CTAs are split over
 * the matrices in proportion to their weight bytes, and (batch 2..8, when a matrix is split into K
 * parts) one kernel adding the parts.  For the matrices of one decode step that a ggml graph keeps
 * as separate tensors and feeds the same activations (attn_q / attn_k / attn_v, ffn_gate / ffn_up),
 * or any set of independent GEMVs: the launch, ramp and tail of a GEMV are paid once per group.
 * Each problem's output is that of iq4xs_gemv_f32 on the same inputs within the GEMV tolerance
 * (batch 1: the same bits; batch 2..8 may split K into parts differently).  Y of one problem must not
 * overlap any W, X or Y of the group.  Groups the grouped kernels do not take (W not 16-byte aligned,
 * K % 512 != 0, batch 1 with K > 24576) run as one iq4xs_gemv_f32_ex per problem.
 * workspace >= iq4xs_gemv_grouped_workspace_bytes(problems, count, B), 256-byte aligned, no zeroing.
 * No counterpart in the reference (one GEMV per MUL_MAT node, patch:278-280). */
#define IQ4XS_MAX_GROUP 8
typedef struct iq4xs_gemv_problem {
    const void* W;  /* IQ4_XS [N][K/256] (8-byte aligned) */
    const float* X; /* fp32 [B][K] */
    float* Y;       /* fp32 [B][N] */
    int64_t K;
    int64_t N;
} iq4xs_gemv_problem;
size_t iq4xs_gemv_grouped_workspace_bytes(const iq4xs_gemv_problem* problems, int count, int64_t B);
int iq4xs_gemv_grouped(const iq4xs_gemv_problem* problems, int count, int64_t B, void* workspace,
                       size_t workspace_bytes, unsigned flags, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Prefill GEMM (tensor cores): Y[M][N] = X[M][K] (fp32, quantised per 32-block with Q8_1
 * semantics inside the call) times W^T (IQ4_XS [N][K/256]), ggml layouts.  Same per-sub-block
 * arithmetic as the stock GEMM (real_stock_dp4a_comparator.hip:375-443).  K % 256 == 0; M, N >= 1.
 * K % 512 == 0 (whole super-block pairs, the tensor-map granule; W 16-byte aligned) runs the
 * tensor-core kernel.  An odd K/256 gives rows no tensor map can address: those calls quantise X to
 * Q8_1 in the workspace and run the direct-load GEMV kernel 8 tokens at a time (same arithmetic,
 * much slower), for the ggml output layout only (Y [M][N]; other layouts: unsupported shape).
 * The workspace holds the quantised activations (iq4xs_gemm_workspace_bytes(K, M) bytes, 256-byte
 * aligned, no zeroing needed).
 * Replaces gemm_iq4xs_stock_dp4a_gpu / gemm_iq4xs_wmma_stream_gpu (which allocate per call). */
size_t iq4xs_gemm_workspace_bytes(int64_t K, int64_t M);
int iq4xs_gemm(const void* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
               void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* iq4xs_gemm with explicit strides (elements): X(m, k) at X[m*ldx_m + k*ldx_k], Y(m, n) at
 * Y[m*ldy_m + n*ldy_n].  ggml: ldx = (K, 1), ldy = (N, 1); playground X [K][M], Y [N][M]:
 * ldx = (1, M), ldy = (1, M) -- the layout in which a row shard of Y is one contiguous block, as an
 * all-gather of row shards needs.  Strides must be positive; Y must hold every addressed element. */
int iq4xs_gemm_strided(const void* W, const float* X, int64_t ldx_m, int64_t ldx_k, float* Y, int64_t ldy_m,
                       int64_t ldy_n, int64_t K, int64_t N, int64_t M, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream);
/* Operand kind of the tensor-core GEMM (iq4xs_gemm_ex flags).  IQ4XS_GEMM_KIND_I8: int8 codebook
 * values and Q8_1 quants (tcgen05 kind::i8, s32 accumulators); IQ4XS_GEMM_KIND_F16: the same integers
 * as fp16 (kind::f16, fp32 accumulators).  Both form the exact integer sub-block dots; the fp32 scale
 * products are taken in a different order (i8: (sumi*sw)*d_x, f16: (sumi*d_x)*sw), so the outputs
 * agree to fp32 rounding.  Neither flag: the default kind, fp16 (measured the faster on B200, by 2-3%
 * at the 27B-class layer shapes).  The odd-K path ignores the kind.  No counterpart in the reference
 * (its WMMA GEMM has one operand kind). */
#define IQ4XS_GEMM_KIND_F16 0x10u
#define IQ4XS_GEMM_KIND_I8 0x20u
/* iq4xs_gemm_strided with flags (IQ4XS_GEMM_KIND_*); any other bit: IQ4XS_ERR_INVALID_ARGUMENT. */
int iq4xs_gemm_ex(const void* W, const float* X, int64_t ldx_m, int64_t ldx_k, float* Y, int64_t ldy_m,
                  int64_t ldy_n, int64_t K, int64_t N, int64_t M, void* workspace, size_t workspace_bytes,
                  uint32_t flags, cudaStream_t stream);
/* The GEMM's activation quantiser alone, into `workspace` (iq4xs_gemm_workspace_bytes(K, M)): one
 * 17,408-byte block per (128-token tile t, 64-wide K stage s) at offset (t*(K/64) + s)*17408:
 * fp16 q of the tile's tokens (exact integers) in the 128-byte-swizzled K-major layout (token r,
 * 16-byte chunk c at (r/8)*1024 + (r%8)*128 + (c ^ r%8)*16; within each 32-block element 4w+i+16j
 * at position 8w+2i+j), then fp32 d [2][128] (the value of the truncated fp16 d of each Q8_1
 * block) for the stage's two 32-blocks.  Tokens past M are zeros.  For tests. */
int iq4xs_debug_gemm_quantize(const float* X, void* workspace, int64_t K, int64_t M, cudaStream_t stream);
/* The int8 GEMM's quantiser alone: one 18,432-byte block per (128-token tile t, 128-wide K stage s)
 * at offset (t*(K/128) + s)*18432: int8 q in the same swizzled K-major layout (16 values per 16-byte
 * chunk; within each 32-block element 4w+i+16j at position 8w+2i+j), then fp32 d [4][128].
 * K % 128 == 0.  For tests. */
int iq4xs_debug_gemm_i8_quantize(const float* X, void* workspace, int64_t K, int64_t M, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Raw int32 sub-block dot products sum_j kvalues[q_j]*q8_j (before the (ls-32) factor) through
 * the production GEMV kernel's own inner loop: S [B][N][K/32].  Debug / parity entry point for
 * the bit-exact contract of vec_dot_iq4_xs_q8_1 (real_stock_dp4a_comparator.hip:145-160). */
int iq4xs_debug_subblock_dots(const void* W, const void* q8, int32_t* S, int64_t K, int64_t N,
                              int64_t B, cudaStream_t stream);

/* Same as iq4xs_gemv_q8 but forcing the direct-load (non bulk-copy) kernel; for tests. */
int iq4xs_gemv_q8_generic(const void* W, const void* q8, float* Y, int64_t K, int64_t N, int64_t B,
                          cudaStream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Weight-side helpers (data generation, format tools).
 * iq4xs_fill_normal: dst[i] = mean + std * N(0,1) from a counter-based generator (seeded).
 * iq4xs_quantize_weights: fp32 [N][K] -> IQ4_XS rows; the upstream ggml quantize_row_iq4_xs
 *   algorithm without importance matrix (the reference calls it from llama.cpp; not vendored).
 * iq4xs_dequantize: IQ4_XS -> fp32 [N][K] (dequant_mat_iq4xs_cpu semantics, ref_cpu.cpp:115-139). */
int iq4xs_fill_normal(float* dst, int64_t n, uint64_t seed, float mean, float stddev, cudaStream_t stream);
int iq4xs_quantize_weights(const float* src, void* W, int64_t N, int64_t K, cudaStream_t stream);
int iq4xs_dequantize(const void* W, float* out, int64_t K, int64_t N, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------ */
/* Reference-named entry points, same argument meaning, returning cudaError_t like the HIP
 * originals return hipError_t.  The ones without a workspace argument use a library-owned
 * per-(device, stream) workspace that is allocated on the first call of a given size outside
 * stream capture; under capture with no cached workspace they return cudaErrorNotSupported
 * (the reference refuses capture outright, patch:269). */

/* impl_gemv_dp4a_gfx1100.hip:332-341 (the reference's extern "C" symbol), batch 1. */
cudaError_t gemv_iq4xs_dp4a_coop_gpu(const void* W, const float* x, float* y, int64_t K, int64_t N,
                                     cudaStream_t stream);
/* real_stock_dp4a_comparator.hip:480-503, batch 1. */
cudaError_t gemv_iq4xs_stock_dp4a_gpu(const void* W, const float* x, float* y, int64_t K, int64_t N,
                                      cudaStream_t stream);
/* real_stock_dp4a_comparator.hip:266-273: one token, x fp32 [K] -> y [K/32] Q8_1 blocks. */
cudaError_t quantize_row_q8_1_gpu(const float* x, void* y, int64_t K, cudaStream_t stream);
/* real_stock_dp4a_comparator.hip:308-315: playground layout X [K][M] (X[k*M+m]) -> Y [M][K/32]. */
cudaError_t quantize_row_q8_1_batched_gpu(const float* X, void* Y, int64_t K, int64_t M, cudaStream_t stream);

/* real_stock_dp4a_comparator.hip:505-548 and impl_gemm_wmma_stream.hip:321-350: playground layouts
 * X [K][M] (X[k*M+m]) and Y [N][M] (Y[n*M+m]); both run the tensor-core GEMM (K % 512 == 0; an odd
 * K/256 is refused in this output layout). */
cudaError_t gemm_iq4xs_stock_dp4a_gpu(const void* W, const float* X, float* Y, int64_t K, int64_t N,
                                      int64_t M, cudaStream_t stream);
cudaError_t gemm_iq4xs_wmma_stream_gpu(const void* W, const float* X, float* Y, int64_t K, int64_t N,
                                       int64_t M, cudaStream_t stream);

/* ggml MUL_MAT hook (patches/0001-gfx1100-mul-mat-custom.patch).  ggml layouts: W = src0 data
 * (ne00 = K, ne01 = N), x/X = src1 fp32 [M][K], y/Y = dst fp32 [M][N].
 * can_handle: patch:274-277 (GEMV) and :148-151 (GEMM); dispatch: :278-280 and :152-154.
 * GEMV handles M = 1..8 (the patch: M == 1 and three fixed shapes); the batched dispatch is the
 * M > 1 form of the same call.  Any non-success status lets the caller fall back to stock.
 * The GEMV dispatches treat W as static model weights (IQ4XS_FLAG_OVERLAP_PRECEDING).
 * GEMM can_handle: IQ4_XS, M >= 16 (the patch's gate), K % 256 == 0, N >= 1 (patch:148-151; the
 * patch's N % 16 gate is dropped: every N is served). */
bool custom_gemv_iq4xs_can_handle(int64_t K, int64_t N, int64_t M, int type);
cudaError_t custom_gemv_iq4xs_dispatch(const void* W, const float* x, float* y, int64_t K, int64_t N,
                                       cudaStream_t stream);
cudaError_t custom_gemv_iq4xs_dispatch_batched(const void* W, const float* x, float* y, int64_t K,
                                               int64_t N, int64_t M, cudaStream_t stream);
bool custom_gemm_iq4xs_can_handle(int64_t K, int64_t N, int64_t M, int type);
cudaError_t custom_gemm_iq4xs_dispatch(const void* W, const float* X, float* Y, int64_t K, int64_t N,
                                       int64_t M, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* IQ4XS_H */
