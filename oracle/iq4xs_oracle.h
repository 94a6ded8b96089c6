/*
 * iq4xs_oracle.h -- CPU restatement of the reference's IQ4_XS x Q8_1 matmul pipeline.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: it may be loaded by tests/,
 * by __graft_entry__.smoke() and by bench.py's cpu_baseline leg, and by nothing else.
 * The product (qwen_3.8_27b_optimizations_b200/) never links or calls it.
 *
 * Every function restates a piece of the reference (paths relative to the reference
 * project root); the citations are repeated next to each definition in iq4xs_oracle.c.
 *
 *   block_iq4_xs layout, codebook ........ kernels/common/block_iq4_xs.h:10-24
 *   fp16 -> fp32 (exact) .................. kernels/common/block_iq4_xs.h:34-68
 *   fp32 -> fp16 (truncating) ............. kernels/common/block_iq4_xs.h:71-86,
 *                                          kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:43-62
 *   Q8_1 activation quantizer ............. real_stock_dp4a_comparator.hip:230-264 (device form x/d)
 *   codebook gather of 8 nibbles .......... real_stock_dp4a_comparator.hip:105-131
 *   per-sub-block dot (vec_dot_iq4_xs_q8_1) real_stock_dp4a_comparator.hip:145-166
 *   FP64 dequant oracles .................. kernels/matmul_iq4xs/ref_cpu.cpp:12-139
 *   IQ4_XS weight quantizer ............... upstream ggml quantize_row_iq4_xs (llama.cpp bb4caa75,
 *                                          not vendored in the reference; restated algorithm)
 *
 * Parity pin: see tests/golden/make_golden.py -- the FP64 and dequant paths are checked against
 * the reference's own ref_cpu.cpp compiled into oracle/_ref/, the integer pipeline against
 * known-answer vectors derived from the reference formulas.
 */
#ifndef IQ4XS_ORACLE_H
#define IQ4XS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_QK_K 256
#define OR_QK8_1 32

#pragma pack(push, 1)
typedef struct {
    uint16_t d;
    uint16_t scales_h;
    uint8_t scales_l[4];
    uint8_t qs[128];
} or_block_iq4_xs;

typedef struct {
    uint16_t d;   /* low half of ds: truncated fp16 of amax/127 */
    uint16_t s;   /* high half of ds: truncated fp16 of the block sum */
    int8_t qs[32];
} or_block_q8_1;
#pragma pack(pop)

extern const int8_t or_kvalues_iq4nl[16];

float or_fp16_to_fp32(uint16_t h);
uint16_t or_fp32_to_fp16_trunc(float f);
uint16_t or_fp32_to_fp16_rne(float f);

/* Scale code ls (0..63) of sub-block ib of one block. */
int or_iq4xs_scale(const or_block_iq4_xs* b, int ib);

/* X: fp32 [M][K] (token-major) -> Y: [M][K/32] Q8_1 blocks. */
void or_quantize_q8_1(const float* X, or_block_q8_1* Y, int64_t K, int64_t M);

/* Raw int32 dot of one sub-block: sum_j kvalues[q_j] * q8_j (before the (ls-32) factor). */
int32_t or_subblock_dot(const or_block_iq4_xs* b, int ib, const or_block_q8_1* q);

/* S: int32 [M][N][K/32] raw sub-block dots. */
void or_subblock_dots(const or_block_iq4_xs* W, const or_block_q8_1* Q, int32_t* S,
                      int64_t K, int64_t N, int64_t M);

/* Reference fp32 term of one (row, sub-block, token): (d_w*d_x)_f32 * (float)(sumi*(ls-32)). */
float or_term_f32(const or_block_iq4_xs* b, int ib, const or_block_q8_1* q);

/* FP64 oracle of the quantised pipeline.  Y[m][N] = sum_sb (double)term_f32;
 * A[m][N] = sum_sb |term| (for cancellation-aware tolerances).  A may be NULL. */
void or_matmul_q8(const or_block_iq4_xs* W, const or_block_q8_1* Q, double* Y, double* A,
                  int64_t K, int64_t N, int64_t M);

/* Same pipeline, fp32 accumulation in the reference stock GEMV order (one lane per row). */
void or_matmul_q8_f32(const or_block_iq4_xs* W, const or_block_q8_1* Q, float* Y,
                      int64_t K, int64_t N, int64_t M);

/* FP64 dequant-and-dot on unquantised fp32 activations (ref_cpu.cpp restated).
 * X: fp32 [M][K], Y: fp32 [M][N]. */
void or_matmul_f64(const or_block_iq4_xs* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M);

void or_dequantize(const or_block_iq4_xs* W, float* out, int64_t K, int64_t N);

/* IQ4_XS weight quantizer (no importance matrix).  src: fp32 [nrows][n_per_row]. */
void or_quantize_iq4_xs(const float* src, or_block_iq4_xs* dst, int64_t nrows, int64_t n_per_row);

#ifdef __cplusplus
}
#endif

#endif
