/*
 * iq4xs_decoder.h -- decoder-step operations exported by libiq4xs_b200.so.
 *
 * The per-token work of a dense decoder layer between its IQ4_XS GEMVs, fused so that each
 * operation writes the Q8_1 activations of the GEMV that follows it (byte-identical to
 * iq4xs_q8_1_quantize of the same fp32 values).  A decode layer at batch 1 is then
 *
 *   residual_rmsnorm_q8 -> gemv_q8_ex(q|k|v) -> attention_decode_q8 -> gemv_q8_ex(o) [-> all-reduce]
 *   -> residual_rmsnorm_q8 -> gemv_q8_ex(gate|up) -> swiglu_q8 -> gemv_q8_ex(down) [-> all-reduce]
 *
 * The reference has no decoder of its own (its model runs inside llama.cpp, absent from it); these
 * serve the synthetic tensor-parallel decoder of the benchmark configs.  Conventions as in iq4xs.h:
 * status codes, stream-ordered, nothing allocated, graph-capture safe.  flags: IQ4XS_FLAG_PDL lets
 * the kernel launch as a programmatic dependent of the preceding kernel (it waits for it before
 * reading any input); every operation here also lets the kernel after it start early, which is
 * what iq4xs_gemv_q8_ex's IQ4XS_FLAG_OVERLAP_PRECEDING uses.
 */
#ifndef IQ4XS_DECODER_H
#define IQ4XS_DECODER_H

#include <cuda_runtime_api.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IQ4XS_FLAG_PDL 1u
/* iq4xs_dec_attention_decode_q8 with IQ4XS_FLAG_PDL: the position, the cache rows before it and the
 * RoPE tables are not written by the preceding kernel (only qkv is), so the kernel reads them, and
 * requests the K/V rows, before it waits for that kernel.  A decode step qualifies when the position
 * and the cache were last written by earlier tokens' kernels. */
#define IQ4XS_FLAG_ATTN_EARLY_STATE 2u

/* For each of the T rows of x [T][D] (fp32, D % 32 == 0, D <= 8192):
 *   if delta: x += delta (written back; delta [T][D] is e.g. the all-reduced o_proj output)
 *   h = (x * rsqrt(mean(x^2) + eps)) * w          (w [D])
 * and store h as Q8_1 blocks q8 [T][D/32] and/or fp32 h_out [T][D] (either may be null, not both). */
int iq4xs_dec_residual_rmsnorm_q8(float* x, const float* delta, const float* w, int64_t D, int64_t T, float eps,
                                  void* q8, float* h_out, unsigned flags, cudaStream_t stream);

/* Residual + RMSNorm fused into the batch-1 decode GEMV that consumes it:
 *   v = x + delta (delta may be null), h = (v * rsqrt(mean(v^2) + eps)) * w, Y[n] = sum_k W[n][k] q8(h)[k]
 * where q8(h) are the Q8_1 blocks iq4xs_q8_1_quantize would make of h (every CTA of the GEMV builds
 * them in its shared memory; the weight copies start before the kernel waits for x).  If x_out is
 * not null, v is also written there (it must not be x or delta; a decoder alternates two residual
 * buffers).  x, delta, w and x_out 16-byte aligned.  K <= 24576 and the bulk-copy GEMV (K/256 even, W 16-byte aligned), otherwise
 * IQ4XS_ERR_NOT_SUPPORTED.  workspace >= iq4xs_gemv_q8_workspace_bytes(K, N, 1).
 * IQ4XS_FLAG_PDL: W is not written by the preceding kernel (programmatic dependent launch). */
int iq4xs_dec_rmsnorm_gemv(const void* W, const float* x, const float* delta, const float* w, float eps, float* x_out,
                           float* Y, int64_t K, int64_t N, void* workspace, size_t workspace_bytes, unsigned flags,
                           cudaStream_t stream);

/* Attention of one new token at position *pos (a device int64, so a captured graph can advance it):
 *   qkv      fp32 [q_heads + 2*kv_heads][head_dim]: the token's q heads, then k heads, then v heads
 *   k_cache, v_cache  f16 [kv_heads][max_seq][head_dim] (16-byte aligned)
 *   cos_table, sin_table  fp32 [max_seq][head_dim/2]
 * RoPE (rotate-half) is applied to q and the new k; the new k and v are rounded to f16 and written
 * at position *pos; every query head h (kv head h / (q_heads/kv_heads)) attends causally over
 * positions 0..*pos with scores q.k / sqrt(head_dim) and softmax in fp32.  The head outputs
 * [q_heads*head_dim] go to q8 as Q8_1 blocks and, if o_out is not null, as fp32.
 * head_dim == 128, q_heads % kv_heads == 0, max_seq <= 8192.  A position outside [0, max_seq)
 * makes the kernel record device error 5 (iq4xs_device_error) and write nothing. */
int iq4xs_dec_attention_decode_q8(const float* qkv, void* k_cache, void* v_cache, const float* cos_table,
                                  const float* sin_table, const int64_t* pos, int64_t q_heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t max_seq, void* q8, float* o_out, unsigned flags,
                                  cudaStream_t stream);

/* act = silu(gate) * up for gu [T][2F] (gate = columns [0, F), up = [F, 2F)), F % 32 == 0, stored as
 * Q8_1 blocks q8 [T][F/32]. */
int iq4xs_dec_swiglu_q8(const float* gu, int64_t F, int64_t T, void* q8, unsigned flags, cudaStream_t stream);

/* SwiGLU fused into the batch-1 down_proj GEMV: Y[n] = sum_k W[n][k] q8(h)[k] with h = silu(gate) * up
 * from gu [2K] (gate = [0, K), up = [K, 2K)): the Q8_1 blocks iq4xs_dec_swiglu_q8 would write.  For
 * K <= 6144 every CTA of the GEMV builds them in its shared memory; for longer K the standalone SwiGLU
 * kernel writes them into the workspace first (cheaper than K/32 blocks per CTA).  gu 16-byte aligned;
 * the row kernel's K range (K/256 even, K <= 24576, W 16-byte aligned), otherwise
 * IQ4XS_ERR_NOT_SUPPORTED.  workspace >= iq4xs_gemv_workspace_bytes(K, N, 1). */
int iq4xs_dec_swiglu_gemv(const void* W, const float* gu, int64_t K, int64_t N, float* Y, void* workspace,
                          size_t workspace_bytes, unsigned flags, cudaStream_t stream);

/* x [D] fp32 = row *tok of the f16 embedding table emb [vocab][D] (tok: a device int64, so a captured
 * decode step embeds the token the previous step chose).  D % 8 == 0; emb and x 16-byte aligned.  A
 * token outside [0, vocab) makes the kernel record device error 7 and write nothing. */
int iq4xs_dec_embed(const void* emb, const int64_t* tok, int64_t vocab, int64_t D, float* x, unsigned flags,
                    cudaStream_t stream);

/* Greedy sampling: *tok = the index of the largest of logits [n] (the first one on ties; a NaN
 * counts as larger than any number, as in torch.argmax), then *pos += 1 when pos is not null (the
 * decode step's position advances in the same kernel).  tok, pos: device int64. */
int iq4xs_dec_argmax(const float* logits, int64_t n, int64_t* tok, int64_t* pos, unsigned flags, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* IQ4XS_DECODER_H */
