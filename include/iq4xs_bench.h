/*
 * iq4xs_bench.h -- host-side measurement driver exported by libiq4xs_b200.so.
 *
 * Not part of the matmul path: it is the C++ caller a ggml-style host would be, used by bench.py
 * to time the reference-facing entry point end to end (pinned host inputs in, results back to
 * the host, every step).  It has no counterpart in the reference, whose harness does the same
 * from bench_gemv_dp4a.cpp with device-resident inputs.
 */
#ifndef IQ4XS_BENCH_H
#define IQ4XS_BENCH_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Floats of one pass's concatenated layout for row lengths L[0..nmat): the sum over every batch
 * size b and matrix i of b*L[i] rounded up to a multiple of 64 (each call's segment starts on a
 * 256-byte boundary).  L = K gives the input layout, L = N the output layout. */
int64_t iq4xs_bench_e2e_floats(const int64_t* L, int nmat, const int64_t* batches, int nbatch);

/* Runs `steps` passes; one pass = one cudaMemcpyAsync of the pass's inputs (dev x <- host_x, the
 * input layout), then for every batch size b in batches[0..nbatch) and every matrix i
 * custom_gemv_iq4xs_dispatch_batched(W[i], x segment, y segment, K[i], N[i], b) on `stream`, then
 * one cudaMemcpyAsync of the pass's results (host_y <- dev y, the output layout).  The copies run on
 * two copy streams of the driver and overlap the neighbouring passes' GEMVs (two device slots: the
 * caller's dev_x / dev_y and a second pair the driver allocates before the timed region).  host_x /
 * dev_x hold the input layout, host_y / dev_y the output layout; host buffers pinned.  *ms =
 * elapsed device time between events recorded on `stream` before the first upload and after the
 * last download.  Returns 0 or the first failing cudaError_t. */
int iq4xs_bench_e2e_gemv(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                         const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                         float* dev_x, float* dev_y, int steps, cudaStream_t stream, float* ms);

/* iq4xs_bench_e2e_gemv with one iq4xs_gemv_grouped call per batch size over the nmat matrices
 * (nmat <= IQ4XS_MAX_GROUP) instead of one hook call per matrix; `workspace` holds at least
 * iq4xs_gemv_grouped_workspace_bytes for the largest batch (256-byte aligned). */
int iq4xs_bench_e2e_gemv_grouped(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                                 const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                                 float* dev_x, float* dev_y, void* workspace, size_t workspace_bytes, int steps,
                                 cudaStream_t stream, float* ms);

#ifdef __cplusplus
}
#endif

#endif
