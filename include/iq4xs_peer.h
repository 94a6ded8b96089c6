/*
 * iq4xs_peer.h -- collectives over NVLink peer memory, exported by libiq4xs_b200.so.
 *
 * For the row-sharded GEMV (all-gather of the output slices) and the tensor-parallel decoder
 * (all-reduce of the o_proj / down_proj partial sums) of the benchmark configs, at the message
 * sizes of decode (kilobytes), where a library collective's launch and protocol latency exceeds
 * the transfer.  The reference has no multi-GPU code; these have no counterpart there.
 *
 * Memory: each rank allocates one buffer with iq4xs_peer_alloc, exports it with
 * iq4xs_ipc_handle, exchanges the handles out of band (e.g. torch.distributed.all_gather_object)
 * and maps the peers' buffers with iq4xs_ipc_open (CUDA IPC; no multicast object).  The buffer holds
 * the flag array [world] uint32 and the data areas; a separate device counter (2 x uint32, zero
 * initially) belongs to this rank only.
 *
 * iq4xs_peer_collective: launched on `stream` after the kernel that wrote this rank's contribution
 * into its own buffer (src[rank]); signals every peer, waits (bounded) for every peer's signal of
 * the same collective, then
 *   gather == 0: out[i] = sum over q = 0..world-1 (in this order) of src[q][i], i < n
 *   gather != 0: out[q*n + i] = src[q][i]
 * src[q] and rflags[q] are rank q's data area and flag array as mapped on this rank (src[rank],
 * rflags[rank] this rank's own).  n % 4 == 0; src[q] and out 16-byte aligned.  Every rank must issue the same collectives in the same order;
 * consecutive collectives must use different data areas (alternate two).  A wait that exceeds
 * spin_limit polls (0: a few seconds) records device error 6 (iq4xs_device_error) and returns.
 * Graph-capture safe.
 */
#ifndef IQ4XS_PEER_H
#define IQ4XS_PEER_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IQ4XS_MAX_PEERS 8
#define IQ4XS_IPC_HANDLE_BYTES 64

int iq4xs_peer_alloc(size_t bytes, void** ptr);
int iq4xs_peer_free(void* ptr);
int iq4xs_ipc_handle(void* ptr, void* handle);
int iq4xs_ipc_open(const void* handle, void** ptr);
int iq4xs_ipc_close(void* ptr);
int iq4xs_peer_collective(const float* const* src, uint32_t* const* rflags, uint32_t* flags, uint32_t* counter,
                          int rank, int world, int gather, int64_t n, float* out, uint32_t spin_limit,
                          cudaStream_t stream);

/* Row-parallel decode GEMV with the all-reduce fused in (push model, low-latency protocol), for the
 * tensor-parallel decoder's o_proj / down_proj.  One data area of every rank holds `world` slots of
 * N 64-bit words; word i of slot q is rank q's partial output i (fp32 bits, low half) tagged with the
 * epoch of the all-reduce (high half).  The producer, iq4xs_dec_gemv_q8_push, is a batch-1 GEMV whose
 * epilogue stores each output, tagged, into slot `rank` of every rank's area (single 8-byte NVLink
 * stores, no fence, no flag: the tag travels with the value); the last CTA to finish advances this
 * rank's epoch counter.  There is no collective kernel.  The consumers are the next kernel of the
 * decode step: iq4xs_dec_rmsnorm_gemv_peer and iq4xs_dec_residual_rmsnorm_q8_peer read each word until
 * its tag is the current epoch (bounded polls) and take delta[i] = sum over q = 0..world-1, in this
 * order, of slot q's value -- the same bits as iq4xs_peer_collective's all-reduce.  The epoch counter
 * is the one iq4xs_peer_collective advances (the two can be mixed in one sequence; every rank runs
 * the same sequence).  The descriptor lives in DEVICE memory (the kernels read it) and is built
 * once per area by the caller.  A consumer must directly follow its producer's kernel on the stream
 * (or follow its completion); two consecutive fused all-reduces must use different areas.
 * Graph-capture safe. */
typedef struct iq4xs_peer_slots {
    uint64_t* dst[IQ4XS_MAX_PEERS];  /* slot `rank` of rank q's area, as mapped on this rank */
    const uint64_t* local;           /* this rank's area: slot q at local + q*N */
    uint32_t* counter;               /* this rank's epoch counter (2 x uint32, as for iq4xs_peer_collective) */
    int32_t rank, world;
    uint32_t spin_limit;             /* polls before a read gives up (device error 6); 0: a few seconds */
    uint32_t reserved;
} iq4xs_peer_slots;

/* Y = W . q8 (batch 1, iq4xs_gemv_q8 arithmetic) into slot `rank` of every rank's area (`slots`, a
 * device pointer), each output tagged with the all-reduce's epoch; the grid's last CTA advances this
 * rank's epoch counter.  The row kernel's K range (K % 512 == 0, K <= 24576, W 16-byte aligned);
 * otherwise IQ4XS_ERR_NOT_SUPPORTED.  flags: IQ4XS_FLAG_PDL. */
int iq4xs_dec_gemv_q8_push(const void* W, const void* q8, int64_t K, int64_t N, const iq4xs_peer_slots* slots,
                           void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream);
/* iq4xs_dec_swiglu_gemv with the outputs pushed into slot `rank` of every rank's area, as
 * iq4xs_dec_gemv_q8_push does. */
int iq4xs_dec_swiglu_gemv_push(const void* W, const float* gu, int64_t K, int64_t N, const iq4xs_peer_slots* slots,
                               void* workspace, size_t workspace_bytes, unsigned flags, cudaStream_t stream);
/* iq4xs_dec_rmsnorm_gemv with delta = the fused all-reduce of `slots` (K = the slots' N). */
int iq4xs_dec_rmsnorm_gemv_peer(const void* W, const float* x, const iq4xs_peer_slots* slots, const float* w, float eps,
                                float* x_out, float* Y, int64_t K, int64_t N, void* workspace, size_t workspace_bytes,
                                unsigned flags, cudaStream_t stream);
/* iq4xs_dec_residual_rmsnorm_q8 (one token, T = 1) with delta = the fused all-reduce of `slots`. */
int iq4xs_dec_residual_rmsnorm_q8_peer(float* x, const iq4xs_peer_slots* slots, const float* w, int64_t D, float eps,
                                       void* q8, float* h_out, unsigned flags, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* IQ4XS_PEER_H */
