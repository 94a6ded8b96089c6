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

#ifdef __cplusplus
}
#endif

#endif /* IQ4XS_PEER_H */
