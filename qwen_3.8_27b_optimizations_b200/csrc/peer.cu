// peer.cu -- small collectives over NVLink peer memory (CUDA IPC), for the row-sharded GEMV and the
// tensor-parallel decoder of the benchmark configs (the reference has no multi-GPU code).
//
// Every rank owns one shared buffer (cudaMalloc'd here, mapped into the other ranks with CUDA IPC;
// no multicast object, no NVLS).  A collective is one kernel launched after the kernel that wrote
// this rank's contribution into its own shared buffer (plain local stores, completed at that
// kernel's end):
//   1. CTA 0, thread 0: fence.sc.sys, then st.release.sys of the epoch into flags[rank] of every
//      peer;
//   2. every CTA waits (bounded, nanosleep backoff) until its own flags[q] has reached the epoch for
//      every peer q, with ld.acquire.sys;
//   3. every CTA pulls its share of the data from all ranks' buffers with plain P2P loads:
//      all-reduce = sum over ranks in rank order (identical bits on every rank), all-gather =
//      concatenation of equal slices.
// The epoch is this rank's device-side counter + 1 (every rank runs the same collectives in the same
// order, so the counters agree; CUDA graphs replay it correctly).  The last CTA to finish advances
// the counter.  A wait that gives up records kDevErrPeerWait in the device error word and the kernel
// goes on (the data of that call is then undefined, nothing hangs).  Callers alternate two buffers
// between consecutive collectives: a rank overwrites a buffer only after the next barrier, which no
// peer passes before it has finished reading that buffer.
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/iq4xs.h"
#include "../../include/iq4xs_peer.h"
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {
namespace {
constexpr int kPeerThreads = 256;

struct PeerArgs {
    const float* src[IQ4XS_MAX_PEERS];   // rank q's contribution, as mapped on this rank
    uint32_t* rflags[IQ4XS_MAX_PEERS];   // rank q's flag array, as mapped on this rank
    uint32_t* flags;                     // this rank's flag array [world] (written by the peers)
    uint32_t* counter;                   // [0] epoch counter, [1] finished-CTA count
    float* out;
    int64_t n;                           // all-reduce: elements; all-gather: elements per slice
    int rank, world, gather;
    uint32_t spin_limit;
    uint32_t* err;
};

__global__ void __launch_bounds__(kPeerThreads) peer_collective_kernel(const PeerArgs a) {
    __shared__ uint32_t epoch;
    if (threadIdx.x == 0) epoch = a.counter[0] + 1u;
    __syncthreads();
    const uint32_t e = epoch;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < a.world; ++q)
            if (q != a.rank) st_release_sys(a.rflags[q] + a.rank, e);
    }
    if (threadIdx.x < a.world && (int)threadIdx.x != a.rank) {
        const uint32_t* f = a.flags + threadIdx.x;
        uint32_t i = 0;
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            if (++i > a.spin_limit) {
                record_error(a.err, kDevErrPeerWait);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    // One float4 per thread and source, every load issued before any is used (n % 4 == 0): a
    // single NVLink round trip for the decode-size messages (the grid covers them in one pass).
    const int64_t n4 = a.n >> 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (a.gather) {
        const int64_t total = n4 * a.world;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int q = (int)(i / n4);
            reinterpret_cast<float4*>(a.out)[i] = reinterpret_cast<const float4*>(a.src[q])[i - (int64_t)q * n4];
        }
    } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
            float4 v[IQ4XS_MAX_PEERS];
#pragma unroll
            for (int q = 0; q < IQ4XS_MAX_PEERS; ++q)
                if (q < a.world) v[q] = reinterpret_cast<const float4*>(a.src[q])[i];
            float4 s = v[0];
#pragma unroll
            for (int q = 1; q < IQ4XS_MAX_PEERS; ++q)
                if (q < a.world) {
                    s.x += v[q].x;
                    s.y += v[q].y;
                    s.z += v[q].z;
                    s.w += v[q].w;
                }
            reinterpret_cast<float4*>(a.out)[i] = s;
        }
    }
    // the last CTA to finish advances the epoch counter (every CTA has read it by now)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.counter + 1, 1u) == gridDim.x - 1) {
            a.counter[1] = 0u;
            a.counter[0] = e;
        }
    }
}

bool aligned(const void* p, uintptr_t al) { return (reinterpret_cast<uintptr_t>(p) & (al - 1)) == 0; }
}  // namespace
}  // namespace iq4xs

using namespace iq4xs;

extern "C" {

int iq4xs_peer_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    *ptr = nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return IQ4XS_ERR_CUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess) {
        cudaFree(p);
        return IQ4XS_ERR_CUDA;
    }
    *ptr = p;
    return IQ4XS_OK;
}

int iq4xs_peer_free(void* ptr) {
    if (!ptr) return IQ4XS_ERR_INVALID_ARGUMENT;
    return cudaFree(ptr) == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
}

int iq4xs_ipc_handle(void* ptr, void* handle) {
    if (!ptr || !handle) return IQ4XS_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return IQ4XS_ERR_CUDA;
    static_assert(sizeof(h) == IQ4XS_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof h);
    return IQ4XS_OK;
}

int iq4xs_ipc_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return IQ4XS_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    *ptr = nullptr;
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
}

int iq4xs_ipc_close(void* ptr) {
    if (!ptr) return IQ4XS_ERR_INVALID_ARGUMENT;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
}

int iq4xs_peer_collective(const float* const* src, uint32_t* const* rflags, uint32_t* flags, uint32_t* counter,
                          int rank, int world, int gather, int64_t n, float* out, uint32_t spin_limit,
                          cudaStream_t stream) {
    if (!src || !rflags || !flags || !counter || !out || n <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (n % 4 != 0) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if (world < 1 || world > IQ4XS_MAX_PEERS || rank < 0 || rank >= world) return IQ4XS_ERR_INVALID_ARGUMENT;
    PeerArgs a = {};
    for (int q = 0; q < world; ++q) {
        if (!src[q] || !rflags[q]) return IQ4XS_ERR_INVALID_ARGUMENT;
        if (!aligned(src[q], 16) || !aligned(rflags[q], 4)) return IQ4XS_ERR_MISALIGNED;
        a.src[q] = src[q];
        a.rflags[q] = rflags[q];
    }
    if (!aligned(flags, 4) || !aligned(counter, 8) || !aligned(out, 16)) return IQ4XS_ERR_MISALIGNED;
    a.flags = flags;
    a.counter = counter;
    a.out = out;
    a.n = n;
    a.rank = rank;
    a.world = world;
    a.gather = gather ? 1 : 0;
    a.spin_limit = spin_limit ? spin_limit : (1u << 24);  // a few seconds: ranks may arrive skewed
    a.err = device_error_word();
    if (!a.err) return IQ4XS_ERR_CUDA;
    const int64_t total4 = (gather ? n * world : n) / 4;
    const int grid = (int)imin64((total4 + kPeerThreads - 1) / kPeerThreads, (int64_t)device_sm_count() * 4);
    peer_collective_kernel<<<grid < 1 ? 1 : grid, kPeerThreads, 0, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? IQ4XS_OK : IQ4XS_ERR_CUDA;
}

}  // extern "C"
