// bench_host.cu -- the C++ end-to-end driver declared in include/iq4xs_bench.h.
//
// A host that feeds the ggml hook from host memory the way a serving loop would: every GEMV's
// activations are copied in from pinned host memory and its result copied back, on two copy
// streams, so that GEMV i's kernels overlap the upload of GEMV i+1's activations and the download
// of GEMV i-1's result (two device slots for x and y, events between the three streams).
#include <cuda_runtime.h>

#include "../../include/iq4xs.h"
#include "../../include/iq4xs_bench.h"

extern "C" int iq4xs_bench_e2e_gemv(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                                    const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                                    float* dev_x, float* dev_y, int steps, cudaStream_t stream, float* ms) {
    int64_t max_x = 0, max_y = 0;
    for (int bi = 0; bi < nbatch; ++bi)
        for (int i = 0; i < nmat; ++i) {
            max_x = batches[bi] * K[i] > max_x ? batches[bi] * K[i] : max_x;
            max_y = batches[bi] * N[i] > max_y ? batches[bi] * N[i] : max_y;
        }
    // the second device slot (the caller's buffers are slot 0)
    float *dx1 = nullptr, *dy1 = nullptr;
    cudaError_t e = cudaMalloc(&dx1, (size_t)max_x * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&dy1, (size_t)max_y * sizeof(float));
    cudaStream_t up = nullptr, down = nullptr;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&up, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&down, cudaStreamNonBlocking);
    cudaEvent_t e0 = nullptr, e1 = nullptr, x_ready[2] = {}, done[2] = {}, y_free[2] = {};
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    for (int s = 0; s < 2 && e == cudaSuccess; ++s) {
        e = cudaEventCreateWithFlags(&x_ready[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&y_free[s], cudaEventDisableTiming);
    }
    int rc = (int)e;
    float* dx[2] = {dev_x, dx1};
    float* dy[2] = {dev_y, dy1};
    float* hy[2] = {host_y, host_y + max_y};  // host_y holds two results
    if (!rc) {
        cudaEventRecord(e0, stream);
        cudaStreamWaitEvent(up, e0, 0);
        cudaStreamWaitEvent(down, e0, 0);
        int64_t call = 0;
        for (int s = 0; s < steps && !rc; ++s)
            for (int bi = 0; bi < nbatch && !rc; ++bi)
                for (int i = 0; i < nmat && !rc; ++i, ++call) {
                    const int slot = (int)(call & 1);
                    const int64_t b = batches[bi];
                    // upload: slot's x is free once the GEMV two calls back has finished
                    if (call >= 2) cudaStreamWaitEvent(up, done[slot], 0);
                    e = cudaMemcpyAsync(dx[slot], host_x, (size_t)(b * K[i]) * sizeof(float), cudaMemcpyHostToDevice, up);
                    if (e == cudaSuccess) e = cudaEventRecord(x_ready[slot], up);
                    // compute: needs the upload and the slot's y read back from two calls ago
                    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, x_ready[slot], 0);
                    if (e == cudaSuccess && call >= 2) e = cudaStreamWaitEvent(stream, y_free[slot], 0);
                    if (e == cudaSuccess) e = custom_gemv_iq4xs_dispatch_batched(W[i], dx[slot], dy[slot], K[i], N[i], b, stream);
                    if (e == cudaSuccess) e = cudaEventRecord(done[slot], stream);
                    // download
                    if (e == cudaSuccess) e = cudaStreamWaitEvent(down, done[slot], 0);
                    if (e == cudaSuccess)
                        e = cudaMemcpyAsync(hy[slot], dy[slot], (size_t)(b * N[i]) * sizeof(float), cudaMemcpyDeviceToHost, down);
                    if (e == cudaSuccess) e = cudaEventRecord(y_free[slot], down);
                    if (e != cudaSuccess) rc = (int)e;
                }
        // join: the last download ends the timed region
        cudaEventRecord(y_free[0], down);
        cudaStreamWaitEvent(stream, y_free[0], 0);
        cudaEventRecord(e1, stream);
        e = cudaStreamSynchronize(stream);
        if (!rc && e != cudaSuccess) rc = (int)e;
        float t = 0.0f;
        cudaEventElapsedTime(&t, e0, e1);
        if (ms) *ms = t;
    }
    cudaStreamSynchronize(up);
    cudaStreamSynchronize(down);
    for (int s = 0; s < 2; ++s) {
        if (x_ready[s]) cudaEventDestroy(x_ready[s]);
        if (done[s]) cudaEventDestroy(done[s]);
        if (y_free[s]) cudaEventDestroy(y_free[s]);
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (up) cudaStreamDestroy(up);
    if (down) cudaStreamDestroy(down);
    if (dx1) cudaFree(dx1);
    if (dy1) cudaFree(dy1);
    return rc;
}
