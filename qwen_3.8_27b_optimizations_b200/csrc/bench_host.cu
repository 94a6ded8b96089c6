// bench_host.cu -- the C++ end-to-end driver declared in include/iq4xs_bench.h.
#include "../../include/iq4xs.h"
#include "../../include/iq4xs_bench.h"

extern "C" int iq4xs_bench_e2e_gemv(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                                    const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                                    float* dev_x, float* dev_y, int steps, cudaStream_t stream, float* ms) {
    cudaEvent_t e0, e1;
    cudaError_t e = cudaEventCreate(&e0);
    if (e != cudaSuccess) return (int)e;
    if ((e = cudaEventCreate(&e1)) != cudaSuccess) return (int)e;
    int rc = 0;
    cudaEventRecord(e0, stream);
    for (int s = 0; s < steps && !rc; ++s)
        for (int bi = 0; bi < nbatch && !rc; ++bi)
            for (int i = 0; i < nmat && !rc; ++i) {
                const int64_t b = batches[bi];
                e = cudaMemcpyAsync(dev_x, host_x, (size_t)(b * K[i]) * sizeof(float), cudaMemcpyHostToDevice, stream);
                if (e == cudaSuccess) e = custom_gemv_iq4xs_dispatch_batched(W[i], dev_x, dev_y, K[i], N[i], b, stream);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(host_y, dev_y, (size_t)(b * N[i]) * sizeof(float), cudaMemcpyDeviceToHost, stream);
                if (e != cudaSuccess) rc = (int)e;
            }
    cudaEventRecord(e1, stream);
    e = cudaStreamSynchronize(stream);
    if (!rc && e != cudaSuccess) rc = (int)e;
    float t = 0.0f;
    cudaEventElapsedTime(&t, e0, e1);
    if (ms) *ms = t;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return rc;
}
