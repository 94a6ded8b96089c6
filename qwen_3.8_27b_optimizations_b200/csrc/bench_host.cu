// bench_host.cu -- the C++ end-to-end driver declared in include/iq4xs_bench.h.
//
// A host that feeds the ggml hook from host memory the way a pipelined serving loop would: each
// pass's activations are uploaded from pinned host memory in one copy and its results downloaded in
// one copy, on two copy streams, so that pass p's GEMVs overlap the upload of pass p+1's inputs and
// the download of pass p-1's results (two device slots for x and y, events between the three
// streams; the compute stream waits once per pass, so consecutive hook calls of a pass run back to
// back as they would inside one ggml graph).
#include <cuda_runtime.h>

#include "../../include/iq4xs.h"
#include "../../include/iq4xs_bench.h"

namespace {

// Offsets of the calls of one pass in the concatenated x / y layouts (floats; every segment starts
// on a 256-byte boundary).
constexpr int64_t kSegAlign = 64;
int64_t seg_round(int64_t n) { return (n + kSegAlign - 1) / kSegAlign * kSegAlign; }

struct Pipe {
    float* dx[2] = {};
    float* dy[2] = {};
    int64_t x_total = 0, y_total = 0;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t x_ready[2] = {}, done[2] = {}, y_free[2] = {};
};

int64_t pass_floats(const int64_t* L, int nmat, const int64_t* batches, int nbatch) {
    int64_t t = 0;
    for (int bi = 0; bi < nbatch; ++bi)
        for (int i = 0; i < nmat; ++i) t += seg_round(batches[bi] * L[i]);
    return t;
}

cudaError_t pipe_create(Pipe& p, const int64_t* K, const int64_t* N, int nmat, const int64_t* batches, int nbatch,
                        float* dev_x, float* dev_y) {
    p.x_total = pass_floats(K, nmat, batches, nbatch);
    p.y_total = pass_floats(N, nmat, batches, nbatch);
    p.dx[0] = dev_x;
    p.dy[0] = dev_y;
    cudaError_t e = cudaMalloc(&p.dx[1], (size_t)p.x_total * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&p.dy[1], (size_t)p.y_total * sizeof(float));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking);
    for (int s = 0; s < 2 && e == cudaSuccess; ++s) {
        e = cudaEventCreateWithFlags(&p.x_ready[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.done[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p.y_free[s], cudaEventDisableTiming);
    }
    return e;
}

void pipe_destroy(Pipe& p) {
    if (p.up) cudaStreamSynchronize(p.up);
    if (p.down) cudaStreamSynchronize(p.down);
    for (int s = 0; s < 2; ++s) {
        if (p.x_ready[s]) cudaEventDestroy(p.x_ready[s]);
        if (p.done[s]) cudaEventDestroy(p.done[s]);
        if (p.y_free[s]) cudaEventDestroy(p.y_free[s]);
    }
    if (p.up) cudaStreamDestroy(p.up);
    if (p.down) cudaStreamDestroy(p.down);
    if (p.dx[1]) cudaFree(p.dx[1]);
    if (p.dy[1]) cudaFree(p.dy[1]);
}

// Pass `pass`: upload -> every hook call of the pass -> download.  Passes two apart share a slot and
// are ordered by events.
// Grouped mode: one iq4xs_gemv_grouped call per batch size over all matrices (workspace != null).
struct Grouped {
    void* ws = nullptr;
    size_t ws_bytes = 0;
};

cudaError_t enqueue_pass(Pipe& p, int pass, const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                         const int64_t* batches, int nbatch, const float* host_x, float* host_y, cudaStream_t stream,
                         const Grouped& grouped) {
    const int slot = pass & 1;
    cudaError_t e = cudaSuccess;
    // upload: the slot's x is free once the compute of pass-2 has finished
    if (pass >= 2) e = cudaStreamWaitEvent(p.up, p.done[slot], 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p.dx[slot], host_x, (size_t)p.x_total * sizeof(float), cudaMemcpyHostToDevice, p.up);
    if (e == cudaSuccess) e = cudaEventRecord(p.x_ready[slot], p.up);
    // compute: needs this pass's upload and the slot's y read back by the download of pass-2
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, p.x_ready[slot], 0);
    if (e == cudaSuccess && pass >= 2) e = cudaStreamWaitEvent(stream, p.y_free[slot], 0);
    int64_t xo = 0, yo = 0;
    for (int bi = 0; bi < nbatch && e == cudaSuccess; ++bi) {
        const int64_t b = batches[bi];
        iq4xs_gemv_problem prob[IQ4XS_MAX_GROUP];
        for (int i = 0; i < nmat && e == cudaSuccess; ++i) {
            if (grouped.ws) {
                prob[i] = {W[i], p.dx[slot] + xo, p.dy[slot] + yo, K[i], N[i]};
            } else {
                e = custom_gemv_iq4xs_dispatch_batched(W[i], p.dx[slot] + xo, p.dy[slot] + yo, K[i], N[i], b, stream);
            }
            xo += seg_round(b * K[i]);
            yo += seg_round(b * N[i]);
        }
        if (grouped.ws && e == cudaSuccess &&
            iq4xs_gemv_grouped(prob, nmat, b, grouped.ws, grouped.ws_bytes, IQ4XS_FLAG_OVERLAP_PRECEDING, stream) != 0)
            e = cudaErrorLaunchFailure;
    }
    if (e == cudaSuccess) e = cudaEventRecord(p.done[slot], stream);
    // download
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p.down, p.done[slot], 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(host_y, p.dy[slot], (size_t)p.y_total * sizeof(float), cudaMemcpyDeviceToHost, p.down);
    if (e == cudaSuccess) e = cudaEventRecord(p.y_free[slot], p.down);
    return e;
}
}  // namespace

extern "C" int64_t iq4xs_bench_e2e_floats(const int64_t* L, int nmat, const int64_t* batches, int nbatch) {
    return pass_floats(L, nmat, batches, nbatch);
}

namespace {
int run_e2e(const void* const* W, const int64_t* K, const int64_t* N, int nmat, const int64_t* batches, int nbatch,
            const float* host_x, float* host_y, float* dev_x, float* dev_y, int steps, cudaStream_t stream, float* ms,
            const Grouped& grouped) {
    if (grouped.ws && (nmat < 1 || nmat > IQ4XS_MAX_GROUP)) return (int)cudaErrorInvalidValue;
    Pipe p;
    cudaEvent_t e0 = nullptr, e1 = nullptr, ju = nullptr, jd = nullptr;
    cudaError_t e = pipe_create(p, K, N, nmat, batches, nbatch, dev_x, dev_y);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ju, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&jd, cudaEventDisableTiming);
    if (e == cudaSuccess) {
        // fork the copy streams off `stream` at e0, run the passes, join them back before e1
        e = cudaEventRecord(e0, stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p.up, e0, 0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p.down, e0, 0);
        for (int s = 0; s < steps && e == cudaSuccess; ++s)
            e = enqueue_pass(p, s, W, K, N, nmat, batches, nbatch, host_x, host_y, stream, grouped);
        if (e == cudaSuccess) e = cudaEventRecord(ju, p.up);
        if (e == cudaSuccess) e = cudaEventRecord(jd, p.down);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ju, 0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, jd, 0);  // the last download ends the timed region
        cudaEventRecord(e1, stream);
        const cudaError_t es = cudaStreamSynchronize(stream);
        if (e == cudaSuccess) e = es;
        float t = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
        if (ms) *ms = t;
    }
    pipe_destroy(p);
    for (cudaEvent_t ev : {e0, e1, ju, jd})
        if (ev) cudaEventDestroy(ev);
    return (int)e;
}
}  // namespace

extern "C" int iq4xs_bench_e2e_gemv(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                                    const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                                    float* dev_x, float* dev_y, int steps, cudaStream_t stream, float* ms) {
    return run_e2e(W, K, N, nmat, batches, nbatch, host_x, host_y, dev_x, dev_y, steps, stream, ms, Grouped{});
}

extern "C" int iq4xs_bench_e2e_gemv_grouped(const void* const* W, const int64_t* K, const int64_t* N, int nmat,
                                            const int64_t* batches, int nbatch, const float* host_x, float* host_y,
                                            float* dev_x, float* dev_y, void* workspace, size_t workspace_bytes,
                                            int steps, cudaStream_t stream, float* ms) {
    if (!workspace) return (int)cudaErrorInvalidValue;
    Grouped g;
    g.ws = workspace;
    g.ws_bytes = workspace_bytes;
    return run_e2e(W, K, N, nmat, batches, nbatch, host_x, host_y, dev_x, dev_y, steps, stream, ms, g);
}
