// gemv_grouped.cu -- iq4xs_gemv_grouped: several independent decode GEMVs of one batch size in one
// launch sequence.
//
// A decode step of a ggml graph reads one activation vector with several IQ4_XS matrices that are
// separate tensors (attn_q / attn_k / attn_v, ffn_gate / ffn_up), and the reference runs each as its
// own GEMV (patches/0001-gfx1100-mul-mat-custom.patch:278-280, one call per MUL_MAT node).  On B200 a
// GEMV launch pays a fixed cost of a few microseconds (launch, the first weight bytes, the tail of
// the last CTAs) that a 2.8 MB k_proj cannot hide.  Here the matrices share one grid: matrix i gets a
// contiguous slice of the CTAs, handed out one at a time to the matrix whose busiest CTA is estimated
// slowest at the kernels' own work granularity (cta_cost), so that the whole group ends together.
//
//  1. q8_1_grouped_kernel quantises every problem's activations into its slice of the workspace
//     (q8_1_block_store: the bytes of iq4xs_q8_1_quantize);
//  2. the grouped GEMV (batch 1: row kernel, gemv.cu; batch 2..8: tensor-core kernel, gemv_mma.cu)
//     runs as a programmatic dependent: its weight copies start while the quantiser runs;
//  3. when a tensor-core matrix is split into K parts, reduce_grouped_kernel adds the parts in part
//     order (deterministic), again as a programmatic dependent.
// Groups the grouped kernels do not take (a W that is not 16-byte aligned, K % 512 != 0, batch 1 with
// K > 24576) run as one iq4xs_gemv_f32_ex call per problem on the same workspace slices.
#include <algorithm>
#include <cstring>

#include "../../include/iq4xs.h"
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

namespace {
struct GroupQuantParams {
    const float* x[kMaxGroup];
    uint8_t* q8[kMaxGroup];
    int64_t off[kMaxGroup + 1];  // first Q8_1 block of each problem in the concatenated block index
    int count;
};

// One warp per Q8_1 block of the concatenated [problem][token][K/32] block list.  Problem p's x is
// [B][K] contiguous, so its local block j covers x[32j .. 32j+31] and lands at q8 + 36j.
__global__ void __launch_bounds__(256) q8_1_grouped_kernel(const __grid_constant__ GroupQuantParams G) {
    grid_dependency_wait();
    grid_launch_dependents();  // the GEMV's weight stream may start; it waits for this grid before reading q8
    const int lane = threadIdx.x & 31;
    const int64_t total = G.off[G.count];
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total; blk += nwarps) {
        int p = 0;
        while (p + 1 < G.count && blk >= G.off[p + 1]) ++p;
        const int64_t j = blk - G.off[p];
        q8_1_block_store(G.x[p][j * kQK8 + lane], G.q8[p] + j * kQ8Bytes, lane);
    }
}

struct GroupReduceParams {
    const float* partial[kMaxGroup];  // [parts][B*N]
    float* y[kMaxGroup];              // [B*N]
    int parts[kMaxGroup];
    int64_t bn[kMaxGroup];
    int64_t off[kMaxGroup + 1];       // first output of each problem in the concatenated output index
    int count;
};

// y = sum of the K parts in part order, for every problem of the group that was split.
__global__ void __launch_bounds__(256) reduce_grouped_kernel(const __grid_constant__ GroupReduceParams G) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int64_t total = G.off[G.count];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int p = 0;
        while (p + 1 < G.count && i >= G.off[p + 1]) ++p;
        const int64_t j = i - G.off[p];
        const float* src = G.partial[p] + j;
        const int64_t bn = G.bn[p];
        const int parts = G.parts[p];
        // the loads of four parts are issued before any is added (their latencies overlap); the adds
        // stay in part order
        float sum = 0.0f;
        int q = 0;
        for (; q + 4 <= parts; q += 4) {
            const float v0 = src[(int64_t)q * bn], v1 = src[(int64_t)(q + 1) * bn];
            const float v2 = src[(int64_t)(q + 2) * bn], v3 = src[(int64_t)(q + 3) * bn];
            sum = (((sum + v0) + v1) + v2) + v3;
        }
        for (; q < parts; ++q) sum += src[(int64_t)q * bn];
        G.y[p][j] = sum;
    }
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

size_t q8_area(int64_t K, int64_t B) { return align256((size_t)(K / kQK8) * (size_t)B * kQ8Bytes); }

size_t partial_area(int64_t K, int64_t N, int64_t B) { return align256(gemv_mma_partial_bytes(K, N, (int)B)); }

// Relative compute time per weight byte of a matrix with K columns at batch B (against K = 5120),
// tuned on B200 by timing the grouped launch of the benchmark's six layer shapes: the row kernel
// splits rows of K > 6144 over 2-4 warps (per-row combine, idle lane slots), the tensor-core kernel
// pays more K parts and a longer activation staging for long K.
double cost_per_byte(int64_t K, int64_t B) {
    if (B == 1) {
        int kw = 1, spl = 1;
        row_split(K, 1, &kw, &spl);
        return kw == 1 ? 1.0 : (kw == 2 ? 1.45 : (kw == 3 ? 1.3 : 1.6));
    }
    const double x = std::min(std::max((double)(K - 5120) / (17408 - 5120), 0.0), 1.0);
    return 1.0 + 0.25 * x;
}

// Estimated time of the busiest CTA of matrix q on `ctas` CTAs.  Batch 2..8: the tensor-core
// kernel's own cost model (gemv_mma_cta_cost: whole units per warp pair).  Batch 1: the row kernel
// streams whole stages of R rows, and a partly filled last stage takes as long as a full one (a
// warp's rows are computed together), so a CTA costs its stage count x R rows x the matrix's cost
// per byte.
double cta_cost(const iq4xs_gemv_problem& q, int64_t B, int ctas, int smem_optin) {
    if (B > 1) return gemv_mma_cta_cost(q.K, q.N, ctas, smem_optin);
    const int64_t R = gemv_rows_per_stage(q.K);
    const int64_t rows = (q.N + ctas - 1) / ctas;
    const int64_t stages = (rows + R - 1) / R;
    return (double)(stages * R) * (double)q.K * cost_per_byte(q.K, 1);
}

// CTAs handed out one at a time to the matrix whose busiest CTA is estimated slowest (cta_cost),
// starting from one each, so that the matrices' last CTAs finish together at the granularity the
// kernels work in.
void split_ctas_balanced(const iq4xs_gemv_problem* p, int count, int64_t B, int total, int smem_optin, int* out) {
    double cost[kMaxGroup];
    int used = 0;
    for (int i = 0; i < count; ++i) {
        out[i] = 1;
        cost[i] = cta_cost(p[i], B, 1, smem_optin);
        ++used;
    }
    while (used < total) {
        int best = 0;
        for (int i = 1; i < count; ++i)
            if (cost[i] > cost[best]) best = i;
        ++out[best];
        cost[best] = cta_cost(p[best], B, out[best], smem_optin);
        ++used;
    }
}

bool grouped_kernels_take(const iq4xs_gemv_problem* p, int count, int64_t B) {
    for (int i = 0; i < count; ++i) {
        const uint8_t* W = static_cast<const uint8_t*>(p[i].W);
        if (p[i].K % 512 != 0 || !gemv_bulk_path(W, p[i].K)) return false;
        if (B == 1 && gemv_takes_mma(W, p[i].K, 1)) return false;  // beyond the row kernel's K
    }
    return true;
}

int check_problem(const iq4xs_gemv_problem& q) {
    if (!q.W || !q.X || !q.Y || q.K <= 0 || q.N <= 0) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (q.K % kQK != 0 || q.K > (int64_t)1 << 30 || q.N > ((int64_t)1 << 31) - 1) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q.W) & 7u) || (reinterpret_cast<uintptr_t>(q.X) & 3u) ||
        (reinterpret_cast<uintptr_t>(q.Y) & 3u))
        return IQ4XS_ERR_MISALIGNED;
    return IQ4XS_OK;
}
}  // namespace

}  // namespace iq4xs

using namespace iq4xs;

extern "C" size_t iq4xs_gemv_grouped_workspace_bytes(const iq4xs_gemv_problem* problems, int count, int64_t B) {
    if (!problems || count < 1 || count > IQ4XS_MAX_GROUP || B < 1 || B > IQ4XS_MAX_GEMV_BATCH) return 0;
    size_t total = 0;
    for (int i = 0; i < count; ++i) {
        if (problems[i].K <= 0 || problems[i].N <= 0 || problems[i].K % kQK != 0) return 0;
        total += q8_area(problems[i].K, B) + partial_area(problems[i].K, problems[i].N, B);
    }
    return total;
}

extern "C" int iq4xs_gemv_grouped(const iq4xs_gemv_problem* problems, int count, int64_t B, void* workspace,
                                  size_t workspace_bytes, unsigned flags, cudaStream_t stream) {
    if (!problems || count < 1) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (count > IQ4XS_MAX_GROUP || B < 1 || B > IQ4XS_MAX_GEMV_BATCH) return IQ4XS_ERR_UNSUPPORTED_SHAPE;
    for (int i = 0; i < count; ++i) {
        const int s = check_problem(problems[i]);
        if (s) return s;
    }
    const size_t need = iq4xs_gemv_grouped_workspace_bytes(problems, count, B);
    if (!workspace) return IQ4XS_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < need) return IQ4XS_ERR_WORKSPACE_TOO_SMALL;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return IQ4XS_ERR_MISALIGNED;

    // Workspace slice of problem i: [Q8_1 activations][partial sums], each 256-byte aligned -- the
    // layout of iq4xs_gemv_f32's workspace, so the per-problem fallback uses the slices as they are.
    uint8_t* slice[kMaxGroup];
    size_t slice_bytes[kMaxGroup];
    {
        uint8_t* base = static_cast<uint8_t*>(workspace);
        for (int i = 0; i < count; ++i) {
            slice[i] = base;
            slice_bytes[i] = q8_area(problems[i].K, B) + partial_area(problems[i].K, problems[i].N, B);
            base += slice_bytes[i];
        }
    }
    if (!grouped_kernels_take(problems, count, B)) {
        for (int i = 0; i < count; ++i) {
            const iq4xs_gemv_problem& q = problems[i];
            const int s = iq4xs_gemv_f32_ex(q.W, q.X, q.Y, q.K, q.N, B, slice[i], slice_bytes[i], flags, stream);
            if (s) return s;
        }
        return IQ4XS_OK;
    }

    int sms = 0, smem_optin = 0;
    device_limits_current(&sms, &smem_optin);
    uint32_t* err = device_error_word();
    const uint32_t lut[4] = {kNegLo0, kNegLo1, kPosHi0, kPosHi1};
    int ctas[kMaxGroup];
    split_ctas_balanced(problems, count, B, std::max(sms, count), smem_optin, ctas);

    // 1. activations -> Q8_1 (one launch for the group)
    GroupQuantParams Q;
    std::memset(&Q, 0, sizeof Q);
    Q.count = count;
    for (int i = 0; i < count; ++i) {
        Q.x[i] = problems[i].X;
        Q.q8[i] = slice[i];
        Q.off[i + 1] = Q.off[i] + (problems[i].K / kQK8) * B;
    }
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)std::min<int64_t>((Q.off[count] + 7) / 8, (int64_t)sms * 8));
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = (flags & IQ4XS_FLAG_OVERLAP_PRECEDING) ? 1 : 0;
        if (cudaLaunchKernelEx(&cfg, q8_1_grouped_kernel, Q) != cudaSuccess) return IQ4XS_ERR_CUDA;
    }

    // 2. the grouped GEMV, programmatic dependent of the quantiser
    GroupedProblem g[kMaxGroup];
    GroupReduceParams R;
    std::memset(&R, 0, sizeof R);
    for (int i = 0; i < count; ++i) {
        const iq4xs_gemv_problem& q = problems[i];
        g[i].W = static_cast<const uint8_t*>(q.W);
        g[i].q8 = slice[i];
        g[i].y = q.Y;
        g[i].partials = nullptr;
        g[i].K = q.K;
        g[i].N = q.N;
        g[i].ctas = ctas[i];
        if (B > 1) {
            const int parts = gemv_mma_grouped_parts(q.K, q.N, ctas[i], smem_optin);
            if (parts > 1) {
                g[i].partials = reinterpret_cast<float*>(slice[i] + q8_area(q.K, B));
                const int r = R.count++;
                R.partial[r] = g[i].partials;
                R.y[r] = q.Y;
                R.parts[r] = parts;
                R.bn[r] = B * q.N;
                R.off[r + 1] = R.off[r] + B * q.N;
            }
        }
    }
    cudaError_t e = (B == 1) ? launch_gemv_rows_grouped(g, count, stream, true, err, lut)
                             : launch_gemv_mma_grouped(g, count, (int)B, stream, true, err, lut);
    if (e != cudaSuccess) return IQ4XS_ERR_CUDA;

    // 3. K parts of the split matrices, added in part order
    if (R.count > 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)std::min<int64_t>((R.off[R.count] + 255) / 256, (int64_t)sms * 4));
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, reduce_grouped_kernel, R) != cudaSuccess) return IQ4XS_ERR_CUDA;
    }
    return IQ4XS_OK;
}
