// gemv.cu -- IQ4_XS x Q8_1 decode GEMV for batch 1..8 on sm_100a.
//
// Replaces the reference's decode path: quantize_row_q8_1 + vec_dot_iq4_xs_q8_1 in
// gemv_iq4xs_stock_dp4a_kernel (kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:325-360) and the
// cooperative gemv_iq4xs_dp4a_coop_kernel (kernels/matmul_iq4xs/impl_gemv_dp4a_gfx1100.hip:178-283,
// vendored as patches/0001-gfx1100-mul-mat-custom.patch:237-260).
//
// Design (HBM-streaming, one CTA per SM):
//  * every CTA owns a contiguous, balanced range of output rows and streams those rows' IQ4_XS
//    bytes through a ring of shared-memory stages filled by 1-D bulk copies (cp.async.bulk, one
//    copy per row segment, completion on an mbarrier, L2 evict-first);
//  * warp 0 is the producer; NCW consumer warps compute.  Consumer lane layout: 8 lanes per row
//    (lane & 7 = sub-block ib of each super-block), 4 rows per warp step, RPL steps per warp;
//  * the Q8_1 activations of all B tokens are staged once per CTA in shared memory, permuted to
//    the order of the codebook lookup and read back as 16-byte vectors;
//  * the codebook gather is two prmt lookups per 4 codes with no merge (sign-replication zeroes
//    the half that does not apply), the int8 dot products are dp4a, giving the exact int32
//    sub-block dot of the reference; the term (d_w*d_x)*(float)(sumi*(ls-32)) is the reference's
//    fp32 expression; per-row sums are reduced over the 8 sub-block lanes with xor shuffles.
//  * every mbarrier wait is bounded; a timeout records a device error code and the kernel
//    drains its in-flight copies and returns.
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

constexpr int kMaxStages = 16;

template <int B, int NCW, int RPL, int KC>
struct GemvCfg {
    static constexpr int kThreads = 32 * (1 + NCW);
    static constexpr int kRowsPerWarp = 4 * RPL;
    static constexpr int kRT = kRowsPerWarp * NCW;           // rows per tile
    static constexpr int kRowStride = KC * kBlockBytes + 16;  // smem bytes per row segment (16-aligned)
    static constexpr int kStageBytes = kRT * kRowStride;
    static constexpr int kActBytesPerSB = 256 + 32;            // permuted q8 (256) + 8 fp32 d_x (32)
};

struct SmemLayout {
    uint32_t bar_off, abort_off, act_off, dx_off, ring_off, total;
};

// Barriers first, then the activation area, then the 128-byte aligned ring.
template <int B, int NCW, int RPL, int KC>
__host__ __device__ inline SmemLayout gemv_smem_layout(int kb_per_part, int stages) {
    using Cfg = GemvCfg<B, NCW, RPL, KC>;
    SmemLayout L;
    L.bar_off = 0;
    L.abort_off = 2 * kMaxStages * 8;
    L.act_off = (L.abort_off + 16 + 127) & ~127u;
    L.dx_off = L.act_off + (uint32_t)B * kb_per_part * 256;
    L.ring_off = (L.dx_off + (uint32_t)B * kb_per_part * 32 + 127) & ~127u;
    L.total = L.ring_off + (uint32_t)stages * Cfg::kStageBytes;
    return L;
}

// Wait on an mbarrier phase, giving up when another warp already aborted or the spin limit hits.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                              uint32_t* err, uint32_t code) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *abort_flag) return false;
    }
    record_error(err, code);
    *abort_flag = 1u;
    return false;
}

template <int B, int NCW, int RPL, int KC, bool kDebug>
__global__ void __launch_bounds__(GemvCfg<B, NCW, RPL, KC>::kThreads, 1)
    gemv_iq4xs_q8_kernel(const GemvArgs a) {
    using Cfg = GemvCfg<B, NCW, RPL, KC>;
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemLayout L = gemv_smem_layout<B, NCW, RPL, KC>(a.kb_per_part, a.stages);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + kMaxStages;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.abort_off);
    uint8_t* ring = smem + L.ring_off;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int stages = a.stages;

    // Balanced contiguous row range of this CTA.
    const int64_t r0 = a.N * (int64_t)blockIdx.x / gridDim.x;
    const int64_t r1 = a.N * (int64_t)(blockIdx.x + 1) / gridDim.x;
    const int ntiles = (int)((r1 - r0 + Cfg::kRT - 1) / Cfg::kRT);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        *abort_flag = 0u;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        const uint64_t policy = l2_policy_evict_first();
        uint32_t it = 0;
        bool ok = true;
        for (int p = 0; p < a.kparts && ok; ++p) {
            const int pb0 = p * a.kb_per_part;
            const int pb1 = min(a.kb, pb0 + a.kb_per_part);
            const int nchunks = (pb1 - pb0 + KC - 1) / KC;
            for (int t = 0; t < ntiles && ok; ++t) {
                const int64_t row0 = r0 + (int64_t)t * Cfg::kRT;
                const int rows = (int)imin64(Cfg::kRT, r1 - row0);
                for (int c = 0; c < nchunks; ++c) {
                    const int s = (int)(it % stages);
                    const uint32_t use = it / stages;
                    if (use > 0 && !wait_or_abort(&empty[s], (use - 1) & 1u, abort_flag, a.err, kDevErrEmptyWait)) {
                        ok = false;
                        break;
                    }
                    const int b0 = pb0 + c * KC;
                    const uint32_t bytes = (uint32_t)min(KC, pb1 - b0) * kBlockBytes;
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes * (uint32_t)rows);
                    __syncwarp();
                    uint8_t* dst = ring + (size_t)s * Cfg::kStageBytes;
                    for (int r = lane; r < rows; r += 32)
                        bulk_g2s_evict_first(dst + r * Cfg::kRowStride, a.W + (row0 + r) * a.rb + (int64_t)b0 * kBlockBytes,
                                             bytes, &full[s], policy);
                    ++it;
                }
            }
        }
        // Drain: every issued stage must have landed before this CTA's shared memory goes away.
        if (lane == 0) {
            const uint32_t first = it > (uint32_t)stages ? it - stages : 0u;
            for (uint32_t j = first; j < it; ++j) {
                bool landed = false;
                for (uint32_t i = 0; i < kSpinLimit && !landed; ++i) landed = mbar_try_wait(&full[j % stages], (j / stages) & 1u);
                if (!landed) record_error(a.err, kDevErrDrainWait);
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int cw = warp - 1;
    const int g = lane >> 3;   // row within a 4-row warp step
    const int ib = lane & 7;   // sub-block within each super-block
    const int ctid = threadIdx.x - 32;
    const int nct = NCW * 32;
    const uint32_t act_base = smem_addr(smem + L.act_off);
    const uint32_t dx_base = smem_addr(smem + L.dx_off);
    const uint32_t ring_base = smem_addr(ring);
    const int nsb = a.K / kQK8;  // Q8_1 blocks per token

    grid_dependency_wait();  // activations may come from the immediately preceding kernel

    uint32_t it = 0;
    for (int p = 0; p < a.kparts; ++p) {
        const int pb0 = p * a.kb_per_part;
        const int pb1 = min(a.kb, pb0 + a.kb_per_part);
        const int nchunks = (pb1 - pb0 + KC - 1) / KC;
        const int pkb = pb1 - pb0;

        // Stage this part's activations: per (token, super-block) 256 B of permuted q8 laid out as
        // [half][ib][16 B] (8 lanes read 128 contiguous bytes) and 8 fp32 d_x.
        if (p > 0) named_barrier(1, nct);  // everyone finished with the previous part
        for (int e = ctid; e < B * pkb * 8; e += nct) {
            const int t = e / (pkb * 8);
            const int rem = e - t * pkb * 8;
            const int bl = rem >> 3, sib = rem & 7;
            const uint32_t* blk =
                reinterpret_cast<const uint32_t*>(a.q8 + ((int64_t)t * nsb + (int64_t)(pb0 + bl) * 8 + sib) * kQ8Bytes);
            uint32_t w[9];
#pragma unroll
            for (int i = 0; i < 9; ++i) w[i] = __ldg(blk + i);
            uint4 lo, hi;
            lo.x = act_perm_lo(w[1], w[5]);
            lo.y = act_perm_lo(w[2], w[6]);
            lo.z = act_perm_lo(w[3], w[7]);
            lo.w = act_perm_lo(w[4], w[8]);
            hi.x = act_perm_hi(w[1], w[5]);
            hi.y = act_perm_hi(w[2], w[6]);
            hi.z = act_perm_hi(w[3], w[7]);
            hi.w = act_perm_hi(w[4], w[8]);
            uint8_t* dst = smem + L.act_off + ((size_t)(t * a.kb_per_part + bl) * 256) + sib * 16;
            *reinterpret_cast<uint4*>(dst) = lo;
            *reinterpret_cast<uint4*>(dst + 128) = hi;
            reinterpret_cast<float*>(smem + L.dx_off)[(t * a.kb_per_part + bl) * 8 + sib] = f16_bits_to_f32(w[0]);
        }
        named_barrier(1, nct);

        for (int tl = 0; tl < ntiles; ++tl) {
            const int64_t row0 = r0 + (int64_t)tl * Cfg::kRT;
            const int rows = (int)imin64(Cfg::kRT, r1 - row0);
            float acc[RPL][B];
#pragma unroll
            for (int j = 0; j < RPL; ++j)
#pragma unroll
                for (int t = 0; t < B; ++t) acc[j][t] = 0.0f;

            for (int c = 0; c < nchunks; ++c) {
                const int s = (int)(it % stages);
                const bool ready = !*abort_flag && wait_or_abort(&full[s], (it / stages) & 1u, abort_flag, a.err, kDevErrFullWait);
                if (ready) {
                    const int b0 = pb0 + c * KC;
                    const int nblk = min(KC, pb1 - b0);
                    const uint32_t stage = ring_base + (uint32_t)s * Cfg::kStageBytes;
                    for (int cb = 0; cb < nblk; ++cb) {
                        const int bl = b0 - pb0 + cb;
                        uint32_t alo[B][4], ahi[B][4];
                        float dx[B];
#pragma unroll
                        for (int t = 0; t < B; ++t) {
                            const uint32_t ab = act_base + (uint32_t)(t * a.kb_per_part + bl) * 256 + ib * 16;
                            const uint4 l4 = lds_u4(ab), h4 = lds_u4(ab + 128);
                            alo[t][0] = l4.x; alo[t][1] = l4.y; alo[t][2] = l4.z; alo[t][3] = l4.w;
                            ahi[t][0] = h4.x; ahi[t][1] = h4.y; ahi[t][2] = h4.z; ahi[t][3] = h4.w;
                            dx[t] = lds_f32(dx_base + (uint32_t)((t * a.kb_per_part + bl) * 8 + ib) * 4);
                        }
#pragma unroll
                        for (int j = 0; j < RPL; ++j) {
                            const int rloc = cw * Cfg::kRowsPerWarp + j * 4 + g;
                            const uint32_t rb = stage + (uint32_t)rloc * Cfg::kRowStride + cb * kBlockBytes;
                            const uint2 h = lds_u2(rb);
                            const uint2 qa = lds_u2(rb + 8 + 16 * ib);
                            const uint2 qb = lds_u2(rb + 16 + 16 * ib);
                            // Weight side of the lookup, shared by all tokens.
                            uint32_t wh[8], wl[8];
                            const uint32_t qw[4] = {qa.x, qa.y, qb.x, qb.y};
#pragma unroll
                            for (int w = 0; w < 4; ++w) {
                                const uint32_t x = qw[w], xf = x ^ 0x88888888u;
                                wh[2 * w] = prmt(kPosHi0, kPosHi1, xf);
                                wl[2 * w] = prmt(kNegLo0, kNegLo1, x);
                                wh[2 * w + 1] = prmt(kPosHi0, kPosHi1, xf >> 16);
                                wl[2 * w + 1] = prmt(kNegLo0, kNegLo1, x >> 16);
                            }
                            const float dw = f16_bits_to_f32(h.x);
                            const int scale = subblock_scale(h.x, h.y, ib) - 32;
#pragma unroll
                            for (int t = 0; t < B; ++t) {
                                int sh = 0, sl = 0;
#pragma unroll
                                for (int w = 0; w < 4; ++w) {
                                    sh = dp4a((int)wh[2 * w], (int)alo[t][w], sh);
                                    sl = dp4a((int)wl[2 * w], (int)alo[t][w], sl);
                                    sh = dp4a((int)wh[2 * w + 1], (int)ahi[t][w], sh);
                                    sl = dp4a((int)wl[2 * w + 1], (int)ahi[t][w], sl);
                                }
                                const int sumi = sh - sl;
                                if constexpr (kDebug) {
                                    if (rloc < rows)
                                        a.sumi[((int64_t)t * a.N + row0 + rloc) * nsb + (int64_t)(b0 + cb) * 8 + ib] = sumi;
                                }
                                acc[j][t] += (dw * dx[t]) * (float)(sumi * scale);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                ++it;
            }

            // Reduce over the 8 sub-block lanes of each row and store.
#pragma unroll
            for (int j = 0; j < RPL; ++j) {
                const int rloc = cw * Cfg::kRowsPerWarp + j * 4 + g;
#pragma unroll
                for (int t = 0; t < B; ++t) {
                    float v = acc[j][t];
                    v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
                    v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
                    v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
                    if (ib == 0 && rloc < rows && !*abort_flag && a.y) {
                        float* yp = a.y + (int64_t)t * a.N + row0 + rloc;
                        *yp = (p == 0) ? v : (*yp + v);
                    }
                }
            }
        }
    }
}

// --------------------------------------------------------------------------------------------
// Generic path for shapes the bulk-copy kernel does not take (K/256 odd, unaligned W): one warp
// per row, lane = sub-block, direct global loads.  Same per-term arithmetic.
template <int B, bool kDebug>
__global__ void __launch_bounds__(256) gemv_iq4xs_q8_generic_kernel(const GemvArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int nsb = a.K / kQK8;
    grid_dependency_wait();
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < a.N; row += nwarps) {
        float acc[B];
#pragma unroll
        for (int t = 0; t < B; ++t) acc[t] = 0.0f;
        const uint8_t* wrow = a.W + row * a.rb;
        for (int sb = lane; sb < nsb; sb += 32) {
            const uint8_t* blk = wrow + (sb >> 3) * kBlockBytes;
            const int ib = sb & 7;
            const uint2 h = *reinterpret_cast<const uint2*>(blk);
            const uint2 qa = *reinterpret_cast<const uint2*>(blk + 8 + 16 * ib);
            const uint2 qb = *reinterpret_cast<const uint2*>(blk + 16 + 16 * ib);
            const uint32_t qw[4] = {qa.x, qa.y, qb.x, qb.y};
            const float dw = f16_bits_to_f32(h.x);
            const int scale = subblock_scale(h.x, h.y, ib) - 32;
#pragma unroll
            for (int t = 0; t < B; ++t) {
                const uint32_t* q = reinterpret_cast<const uint32_t*>(a.q8 + ((int64_t)t * nsb + sb) * kQ8Bytes);
                uint32_t alo[4], ahi[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const uint32_t lo = __ldg(q + 1 + w), hi = __ldg(q + 5 + w);
                    alo[w] = act_perm_lo(lo, hi);
                    ahi[w] = act_perm_hi(lo, hi);
                }
                const float dx = f16_bits_to_f32(__ldg(q));
                const int sumi = subblock_dot(qw, alo, ahi);
                if constexpr (kDebug) a.sumi[((int64_t)t * a.N + row) * nsb + sb] = sumi;
                acc[t] += (dw * dx) * (float)(sumi * scale);
            }
        }
#pragma unroll
        for (int t = 0; t < B; ++t) {
            float v = acc[t];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
            if (lane == 0 && a.y) a.y[(int64_t)t * a.N + row] = v;
        }
    }
}

// --------------------------------------------------------------------------------------------
// Host-side launch helpers.
namespace {
constexpr int kNCW = 8, kRPL = 2, kKC = 4;

int g_num_sms[64];
int g_max_smem[64];

void device_limits(int dev, int* sms, int* smem_optin) {
    if (dev < 0 || dev >= 64) {
        cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        return;
    }
    if (g_num_sms[dev] == 0) {
        cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&g_max_smem[dev], cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    *sms = g_num_sms[dev];
    *smem_optin = g_max_smem[dev];
}

template <int B, bool kDebug>
cudaError_t launch_bulk(GemvArgs a, cudaStream_t stream, bool pdl, int sms, int smem_optin) {
    using Cfg = GemvCfg<B, kNCW, kRPL, kKC>;
    // Activation part: all of K when it fits next to a 4-stage ring, otherwise even halves.
    const int ring4 = 4 * Cfg::kStageBytes;
    int kparts = 1, kbpp = a.kb;
    while ((int)gemv_smem_layout<B, kNCW, kRPL, kKC>(kbpp, 4).total > smem_optin && kbpp > 2) {
        ++kparts;
        kbpp = (a.kb + kparts - 1) / kparts;
        kbpp += kbpp & 1;
    }
    (void)ring4;
    int stages = 4;
    while (stages < kMaxStages && (int)gemv_smem_layout<B, kNCW, kRPL, kKC>(kbpp, stages + 1).total <= smem_optin) ++stages;
    a.kparts = kparts;
    a.kb_per_part = kbpp;
    a.stages = stages;
    const SmemLayout L = gemv_smem_layout<B, kNCW, kRPL, kKC>(kbpp, stages);
    if ((int)L.total > smem_optin) return cudaErrorInvalidConfiguration;
    auto kern = gemv_iq4xs_q8_kernel<B, kNCW, kRPL, kKC, kDebug>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    const int grid = (int)imin64((int64_t)sms, a.N);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int B, bool kDebug>
cudaError_t launch_generic(GemvArgs a, cudaStream_t stream, bool pdl, int sms) {
    const int64_t warps_needed = a.N;
    const int grid = (int)imin64((warps_needed + 7) / 8, (int64_t)sms * 8);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_iq4xs_q8_generic_kernel<B, kDebug>, a);
}

template <bool kDebug>
cudaError_t dispatch(int B, GemvArgs a, cudaStream_t stream, bool pdl) {
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0, smem_optin = 0;
    device_limits(dev, &sms, &smem_optin);
    const bool bulk_ok = (a.kb % 2 == 0) && ((reinterpret_cast<uintptr_t>(a.W) & 15u) == 0) && !a.force_generic;
    switch (B) {
#define IQ4XS_CASE(BB)                                                                                 \
    case BB:                                                                                           \
        return bulk_ok ? launch_bulk<BB, kDebug>(a, stream, pdl, sms, smem_optin)                      \
                       : launch_generic<BB, kDebug>(a, stream, pdl, sms);
        IQ4XS_CASE(1)
        IQ4XS_CASE(2)
        IQ4XS_CASE(3)
        IQ4XS_CASE(4)
        IQ4XS_CASE(5)
        IQ4XS_CASE(6)
        IQ4XS_CASE(7)
        IQ4XS_CASE(8)
#undef IQ4XS_CASE
        default:
            return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t launch_gemv_q8(GemvArgs a, int B, cudaStream_t stream, bool pdl) {
    a.sumi = nullptr;
    return dispatch<false>(B, a, stream, pdl);
}

cudaError_t launch_gemv_q8_debug(GemvArgs a, int B, cudaStream_t stream) { return dispatch<true>(B, a, stream, false); }

}  // namespace iq4xs
