// gemv.cu -- IQ4_XS x Q8_1 decode GEMV for batch 1..8 on sm_100a.
//
// Replaces the reference's decode path: quantize_row_q8_1 + vec_dot_iq4_xs_q8_1 in
// gemv_iq4xs_stock_dp4a_kernel (kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:325-360) and the
// cooperative gemv_iq4xs_dp4a_coop_kernel (kernels/matmul_iq4xs/impl_gemv_dp4a_gfx1100.hip:178-283,
// vendored as patches/0001-gfx1100-mul-mat-custom.patch:237-260).
//
// Batch 1 runs here (dp4a); batch 2..8 run on the tensor cores (gemv_mma.cu).
// Design (HBM-streaming, one CTA per SM):
//  * every CTA owns a contiguous, balanced range of output rows and streams them through a ring of
//    shared-memory stages; one stage = R consecutive full rows = ONE 1-D bulk copy (cp.async.bulk,
//    completion on an mbarrier, L2 evict-first) -- many small copies starve the copy engine;
//  * warp 0 is the producer; the consumer warps own rows (or, for long K, K slices of a row): lane l
//    owns sub-blocks l, l+32, ... of its K slice, the same K positions for every row, so its Q8_1
//    activations (permuted to the order of the codebook lookup) live in registers for the whole kernel;
//  * the codebook gather is two prmt lookups per 4 codes with no merge (sign-replication zeroes
//    the half that does not apply), the int8 dot products are dp4a, giving the exact int32
//    sub-block dot of the reference; the term (d_w*d_x)*(float)(sumi*(ls-32)) is the reference's
//    fp32 expression; per-row sums are reduced over the 8 sub-block lanes with xor shuffles.
//  * every mbarrier wait is bounded; a timeout records a device error code and the kernel
//    drains its in-flight copies and returns.
#include <atomic>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

constexpr int kMaxStages = 16;

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

// Sleeping variant: each try_wait suspends up to 1 ms; 20000 tries bound the wait to ~20 s.
__device__ __forceinline__ bool wait_sleep_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                    uint32_t* err, uint32_t code) {
    for (uint32_t i = 0; i < 20000u; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (*abort_flag) return false;
    }
    record_error(err, code);
    *abort_flag = 1u;
    return false;
}

// --------------------------------------------------------------------------------------------
// Row-stage kernel (batch 1..2): one stage = R consecutive full rows = ONE bulk copy of R*rb bytes.
// Warp (kw, slot) handles stage row `slot` over its contiguous K range kw; lane l owns sub-blocks
// kw*32*SPL + l + 32*i (i < SPL), the same K positions for every row, so its Q8_1 activations are
// loaded into registers once per kernel.  With KW > 1 warps per row, each warp leaves its partial
// sum in shared memory and the last of the KW warps (shared-memory ticket) adds them in kw order:
// deterministic.
struct RowSmem {
    uint32_t bar_off, abort_off, red_off, part_off, cnt_off, q8_off, ring_off, total;
};

// q8_bytes: Q8_1 activations built in shared memory from an fp32 source (0 for kActQ8).
__host__ __device__ inline RowSmem gemv_row_smem(int B, int R, int KW, int stages, int64_t stage_bytes,
                                                 uint32_t q8_bytes = 0) {
    RowSmem L;
    L.bar_off = 0;
    L.abort_off = 2 * kMaxStages * 8;
    L.red_off = L.abort_off + 16;  // 32 floats: per-warp sums of squares of the RMSNorm source
    L.part_off = L.red_off + 128;
    L.cnt_off = L.part_off + (uint32_t)kMaxStages * R * KW * B * 4;
    L.q8_off = (L.cnt_off + (uint32_t)kMaxStages * R * 4 + 15) & ~15u;
    L.ring_off = (L.q8_off + q8_bytes + 127) & ~127u;
    L.total = L.ring_off + (uint32_t)(stages * stage_bytes);
    return L;
}

// Shared memory of an activation source: the Q8_1 blocks [B][K/32] (every source but kActQ8), then
// for kActNormPeer the all-reduced delta [K] fp32 (16-byte aligned).
__host__ __device__ inline uint32_t act_q8_bytes(int B, int K) { return (uint32_t)(B * (K / kQK8) * kQ8Bytes); }
__host__ __device__ inline uint32_t act_smem_bytes(int mode, int B, int K) {
    if (mode == kActQ8) return 0u;
    const uint32_t q8 = act_q8_bytes(B, K);
    return mode == kActNormPeer ? ((q8 + 15u) & ~15u) + (uint32_t)K * 4u : q8;
}

// Consumer warps (warp index cw of ncw) build the Q8_1 activations of an fp32 source in shared
// memory, four blocks (128 values, one float4 per lane) at a time with q8_1_quad_store; each warp
// issues the loads of a batch of quads (kActQ / kActQF) before using any (one round trip per batch).
// kActNorm (batch 1): v = x (+ delta) (CTA 0 also writes v to x_out), the sum of v^2 per lane, per
// warp (xor butterfly) and then over warps in warp order (the same order in every CTA),
// r = rsqrt(mean + eps), h = (v * r) * w.  The first batch of v and w stays in registers for the
// second pass; later batches (K > 6144) are re-read.  Ends with a barrier of the consumer warps
// (named barrier `bar_id`).
constexpr int kActQ = 4;    // kActNorm: quads per warp per batch (v and w of the first batch stay in registers)
constexpr int kActQF = 12;  // kActF32: quads per warp per batch (one batch up to K = 18432 at batch 1)

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float4 add4_rn(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

template <int kAct>
__device__ __forceinline__ void build_act_q8(const ActSource& act, int B, int K, uint8_t* q8s, float* red, int cw,
                                             int ncw, int lane, int bar_id, bool first_cta, uint32_t* err) {
    const int nq = B * K / 128;
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (kAct == kActNorm || kAct == kActNormPeer) {
        // delta: a plain vector (kActNorm), or the fused all-reduce of the ranks' slots (kActNormPeer:
        // each word read until it carries the current epoch)
        constexpr bool kPeer = kAct == kActNormPeer;
        const bool has_delta = kPeer || act.delta != nullptr;
        // kPeer: the all-reduced delta of this warp's quads is summed first into shared memory (after
        // the Q8_1 blocks), with up to eight (quad, rank) slot reads in flight at a time; the warp
        // reads back only its own quads
        float* dsm = reinterpret_cast<float*>(q8s + ((act_q8_bytes(B, K) + 15u) & ~15u));
        if constexpr (kPeer) {
            const uint32_t ep = peer_slots_epoch(act.peer);
            peer_slots_sum_to_smem(act.peer, K, nq, cw, ncw, lane, ep, err, dsm);
            __syncwarp();
        }
        // delta of the batch's quads (global memory, or the peer pre-pass's shared memory), in halves
        // of the batch
        auto delta_batch = [&](int base, float4(&da)[kActQ]) {
            constexpr int H = kActQ / 2;
#pragma unroll
            for (int h = 0; h < kActQ; h += H) {
                int off[H];
                bool ok[H];
                float4 d[H];
#pragma unroll
                for (int i = 0; i < H; ++i) {
                    const int qd = base + (h + i) * ncw;
                    ok[i] = qd < nq;
                    off[i] = qd * 128 + 4 * lane;
                    d[i] = zero4;
                }
                if constexpr (kPeer) {
#pragma unroll
                    for (int i = 0; i < H; ++i)
                        if (ok[i]) d[i] = *reinterpret_cast<const float4*>(dsm + off[i]);
                } else {
#pragma unroll
                    for (int i = 0; i < H; ++i)
                        if (ok[i]) d[i] = ldg4(act.delta + off[i]);
                }
#pragma unroll
                for (int i = 0; i < H; ++i) da[h + i] = d[i];
            }
        };
        float4 v0[kActQ], w0[kActQ];
        float ss = 0.0f;
        for (int base = cw; base < nq; base += ncw * kActQ) {
            float4 xa[kActQ], da[kActQ];
#pragma unroll
            for (int i = 0; i < kActQ; ++i) {
                const int qd = base + i * ncw;
                xa[i] = zero4;
                if (qd < nq) {
                    xa[i] = ldg4(act.x + qd * 128 + 4 * lane);
                    if (base == cw) w0[i] = ldg4(act.w + qd * 128 + 4 * lane);
                }
            }
            if (has_delta) delta_batch(base, da);
#pragma unroll
            for (int i = 0; i < kActQ; ++i) {
                const int qd = base + i * ncw;
                if (qd >= nq) continue;
                const float4 v = has_delta ? add4_rn(xa[i], da[i]) : xa[i];
                if (act.x_out && first_cta) *reinterpret_cast<float4*>(act.x_out + qd * 128 + 4 * lane) = v;
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
                if (base == cw) v0[i] = v;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
        if (lane == 0) red[cw] = ss;
        named_barrier(bar_id, ncw * 32);
        float tot = 0.0f;
        for (int i = 0; i < ncw; ++i) tot += red[i];
        const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)K), act.eps));
        for (int base = cw; base < nq; base += ncw * kActQ) {
            float4 va[kActQ], wa[kActQ], da[kActQ];
#pragma unroll
            for (int i = 0; i < kActQ; ++i) {
                const int qd = base + i * ncw;
                va[i] = wa[i] = zero4;
                if (qd >= nq) continue;
                if (base == cw) {
                    va[i] = v0[i];
                    wa[i] = w0[i];
                } else {
                    va[i] = ldg4(act.x + qd * 128 + 4 * lane);
                    wa[i] = ldg4(act.w + qd * 128 + 4 * lane);
                }
            }
            if (has_delta && base != cw) {
                delta_batch(base, da);
#pragma unroll
                for (int i = 0; i < kActQ; ++i) va[i] = add4_rn(va[i], da[i]);
            }
#pragma unroll
            for (int i = 0; i < kActQ; ++i) {
                const int qd = base + i * ncw;
                if (qd >= nq) continue;
                float4 h;
                h.x = __fmul_rn(__fmul_rn(va[i].x, r), wa[i].x);
                h.y = __fmul_rn(__fmul_rn(va[i].y, r), wa[i].y);
                h.z = __fmul_rn(__fmul_rn(va[i].z, r), wa[i].z);
                h.w = __fmul_rn(__fmul_rn(va[i].w, r), wa[i].w);
                q8_1_quad_store(h, q8s + (size_t)qd * 4 * kQ8Bytes, lane);
            }
        }
    } else if constexpr (kAct == kActSwiGLU) {
        // the values of swiglu_q8_kernel (silu(g) = g / (1 + exp(-g)), then * u, each rounded once)
        constexpr int kQS = kActQF / 2;
        for (int base = cw; base < nq; base += ncw * kQS) {
            float4 ga[kQS], ua[kQS];
#pragma unroll
            for (int i = 0; i < kQS; ++i) {
                const int qd = base + i * ncw;
                ga[i] = ua[i] = zero4;
                if (qd < nq) {
                    ga[i] = ldg4(act.x + (int64_t)qd * 128 + 4 * lane);
                    ua[i] = ldg4(act.x + K + (int64_t)qd * 128 + 4 * lane);
                }
            }
#pragma unroll
            for (int i = 0; i < kQS; ++i) {
                const int qd = base + i * ncw;
                if (qd >= nq) continue;
                float4 h;
                h.x = __fmul_rn(__fdiv_rn(ga[i].x, __fadd_rn(1.0f, expf(-ga[i].x))), ua[i].x);
                h.y = __fmul_rn(__fdiv_rn(ga[i].y, __fadd_rn(1.0f, expf(-ga[i].y))), ua[i].y);
                h.z = __fmul_rn(__fdiv_rn(ga[i].z, __fadd_rn(1.0f, expf(-ga[i].z))), ua[i].z);
                h.w = __fmul_rn(__fdiv_rn(ga[i].w, __fadd_rn(1.0f, expf(-ga[i].w))), ua[i].w);
                q8_1_quad_store(h, q8s + (size_t)qd * 4 * kQ8Bytes, lane);
            }
        }
    } else {
        for (int base = cw; base < nq; base += ncw * kActQF) {
            float4 xa[kActQF];
#pragma unroll
            for (int i = 0; i < kActQF; ++i) {
                const int qd = base + i * ncw;
                xa[i] = qd < nq ? ldg4(act.x + (int64_t)qd * 128 + 4 * lane) : zero4;
            }
#pragma unroll
            for (int i = 0; i < kActQF; ++i) {
                const int qd = base + i * ncw;
                if (qd < nq) q8_1_quad_store(xa[i], q8s + (size_t)qd * 4 * kQ8Bytes, lane);
            }
        }
    }
    named_barrier(bar_id, ncw * 32);
}

// The upper 16 selector bits of a qs word.  A plain shift: mul.hi.u32 by 2^16 would move it to the
// FMA pipe, but that instruction issues at a quarter of the rate and sits in the lookup's dependency
// chain (measured on B200: the shift makes the 190 MB batch-1 GEMV 7% faster).
__device__ __forceinline__ uint32_t sel_hi16(uint32_t x) {
    return x >> 16;
}

// Weight side of the split codebook lookup for one qs word: hi/lo halves of both 16-bit selectors.
// The table words come from the kernel parameters so prmt can read them from the constant bank.
__device__ __forceinline__ void lut_word(const uint32_t (&tab)[4], uint32_t x, uint32_t& h0, uint32_t& l0, uint32_t& h1,
                                         uint32_t& l1) {
    const uint32_t xf = x ^ 0x88888888u;
    h0 = prmt(tab[2], tab[3], xf);
    l0 = prmt(tab[0], tab[1], x);
    h1 = prmt(tab[2], tab[3], sel_hi16(xf));
    l1 = prmt(tab[0], tab[1], sel_hi16(x));
}

// kAct: where the activations come from (ActMode).  Every source but kActQ8 builds them into shared memory
// (build_act_q8); each instance carries only its own prologue (code size costs instruction-cache
// misses in the hot loop).
// The kernel body, for CTA `cta` of the `ncta` CTAs that share the matrix (the single-matrix kernel
// passes its grid; the grouped kernel a slice of it).
template <int B, int SPL, int RPW, int NCW, bool kTail, bool kDebug, int kAct>
__device__ __forceinline__ void gemv_rows_body(const GemvArgs& a, int cta, int ncta, uint8_t* smem) {
    const int R = a.rows_per_stage, KW = a.kw;
    const int stages = a.stages;
    const int64_t stage_bytes = (int64_t)R * a.rb;
    constexpr bool smem_act = kAct != kActQ8;
    const RowSmem L = gemv_row_smem(B, R, KW, stages, stage_bytes, act_smem_bytes(kAct, B, a.K));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + kMaxStages;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.abort_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + L.cnt_off);
    uint8_t* ring = smem + L.ring_off;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = a.N * (int64_t)cta / ncta;
    const int64_t r1 = a.N * (int64_t)(cta + 1) / ncta;
    const int ntiles = (int)((r1 - r0 + R - 1) / R);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        *abort_flag = 0u;
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < kMaxStages * R; i += blockDim.x) cnt[i] = 0u;
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------------ producer: one copy per stage
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            uint32_t it = 0;
            for (int t = 0; t < ntiles; ++t, ++it) {
                const int s = (int)(it % stages);
                const uint32_t use = it / stages;
                if (use > 0 && !wait_sleep_or_abort(&empty[s], (use - 1) & 1u, abort_flag, a.err, kDevErrEmptyWait)) break;
                const int64_t row0 = r0 + (int64_t)t * R;
                const uint32_t bytes = (uint32_t)(imin64(R, r1 - row0) * a.rb);
                fence_generic_async_smem();  // the consumers' ld.shared of this stage come first
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s_evict_first(ring + (size_t)s * stage_bytes, a.W + row0 * a.rb, bytes, &full[s], policy);
            }
            const uint32_t first = it > (uint32_t)stages ? it - stages : 0u;
            for (uint32_t j = first; j < it; ++j) {
                bool landed = false;
                for (uint32_t i = 0; i < 20000u && !landed; ++i)
                    landed = mbar_try_wait_sleep(&full[j % stages], (j / stages) & 1u, 1000000u);
                if (!landed) record_error(a.err, kDevErrDrainWait);
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int cw = warp - 1;
    const int kw = cw % KW, slot = cw / KW;     // rows slot*RPW .. slot*RPW+RPW-1 of every stage
    const int nsb = a.K / kQK8;
    const int sb0 = kw * 32 * SPL + lane;       // this lane's first sub-block; ib = lane & 7
    const int ib = lane & 7;
    const uint32_t sh_lo = 4u * ib, sh_hi = 12u + 2u * ib;  // scale bit positions
    // offsets inside a row of this lane's super-block header and qs words (sub-block i adds 4*136)
    const uint32_t off_h = (uint32_t)(sb0 >> 3) * kBlockBytes;
    const uint32_t off_q = off_h + 8 + 16 * ib;

    grid_dependency_wait();
    if constexpr (smem_act)
        build_act_q8<kAct>(a.act, B, a.K, smem + L.q8_off, reinterpret_cast<float*>(smem + L.red_off), cw, NCW, lane, 1,
                           cta == 0, a.err);
    uint32_t alo[SPL][B][4], ahi[SPL][B][4];
    float dx[SPL][B];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
        const int sb = sb0 + 32 * i;
#pragma unroll
        for (int t = 0; t < B; ++t) {
            if (!kTail || sb < nsb) {
                uint32_t w[9];
                if constexpr (smem_act) {
                    const uint32_t* q = reinterpret_cast<const uint32_t*>(smem + L.q8_off + ((size_t)t * nsb + sb) * kQ8Bytes);
#pragma unroll
                    for (int j = 0; j < 9; ++j) w[j] = q[j];
                } else {
                    const uint32_t* q = reinterpret_cast<const uint32_t*>(a.q8 + ((int64_t)t * nsb + sb) * kQ8Bytes);
#pragma unroll
                    for (int j = 0; j < 9; ++j) w[j] = __ldg(q + j);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    alo[i][t][j] = act_perm_lo(w[1 + j], w[5 + j]);
                    ahi[i][t][j] = act_perm_hi(w[1 + j], w[5 + j]);
                }
                dx[i][t] = f16_bits_to_f32(w[0]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) alo[i][t][j] = ahi[i][t][j] = 0u;
                dx[i][t] = 0.0f;
            }
        }
    }
    // Activations are in registers: a dependent kernel may now overwrite the Q8_1 workspace.
    grid_launch_dependents();
    const uint32_t push_epoch = a.push ? peer_slots_epoch_next(a.push) : 0u;  // after the grid dependency wait
    const uint8_t* lane_h = ring + (size_t)(slot * RPW) * a.rb + off_h;  // + stage, row, sub-block offsets

    for (int t = 0; t < ntiles; ++t) {
        const int s = (int)((uint32_t)t % stages);
        const bool ready =
            !*abort_flag && wait_sleep_or_abort(&full[s], ((uint32_t)t / stages) & 1u, abort_flag, a.err, kDevErrFullWait);
        const int64_t row0 = r0 + (int64_t)t * R;
        const int rows = (int)imin64(R, r1 - row0);
        if (ready && slot * RPW < rows) {
            const uint8_t* sbase = lane_h + (size_t)s * stage_bytes;
            float acc[RPW][B];
#pragma unroll
            for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int tt = 0; tt < B; ++tt) acc[r][tt] = 0.0f;
#pragma unroll
            for (int i = 0; i < SPL; ++i) {
                if (!kTail || sb0 + 32 * i < nsb) {
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        // rows past the tile read stale shared memory; their sums are discarded
                        const uint8_t* rowp = sbase + (size_t)r * a.rb + i * 4 * kBlockBytes;
                        const uint2 h = *reinterpret_cast<const uint2*>(rowp);
                        const uint2 qa = *reinterpret_cast<const uint2*>(rowp + (off_q - off_h));
                        const uint2 qb = *reinterpret_cast<const uint2*>(rowp + (off_q - off_h) + 8);
                        uint32_t wh[8], wl[8];
                        lut_word(a.lut, qa.x, wh[0], wl[0], wh[1], wl[1]);
                        lut_word(a.lut, qa.y, wh[2], wl[2], wh[3], wl[3]);
                        lut_word(a.lut, qb.x, wh[4], wl[4], wh[5], wl[5]);
                        lut_word(a.lut, qb.y, wh[6], wl[6], wh[7], wl[7]);
                        const float dw = f16_bits_to_f32(h.x);
                        const int scale = (int)(((h.y >> sh_lo) & 0xFu) | ((h.x >> sh_hi) & 0x30u)) - 32;
#pragma unroll
                        for (int tt = 0; tt < B; ++tt) {
                            int s0 = dp4a((int)wh[0], (int)alo[i][tt][0], 0);
                            int s1 = dp4a((int)wl[0], (int)alo[i][tt][0], 0);
                            int s2 = dp4a((int)wh[1], (int)ahi[i][tt][0], 0);
                            int s3 = dp4a((int)wl[1], (int)ahi[i][tt][0], 0);
#pragma unroll
                            for (int w = 1; w < 4; ++w) {
                                s0 = dp4a((int)wh[2 * w], (int)alo[i][tt][w], s0);
                                s1 = dp4a((int)wl[2 * w], (int)alo[i][tt][w], s1);
                                s2 = dp4a((int)wh[2 * w + 1], (int)ahi[i][tt][w], s2);
                                s3 = dp4a((int)wl[2 * w + 1], (int)ahi[i][tt][w], s3);
                            }
                            const int sumi = (s0 + s2) - (s1 + s3);
                            if constexpr (kDebug) {
                                if (slot * RPW + r < rows)
                                    a.sumi[((int64_t)tt * a.N + row0 + slot * RPW + r) * nsb + sb0 + 32 * i] = sumi;
                            }
                            acc[r][tt] += (dw * dx[i][tt]) * (float)(sumi * scale);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                const int rl = slot * RPW + r;
#pragma unroll
                for (int tt = 0; tt < B; ++tt) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) acc[r][tt] += __shfl_xor_sync(0xFFFFFFFFu, acc[r][tt], off);
                }
                if (rl >= rows) continue;
                const int64_t row = row0 + rl;
                if (KW == 1) {
                    if (lane == 0 && a.push) {
                        peer_slots_store(a.push, row, acc[r][0], push_epoch);
                    } else if (lane == 0 && a.y) {
#pragma unroll
                        for (int tt = 0; tt < B; ++tt) a.y[(int64_t)tt * a.N + row] = acc[r][tt];
                    }
                } else if (lane == 0) {
                    float* pp = part + ((s * R + rl) * KW) * B;
#pragma unroll
                    for (int tt = 0; tt < B; ++tt) pp[kw * B + tt] = acc[r][tt];
                    __threadfence_block();
                    const uint32_t old = atomicAdd(&cnt[s * R + rl], 1u);
                    if (old == (uint32_t)KW - 1) {
                        __threadfence_block();
                        cnt[s * R + rl] = 0u;
                        if (a.push) {
                            float v = 0.0f;
                            for (int k = 0; k < KW; ++k) v += reinterpret_cast<volatile float*>(pp)[k * B];
                            peer_slots_store(a.push, row, v, push_epoch);
                        } else if (a.y) {
#pragma unroll
                            for (int tt = 0; tt < B; ++tt) {
                                float v = 0.0f;
                                for (int k = 0; k < KW; ++k) v += reinterpret_cast<volatile float*>(pp)[k * B + tt];
                                a.y[(int64_t)tt * a.N + row] = v;
                            }
                        }
                    }
                }
            }
        }
        fence_generic_async_smem();  // this warp's reads of the stage before its refill
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (a.push) {  // every consumer warp has stored: the grid's last CTA advances the epoch counter
        named_barrier(2, NCW * 32);
        if (cw == 0 && lane == 0) peer_slots_done(a.push, ncta, push_epoch);
    }
}

template <int B, int SPL, int RPW, int NCW, bool kTail, bool kDebug, int kAct>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) gemv_iq4xs_q8_rows_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    gemv_rows_body<B, SPL, RPW, NCW, kTail, kDebug, kAct>(a, (int)blockIdx.x, (int)gridDim.x, smem);
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
// Grouped row kernel (batch 1): block b belongs to matrix p with cta0[p] <= b < cta0[p+1] and runs
// the row-kernel body on that matrix's row range share.  Every instance of the body a matrix may need
// (sub-block slots per lane, tail) is compiled in; each CTA executes one.
constexpr int kRowGroupNCW = 12, kRowGroupRPW = 2;  // the row kernel's geometry (kRowNCW, kRowRPW below)
struct GroupRowsParams {
    GemvArgs args[kMaxGroup];
    int cta0[kMaxGroup + 1];
    int code[kMaxGroup];  // 2 * sub-block slots per lane + tail
    int count;
};

__global__ void __launch_bounds__(32 * (kRowGroupNCW + 1), 1)
    gemv_rows_grouped_kernel(const __grid_constant__ GroupRowsParams G) {
    extern __shared__ __align__(128) uint8_t smem[];
    int p = 0;
    while (p + 1 < G.count && (int)blockIdx.x >= G.cta0[p + 1]) ++p;
    const int cta = (int)blockIdx.x - G.cta0[p], ncta = G.cta0[p + 1] - G.cta0[p];
    const GemvArgs a = G.args[p];
    switch (G.code[p]) {
#define IQ4XS_ROWS_CASE(SPL, TAIL)                                                                           \
    case 2 * SPL + TAIL:                                                                                     \
        gemv_rows_body<1, SPL, kRowGroupRPW, kRowGroupNCW, TAIL != 0, false, kActQ8>(a, cta, ncta, smem); \
        break;
        IQ4XS_ROWS_CASE(1, 0) IQ4XS_ROWS_CASE(1, 1) IQ4XS_ROWS_CASE(2, 0) IQ4XS_ROWS_CASE(2, 1)
        IQ4XS_ROWS_CASE(3, 0) IQ4XS_ROWS_CASE(3, 1) IQ4XS_ROWS_CASE(4, 0) IQ4XS_ROWS_CASE(4, 1)
        IQ4XS_ROWS_CASE(5, 0) IQ4XS_ROWS_CASE(5, 1)
        IQ4XS_ROWS_CASE(6, 0) IQ4XS_ROWS_CASE(6, 1)
#undef IQ4XS_ROWS_CASE
        default: break;
    }
}

// --------------------------------------------------------------------------------------------
// Host-side launch helpers.
// Warps per row (kw) and sub-block slots per lane (spl) of the row kernel for K at batch B; false when
// even four warps per row would need more than the lane's register budget (the launch then takes the
// tensor-core kernel).
int gemv_rows_per_stage(int64_t K) {
    int kw = 1, spl = 1;
    row_split(K, 1, &kw, &spl);
    return (kRowGroupNCW / kw) * kRowGroupRPW;
}

bool row_split(int64_t K, int B, int* kw_out, int* spl_out) {
    const int64_t nsb = K / kQK8;
    // the fewest warps per row (1..4, all dividing the 12 consumer warps) that fit the lane budget;
    // 3 warps at K = 17408 leave 5.6% of the lane slots idle where 4 warps left 15% (measured on
    // B200: down_proj at batch 1 18.4 -> 16.4 us)
    const int spl_max = (B == 1) ? 6 : 2;
    int kw = 1;
    while (kw < 4 && (nsb + 32 * kw - 1) / (32 * kw) > spl_max) ++kw;
    const int64_t spl = (nsb + 32 * kw - 1) / (32 * kw);
    *kw_out = kw;
    *spl_out = (int)(spl < 1 << 20 ? spl : 1 << 20);
    return spl <= spl_max;
}

namespace {

// Per-device cache of the two attributes.  Host threads may launch on one device concurrently: the
// shared-memory limit is published before the SM count (release), and a reader that sees the SM
// count (acquire) sees the limit too, so no caller reads a half-filled entry.
std::atomic<int> g_num_sms[64];
std::atomic<int> g_max_smem[64];

void device_limits(int dev, int* sms, int* smem_optin) {
    if (dev < 0 || dev >= 64) {
        cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        return;
    }
    int n = g_num_sms[dev].load(std::memory_order_acquire);
    if (n == 0) {
        int smem = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        *sms = n;
        *smem_optin = smem;
        if (n > 0 && smem > 0) {
            g_max_smem[dev].store(smem, std::memory_order_relaxed);
            g_num_sms[dev].store(n, std::memory_order_release);
        }
        return;
    }
    *sms = n;
    *smem_optin = g_max_smem[dev].load(std::memory_order_relaxed);
}

// Row-stage kernel configuration for batch B: 16 consumer warps, one row each per stage; KW warps
// per row so that a lane holds at most SPLMAX(B) sub-blocks of activations in registers.
constexpr int kRowNCW = kRowGroupNCW, kRowRPW = kRowGroupRPW;
// fp32 sources are quantised inside the row kernel up to this K (every CTA quantises all of K; beyond
// it the standalone quantizer launch is cheaper, measured on B200 at K = 8192 and 17408)
constexpr int kRowFusedMaxK = 6144;


template <int B, int SPL, bool kDebug, int kAct>
void* rows_kernel_ptr_t(bool tail) {
    return tail ? (void*)gemv_iq4xs_q8_rows_kernel<B, SPL, kRowRPW, kRowNCW, true, kDebug, kAct>
                : (void*)gemv_iq4xs_q8_rows_kernel<B, SPL, kRowRPW, kRowNCW, false, kDebug, kAct>;
}

template <int B, int SPL, bool kDebug>
void* rows_kernel_ptr(bool tail, int mode) {
    if constexpr (kDebug) {  // the debug path reads Q8_1 from global memory only
        return rows_kernel_ptr_t<B, SPL, true, kActQ8>(tail);
    } else {
        if constexpr (B == 1) {
            if (mode == kActNormPeer) return rows_kernel_ptr_t<B, SPL, false, kActNormPeer>(tail);
            if (mode == kActSwiGLU) return rows_kernel_ptr_t<B, SPL, false, kActSwiGLU>(tail);
        }
        if (mode == kActNorm) return rows_kernel_ptr_t<B, SPL, false, kActNorm>(tail);
        if (mode == kActF32) return rows_kernel_ptr_t<B, SPL, false, kActF32>(tail);
        return rows_kernel_ptr_t<B, SPL, false, kActQ8>(tail);
    }
}

// Row-kernel geometry of `a` at batch B: warps per row, rows per stage and ring depth are set in
// `a`; *spl / *tail select the kernel instance, *smem_total its dynamic shared memory.  cudaErrorNotSupported when K is too long for the row kernel.
cudaError_t row_geometry(GemvArgs& a, int B, int smem_optin, int* spl_out, bool* tail_out, uint32_t* smem_total) {
    constexpr int NCW = kRowNCW, RPW = kRowRPW;
    const int nsb = a.K / kQK8;
    int kw = 1, spl = 1;
    if (!row_split(a.K, B, &kw, &spl)) return cudaErrorNotSupported;
    const bool tail = (nsb != 32 * kw * spl);
    const int R = (NCW / kw) * RPW;
    a.kw = kw;
    a.rows_per_stage = R;
    const int64_t stage_bytes = (int64_t)R * a.rb;
    // At most ~110 KB of stages (two of them always): deeper rings did not stream faster, and a CTA
    // that leaves half the shared memory free lets the next kernel's CTA start on the same SM.
    constexpr int64_t kRowSmemTarget = 110000;
    const uint32_t q8b = act_smem_bytes(a.act.mode, B, a.K);
    int stages = kMaxStages;
    while (stages > 2 && ((int64_t)gemv_row_smem(B, R, kw, stages, stage_bytes, q8b).total > smem_optin ||
                          (int64_t)gemv_row_smem(B, R, kw, stages, stage_bytes, q8b).total > kRowSmemTarget + q8b))
        --stages;
    a.stages = stages;
    const RowSmem L = gemv_row_smem(B, R, kw, stages, stage_bytes, q8b);
    if ((int64_t)L.total > smem_optin || stage_bytes >= (1 << 20)) return cudaErrorInvalidConfiguration;
    *spl_out = spl;
    *tail_out = tail;
    *smem_total = L.total;
    return cudaSuccess;
}

template <int B, bool kDebug>
cudaError_t launch_rows(GemvArgs a, cudaStream_t stream, bool pdl, int sms, int smem_optin) {
    constexpr int NCW = kRowNCW;
    int kw = 1, spl = 1;
    if (!row_split(a.K, B, &kw, &spl)) {  // K too long for register-resident activations: tensor-core kernel
        if (a.act.mode == kActNorm || a.act.mode == kActNormPeer || a.act.mode == kActSwiGLU)
            return cudaErrorNotSupported;
        return launch_gemv_mma(a.W, a.q8, a.y, kDebug ? a.sumi : nullptr, a.partials, a.partial_bytes, a.K, a.N,
                               B, stream, pdl, sms, smem_optin, a.err, a.lut, &a.act);
    }
    if (a.act.mode == kActF32 && a.K > kRowFusedMaxK) {
        // every CTA would quantise all of K: the standalone quantizer (programmatic launch) is cheaper
        cudaError_t eq = launch_q8_1_quantize(a.act.x, const_cast<uint8_t*>(a.q8), a.K, B, a.K, 1, stream, true, pdl);
        if (eq != cudaSuccess) return eq;
        a.act.mode = kActQ8;
        pdl = true;
    }
    if (a.act.mode == kActSwiGLU && (B != 1 || a.K > kRowFusedMaxK)) {
        // the same policy for the SwiGLU source: the standalone SwiGLU kernel writes the Q8_1 blocks
        cudaError_t eq = launch_swiglu_q8(a.act.x, a.K, 1, const_cast<uint8_t*>(a.q8), stream, pdl);
        if (eq != cudaSuccess) return eq;
        a.act.mode = kActQ8;
        pdl = true;
    }
    bool tail = false;
    uint32_t smem_total = 0;
    cudaError_t eg = row_geometry(a, B, smem_optin, &spl, &tail, &smem_total);
    if (eg != cudaSuccess) return eg;
    void* kern = nullptr;
    const int sa = a.act.mode;
    switch (spl) {
        case 1: kern = rows_kernel_ptr<B, 1, kDebug>(tail, sa); break;
        case 2: kern = rows_kernel_ptr<B, 2, kDebug>(tail, sa); break;
        case 3: kern = B == 1 ? rows_kernel_ptr<1, 3, kDebug>(tail, sa) : nullptr; break;
        case 4: kern = B == 1 ? rows_kernel_ptr<1, 4, kDebug>(tail, sa) : nullptr; break;
        case 5: kern = B == 1 ? rows_kernel_ptr<1, 5, kDebug>(tail, sa) : nullptr; break;
        case 6: kern = B == 1 ? rows_kernel_ptr<1, 6, kDebug>(tail, sa) : nullptr; break;
        default: break;
    }
    if (!kern) return cudaErrorInvalidConfiguration;
    cudaError_t e = ensure_dynamic_smem(kern, (int)smem_total);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)imin64((int64_t)sms, a.N));
    cfg.blockDim = dim3(32 * (NCW + 1));
    cfg.dynamicSmemBytes = smem_total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, kern, args);
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
    const bool bulk_ok = gemv_bulk_path(a.W, a.K) && !a.force_generic;
    if (!bulk_ok) {
        if (a.act.mode != kActQ8) return cudaErrorNotSupported;  // the generic kernel reads Q8_1 from global
        switch (B) {
#define IQ4XS_GEN(BB) case BB: return launch_generic<BB, kDebug>(a, stream, pdl, sms);
            IQ4XS_GEN(1) IQ4XS_GEN(2) IQ4XS_GEN(3) IQ4XS_GEN(4) IQ4XS_GEN(5) IQ4XS_GEN(6) IQ4XS_GEN(7) IQ4XS_GEN(8)
#undef IQ4XS_GEN
            default: return cudaErrorInvalidValue;
        }
    }
    if (B == 1) return launch_rows<1, kDebug>(a, stream, pdl, sms, smem_optin);
    if (a.act.mode == kActNorm || a.act.mode == kActNormPeer || a.act.mode == kActSwiGLU) return cudaErrorNotSupported;
    return launch_gemv_mma(a.W, a.q8, a.y, kDebug ? a.sumi : nullptr, a.partials, a.partial_bytes, a.K, a.N, B,
                           stream, pdl, sms, smem_optin, a.err, a.lut, &a.act);
}
}  // namespace

bool gemv_bulk_path(const uint8_t* W, int64_t K) {
    return ((K / kQK) % 2 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15u) == 0);
}

void device_limits_current(int* sms, int* smem_optin) {
    int dev = 0;
    cudaGetDevice(&dev);
    device_limits(dev, sms, smem_optin);
}

cudaError_t launch_gemv_rows_grouped(const GroupedProblem* p, int count, cudaStream_t stream, bool pdl, uint32_t* err,
                                     const uint32_t lut[4]) {
    if (count < 1 || count > kMaxGroup) return cudaErrorInvalidValue;
    int sms = 0, smem_optin = 0;
    device_limits_current(&sms, &smem_optin);
    GroupRowsParams G;
    std::memset(&G, 0, sizeof G);
    uint32_t smem_max = 0;
    int cta = 0;
    for (int i = 0; i < count; ++i) {
        if (!gemv_bulk_path(p[i].W, p[i].K)) return cudaErrorNotSupported;
        GemvArgs a;
        std::memset(&a, 0, sizeof a);
        a.W = p[i].W;
        a.q8 = p[i].q8;
        a.y = p[i].y;
        a.err = err;
        a.N = p[i].N;
        a.K = (int)p[i].K;
        a.kb = (int)(p[i].K / kQK);
        a.rb = (int64_t)a.kb * kBlockBytes;
        for (int j = 0; j < 4; ++j) a.lut[j] = lut[j];
        a.act.mode = kActQ8;
        int spl = 1;
        bool tail = false;
        uint32_t sm = 0;
        const cudaError_t e = row_geometry(a, 1, smem_optin, &spl, &tail, &sm);
        if (e != cudaSuccess) return e;
        G.args[i] = a;
        G.code[i] = 2 * spl + (tail ? 1 : 0);
        G.cta0[i] = cta;
        cta += (int)imin64(std::max(p[i].ctas, 1), p[i].N);
        smem_max = std::max(smem_max, sm);
    }
    G.cta0[count] = cta;
    G.count = count;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemv_rows_grouped_kernel), (int)smem_max);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cta);
    cfg.blockDim = dim3(32 * (kRowNCW + 1));
    cfg.dynamicSmemBytes = smem_max;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_rows_grouped_kernel, G);
}

bool gemv_takes_mma(const uint8_t* W, int64_t K, int B) {
    if (!gemv_bulk_path(W, K)) return false;  // the direct-load kernel writes no partial sums
    if (B > 1) return true;
    int kw = 1, spl = 1;
    return !row_split(K, 1, &kw, &spl);
}

cudaError_t ensure_dynamic_smem(const void* kern, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, int> done;  // (device, kernel) -> bytes allowed
    int dev = 0, sms = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    device_limits(dev, &sms, &optin);
    if (bytes > optin) return cudaErrorInvalidValue;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(dev, kern);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e == cudaSuccess) done[key] = optin;
    return e;
}

int device_sm_count() {
    int dev = 0, sms = 0, smem = 0;
    cudaGetDevice(&dev);
    device_limits(dev, &sms, &smem);
    return sms;
}

int device_smem_optin() {
    int dev = 0, sms = 0, smem = 0;
    cudaGetDevice(&dev);
    device_limits(dev, &sms, &smem);
    return smem;
}

cudaError_t launch_gemv_q8(GemvArgs a, int B, cudaStream_t stream, bool pdl) {
    a.sumi = nullptr;
    return dispatch<false>(B, a, stream, pdl);
}

cudaError_t launch_gemv_q8_debug(GemvArgs a, int B, cudaStream_t stream) { return dispatch<true>(B, a, stream, false); }

}  // namespace iq4xs
