// gemm.cu -- IQ4_XS x Q8_1 prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Arithmetic contract: the reference's stock GEMM (real_stock_dp4a_comparator.hip:375-443): every
// 32-weight sub-block of a weight row meets every token's Q8_1 block as an exact integer dot
// sumi = sum_j kv[q_j] * x_j, and the output is sum over sub-blocks of (d_w*(ls-32)) * d_x * sumi in
// fp32.  Here:
//
//  * Operands are fp16 tensors holding exact small integers: the codebook values kv (|kv| <= 127)
//    and the Q8_1 quants (|q| <= 127).  Products are exact, and the fp32 tensor-core sum of one
//    sub-block (|sumi| <= 32*127*127 < 2^24) is exact too, so each TMEM accumulator holds the exact
//    integer sumi of one (row, token, sub-block).  int8 operands (kind::i8) would halve the MMA time
//    but leave an s32 -> f32 conversion on every drained element, and the drain is this kernel's
//    bound (below); fp16 integers come out of TMEM as fp32 directly.
//  * Per 32-wide sub-block the MMA (M = 128 weight rows, N = 128 tokens, two K = 16 steps) writes a
//    fresh TMEM accumulator; drain warps load it (tcgen05.ld) and fold the scale in:
//    acc[row][token] += (sumi * d_x[token]) * (d_w*(ls-32))[row] in fp32 registers.  Four TMEM
//    accumulators (4 x 128 columns) let the MMA run up to four sub-blocks ahead of the drain.
//    A drain warp reads its 32 columns of a stage's two accumulators in four 16-column chunks and
//    issues each chunk's load before the arithmetic of the previous one, so the TMEM load latency
//    hides behind the scale folding (+4-5% over load-all-then-compute, measured on B200).
//  * Weights: the IQ4_XS rows as stored, viewed as uint64 [N][K/512 pairs][34] and loaded by TMA
//    128 rows x one super-block pair (34,816 bytes) at a time.  Converter warps (one thread per row)
//    expand each 64-wide K chunk to fp16 in the canonical K-major 128-byte-swizzled layout that
//    tcgen05 descriptors read: split codebook lookup by prmt (tables -kv[0..7] and kv[8..15]), one
//    IADD3 to the biased byte kv+128, prmt into the fp16 pattern 0x64XX (= 1024 + byte), HADD2 with
//    -1152.  Within a sub-block the K order is the lookup's natural order: position 8w + 2i + j holds
//    element 4w + i + 16j (w = qs word, i = byte in word, j = nibble); the activation quantizer
//    writes the same order, and a permutation of K inside a sub-block leaves the dot unchanged.
//  * Activations: quantised once per call into stage blocks, one per (128-token tile, 64-wide K
//    stage): 16 KB of fp16 q (exact integers, that K order) already in the 128-byte-swizzled K-major
//    layout, then 2 x 128 fp32 d_x (the fp32 value of the truncated fp16 d of each Q8_1 block: the
//    reference's low2float(ds)).  A stage is one contiguous 17,408-byte bulk copy: a 2-D tensor box
//    of 128 rows x 128 bytes moves as 128 separate rows and ran several times slower.
//  * Persistent kernel, one CTA per SM; tiles (128 rows x 128 tokens) in row-tile-major order so the
//    CTAs running at once share weight rows in L2.  Warp roles: 0 weight TMA, 1 TMEM allocation and
//    MMA issue (one thread), 2 activation TMA, 3 spare, 4-7 converters, 8-23 drain +
//    epilogue.
//  * Synchronisation is per 64-wide stage, not per sub-block: an mbarrier operation costs a few
//    hundred cycles of latency here, so the single MMA-issuing thread waits on one "stage full"
//    barrier (activation copy + four converter warps) and one "TMEM pair free" barrier per stage,
//    and the two sub-block accumulators of a stage form a TMEM pair (two pairs, 512 columns).
//    Waiters sleep on their barriers in turn (try_wait with a suspend hint): a polling loop of
//    non-blocking tests in the 16 drain warps took more issue slots than the drain arithmetic.
//  * Every mbarrier wait is bounded (sleeping try_wait); a wait that gives up records a device
//    error, raises the CTA's abort flag, and every role leaves its loop; in-flight TMA copies and
//    MMAs are waited for (bounded) and TMEM is freed before the CTA exits.  No cluster multicast.
#include <cuda.h>

#include <algorithm>

#include "gemm_tc.cuh"
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

using namespace gemm_tc;

namespace {
constexpr int kBM = 128;         // weight rows per tile = MMA M = TMEM lanes
constexpr int kBN = 128;         // tokens per tile = MMA N = TMEM columns per accumulator
constexpr int kBK = 64;          // K per stage (two sub-blocks, one 128-byte swizzle atom of fp16)
constexpr int kStages = 4;       // A / B / scale ring depth
constexpr int kRawStages = 2;    // raw weight ring depth (one super-block pair each)
constexpr int kAccBufs = 4;      // TMEM accumulators (4 x 128 = 512 columns)
constexpr int kConvWarps = 4;
constexpr int kDrainWarps = 16;  // 4 per TMEM lane quarter, 32 token columns each
constexpr int kFirstConvWarp = 4;                             // warps 0-3: weight TMA, MMA, act TMA, spare
constexpr int kFirstDrainWarp = kFirstConvWarp + kConvWarps;  // 8
constexpr int kThreads = 32 * (kFirstDrainWarp + kDrainWarps);  // 768


constexpr uint32_t kRawBytes = kBM * 272;        // 34,816
constexpr uint32_t kABytes = kBM * kBK * 2;      // 16,384
constexpr uint32_t kBBytes = kBN * kBK * 2;      // 16,384
constexpr uint32_t kSxBytes = 2 * kBN * 4;       // 1,024
constexpr uint32_t kSwBytes = 2 * kBM * 4;       // 1,024

constexpr uint32_t kActStageBytes = kBBytes + kSxBytes;  // 17,408: one activation stage block

constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffB = kOffA + kStages * kABytes;          // stage s: B at kOffB + s*17408, d_x after it
constexpr uint32_t kOffRaw = kOffB + kStages * kActStageBytes;
constexpr uint32_t kOffSw = kOffRaw + kRawStages * kRawBytes;
constexpr uint32_t kOffBar = kOffSw + kStages * kSwBytes;
constexpr int kNumBars = 2 * kRawStages + 2 * kStages + 2 * (kAccBufs / 2) + 1;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;  // TMEM address, abort flag, stage verdict
constexpr uint32_t kSmemBytes = kOffMisc + 16 + 1024;  // + slack to align the base to 1024

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B fp16 (bits 7-9, 10-12 = 0),
// both K-major (bits 15, 16 = 0), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// fp16x2 add on raw bits.
__device__ __forceinline__ uint32_t hadd2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Four fp16 pairs (8 weights) of one qs word in the lookup order, exact codebook values:
// [e(4w), e(4w+16)], [e(4w+1), e(4w+17)], [e(4w+2), e(4w+18)], [e(4w+3), e(4w+19)].
__device__ __forceinline__ uint4 expand_word(uint32_t x, const uint32_t (&lut)[4]) {
    const uint32_t xf = x ^ 0x88888888u;
    const uint32_t lo_l = prmt(lut[0], lut[1], x), lo_h = prmt(lut[2], lut[3], xf);
    const uint32_t hi_l = prmt(lut[0], lut[1], x >> 16), hi_h = prmt(lut[2], lut[3], xf >> 16);
    // Biased bytes kv + 128: 128 - (-kv) for codes < 8, 128 + kv for codes >= 8 (no carries).
    const uint32_t blo = 0x80808080u - lo_l + lo_h;
    const uint32_t bhi = 0x80808080u - hi_l + hi_h;
    // prmt with 0x64 high bytes makes fp16 1024 + byte; adding -1152 (0xE480) leaves kv exactly.
    constexpr uint32_t kBias = 0xE480E480u;
    uint4 r;
    r.x = hadd2_bits(prmt(blo, 0x64646464u, 0x4140u), kBias);
    r.y = hadd2_bits(prmt(blo, 0x64646464u, 0x4342u), kBias);
    r.z = hadd2_bits(prmt(bhi, 0x64646464u, 0x4140u), kBias);
    r.w = hadd2_bits(prmt(bhi, 0x64646464u, 0x4342u), kBias);
    return r;
}

// The loaded registers are redefined after the wait, so no use can be scheduled before it.
__device__ __forceinline__ void regs_after_wait(uint32_t (&v)[16]) {
    asm volatile("" : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]));
}

// acc[c0 + j] += (v[j] * d_x[32 cg + c0 + j]) * sw for the 16 columns of one chunk of sub-block h.
__device__ __forceinline__ void drain_chunk(float (&acc)[32], const uint32_t (&v)[16], int c0, uint32_t sw_base,
                                            uint32_t sx_base, int s, int h) {
    const float wsc = lds_f32(sw_base + (uint32_t)(s * kSwBytes + h * kBM * 4));
    const uint32_t sxa = sx_base + (uint32_t)(s * kActStageBytes + h * kBN * 4 + 4 * c0);
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
        const uint4 x = lds_u4(sxa + 16u * c4);
        float t0, t1, t2, t3;
        mul2(t0, t1, __uint_as_float(v[4 * c4 + 0]), __uint_as_float(v[4 * c4 + 1]), __uint_as_float(x.x), __uint_as_float(x.y));
        mul2(t2, t3, __uint_as_float(v[4 * c4 + 2]), __uint_as_float(v[4 * c4 + 3]), __uint_as_float(x.z), __uint_as_float(x.w));
        fma2(acc[c0 + 4 * c4 + 0], acc[c0 + 4 * c4 + 1], t0, t1, wsc, wsc);
        fma2(acc[c0 + 4 * c4 + 2], acc[c0 + 4 * c4 + 3], t2, t3, wsc, wsc);
    }
}
}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    gemm_iq4xs_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* raw_full = bars;                       // weight pair landed (TMA bytes)
    uint64_t* raw_empty = raw_full + kRawStages;     // converters done with a weight pair
    uint64_t* full = raw_empty + kRawStages;         // stage: activation copy landed + 4 converter warps
    uint64_t* freeb = full + kStages;                // stage: MMAs done (commit) + drain done with its scales
    uint64_t* t_full = freeb + kStages;              // TMEM pair: both sub-block MMAs of a stage done
    uint64_t* t_empty = t_full + kAccBufs / 2;       // TMEM pair: drain warps have loaded it
    uint64_t* mma_done = t_empty + kAccBufs / 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = a.tiles_m;
    const int64_t T = (int64_t)a.tiles_n * tiles_m;
    const int pairs = a.K / 512;
    const int S = a.K / kBK;  // stages per tile

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRawStages; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kConvWarps);
        }
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1 + kConvWarps);
            mbar_init(&freeb[i], 1 + kDrainWarps);
        }
        for (int i = 0; i < kAccBufs / 2; ++i) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], kDrainWarps);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0u;
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kAccBufs * kBN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // X (and so the quantised activations) may come from the preceding kernel.
    grid_dependency_wait();

    if (warp == 0) {
        // ------------------------------------------------------------------ weight TMA
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < T && ok; t += gridDim.x) {
                const int row0 = (int)(t / tiles_m) * kBM;
                for (int p = 0; p < pairs && ok; ++p, ++it) {
                    const int s = (int)(it % kRawStages);
                    const uint32_t u = it / kRawStages;
                    if (!(ok = gwait(&raw_empty[s], (u & 1u) ^ 1u, abort_flag, a.err, kDevErrEmptyWait))) break;
                    fence_generic_async_smem();  // the converters' ld.shared of this stage come first
                    mbar_arrive_expect_tx(&raw_full[s], kRawBytes);
                    tma_load_3d_nohint(smem + kOffRaw + s * kRawBytes, &tmap_w, 0, p, row0, &raw_full[s]);
                }
            }
            // Let the last copies land before the CTA can exit.
            for (uint32_t j = it > (uint32_t)kRawStages ? it - kRawStages : 0; j < it; ++j)
                gdrain(&raw_full[j % kRawStages], (j / kRawStages) & 1u, a.err);
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------------ activation TMA
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < T && ok; t += gridDim.x) {
                const int64_t mt = t % tiles_m;
                for (int st = 0; st < S; ++st, ++it) {
                    const int s = (int)(it % kStages);
                    const uint32_t u = it / kStages;
                    if (!(ok = gwait_fast(&freeb[s], (u & 1u) ^ 1u, abort_flag, a.err, kDevErrEmptyWait))) break;
                    fence_generic_async_smem();  // the drain's ld.shared of this stage's d_x come first
                    mbar_arrive_expect_tx(&full[s], kActStageBytes);
                    bulk_g2s(smem + kOffB + s * kActStageBytes, a.act + ((size_t)mt * S + st) * kActStageBytes,
                             kActStageBytes, &full[s]);
                }
            }
            for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0; j < it; ++j)
                gdrain(&full[j % kStages], (j / kStages) & 1u, a.err);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < T && ok; t += gridDim.x) {
                for (int st = 0; st < S && ok; ++st, ++it) {
                    const int s = (int)(it % kStages);
                    const uint32_t u = it / kStages;
                    const int g = (int)(it & 1u);
                    const uint32_t ug = it >> 1;
                    if (!(ok = gwait_seq(&full[s], u & 1u, &t_empty[g], (ug & 1u) ^ 1u, abort_flag, a.err, kDevErrMmaWait)))
                        break;
                    tc_fence_after();
                    const uint64_t ad = smem_desc_sw128(smem_addr(smem + kOffA + s * kABytes));
                    const uint64_t bd = smem_desc_sw128(smem_addr(smem + kOffB + s * kActStageBytes));
                    const uint32_t d = tmem_base + (uint32_t)(g * 2 * kBN);
                    // Sub-block h -> accumulator d + h*128; K offsets 32h, 32h+16 fp16 = 4h, 4h+2 in 16-byte units.
                    tc_mma_f16(d, ad, bd, 0u);
                    tc_mma_f16(d, ad + 2, bd + 2, 1u);
                    tc_mma_f16(d + kBN, ad + 4, bd + 4, 0u);
                    tc_mma_f16(d + kBN, ad + 6, bd + 6, 1u);
                    tc_commit(&t_full[g]);
                    tc_commit(&freeb[s]);
                }
            }
            // All issued MMAs complete before TMEM is released.
            tc_commit(mma_done);
            gdrain(mma_done, 0u, a.err);
        }
        __syncwarp();
    } else if (warp == 3) {
        // spare warp (keeps the converter and drain warps on fixed sub-partitions)
    } else if (warp < kFirstDrainWarp) {
        // ------------------------------------------------------------------ converters: thread = row
        const int r = threadIdx.x - 32 * kFirstConvWarp;
        const uint32_t lut[4] = {a.lut[0], a.lut[1], a.lut[2], a.lut[3]};
        uint32_t rit = 0, it = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < T && ok; t += gridDim.x) {
            for (int p = 0; p < pairs && ok; ++p, ++rit) {
                const int rs = (int)(rit % kRawStages);
                if (!(ok = gwait_fast(&raw_full[rs], (rit / kRawStages) & 1u, abort_flag, a.err, kDevErrFullWait))) break;
                const uint32_t rowp = smem_addr(smem + kOffRaw + rs * kRawBytes) + (uint32_t)r * 272u;
                for (int sp = 0; sp < 8; ++sp, ++it) {
                    const int s = (int)(it % kStages);
                    const uint32_t u = it / kStages;
                    if (!(ok = gwait_fast(&freeb[s], (u & 1u) ^ 1u, abort_flag, a.err, kDevErrEmptyWait))) break;
                    const uint32_t sbp = rowp + (uint32_t)(sp >> 2) * 136u;
                    const uint2 hdr = lds_u2(sbp);
                    const float dw = f16_bits_to_f32(hdr.x);
                    const int ib0 = 2 * (sp & 3);
                    const uint32_t sw = smem_addr(smem + kOffSw + s * kSwBytes) + 4u * (uint32_t)r;
                    sts_f32(sw, dw * (float)(subblock_scale(hdr.x, hdr.y, ib0) - 32));
                    sts_f32(sw + 4u * kBM, dw * (float)(subblock_scale(hdr.x, hdr.y, ib0 + 1) - 32));
                    const uint32_t qp = sbp + 8u + 32u * (uint32_t)(sp & 3);
                    uint32_t qw[8];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint2 v = lds_u2(qp + 8u * k);
                        qw[2 * k] = v.x;
                        qw[2 * k + 1] = v.y;
                    }
                    const uint32_t arow = smem_addr(smem + kOffA + s * kABytes) + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) sts_u4(arow + (uint32_t)((c ^ (r & 7)) << 4), expand_word(qw[c], lut));
                    fence_proxy_async_smem();  // generic-proxy writes -> tensor-core (async proxy) reads
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                }
                fence_generic_async_smem();  // this warp's reads of the raw stage before its TMA refill
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&raw_empty[rs]);
            }
        }
    } else {
        // ------------------------------------------------------------------ drain + epilogue
        const int dw = warp - kFirstDrainWarp;        // 0..15
        const int lq = warp & 3;                      // TMEM lane quarter this warp may access
        const int cg = dw >> 2;                       // token columns 32*cg .. 32*cg+31
        const int r = 32 * lq + lane;                 // tile row = TMEM lane
        const uint32_t lane_base = tmem_base + ((uint32_t)(32 * lq) << 16) + (uint32_t)(32 * cg);
        const uint32_t sw_base = smem_addr(smem + kOffSw) + 4u * (uint32_t)r;
        const uint32_t sx_base = smem_addr(smem + kOffB + kBBytes) + 4u * (uint32_t)(32 * cg);
        uint32_t it = 0;
        bool go = true;
        for (int64_t t = blockIdx.x; t < T && go; t += gridDim.x) {
            const int row0 = (int)(t / tiles_m) * kBM;
            const int m0 = (int)(t % tiles_m) * kBN;
            float acc[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
            for (int st = 0; st < S; ++st, ++it) {
                const int s = (int)(it % kStages);
                const int g = (int)(it & 1u);
                // t_full: both sub-block MMAs of the stage are done; full[s] (complete before the MMAs were
                // issued) makes the activation and weight scales of the stage visible to this warp.
                if (lane == 0)
                    go = gwait_seq(&t_full[g], (it >> 1) & 1u, &full[s], (it / kStages) & 1u, abort_flag, a.err, kDevErrMmaWait);
                go = __shfl_sync(0xFFFFFFFFu, go ? 1 : 0, 0) != 0;
                if (!go) break;
                tc_fence_after();
                {
                    // 16-column chunks q = 0..3 (sub-block q >> 1, columns 16*(q & 1)), each load issued
                    // before the arithmetic of the previous chunk; the pair is released after the last load.
                    uint32_t va[16], vb[16];
                    const uint32_t tb = lane_base + (uint32_t)(g * 2 * kBN);
                    tmem_ld16(tb, va);
                    tmem_wait_ld();
                    regs_after_wait(va);
                    tmem_ld16(tb + 16u, vb);
                    drain_chunk(acc, va, 0, sw_base, sx_base, s, 0);
                    tmem_wait_ld();
                    regs_after_wait(vb);
                    tmem_ld16(tb + (uint32_t)kBN, va);
                    drain_chunk(acc, vb, 16, sw_base, sx_base, s, 0);
                    tmem_wait_ld();
                    regs_after_wait(va);
                    tmem_ld16(tb + (uint32_t)kBN + 16u, vb);
                    drain_chunk(acc, va, 0, sw_base, sx_base, s, 1);
                    tmem_wait_ld();
                    regs_after_wait(vb);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&t_empty[g]);
                    drain_chunk(acc, vb, 16, sw_base, sx_base, s, 1);
                }
                fence_generic_async_smem();  // this warp's reads of d_x and the weight scales before the refill
                __syncwarp();
                if (lane == 0) mbar_arrive(&freeb[s]);
            }
            if (!go) break;
            // Epilogue: Y[m][n] at Y + m*ldy_m + n*ldy_n.
            const int64_t n = (int64_t)row0 + r;
            if (n < a.N) {
                float* yrow = a.y + n * a.ldy_n;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int64_t m = (int64_t)m0 + 32 * cg + c;
                    if (m < a.M) yrow[m * a.ldy_m] = acc[c];
                }
            }
        }
    }

    // ---------------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kAccBufs * kBN)
                     : "memory");
    }
}

// ------------------------------------------------------------------------------------------
// Activation quantizer for the GEMM: Q8_1 semantics bit for bit (amax / sum butterflies,
// d = amax/127, q = roundf(x/d), q = 0 for an all-zero block), written as the kernel's stage blocks:
// block (tile mt, stage st) at act + (mt*S + st)*17408 holds fp16 q of tokens 128mt..128mt+127 for
// K = 64st..64st+63 in the 128-byte-swizzled K-major layout (token r, 16-byte chunk c at
// (r/8)*1024 + (r%8)*128 + ((c ^ r%8)*16)), K in the lookup order within each 32-block (element
// e = 4w+i+16j at position 8w+2i+j), then fp32 d_x[h][r] for the stage's two sub-blocks h.  Tokens
// past M (tail of the last tile) are written as zeros.  One warp per Q8_1 block.
__global__ void __launch_bounds__(256) gemm_act_quantize_kernel(const float* __restrict__ X, uint8_t* __restrict__ act,
                                                                int64_t K, int64_t M, int64_t Mpad, int64_t stride_m,
                                                                int64_t stride_k) {
    grid_dependency_wait();
    const unsigned full = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const int64_t nb = K / kQK8;
    const int64_t S = K / kBK;
    const int64_t total = nb * Mpad;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int pos = 8 * ((lane & 15) >> 2) + 2 * (lane & 3) + (lane >> 4);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total; blk += nwarps) {
        const int64_t m = blk / nb;
        const int64_t ib = blk - m * nb;
        const float x = m < M ? X[m * stride_m + (ib * kQK8 + lane) * stride_k] : 0.0f;
        float amax = fabsf(x), sum = x;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(full, amax, off));
            sum += __shfl_xor_sync(full, sum, off);
        }
        const float d = amax / 127.0f;
        int q = 0;
        if (amax != 0.0f) q = (int)roundf(x / d);
        const int64_t mt = m >> 7;
        const int r = (int)(m & 127);
        const int64_t st = ib >> 1;
        const int h = (int)(ib & 1);
        uint8_t* blkp = act + (mt * S + st) * (int64_t)kActStageBytes;
        const int p = 32 * h + pos;                       // K position within the 64-wide stage
        const int off = (r >> 3) * 1024 + (r & 7) * 128 + ((((p >> 3) ^ (r & 7))) << 4) + ((p & 7) << 1);
        *reinterpret_cast<__half*>(blkp + off) = __int2half_rn(q);
        if (lane == 0)
            *reinterpret_cast<float*>(blkp + kBBytes + h * 512 + 4 * r) = f16_bits_to_f32(f32_to_f16_trunc(d));
    }
    grid_launch_dependents();
}

// ------------------------------------------------------------------------------------------
// Host side.
namespace {
int64_t mpad_of(int64_t M) { return (M + kBN - 1) / kBN * kBN; }
}  // namespace

size_t gemm_workspace_bytes(int64_t K, int64_t M) {
    return (size_t)(mpad_of(M) / kBN) * (size_t)(K / kBK) * kActStageBytes;
}

cudaError_t launch_gemm_quantize(const float* X, void* workspace, int64_t K, int64_t M, int64_t stride_m,
                                 int64_t stride_k, cudaStream_t stream) {
    if (K % kBK != 0) return cudaErrorInvalidValue;
    const int64_t total = (K / kQK8) * mpad_of(M);
    const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
    const int64_t grid = std::min<int64_t>((total + 7) / 8, (int64_t)sms * 16);
    gemm_act_quantize_kernel<<<(unsigned)grid, 256, 0, stream>>>(X, static_cast<uint8_t*>(workspace), K, M, mpad_of(M),
                                                                 stride_m, stride_k);
    return cudaGetLastError();
}

cudaError_t launch_gemm(const uint8_t* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M, int64_t x_stride_m,
                        int64_t x_stride_k, int64_t y_stride_m, int64_t y_stride_n, void* workspace, cudaStream_t stream,
                        uint32_t* err, const uint32_t lut[4]) {
    if (K % 512 != 0 || K <= 0 || N <= 0 || M <= 0 || (reinterpret_cast<uintptr_t>(W) & 15u)) return cudaErrorInvalidValue;
    if (K > (int64_t)1 << 24 || M > (int64_t)1 << 30 || N > (int64_t)1 << 30) return cudaErrorInvalidValue;
    EncodeTiledFn2 enc = encode_fn2();
    if (!enc) return cudaErrorNotSupported;
    cudaError_t e = launch_gemm_quantize(X, workspace, K, M, x_stride_m, x_stride_k, stream);
    if (e != cudaSuccess) return e;
    CUtensorMap mw;
    const int pairs = (int)(K / 512);
    {
        const cuuint64_t dims[3] = {34, (cuuint64_t)pairs, (cuuint64_t)N};
        const cuuint64_t strides[2] = {272, (cuuint64_t)pairs * 272};
        const cuuint32_t box[3] = {34, 1, (cuuint32_t)kBM};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint8_t*>(W), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }

    GemmArgs a = {};
    a.act = static_cast<const uint8_t*>(workspace);
    a.y = Y;
    a.err = err;
    a.N = N;
    a.M = M;
    a.K = (int)K;
    a.ldy_m = y_stride_m;
    a.ldy_n = y_stride_n;
    a.tiles_n = (int)((N + kBM - 1) / kBM);
    a.tiles_m = (int)((M + kBN - 1) / kBN);
    for (int i = 0; i < 4; ++i) a.lut[i] = lut[i];
    const int64_t T = (int64_t)a.tiles_n * a.tiles_m;
    const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
    const int grid = (int)std::min<int64_t>(T, sms);

    e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_iq4xs_tc_kernel), (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_iq4xs_tc_kernel, mw, a);
}

}  // namespace iq4xs
