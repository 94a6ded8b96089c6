// gemm_i8.cu -- IQ4_XS x Q8_1 prefill GEMM on the tcgen05 tensor cores with int8 operands
// (kind::i8, s8 x s8 -> s32 in TMEM), sm_100a.  Same arithmetic contract as gemm.cu (the reference's
// stock GEMM, real_stock_dp4a_comparator.hip:375-443): the exact integer dot sumi of every
// (row, token, 32-wide sub-block), then sum over sub-blocks of (d_w*(ls-32)) * d_x * sumi in fp32.
//
//  * Operands are the int8 values themselves: the codebook values kv (-127..113) expanded from the
//    IQ4_XS nibbles, and the Q8_1 quants (-127..127) as the activation quantiser writes them.  One MMA
//    (M = 128 weight rows, N = 128 tokens, K = 32) is one whole sub-block, into its own TMEM
//    accumulator: half the MMA instructions of the fp16 kernel, half the activation bytes, and a
//    shorter weight expansion (no fp16 conversion).
//  * int32 -> fp32 without conversion instructions: every accumulator starts at the bit pattern of
//    M = 1.5 * 2^23 (the drain warps write it back with tcgen05.st right after reading), and the MMA
//    adds sumi to it as an integer (|sumi| <= 32*127*127 < 2^22), so the bits read back are the float
//    M + sumi exactly.  The drain takes t = fma(M + sumi, sw, -M*sw) = round(sumi * sw) (M*sw is exact:
//    sw = d_w*(ls-32) has at most 17 significant bits) and acc = fma(t, d_x, acc): two packed fp32
//    instructions per two elements, as in the fp16 kernel, with sw and -M*sw per TMEM lane (= weight
//    row) and d_x per column (= token).
//  * Stage = 128-wide K slice (four sub-blocks, one 128-byte swizzle atom of int8 per row).  The four
//    accumulators of a stage fill the 512 TMEM columns; they form two pairs (sub-blocks 0-1, 2-3) so
//    the MMAs of the next stage's first pair run while the drain works on the second.
//  * Weights: IQ4_XS rows as stored, 128 rows x one super-block pair (34,816 bytes) per TMA copy, as in
//    gemm.cu.  Converter warps (thread = row) expand each 128-wide K slice to int8 in the K-major
//    128-byte-swizzled layout: split codebook lookup by prmt, one IADD3 to the biased byte kv + 128
//    (no carries), one LOP3 back to the signed byte.  K order inside a sub-block is the lookup's
//    natural order (position 8w + 2i + j holds element 4w + i + 16j: word w, byte i, nibble j); the
//    activation quantiser writes the same order.
//  * Activations: quantised once per call into stage blocks of 18,432 bytes, one per (128-token tile,
//    128-wide K slice): 16 KB of int8 q in the swizzled K-major layout, then fp32 d_x [4][128].
//  * Roles, barriers, bounded waits, abort handling and TMEM release follow gemm.cu.  No cluster
//    multicast.
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
constexpr int kBK = 128;         // K per stage: four sub-blocks, one 128-byte swizzle atom of int8
constexpr int kSub = kBK / kQK8;  // 4 sub-blocks per stage
constexpr int kStages = 4;       // A / B / scale ring depth
constexpr int kRawStages = 2;    // raw weight ring depth (one super-block pair = 4 stages each)
constexpr int kConvWarps = 4;
constexpr int kDrainWarps = 16;  // 4 per TMEM lane quarter, 32 token columns each
constexpr int kFirstConvWarp = 3;                               // warps 0-2: weight TMA, MMA, act TMA
constexpr int kFirstDrainWarp = kFirstConvWarp + kConvWarps;    // 7
constexpr int kThreads = 32 * (kFirstDrainWarp + kDrainWarps);  // 736 (88 registers per thread)
constexpr int kTmemCols = kSub * kBN;                           // 512

constexpr uint32_t kRawBytes = kBM * 272;     // 34,816
constexpr uint32_t kABytes = kBM * kBK;       // 16,384
constexpr uint32_t kBBytes = kBN * kBK;       // 16,384
constexpr uint32_t kSxBytes = kSub * kBN * 4;  // 2,048: d_x [4][128]
constexpr uint32_t kSwBytes = kSub * kBM * 8;  // 4,096: {sw, -M*sw} [4][128]
constexpr uint32_t kActStageBytes = kBBytes + kSxBytes;  // 18,432

constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffB = kOffA + kStages * kABytes;
constexpr uint32_t kOffRaw = kOffB + kStages * kActStageBytes;
constexpr uint32_t kOffSw = kOffRaw + kRawStages * kRawBytes;
constexpr uint32_t kOffBar = kOffSw + kStages * kSwBytes;
constexpr int kNumBars = 2 * kRawStages + 2 * kStages + 2 * 2 + 1;
constexpr uint32_t kOffMisc = kOffBar + kNumBars * 8;  // TMEM address, abort flag
constexpr uint32_t kSmemBytes = kOffMisc + 16 + 1024;  // + slack to align the base to 1024
static_assert(kSmemBytes + 4096 <= 232448, "shared memory of the int8 GEMM");

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1),
// both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdescI8 =
    (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc) {
    // enable-input-d always set: the accumulator holds M (written by the drain) before every MMA.
    asm volatile("tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, 1;" ::"r"(d_tmem), "l"(adesc), "l"(bdesc),
                 "r"(kIdescI8)
                 : "memory");
}

// 16 consecutive columns of this warp's 32 TMEM lanes set to v.
__device__ __forceinline__ void tmem_st16_const(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
        "r"(v)
        : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void sts_f2(uint32_t addr, float a, float b) {
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

// Eight signed codebook bytes of one qs word in the lookup order: [e(4w), e(4w+16), e(4w+1),
// e(4w+17)] and [e(4w+2), e(4w+18), e(4w+3), e(4w+19)].
__device__ __forceinline__ uint2 expand_word_s8(uint32_t x, const uint32_t (&lut)[4]) {
    const uint32_t xf = x ^ 0x88888888u;
    const uint32_t lo_l = prmt(lut[0], lut[1], x), lo_h = prmt(lut[2], lut[3], xf);
    const uint32_t hi_l = prmt(lut[0], lut[1], x >> 16), hi_h = prmt(lut[2], lut[3], xf >> 16);
    // Biased bytes kv + 128 (128 - (-kv) for codes < 8, 128 + kv for codes >= 8; no carries), then the
    // sign bit of every byte flipped: kv as a two's-complement byte.
    return make_uint2((0x80808080u - lo_l + lo_h) ^ 0x80808080u, (0x80808080u - hi_l + hi_h) ^ 0x80808080u);
}
}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    gemm_iq4xs_i8_kernel(const __grid_constant__ CUtensorMap tmap_w, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* raw_full = bars;                    // weight pair landed (TMA bytes)
    uint64_t* raw_empty = raw_full + kRawStages;  // converters done with a weight pair
    uint64_t* full = raw_empty + kRawStages;      // stage: activation copy landed + 4 converter warps
    uint64_t* freeb = full + kStages;             // stage: MMAs done (commit) + drain done with its scales
    uint64_t* t_full = freeb + kStages;           // TMEM pair q (sub-blocks 2q, 2q+1): both MMAs done
    uint64_t* t_empty = t_full + 2;               // TMEM pair q: drained and reset to M
    uint64_t* mma_done = t_empty + 2;
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
        for (int i = 0; i < 2; ++i) {
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
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    // Every accumulator starts at M before the first MMA (the drain warps own all 128 x 512 cells).
    if (warp >= kFirstDrainWarp) {
        const int lq = warp & 3, cg = (warp - kFirstDrainWarp) >> 2;
        const uint32_t lb = tmem_base + ((uint32_t)(32 * lq) << 16) + (uint32_t)(32 * cg);
#pragma unroll
        for (int h = 0; h < kSub; ++h) {
            tmem_st16_const(lb + (uint32_t)(h * kBN), kMagicBits);
            tmem_st16_const(lb + (uint32_t)(h * kBN + 16), kMagicBits);
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

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
                    const uint64_t ad = smem_desc_sw128(smem_addr(smem + kOffA + s * kABytes));
                    const uint64_t bd = smem_desc_sw128(smem_addr(smem + kOffB + s * kActStageBytes));
                    // Pair q: sub-blocks 2q, 2q+1 -> accumulators at columns 128*(2q), 128*(2q+1); the K
                    // offset of sub-block h inside the swizzle atom is 32h bytes = 2h in 16-byte units.
                    for (int q = 0; q < 2 && ok; ++q) {
                        if (q == 0)
                            ok = gwait_seq(&full[s], u & 1u, &t_empty[0], (it & 1u) ^ 1u, abort_flag, a.err, kDevErrMmaWait);
                        else
                            ok = gwait(&t_empty[1], (it & 1u) ^ 1u, abort_flag, a.err, kDevErrMmaWait);
                        if (!ok) break;
                        tc_fence_after();
                        const int h0 = 2 * q;
                        tc_mma_i8(tmem_base + (uint32_t)(h0 * kBN), ad + 2 * h0, bd + 2 * h0);
                        tc_mma_i8(tmem_base + (uint32_t)((h0 + 1) * kBN), ad + 2 * (h0 + 1), bd + 2 * (h0 + 1));
                        tc_commit(&t_full[q]);
                    }
                    if (ok) tc_commit(&freeb[s]);
                }
            }
            // All issued MMAs complete before TMEM is released.
            tc_commit(mma_done);
            gdrain(mma_done, 0u, a.err);
        }
        __syncwarp();
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
                for (int sp = 0; sp < 4; ++sp, ++it) {  // 4 stages of 128 K per super-block pair
                    const int s = (int)(it % kStages);
                    const uint32_t u = it / kStages;
                    if (!(ok = gwait_fast(&freeb[s], (u & 1u) ^ 1u, abort_flag, a.err, kDevErrEmptyWait))) break;
                    const uint32_t sbp = rowp + (uint32_t)(sp >> 1) * 136u;  // super-block of this stage
                    const uint2 hdr = lds_u2(sbp);
                    const float dw = f16_bits_to_f32(hdr.x);
                    const int ib0 = 4 * (sp & 1);  // first sub-block of the stage within the super-block
                    const uint32_t swa = smem_addr(smem + kOffSw + s * kSwBytes) + 8u * (uint32_t)r;
#pragma unroll
                    for (int h = 0; h < kSub; ++h) {
                        const float sw = dw * (float)(subblock_scale(hdr.x, hdr.y, ib0 + h) - 32);
                        sts_f2(swa + (uint32_t)(h * kBM * 8), sw, -kMagicF * sw);
                    }
                    const uint32_t qp = sbp + 8u + 64u * (uint32_t)(sp & 1);
                    const uint32_t arow = smem_addr(smem + kOffA + s * kABytes) + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = words 2c, 2c+1 of the stage's 64 qs bytes
                        const uint2 v = lds_u2(qp + 8u * c);
                        const uint2 e0 = expand_word_s8(v.x, lut), e1 = expand_word_s8(v.y, lut);
                        sts_u4(arow + (uint32_t)((c ^ (r & 7)) << 4), make_uint4(e0.x, e0.y, e1.x, e1.y));
                    }
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
        const int dw = warp - kFirstDrainWarp;  // 0..15
        const int lq = warp & 3;                // TMEM lane quarter this warp may access (warp id % 4)
        const int cg = dw >> 2;                 // token columns 32*cg .. 32*cg+31 (the four warps of a
                                                // lane quarter have dw = 4k + const: distinct cg)
        const int r = 32 * lq + lane;           // tile row = TMEM lane
        const uint32_t lane_base = tmem_base + ((uint32_t)(32 * lq) << 16) + (uint32_t)(32 * cg);
        const uint32_t sw_base = smem_addr(smem + kOffSw) + 8u * (uint32_t)r;
        const uint32_t sx_base = smem_addr(smem + kOffB + kBBytes) + 4u * (uint32_t)(32 * cg);
        uint32_t it = 0;
        bool go = true;
        for (int64_t t = blockIdx.x; t < T && go; t += gridDim.x) {
            const int row0 = (int)(t / tiles_m) * kBM;
            const int m0 = (int)(t % tiles_m) * kBN;
            float acc[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
            for (int st = 0; st < S && go; ++st, ++it) {
                const int s = (int)(it % kStages);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    // t_full[q]: both MMAs of the pair are done; full[s] (complete before they were issued)
                    // makes the stage's weight scales and d_x visible to this warp.
                    if (lane == 0) {
                        go = q == 0 ? gwait_seq(&t_full[0], it & 1u, &full[s], (it / kStages) & 1u, abort_flag, a.err,
                                                kDevErrMmaWait)
                                    : gwait(&t_full[1], it & 1u, abort_flag, a.err, kDevErrMmaWait);
                    }
                    go = __shfl_sync(0xFFFFFFFFu, go ? 1 : 0, 0) != 0;
                    if (!go) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int hh = 0; hh < 2; ++hh) {
                        const int h = 2 * q + hh;
                        const uint32_t ta = lane_base + (uint32_t)(h * kBN);
                        const float2 swp = lds_f2(sw_base + (uint32_t)(s * kSwBytes + h * kBM * 8));
                        const uint32_t sxa = sx_base + (uint32_t)(s * kActStageBytes + h * kBN * 4);
                        // Four quarters of 8 columns (8 live accumulator registers at a time); the cells are
                        // reset to M once all 32 columns are in registers.
#pragma unroll
                        for (int qt = 0; qt < 4; ++qt) {
                            uint32_t v[8];
                            tmem_ld8(ta + (uint32_t)(8 * qt), v);
                            tmem_wait_ld();
                            if (qt == 3) {
                                tmem_st16_const(ta, kMagicBits);
                                tmem_st16_const(ta + 16, kMagicBits);
                                if (hh == 1) {
                                    tmem_wait_st();
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(&t_empty[q]);
                                }
                            }
#pragma unroll
                            for (int c4 = 0; c4 < 2; ++c4) {
                                const int c = 8 * qt + 4 * c4;
                                const uint4 x = lds_u4(sxa + 4u * (uint32_t)c);
                                float t0, t1, t2, t3;
                                fma2c(t0, t1, __uint_as_float(v[4 * c4 + 0]), __uint_as_float(v[4 * c4 + 1]), swp.x, swp.x,
                                      swp.y, swp.y);
                                fma2c(t2, t3, __uint_as_float(v[4 * c4 + 2]), __uint_as_float(v[4 * c4 + 3]), swp.x, swp.x,
                                      swp.y, swp.y);
                                fma2(acc[c + 0], acc[c + 1], t0, t1, __uint_as_float(x.x), __uint_as_float(x.y));
                                fma2(acc[c + 2], acc[c + 3], t2, t3, __uint_as_float(x.z), __uint_as_float(x.w));
                            }
                        }
                    }
                }
                if (!go) break;
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                     : "memory");
    }
}

// ------------------------------------------------------------------------------------------
// Activation quantiser for the int8 GEMM: Q8_1 semantics bit for bit (the same amax / sum
// butterflies, d = amax/127, q = roundf(x/d), q = 0 for an all-zero block as the fp16 GEMM's
// quantiser), written as stage blocks: block (tile mt, stage st) at act + (mt*S + st)*18432 holds the
// int8 q of tokens 128mt..128mt+127 for K = 128st..128st+127 in the 128-byte-swizzled K-major layout
// (token r, 16-byte chunk c at (r/8)*1024 + (r%8)*128 + ((c ^ r%8)*16)), K in the lookup order within
// each 32-block (element e = 4w+i+16j at position 8w+2i+j), then fp32 d_x[h][r] for the stage's four
// sub-blocks h.  Tokens past M are written as zeros.  One warp per Q8_1 block.
__global__ void __launch_bounds__(256) gemm_i8_act_quantize_kernel(const float* __restrict__ X, uint8_t* __restrict__ act,
                                                                   int64_t K, int64_t M, int64_t Mpad, int64_t stride_m,
                                                                   int64_t stride_k) {
    grid_dependency_wait();
    const unsigned fullm = 0xFFFFFFFFu;
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
            amax = fmaxf(amax, __shfl_xor_sync(fullm, amax, off));
            sum += __shfl_xor_sync(fullm, sum, off);
        }
        const float d = amax / 127.0f;
        int q = 0;
        if (amax != 0.0f) q = (int)roundf(x / d);
        const int64_t mt = m >> 7;
        const int r = (int)(m & 127);
        const int64_t st = ib / kSub;
        const int h = (int)(ib % kSub);
        uint8_t* blkp = act + (mt * S + st) * (int64_t)kActStageBytes;
        const int p = 32 * h + pos;  // K position within the 128-wide stage
        const int off = (r >> 3) * 1024 + (r & 7) * 128 + ((((p >> 4) ^ (r & 7))) << 4) + (p & 15);
        blkp[off] = (uint8_t)(int8_t)q;
        if (lane == 0)
            *reinterpret_cast<float*>(blkp + kBBytes + h * (kBN * 4) + 4 * r) = f16_bits_to_f32(f32_to_f16_trunc(d));
    }
    grid_launch_dependents();
}

// ------------------------------------------------------------------------------------------
// Host side.
namespace {
int64_t mpad_i8(int64_t M) { return (M + kBN - 1) / kBN * kBN; }
}  // namespace

size_t gemm_i8_workspace_bytes(int64_t K, int64_t M) {
    return (size_t)(mpad_i8(M) / kBN) * (size_t)(K / kBK) * kActStageBytes;
}

cudaError_t launch_gemm_i8_quantize(const float* X, void* workspace, int64_t K, int64_t M, int64_t stride_m,
                                    int64_t stride_k, cudaStream_t stream) {
    if (K % kBK != 0) return cudaErrorInvalidValue;
    const int64_t total = (K / kQK8) * mpad_i8(M);
    const int sms = device_sm_count() > 0 ? device_sm_count() : 148;
    const int64_t grid = std::min<int64_t>((total + 7) / 8, (int64_t)sms * 16);
    gemm_i8_act_quantize_kernel<<<(unsigned)grid, 256, 0, stream>>>(X, static_cast<uint8_t*>(workspace), K, M,
                                                                    mpad_i8(M), stride_m, stride_k);
    return cudaGetLastError();
}

cudaError_t launch_gemm_i8(const uint8_t* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M,
                           int64_t x_stride_m, int64_t x_stride_k, int64_t y_stride_m, int64_t y_stride_n,
                           void* workspace, cudaStream_t stream, uint32_t* err, const uint32_t lut[4]) {
    if (K % 512 != 0 || K <= 0 || N <= 0 || M <= 0 || (reinterpret_cast<uintptr_t>(W) & 15u)) return cudaErrorInvalidValue;
    if (K > (int64_t)1 << 24 || M > (int64_t)1 << 30 || N > (int64_t)1 << 30) return cudaErrorInvalidValue;
    EncodeTiledFn2 enc = encode_fn2();
    if (!enc) return cudaErrorNotSupported;
    cudaError_t e = launch_gemm_i8_quantize(X, workspace, K, M, x_stride_m, x_stride_k, stream);
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

    e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_iq4xs_i8_kernel), (int)kSmemBytes);
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
    return cudaLaunchKernelEx(&cfg, gemm_iq4xs_i8_kernel, mw, a);
}

}  // namespace iq4xs
