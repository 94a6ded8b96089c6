// gemv_mma.cu -- IQ4_XS x Q8_1 decode GEMV for batch 2..8 on the tensor cores (mma.sync m16n8k32 s8).
//
// Same arithmetic contract as the dp4a GEMV (real_stock_dp4a_comparator.hip:145-166 per sub-block):
// the int32 dot of one 32-weight sub-block with one Q8_1 block is exact, then
// term = (d_w*(ls-32)) * d_x * sumi in fp32, summed over sub-blocks.
//
//  * The weight matrix is viewed as a 2-D tensor of uint64 [N rows][34 * K/512] (one super-block
//    pair = 272 bytes) and staged by TMA (cp.async.bulk.tensor.2d, no multicast) in units of
//    16 rows x `pk` pairs (one box: 16 rows of pk*272 bytes).  pk is odd, so the shared-memory row pitch pk*272 bytes = 68*pk words is an
//    odd multiple of 4 words: the 8 rows of an MMA fragment load hit 8 disjoint 4-bank groups.
//    Rows and pairs past the matrix are zero-filled by TMA and never read from memory.
//  * Work unit = (16-row tile, K part of pk pairs), ordered part-major and split in balanced
//    contiguous ranges over one CTA per SM.  With more than one part, the parts leave partial sums in
//    the workspace (plain stores) and a small follow-on kernel adds them in part order
//    (deterministic); a fence + ticket per unit to combine in-kernel cost ~11 us on a 95 MB matrix.
//  * Lookup: the two split-table prmt lookups (tables -kv[0..7] and kv[8..15], zero elsewhere) feed
//    one s8 x s8 MMA each (no merge on the integer pipe, which is the busiest one); both accumulators
//    start at the bit pattern of 1.5*2^23, so the two sums are read as floats and one packed fp32
//    subtraction gives the exact int32 sub-block dot sumi as an fp32 value.
//  * A unit is processed by a pair of consumer warps (8 pairs per CTA, units it = pair, pair+8, ...
//    over a stage ring sized to shared memory); the two warps split the unit's super-blocks (even /
//    odd) and add their partial sums through the stage buffer once both are done reading it (half 0
//    + half 1, a fixed order).  Lane (g = lane/4, c = lane%4) holds A = qs word c of each sub-block
//    for rows g and g+8 (looked up as above); B = the 8 tokens' Q8_1 values of the sub-block in the
//    lookup's k order (staged once per part in shared memory).  The weight scales d*(ls-32) of a
//    super-block are computed once by the four lanes of a row group and fetched by shuffle; the fp32
//    update (d_w*(ls-32)*d_x)*sumi is one packed multiply and one packed fused add per two outputs.
//  * Every mbarrier wait is bounded (sleeping try_wait, error word, drain before exit).
#include <cuda.h>

#include <algorithm>
#include <cstring>

#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

namespace {
constexpr int kMaxMmaStages = 16;  // stage ring depth: as many as fit, at least one per consumer warp
constexpr int kPairs = 8;          // consumer warp pairs: one unit (tile x part) per pair at a time
                                   // (measured on B200: 6 and 10 pairs are slower)
constexpr int kNCW = 2 * kPairs;   // consumer warps; the two warps of a pair split the unit's super-blocks

struct MmaSmem {
    uint32_t bar_off, flag_off, act_off, dx_off, scr_off, ring_off, total;
};

constexpr int kStageChunk = 8;                      // Q8_1 blocks per coalesced staging chunk
constexpr int kF32MaxPkB = 12;  // fp32 sources are quantised in the kernel while pk * B <= this
                                // (= the chunks a warp holds in registers while staging, see below)
constexpr int kChunkWords = kStageChunk * kQ8Bytes / 4;  // 72

// act: per staged part (up to 2) and sub-block: 32 lanes x uint2 (B fragment words) = 256 B;
// dx: per sub-block, d_x of the 8 tokens (32 B);
// scr: per consumer warp, one chunk of 8 raw Q8_1 blocks (288 B) while staging;
// ring: `stages` x (16 rows x pk pairs x 272 B).
__host__ __device__ inline MmaSmem mma_smem(int pk, int stages) {
    MmaSmem L;
    L.bar_off = 0;
    L.flag_off = 2 * kMaxMmaStages * 8;
    L.act_off = 384;
    L.dx_off = L.act_off + 2u * (uint32_t)pk * 16 * 256;
    L.scr_off = L.dx_off + 2u * (uint32_t)pk * 16 * 32;
    L.ring_off = (L.scr_off + (uint32_t)kNCW * kChunkWords * 4 + 127) & ~127u;
    L.total = L.ring_off + (uint32_t)stages * 16u * (uint32_t)pk * 272u;
    return L;
}

// Staged activations of sub-block sb (counted over both part slots) in shared memory, by pairs of
// sub-blocks: lane L's B-fragment words of sub-blocks 2m and 2m+1 are adjacent (one 16-byte load),
// and so are the d_x of tokens 2c, 2c+1 of both (one 16-byte load for lane column c).
__device__ __forceinline__ int act_index(int sb, int L) { return ((sb >> 1) * 32 + L) * 2 + (sb & 1); }  // uint2
__device__ __forceinline__ int dx_index(int sb, int n) {                                                // float
    return ((sb >> 1) * 4 + (n >> 1)) * 4 + (sb & 1) * 2 + (n & 1);
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Packed fp32 pairs, one instruction each on sm_100 (float2 builtins: the register allocator places
// the pairs, where inline asm packing two scalars into a .b64 operand costs register moves).
// (d0, d1) += (a0, a1) * (b0, b1)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(d0, d1));
    d0 = r.x;
    d1 = r.y;
}

// (d0, d1) = (a0, a1) - (b0, b1)  (a - b == a + (-b) exactly)
__device__ __forceinline__ void sub2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    const float2 r = __fadd2_rn(make_float2(a0, a1), make_float2(-b0, -b1));
    d0 = r.x;
    d1 = r.y;
}

// int32 -> fp32 without conversion instructions: MMA accumulators that start at kMagicI (the bit
// pattern of 1.5 * 2^23) end as the bit pattern of the float 1.5 * 2^23 + s, exact while
// |s| < 2^22 (a half-table sub-block dot is at most 32 * 127 * 127 = 516128 in magnitude).
constexpr int kMagicI = 0x4B400000;

// (d0, d1) = (a0, a1) * (b0, b1)
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    const float2 r = __fmul2_rn(make_float2(a0, a1), make_float2(b0, b1));
    d0 = r.x;
    d1 = r.y;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// d = a*b + (c, c, c, c): every accumulator starts at the same value c.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c));
}

// Upper 16 selector bits: a plain shift (mul.hi.u32 issues at a quarter of the rate, measured slower).
__device__ __forceinline__ uint32_t hi16(uint32_t x) {
    return x >> 16;
}

__device__ __forceinline__ bool wait_sleep(uint64_t* bar, uint32_t parity, volatile uint32_t* flag, uint32_t* err,
                                           uint32_t code) {
    for (uint32_t i = 0; i < 20000u; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (*flag) return false;
    }
    record_error(err, code);
    *flag = 1u;
    return false;
}
}  // namespace

// kF32: the activations are quantised from fp32 while staging (batch <= 2 and small parts); the
// Q8_1-input instances do not carry that code.
// The kernel body for CTA `cta` of the `ncta` CTAs that share the matrix; `tmap` is a kernel-parameter
// tensor map (the single-matrix kernel's own, or one of the grouped kernel's).
template <int B, bool kDebug, bool kF32>
__device__ __forceinline__ void gemv_mma_body(const CUtensorMap* tmap_p, const GemvMmaArgs& a, int cta, int ncta,
                                              uint8_t* smem) {
    const CUtensorMap& tmap = *tmap_p;
    const int pk = a.pk, P = a.parts, S = a.stages;
    const MmaSmem L = mma_smem(pk, S);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + kMaxMmaStages;
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.flag_off);
    uint8_t* ring = smem + L.ring_off;
    const uint32_t stage_bytes = 16u * (uint32_t)pk * 272u;
    const uint32_t row_pitch = (uint32_t)pk * 272u;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t T = (a.N + 15) / 16;
    const int64_t U = T * P;
    const int64_t u0 = U * cta / ncta, u1 = U * (cta + 1) / ncta;
    const int nunits = (int)(u1 - u0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        *abort_flag = 0u;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            int it = 0;
            for (; it < nunits; ++it) {
                const int s = it % S;
                const uint32_t use = (uint32_t)(it / S);
                if (use > 0 && !wait_sleep(&empty[s], (use - 1) & 1u, abort_flag, a.err, kDevErrEmptyWait)) break;
                const int64_t u = u0 + it;
                const int p = (int)(u / T);
                const int64_t t = u - (int64_t)p * T;
                fence_generic_async_smem();  // the consumers' ld.shared of this stage come first
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                tma_load_2d(ring + (size_t)s * stage_bytes, &tmap, p * pk * 34, (int)(t * 16), &full[s], policy);
            }
            const int first = it > S ? it - S : 0;
            for (int j = first; j < it; ++j) {
                bool landed = false;
                for (uint32_t i = 0; i < 20000u && !landed; ++i)
                    landed = mbar_try_wait_sleep(&full[j % S], (uint32_t)(j / S) & 1u, 1000000u);
                if (!landed) record_error(a.err, kDevErrDrainWait);
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int cw = warp - 1;
    const int g = lane >> 2, c = lane & 3;
    const int ctid = threadIdx.x - 32, nct = kNCW * 32;
    const int nsb = a.K / kQK8;
    const uint2* act = reinterpret_cast<const uint2*>(smem + L.act_off);
    const float* dxs = reinterpret_cast<const float*>(smem + L.dx_off);

    // Stage the activations of the (at most two) parts this CTA touches as MMA B fragments in the
    // lookup's k order: slot = part - first part.
    grid_dependency_wait();
    const int pfirst = nunits > 0 ? (int)(u0 / T) : 0;
    const int plast = nunits > 0 ? (int)((u1 - 1) / T) : -1;
    {
        // One warp per chunk of 8 consecutive Q8_1 blocks of one token (288 contiguous bytes): three
        // coalesced word loads into the warp's scratch, then lane (b, j) = (lane/4, lane%4) builds
        // B-fragment word pair j of block b and lane (b, 0) its d_x.  Tokens >= B stay zero.
        const int nslot = min(plast - pfirst + 1, 2);
        int nsubs[2] = {0, 0};
        for (int sl = 0; sl < nslot; ++sl) nsubs[sl] = 16 * min(pk, a.pairs - (pfirst + sl) * pk);
        uint32_t* scr = reinterpret_cast<uint32_t*>(smem + L.scr_off) + cw * kChunkWords;
        uint2* actw = reinterpret_cast<uint2*>(smem + L.act_off);
        float* dxw = reinterpret_cast<float*>(smem + L.dx_off);
        const int ch0 = nsubs[0] / kStageChunk, ch1 = nsubs[1] / kStageChunk;  // chunks per token
        const int nchunks = (ch0 + ch1) * B;
        // fp32 source (batch <= 2): the fp32 values of all of this warp's chunks are requested first
        constexpr int kF32Chunks = (4 * kF32MaxPkB + kNCW - 1) / kNCW;  // 2 slots * (16 pk / 8) * B / kNCW
        float4 xf[kF32Chunks][2];
        if constexpr (kF32) {
#pragma unroll
            for (int k = 0; k < kF32Chunks; ++k) {
                const int q = cw + k * kNCW;
                xf[k][0] = xf[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (q < nchunks) {
                    const int n = q % B, r = q / B;
                    const int slot = r < ch0 ? 0 : 1;
                    const int sb = (pfirst + slot) * pk * 16 + (r - slot * ch0) * kStageChunk;
                    const float4* xs = reinterpret_cast<const float4*>(a.act.x + (int64_t)n * a.K + (int64_t)sb * kQK8) + lane;
                    xf[k][0] = __ldg(xs);
                    xf[k][1] = __ldg(xs + 32);
                }
            }
        }
        // chunk q -> token n, staged part slot, first sub-block (local and global)
        auto chunk_pos = [&](int q, int& n, int& slot, int& sbl0, int& sb) {
            n = q % B;
            const int r = q / B;
            slot = r < ch0 ? 0 : 1;
            sbl0 = (r - slot * ch0) * kStageChunk;
            sb = (pfirst + slot) * pk * 16 + sbl0;
        };
        // the chunk in the warp's scratch -> B-fragment words and d_x of its 8 blocks
        auto chunk_build = [&](int n, int slot, int sbl0) {
            __syncwarp();
            const int bq = lane >> 2, j = lane & 3;
            const uint32_t* blk = scr + bq * (kQ8Bytes / 4);
            const int sbl = sbl0 + bq;
            actw[act_index(slot * pk * 16 + sbl, n * 4 + j)] =
                make_uint2(act_perm_lo(blk[1 + j], blk[5 + j]), act_perm_hi(blk[1 + j], blk[5 + j]));
            if (j == 0) dxw[dx_index(slot * pk * 16 + sbl, n)] = f16_bits_to_f32(blk[0]);
            __syncwarp();
        };
        if constexpr (kF32) {
            for (int q = cw, kq = 0; q < nchunks; q += kNCW, ++kq) {
                int n, slot, sbl0, sb;
                chunk_pos(q, n, slot, sbl0, sb);
                // quantise the chunk's 8 blocks from fp32 into the scratch
                float4 x0 = xf[0][0], x1 = xf[0][1];
#pragma unroll
                for (int k = 1; k < kF32Chunks; ++k)
                    if (kq == k) {
                        x0 = xf[k][0];
                        x1 = xf[k][1];
                    }
                q8_1_quad_store(x0, reinterpret_cast<uint8_t*>(scr), lane);
                q8_1_quad_store(x1, reinterpret_cast<uint8_t*>(scr) + 4 * kQ8Bytes, lane);
                chunk_build(n, slot, sbl0);
            }
        } else {
            // Q8_1 source: the words of all of this warp's chunks (at most kQ8Pre) are loaded before
            // any is used, so the staging costs one global round trip instead of one per chunk.
            constexpr int kQ8Pre = (4 * 5 * 8 + kNCW - 1) / kNCW;  // 2 slots * (16 pk / 8) * B / kNCW, pk <= 5, B <= 8
            uint32_t pv[kQ8Pre][3];
#pragma unroll
            for (int k = 0; k < kQ8Pre; ++k) {
                const int q = cw + k * kNCW;
                pv[k][0] = pv[k][1] = pv[k][2] = 0u;
                if (q < nchunks) {
                    int n, slot, sbl0, sb;
                    chunk_pos(q, n, slot, sbl0, sb);
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.q8 + ((int64_t)n * nsb + sb) * kQ8Bytes);
                    pv[k][0] = __ldg(src + lane);
                    pv[k][1] = __ldg(src + 32 + lane);
                    if (lane < kChunkWords - 64) pv[k][2] = __ldg(src + 64 + lane);
                }
            }
#pragma unroll
            for (int k = 0; k < kQ8Pre; ++k) {
                const int q = cw + k * kNCW;
                if (q >= nchunks) break;
                int n, slot, sbl0, sb;
                chunk_pos(q, n, slot, sbl0, sb);
                scr[lane] = pv[k][0];
                scr[32 + lane] = pv[k][1];
                if (lane < kChunkWords - 64) scr[64 + lane] = pv[k][2];
                chunk_build(n, slot, sbl0);
            }
            for (int q = cw + kQ8Pre * kNCW; q < nchunks; q += kNCW) {  // not reached for pk <= 5, B <= 8
                int n, slot, sbl0, sb;
                chunk_pos(q, n, slot, sbl0, sb);
                const uint32_t* src = reinterpret_cast<const uint32_t*>(a.q8 + ((int64_t)n * nsb + sb) * kQ8Bytes);
                scr[lane] = __ldg(src + lane);
                scr[32 + lane] = __ldg(src + 32 + lane);
                if (lane < kChunkWords - 64) scr[64 + lane] = __ldg(src + 64 + lane);
                chunk_build(n, slot, sbl0);
            }
        }
        if constexpr (B < 8) {
            const int zitems = (nsubs[0] + nsubs[1]) * (8 - B);
            for (int e = ctid; e < zitems; e += nct) {
                const int n = B + e % (8 - B), sbg = e / (8 - B);
                const int slot = sbg < nsubs[0] ? 0 : 1;
                const int sbl = sbg - slot * nsubs[0];
#pragma unroll
                for (int j = 0; j < 4; ++j) actw[act_index(slot * pk * 16 + sbl, n * 4 + j)] = make_uint2(0u, 0u);
                dxw[dx_index(slot * pk * 16 + sbl, n)] = 0.0f;
            }
        }
    }
    named_barrier(kPairs + 1, nct);
    grid_launch_dependents();  // the workspace activations are no longer read

    // Pair pr = cw/2 owns units it = pr, pr + 8, ... of this CTA (16 rows x the part's sub-blocks);
    // warp half hf = cw%2 of the pair takes super-blocks hf, hf+2, ... and the two partial sums are
    // added through the unit's stage buffer once both warps are done reading it.
    const int pr = cw >> 1, hf = cw & 1;
    for (int it = pr; it < nunits; it += kPairs) {
        const int s = it % S;
        const int64_t u = u0 + it;
        const int p = (int)(u / T);
        const int64_t t = u - (int64_t)p * T;
        const int nsup = 2 * min(pk, a.pairs - p * pk);
        const int slot = p - pfirst;
        bool ready = !*abort_flag && wait_sleep(&full[s], (uint32_t)(it / S) & 1u, abort_flag, a.err, kDevErrFullWait);
        ready = __all_sync(0xFFFFFFFFu, ready);  // mma.sync and the shuffles below need the whole warp
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (ready) {
            const uint8_t* rg = ring + (size_t)s * stage_bytes + (size_t)g * row_pitch;
            const uint8_t* rg8 = rg + 8 * row_pitch;
            const int sbs = slot * pk * 16;  // this part's first staged sub-block (even)
            for (int j = hf; j < nsup; j += 2) {
                const uint8_t* b0p = rg + j * kBlockBytes;
                const uint8_t* b8p = rg8 + j * kBlockBytes;
                const uint2 h0 = *reinterpret_cast<const uint2*>(b0p);
                const uint2 h8 = *reinterpret_cast<const uint2*>(b8p);
                // Lane (g, c) computes the weight scale d*(ls-32) of rows g and g+8 for sub-blocks 2c
                // and 2c+1; the sub-block loop fetches the one it needs from lane 4g + ib/2.
                float fq0[2], fq8[2];
                uint4 bf2 = make_uint4(0u, 0u, 0u, 0u);
                float4 dx2 = make_float4(0.f, 0.f, 0.f, 0.f);
                {
                    const float dw0 = f16_bits_to_f32(h0.x), dw8 = f16_bits_to_f32(h8.x);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int ib = 2 * c + e;
                        const int ls0 = (int)(((h0.y >> (4 * ib)) & 0xFu) | ((h0.x >> (12 + 2 * ib)) & 0x30u));
                        const int ls8 = (int)(((h8.y >> (4 * ib)) & 0xFu) | ((h8.x >> (12 + 2 * ib)) & 0x30u));
                        fq0[e] = dw0 * (float)(ls0 - 32);
                        fq8[e] = dw8 * (float)(ls8 - 32);
                    }
                }
#pragma unroll
                for (int ib = 0; ib < 8; ++ib) {
                    const int sbl = j * 8 + ib;
                    const uint32_t x0 = *reinterpret_cast<const uint32_t*>(b0p + 8 + 16 * ib + 4 * c);
                    const uint32_t x8 = *reinterpret_cast<const uint32_t*>(b8p + 8 + 16 * ib + 4 * c);
                    if ((ib & 1) == 0) {  // the B fragments and d_x of sub-blocks ib, ib+1: two 16-byte loads
                        bf2 = *reinterpret_cast<const uint4*>(act + act_index(sbs + sbl, lane));
                        dx2 = *reinterpret_cast<const float4*>(dxs + dx_index(sbs + sbl, 2 * c));
                    }
                    const uint2 bf = (ib & 1) ? make_uint2(bf2.z, bf2.w) : make_uint2(bf2.x, bf2.y);
                    const float2 dx = (ib & 1) ? make_float2(dx2.z, dx2.w) : make_float2(dx2.x, dx2.y);
                    const uint32_t xf0 = x0 ^ 0x88888888u, xf8 = x8 ^ 0x88888888u;
                    // Codebook bytes of the two table halves: ah = kv (codes >= 8, else 0), al = -kv (codes
                    // < 8, else 0), so kv = ah - al.  Two s8 x s8 MMAs (both accumulators starting at
                    // kMagicI) give 1.5*2^23 + sum(ah*a) and 1.5*2^23 + sum(al*a) as float bit patterns, and
                    // their fp32 difference is sumi exactly (both lie in [2^23, 2^24): Sterbenz).
                    const uint32_t ah[4] = {prmt(a.lut[2], a.lut[3], xf0), prmt(a.lut[2], a.lut[3], xf8),
                                            prmt(a.lut[2], a.lut[3], hi16(xf0)), prmt(a.lut[2], a.lut[3], hi16(xf8))};
                    const uint32_t al[4] = {prmt(a.lut[0], a.lut[1], x0), prmt(a.lut[0], a.lut[1], x8),
                                            prmt(a.lut[0], a.lut[1], hi16(x0)), prmt(a.lut[0], a.lut[1], hi16(x8))};
                    int dd[4], dl[4];
                    mma_s8(dd, ah, bf.x, bf.y, kMagicI);
                    mma_s8(dl, al, bf.x, bf.y, kMagicI);
                    const float f0 = __shfl_sync(0xFFFFFFFFu, fq0[ib & 1], 4 * g + (ib >> 1));
                    const float f8 = __shfl_sync(0xFFFFFFFFu, fq8[ib & 1], 4 * g + (ib >> 1));
                    if constexpr (kDebug) {
                        const int s0 = dd[0] - dl[0], s1 = dd[1] - dl[1], s2 = dd[2] - dl[2], s3 = dd[3] - dl[3];
                        const int64_t r0w = t * 16 + g, r8w = r0w + 8;
                        const int sbg = p * pk * 16 + sbl;
                        if (2 * c < B && r0w < a.N) a.sumi[((int64_t)(2 * c) * a.N + r0w) * nsb + sbg] = s0;
                        if (2 * c + 1 < B && r0w < a.N) a.sumi[((int64_t)(2 * c + 1) * a.N + r0w) * nsb + sbg] = s1;
                        if (2 * c < B && r8w < a.N) a.sumi[((int64_t)(2 * c) * a.N + r8w) * nsb + sbg] = s2;
                        if (2 * c + 1 < B && r8w < a.N) a.sumi[((int64_t)(2 * c + 1) * a.N + r8w) * nsb + sbg] = s3;
                    }
                    // acc += (f * dx) * sumi, as one rounding of the product f*dx and one fused add.
                    float c0, c1, c2, c3, v0, v1, v2, v3;
                    sub2(v0, v1, __int_as_float(dd[0]), __int_as_float(dd[1]), __int_as_float(dl[0]), __int_as_float(dl[1]));
                    sub2(v2, v3, __int_as_float(dd[2]), __int_as_float(dd[3]), __int_as_float(dl[2]), __int_as_float(dl[3]));
                    mul2(c0, c1, f0, f0, dx.x, dx.y);
                    mul2(c2, c3, f8, f8, dx.x, dx.y);
                    fma2(acc[0], acc[1], c0, c1, v0, v1);
                    fma2(acc[2], acc[3], c2, c3, v2, v3);
                }
            }
        }
        // Both warps of the pair are done with the weights: half 1 parks its sums in the stage buffer,
        // half 0 adds them (fixed order: half 0 + half 1) and releases the stage.
        float* park = reinterpret_cast<float*>(ring + (size_t)s * stage_bytes) + 4 * lane;
        named_barrier(1 + pr, 64);
        if (hf == 1) {
            park[0] = acc[0];
            park[1] = acc[1];
            park[2] = acc[2];
            park[3] = acc[3];
            fence_proxy_async_shared();  // generic writes before the stage's next TMA fill
        }
        named_barrier(1 + pr, 64);
        if (hf == 1) continue;
        acc[0] += park[0];
        acc[1] += park[1];
        acc[2] += park[2];
        acc[3] += park[3];
        fence_generic_async_smem();  // the reads of the stage (weights, parked sums) before its refill
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        const int64_t r0w = t * 16 + g, r8w = r0w + 8;
        const int tk[4] = {2 * c, 2 * c + 1, 2 * c, 2 * c + 1};
        const int64_t rw[4] = {r0w, r0w, r8w, r8w};
        if (ready && a.y) {
            if (P == 1) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (tk[k] < B && rw[k] < a.N) a.y[(int64_t)tk[k] * a.N + rw[k]] = acc[k];
            } else {
                // Partial sums of this part, plain stores; reduce_parts_kernel adds the parts in order.
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (tk[k] < B && rw[k] < a.N) a.partial[((int64_t)p * B + tk[k]) * a.N + rw[k]] = acc[k];
            }
        }
    }
}

template <int B, bool kDebug, bool kF32>
__global__ void __launch_bounds__(32 * (kNCW + 1), 1)
    gemv_iq4xs_q8_mma_kernel(const __grid_constant__ CUtensorMap tmap, const GemvMmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    gemv_mma_body<B, kDebug, kF32>(&tmap, a, (int)blockIdx.x, (int)gridDim.x, smem);
}

// Grouped tensor-core kernel: block b belongs to matrix p with cta0[p] <= b < cta0[p+1] and runs the
// body on that matrix (its own tensor map, part size, ring depth); Q8_1 activations from global memory.
struct GroupMmaParams {
    CUtensorMap maps[kMaxGroup];
    GemvMmaArgs args[kMaxGroup];
    int cta0[kMaxGroup + 1];
    int count;
};

template <int B>
__global__ void __launch_bounds__(32 * (kNCW + 1), 1) gemv_mma_grouped_kernel(const __grid_constant__ GroupMmaParams G) {
    extern __shared__ __align__(128) uint8_t smem[];
    int p = 0;
    while (p + 1 < G.count && (int)blockIdx.x >= G.cta0[p + 1]) ++p;
    const GemvMmaArgs a = G.args[p];
    gemv_mma_body<B, false, false>(&G.maps[p], a, (int)blockIdx.x - G.cta0[p], G.cta0[p + 1] - G.cta0[p], smem);
}

// y[b][n] = sum over parts p (in part order) of partial[p][b][n].  Launched after the GEMV with
// programmatic serialization: griddepcontrol.wait returns once the GEMV grid has finished and its
// stores are visible, so the GEMV needs no fences or tickets of its own.
__global__ void __launch_bounds__(256) reduce_parts_kernel(const float* __restrict__ partial, float* __restrict__ y,
                                                          int P, int64_t BN) {
    grid_dependency_wait();
    grid_launch_dependents();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < BN; i += (int64_t)gridDim.x * blockDim.x) {
        // four parts' loads in flight before they are added (in part order)
        float sum = 0.0f;
        int q = 0;
        for (; q + 4 <= P; q += 4) {
            const float v0 = partial[(int64_t)q * BN + i], v1 = partial[(int64_t)(q + 1) * BN + i];
            const float v2 = partial[(int64_t)(q + 2) * BN + i], v3 = partial[(int64_t)(q + 3) * BN + i];
            sum = (((sum + v0) + v1) + v2) + v3;
        }
        for (; q < P; ++q) sum += partial[(int64_t)q * BN + i];
        y[i] = sum;
    }
}

// --------------------------------------------------------------------------------------------
// Host side: tensor map, part choice, launch.
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    // Function-local static: initialised once, thread-safe when several host threads launch at once.
    static const EncodeTiledFn fn = []() -> EncodeTiledFn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return nullptr;
    }();
    return fn;
}

// Stage ring depth for part size pk: as many 16-row stages as fit next to the activations (<= 16).
// (4 KB of the per-block limit stay free: tools that instrument kernels reserve some of it.)
int mma_stages(int pk, int smem_optin) {
    const int budget = smem_optin - 4096;
    int st = kMaxMmaStages;
    while (st > kPairs && (int)mma_smem(pk, st).total > budget) --st;
    return st;
}

// Part size: odd number of pairs pk <= 5 (odd: conflict-free fragment loads).  A unit runs on one
// warp pair: cost of the busiest pair = units per pair x (pk + overhead); the overhead of a unit (stage
// latency, stores) is 0.75 pairs with one stage per warp and 0.35 once the ring holds at
// least 1.5 stages per warp (the next unit's copy overlaps the current one).
int choose_pk(int pairs, int64_t tiles, int ctas, int smem_optin) {
    if (ctas < 1) ctas = 1;
    int best = 1;
    double best_cost = 1e300;
    for (int pk = 5; pk >= 1; pk -= 2) {
        if ((int)mma_smem(pk, kPairs).total > smem_optin - 4096) continue;  // a ring of one stage per pair must fit
        const int parts = (pairs + pk - 1) / pk;
        const int64_t U = tiles * parts;
        const int64_t per = (U + (int64_t)ctas * kPairs - 1) / ((int64_t)ctas * kPairs);
        const double ovh = mma_stages(pk, smem_optin) >= 12 ? 0.35 : 0.75;
        const double cost = (double)per * ((double)pk + ovh) + (parts > 1 ? 0.25 : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = pk;
        }
    }
    return best;
}
}  // namespace

// Upper bound over every part choice (one part per pair), so the size does not depend on the device.
size_t gemv_mma_partial_bytes(int64_t K, int64_t N, int B) {
    if (K % 512 != 0 || K < 1024) return 0;
    return (size_t)(K / 512) * B * N * sizeof(float);
}

// Partial-sum bytes the launch below actually uses for (K, N, B) on a device with `sms` SMs.
size_t gemv_mma_partial_bytes_for(int64_t K, int64_t N, int B, int sms, int smem_optin) {
    if (K % 512 != 0) return 0;
    const int pairs = (int)(K / 512);
    const int64_t T = (N + 15) / 16;
    const int pk = choose_pk(pairs, T, sms, smem_optin);
    const int parts = (pairs + pk - 1) / pk;
    return parts > 1 ? (size_t)parts * B * N * sizeof(float) : 0;
}

template <int B, bool kDebug>
static cudaError_t launch_mma_b(const CUtensorMap& map, GemvMmaArgs a, int smem, cudaStream_t stream, bool pdl, int grid) {
    constexpr bool kF32Ok = !kDebug && B <= kF32MaxPkB;
    auto kern = (kF32Ok && a.act.mode == kActF32) ? gemv_iq4xs_q8_mma_kernel<B, kDebug, kF32Ok>
                                                   : gemv_iq4xs_q8_mma_kernel<B, kDebug, false>;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(32 * (kNCW + 1));
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, map, a);
}

cudaError_t launch_gemv_mma(const uint8_t* W, const uint8_t* q8, float* y, int32_t* sumi, float* partials,
                            size_t partial_bytes, int64_t K, int64_t N, int B, cudaStream_t stream,
                            bool pdl, int sms, int smem_optin, uint32_t* err, const uint32_t lut[4],
                            const ActSource* act) {
    if (B < 1 || B > 8 || K % 512 != 0 || (reinterpret_cast<uintptr_t>(W) & 15u)) return cudaErrorInvalidValue;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const int pairs = (int)(K / 512);
    const int64_t T = (N + 15) / 16;
    const int pk = choose_pk(pairs, T, sms, smem_optin);
    const int stages = mma_stages(pk, smem_optin);
    const int parts = (pairs + pk - 1) / pk;
    if (parts > 1 && y) {  // partial sums of the parts (the debug path writes none)
        if (!partials || partial_bytes < (size_t)parts * B * N * sizeof(float)) return cudaErrorInvalidValue;
    }
    const MmaSmem L = mma_smem(pk, stages);
    if ((int)L.total > smem_optin) return cudaErrorInvalidConfiguration;

    // 2-D view uint64 [N][34*pairs]; a unit is one box of 16 rows x pk pairs (pk*272 bytes per row,
    // 16 TMA rows per copy), landing as [16][pk*272] in shared memory.
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)pairs * 34, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)pairs * 272};
    const cuuint32_t box[2] = {(cuuint32_t)(34 * pk), 16};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(W), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;

    GemvMmaArgs a = {};
    a.q8 = q8;
    a.y = y;
    a.sumi = sumi;
    a.err = err;
    a.N = N;
    a.K = (int)K;
    a.pairs = pairs;
    a.pk = pk;
    a.parts = parts;
    a.stages = stages;
    a.partial = partials;
    for (int i = 0; i < 4; ++i) a.lut[i] = lut[i];
    a.act.mode = kActQ8;
    if (act && act->mode != kActQ8) {
        if (act->mode != kActF32) return cudaErrorNotSupported;
        if (pk * B <= kF32MaxPkB) {
            a.act = *act;  // every CTA quantises the <= 2 parts it touches while staging them
        } else {
            // Quantising 16*pk*B blocks per CTA would cost more than one more launch: the standalone
            // quantizer writes the Q8_1 area (q8) and the GEMV waits for it (programmatic launch).
            if (!q8) return cudaErrorInvalidValue;
            cudaError_t eq = launch_q8_1_quantize(act->x, const_cast<uint8_t*>(q8), K, B, K, 1, stream, true, pdl);
            if (eq != cudaSuccess) return eq;
            pdl = true;
        }
    }
    const int64_t U = T * parts;
    // A CTA holds the activations of at most two parts: its unit range must not exceed T units.
    int64_t grid64 = std::min<int64_t>(sms, U);
    while ((U + grid64 - 1) / grid64 > T) ++grid64;
    const int grid = (int)grid64;
    cudaError_t e = cudaErrorInvalidValue;
    switch (B) {
#define IQ4XS_MMA_B(BB)                                                                         \
    case BB:                                                                                    \
        e = sumi ? launch_mma_b<BB, true>(map, a, (int)L.total, stream, pdl, grid)             \
                 : launch_mma_b<BB, false>(map, a, (int)L.total, stream, pdl, grid);            \
        break;
        IQ4XS_MMA_B(1) IQ4XS_MMA_B(2) IQ4XS_MMA_B(3) IQ4XS_MMA_B(4)
        IQ4XS_MMA_B(5) IQ4XS_MMA_B(6) IQ4XS_MMA_B(7) IQ4XS_MMA_B(8)
#undef IQ4XS_MMA_B
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || parts == 1 || !y) return e;
    // Sum the parts: a small follow-on kernel chained by programmatic dependent launch.
    const int64_t BN = (int64_t)B * N;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::min<int64_t>((BN + 255) / 256, (int64_t)sms * 4));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, reduce_parts_kernel, (const float*)partials, y, parts, BN);
}

double gemv_mma_cta_cost(int64_t K, int64_t N, int ctas, int smem_optin) {
    if (K % 512 != 0 || ctas < 1) return 1e300;
    const int pairs = (int)(K / 512);
    const int64_t T = (N + 15) / 16;
    const int pk = choose_pk(pairs, T, ctas, smem_optin);
    const int parts = (pairs + pk - 1) / pk;
    const int64_t U = T * parts;
    int64_t n = std::min<int64_t>(ctas, U);
    while ((U + n - 1) / n > T) ++n;  // the launcher's bound: a CTA's units span at most two parts
    const int64_t rounds = ((U + n - 1) / n + kPairs - 1) / kPairs;
    const double ovh = mma_stages(pk, smem_optin) >= 12 ? 0.35 : 0.75;
    return (double)rounds * ((double)pk + ovh) + (parts > 1 ? 0.25 : 0.0);
}

int gemv_mma_grouped_parts(int64_t K, int64_t N, int ctas, int smem_optin) {
    if (K % 512 != 0) return 0;
    const int pairs = (int)(K / 512);
    const int pk = choose_pk(pairs, (N + 15) / 16, std::max(ctas, 1), smem_optin);
    return (pairs + pk - 1) / pk;
}

cudaError_t launch_gemv_mma_grouped(const GroupedProblem* p, int count, int B, cudaStream_t stream, bool pdl,
                                    uint32_t* err, const uint32_t lut[4]) {
    if (count < 1 || count > kMaxGroup || B < 2 || B > 8) return cudaErrorInvalidValue;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    int sms = 0, smem_optin = 0;
    device_limits_current(&sms, &smem_optin);
    GroupMmaParams G;
    std::memset(&G, 0, sizeof G);
    uint32_t smem_max = 0;
    int cta = 0;
    for (int i = 0; i < count; ++i) {
        const int64_t K = p[i].K, N = p[i].N;
        if (K % 512 != 0 || (reinterpret_cast<uintptr_t>(p[i].W) & 15u)) return cudaErrorInvalidValue;
        const int pairs = (int)(K / 512);
        const int64_t T = (N + 15) / 16;
        int ncta = std::max(p[i].ctas, 1);
        const int pk = choose_pk(pairs, T, ncta, smem_optin);
        const int stages = mma_stages(pk, smem_optin);
        const int parts = (pairs + pk - 1) / pk;
        if (parts > 1 && !p[i].partials) return cudaErrorInvalidValue;
        const MmaSmem L = mma_smem(pk, stages);
        if ((int)L.total > smem_optin) return cudaErrorInvalidConfiguration;
        const cuuint64_t dims[2] = {(cuuint64_t)pairs * 34, (cuuint64_t)N};
        const cuuint64_t strides[1] = {(cuuint64_t)pairs * 272};
        const cuuint32_t box[2] = {(cuuint32_t)(34 * pk), 16};
        const cuuint32_t estr[2] = {1, 1};
        if (enc(&G.maps[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(p[i].W), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
        GemvMmaArgs& a = G.args[i];
        a.q8 = p[i].q8;
        a.y = p[i].y;
        a.partial = p[i].partials;
        a.sumi = nullptr;
        a.err = err;
        a.N = N;
        a.K = (int)K;
        a.pairs = pairs;
        a.pk = pk;
        a.parts = parts;
        a.stages = stages;
            for (int j = 0; j < 4; ++j) a.lut[j] = lut[j];
        a.act.mode = kActQ8;
        // A CTA stages the activations of at most two parts: its unit range must not exceed T units.
        const int64_t U = T * parts;
        int64_t n64 = std::min<int64_t>(ncta, U);
        while ((U + n64 - 1) / n64 > T) ++n64;
        ncta = (int)n64;
        G.cta0[i] = cta;
        cta += ncta;
        smem_max = std::max(smem_max, L.total);
    }
    G.cta0[count] = cta;
    G.count = count;
    void* kern = nullptr;
    switch (B) {
        case 2: kern = (void*)gemv_mma_grouped_kernel<2>; break;
        case 3: kern = (void*)gemv_mma_grouped_kernel<3>; break;
        case 4: kern = (void*)gemv_mma_grouped_kernel<4>; break;
        case 5: kern = (void*)gemv_mma_grouped_kernel<5>; break;
        case 6: kern = (void*)gemv_mma_grouped_kernel<6>; break;
        case 7: kern = (void*)gemv_mma_grouped_kernel<7>; break;
        case 8: kern = (void*)gemv_mma_grouped_kernel<8>; break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = ensure_dynamic_smem(kern, (int)smem_max);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cta);
    cfg.blockDim = dim3(32 * (kNCW + 1));
    cfg.dynamicSmemBytes = smem_max;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {&G};
    return cudaLaunchKernelExC(&cfg, kern, args);
}

}  // namespace iq4xs
