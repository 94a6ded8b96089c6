// iq4xs_device.cuh -- formats and sm_100a device primitives shared by every kernel.
//
// IQ4_XS super-block (136 B, 256 weights; kernels/common/block_iq4_xs.h:10-19 in the reference):
//   bytes 0-1  d         fp16 super-block scale
//   bytes 2-3  scales_h  2 high bits of the 6-bit scale of each of the 8 sub-blocks
//   bytes 4-7  scales_l  4 low bits of each sub-block scale (two per byte)
//   bytes 8-135 qs       4-bit codebook indices; byte j of sub-block ib holds element j (low
//                        nibble) and element j+16 (high nibble) of the 32-weight sub-block
// Q8_1 activation block (36 B, 32 values; real_stock_dp4a_comparator.hip:22-26):
//   bytes 0-1 d = trunc_fp16(amax/127), bytes 2-3 s = trunc_fp16(sum), bytes 4-35 int8 q.
#pragma once

#include "../../include/iq4xs_peer.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace iq4xs {

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

constexpr int kQK = 256;          // weights per super-block
constexpr int kQK8 = 32;          // values per Q8_1 block / weights per sub-block
constexpr int kBlockBytes = 136;  // IQ4_XS super-block
constexpr int kQ8Bytes = 36;      // Q8_1 block

// Device error word: a bounded wait that gives up records its code here (first writer wins)
// and the kernel returns instead of hanging.  Read and cleared by iq4xs_device_error().
enum DeviceError : uint32_t {
    kDevErrNone = 0,
    kDevErrFullWait = 1,    // consumer waited too long for a weight stage
    kDevErrEmptyWait = 2,   // producer waited too long for a free stage
    kDevErrDrainWait = 3,   // copies still in flight after an error
    kDevErrMmaWait = 4,     // tensor-core pipeline barrier timed out
    kDevErrPosition = 5,    // decode attention: the device-side position is outside the KV cache
    kDevErrPeerWait = 6,    // peer collective: a peer's flag did not arrive within the spin limit
    kDevErrToken = 7,       // decode embedding: the device-side token id is outside the vocabulary
};

// Spin limit for every mbarrier wait (each try_wait already suspends for a while in hardware);
// at ~1-2 us per expired try_wait this bounds a wait to well under a minute.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ void record_error(uint32_t* err, uint32_t code) {
    if (err) atomicCAS(err, 0u, code);
}

// ------------------------------------------------------------------------------ fp16 helpers
// The reference's truncating fp32 -> fp16 (block_iq4_xs.h:71-86, comparator.hip:45-58).
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float v) {
    const uint32_t x = __float_as_uint(v);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    uint32_t m = (x >> 13) & 0x3FFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m = (m | 0x400u) >> (1 - e);
        return (uint16_t)(sign | m);
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xFFFFu)));
}

// One Q8_1 block (kernels/matmul_iq4xs/real_stock_dp4a_comparator.hip:230-264): lane i of a full
// warp holds x_i; amax and sum by a 16..1 xor butterfly, d = amax/127, q = (int8)roundf(x/d)
// (0 when amax == 0), ds = {trunc_fp16(d), trunc_fp16(sum)}; the 36 bytes at `out` (4-byte aligned)
// are written as nine 4-byte stores.  Every Q8_1 producer in the library goes through this.
__device__ __forceinline__ void q8_1_block_store(float x, uint8_t* out, int lane) {
    const unsigned full = 0xFFFFFFFFu;
    float amax = fabsf(x), sum = x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(full, amax, off));
        sum += __shfl_xor_sync(full, sum, off);
    }
    const float d = amax / 127.0f;
    int q = 0;
    if (amax != 0.0f) q = (int)roundf(x / d);
    const uint32_t b0 = (uint32_t)q & 0xFFu;
    const uint32_t b1 = __shfl_down_sync(full, b0, 1);
    const uint32_t b2 = __shfl_down_sync(full, b0, 2);
    const uint32_t b3 = __shfl_down_sync(full, b0, 3);
    if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(out + 4 + lane) = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (lane == 0)
        *reinterpret_cast<uint32_t*>(out) = (uint32_t)f32_to_f16_trunc(d) | ((uint32_t)f32_to_f16_trunc(sum) << 16);
}

// Four consecutive Q8_1 blocks (144 bytes at `out`, 4-byte aligned) from 128 values held as one
// float4 per lane (lane l: values 4l..4l+3; lanes 8j..8j+7 form block j).  amax (exact in any order),
// d = amax/127 and q = (int8)roundf(x/d) are those of q8_1_block_store, so the quants and d are
// identical; the block sum (the upper half of ds, which no IQ4_XS dot reads) is added in a
// different order and may differ in its last bit.
__device__ __forceinline__ void q8_1_quad_store(float4 v, uint8_t* out, int lane) {
    const unsigned full = 0xFFFFFFFFu;
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    float sum = (v.x + v.y) + (v.z + v.w);
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(full, amax, off));
        sum += __shfl_xor_sync(full, sum, off);
    }
    const float d = amax / 127.0f;
    int q0 = 0, q1 = 0, q2 = 0, q3 = 0;
    if (amax != 0.0f) {
        q0 = (int)roundf(v.x / d);
        q1 = (int)roundf(v.y / d);
        q2 = (int)roundf(v.z / d);
        q3 = (int)roundf(v.w / d);
    }
    uint8_t* blk = out + (lane >> 3) * 36;
    *reinterpret_cast<uint32_t*>(blk + 4 + 4 * (lane & 7)) =
        ((uint32_t)q0 & 0xFFu) | (((uint32_t)q1 & 0xFFu) << 8) | (((uint32_t)q2 & 0xFFu) << 16) | ((uint32_t)q3 << 24);
    if ((lane & 7) == 0)
        *reinterpret_cast<uint32_t*>(blk) = (uint32_t)f32_to_f16_trunc(d) | ((uint32_t)f32_to_f16_trunc(sum) << 16);
}

// ------------------------------------------------------------------------------ byte permute
// prmt.b32 default mode: bytes {b,a} numbered 0..7 (a = 0..3); selector nibble i: bits 2:0
// pick the source byte, bit 3 replicates that byte's sign bit over the output byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Codebook kvalues_iq4nl (block_iq4_xs.h:22-24) split into two 8-byte prmt tables:
//  kNegLo: -kv[0..7]  = 127,104,83,65,49,35,22,10  (all < 128, sign bit clear)
//  kPosHi:  kv[8..15] = 1,13,25,38,53,69,89,113    (all < 128, sign bit clear)
// prmt(kNegLo, q) returns -kv[n] for codes n<8 and 0 for n>=8 (bit 3 selects sign replication
// of a positive byte); prmt(kPosHi, q^0x8888) returns kv[n] for n>=8 and 0 for n<8.  So
//   sum_j kv[n_j] x_j = dp4a(hi, x) - dp4a(lo, x)
// with two lookups and no merge step.  Output byte order of one lookup on the low 16 bits of a
// qs word w (bytes 4w..4w+3 of the sub-block) is [e(4w), e(4w+16), e(4w+1), e(4w+17)], on the
// high 16 bits [e(4w+2), e(4w+18), e(4w+3), e(4w+19)]; activations are permuted to match.
constexpr uint32_t kNegLo0 = 0x4153687Fu, kNegLo1 = 0x0A162331u;
constexpr uint32_t kPosHi0 = 0x26190D01u, kPosHi1 = 0x71594535u;

// Activation words in the lookup order: from q8 words lo = q[4w..4w+3], hi = q[16+4w..16+4w+3].
__device__ __forceinline__ uint32_t act_perm_lo(uint32_t lo, uint32_t hi) { return prmt(lo, hi, 0x5140u); }
__device__ __forceinline__ uint32_t act_perm_hi(uint32_t lo, uint32_t hi) { return prmt(lo, hi, 0x7362u); }

// Raw sub-block dot of 4 qs words against 8 permuted activation words (exact int32).
__device__ __forceinline__ int subblock_dot(const uint32_t q[4], const uint32_t alo[4], const uint32_t ahi[4]) {
    int hi = 0, lo = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t x = q[w];
        const uint32_t xf = x ^ 0x88888888u;
        const uint32_t xh = x >> 16, xfh = xf >> 16;
        hi = dp4a((int)prmt(kPosHi0, kPosHi1, xf), (int)alo[w], hi);
        lo = dp4a((int)prmt(kNegLo0, kNegLo1, x), (int)alo[w], lo);
        hi = dp4a((int)prmt(kPosHi0, kPosHi1, xfh), (int)ahi[w], hi);
        lo = dp4a((int)prmt(kNegLo0, kNegLo1, xh), (int)ahi[w], lo);
    }
    return hi - lo;
}

// 6-bit scale code of sub-block ib from the two header words (h0 = d | scales_h<<16,
// h1 = scales_l[0..3]); ref_cpu.cpp:30-33.
__device__ __forceinline__ int subblock_scale(uint32_t h0, uint32_t h1, int ib) {
    return (int)(((h1 >> (4 * ib)) & 0xFu) | (((h0 >> (16 + 2 * ib)) & 0x3u) << 4));
}

// ------------------------------------------------------------------------------ smem / PTX
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes (or the hint,
// in ns, elapses) instead of returning at once, so waiting warps issue almost no instructions.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait on one phase parity.  Returns false (and records `code`) when the limit is hit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    record_error(err, code);
    return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on `bar` (bytes).
// dst, src 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same, with an L2 eviction hint: weights are streamed once per call.
__device__ __forceinline__ void bulk_g2s_evict_first(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                     uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy accesses (TMA,
// bulk copies, tensor-core operand reads) to the same memory.  Needed on both sides of a stage
// handed from threads that read it with ld.shared back to a copy engine that refills it: the reader
// before it releases the stage, the producer after it acquires the stage and before it issues the
// copy.  Without it the refill can land before the last generic read of the old contents.
__device__ __forceinline__ void fence_generic_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory (no-op without PDL).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// ------------------------------------------------------------------------------ peer flags
// System-scope release store / acquire load of a 32-bit flag (another GPU's memory or written by
// another GPU).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Fused all-reduce (low-latency protocol): a slot word is {fp32 value bits, epoch}; single 8-byte
// relaxed system-scope accesses, so a reader sees either the old word or the new one whole.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Producer: the epoch of this all-reduce (read by every CTA before it stores; the grid's last CTA
// advances the counter once all CTAs have stored).
__device__ __forceinline__ uint32_t peer_slots_epoch_next(const iq4xs_peer_slots* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p->counter) + 1u;
}

// Producer: output `row` into slot `rank` of every rank's area.
__device__ __forceinline__ void peer_slots_store(const iq4xs_peer_slots* p, int64_t row, float v, uint32_t e) {
    const uint64_t w = ((uint64_t)e << 32) | (uint64_t)__float_as_uint(v);
    const int world = p->world;
    for (int q = 0; q < world && q < IQ4XS_MAX_PEERS; ++q) st_relaxed_sys_u64(p->dst[q] + row, w);
}

// Producer, one thread per CTA after the CTA's stores: the last CTA advances the epoch counter.
__device__ __forceinline__ void peer_slots_done(const iq4xs_peer_slots* p, int ncta, uint32_t e) {
    uint32_t* cnt = p->counter;
    if (atomicAdd(cnt + 1, 1u) == (uint32_t)ncta - 1u) {
        cnt[1] = 0u;
        reinterpret_cast<volatile uint32_t*>(cnt)[0] = e;
    }
}

// Consumer: the epoch the producer on this rank (complete before the consumer reads) advanced to.
__device__ __forceinline__ uint32_t peer_slots_epoch(const iq4xs_peer_slots* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p->counter);
}

// Consumer: value i of slot q once it carries epoch e (bounded: a read that gives up records
// kDevErrPeerWait and returns the stale value; once the device error word is set, by this wait or
// any other, a waiting read gives up within 1024 polls, so a missing peer costs one spin limit).
__device__ __forceinline__ float peer_slot_value(const iq4xs_peer_slots* p, int q, int64_t n, int64_t i, uint32_t e,
                                                 uint32_t* err) {
    const uint64_t* a = p->local + (int64_t)q * n + i;
    uint64_t w = ld_relaxed_sys_u64(a);
    if ((uint32_t)(w >> 32) != e) {
        const uint32_t limit = p->spin_limit ? p->spin_limit : (1u << 24);
        uint32_t k = 0;
        do {
            if (++k > limit) {
                record_error(err, kDevErrPeerWait);
                break;
            }
            if ((k & 1023u) == 0u && err && *reinterpret_cast<volatile uint32_t*>(err) != 0u) break;
            __nanosleep(32);
            w = ld_relaxed_sys_u64(a);
        } while ((uint32_t)(w >> 32) != e);
    }
    return __uint_as_float((uint32_t)w);
}

// Consumer: delta[i] = the ranks' values added in rank order (slot 0 first), the order and rounding
// of iq4xs_peer_collective's all-reduce.
__device__ __forceinline__ float peer_slots_sum1(const iq4xs_peer_slots* p, int64_t n, int64_t i, uint32_t e,
                                                 uint32_t* err) {
    float s = peer_slot_value(p, 0, n, i, e, err);
    const int world = p->world;
    for (int q = 1; q < world && q < IQ4XS_MAX_PEERS; ++q) s = __fadd_rn(s, peer_slot_value(p, q, n, i, e, err));
    return s;
}

__device__ __forceinline__ void ld_relaxed_sys_v2u64(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Consumer, one warp: dsm[i] = delta[i] (the ranks' values added in rank order) for every i in this
// warp's quads qd = cw, cw + ncw, ... < nq (128 values each, 4 per lane).  (quad, rank) pairs go eight
// at a time: every word of a round is loaded before any tag is checked, so a round whose tags are all
// current costs one round trip (1, 2 or 4 rounds for this warp's four quads at 2, 4 or 8 ranks); a
// stale word is then polled on its own (bounded, peer_slot_value).  Each 8-byte word of a vector load
// is a single-copy-atomic access.
__device__ __forceinline__ void peer_slots_sum_to_smem(const iq4xs_peer_slots* p, int64_t n, int nq, int cw, int ncw,
                                                       int lane, uint32_t e, uint32_t* err, float* dsm) {
    constexpr int kRound = 8;
    const int world = p->world < kRound ? (p->world > 0 ? p->world : 1) : kRound;
    const int qpr = kRound / world;  // quads per round
    for (int first = cw; first < nq; first += ncw * qpr) {
        uint64_t w[kRound][4];
#pragma unroll
        for (int u = 0; u < kRound; ++u) {
            const int j = u / world, q = u - j * world;
            const int qd = first + j * ncw;
            if (j < qpr && qd < nq) {
                const uint64_t* a = p->local + (int64_t)q * n + qd * 128 + 4 * lane;
                ld_relaxed_sys_v2u64(a, w[u][0], w[u][1]);
                ld_relaxed_sys_v2u64(a + 2, w[u][2], w[u][3]);
            }
        }
        float4 cur = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kRound; ++u) {
            const int j = u / world, q = u - j * world;
            const int qd = first + j * ncw;
            if (j >= qpr || qd >= nq) continue;
            const int off = qd * 128 + 4 * lane;
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[k] = (uint32_t)(w[u][k] >> 32) == e ? __uint_as_float((uint32_t)w[u][k])
                                                      : peer_slot_value(p, q, n, off + k, e, err);
            }
            if (q == 0) {
                cur = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                cur.x = __fadd_rn(cur.x, v[0]);
                cur.y = __fadd_rn(cur.y, v[1]);
                cur.z = __fadd_rn(cur.z, v[2]);
                cur.w = __fadd_rn(cur.w, v[3]);
            }
            if (q == world - 1) *reinterpret_cast<float4*>(dsm + off) = cur;
        }
    }
}

// Consumer, batched: s[j] = delta[idx[j]] for the NB indices with ok[j] (loads of one slot issued
// together, as in peer_slots_sum4_batch).
template <int NB>
__device__ __forceinline__ void peer_slots_sum1_batch(const iq4xs_peer_slots* p, int64_t n, const int (&idx)[NB],
                                                      const bool (&ok)[NB], uint32_t e, uint32_t* err,
                                                      float (&s)[NB]) {
    const int world = p->world;
    for (int q = 0; q < world && q < IQ4XS_MAX_PEERS; ++q) {
        const uint64_t* base = p->local + (int64_t)q * n;
        uint64_t w[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) w[j] = ok[j] ? ld_relaxed_sys_u64(base + idx[j]) : ((uint64_t)e << 32);
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const float v = (uint32_t)(w[j] >> 32) == e ? __uint_as_float((uint32_t)w[j])
                                                        : peer_slot_value(p, q, n, idx[j], e, err);
            s[j] = q == 0 ? v : __fadd_rn(s[j], v);
        }
    }
}

}  // namespace iq4xs
