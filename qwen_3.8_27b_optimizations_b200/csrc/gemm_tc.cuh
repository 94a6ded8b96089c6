// gemm_tc.cuh -- pieces shared by the tensor-core (tcgen05 + TMEM) prefill GEMM kernels: shared-memory
// matrix descriptors, TMA and tcgen05 wrappers, packed fp32 pair arithmetic, bounded barrier waits,
// and the host-side tensor-map encoder lookup.  Internal to the library (gemm.cu, gemm_i8.cu).
#pragma once
#include <cuda.h>

#include "iq4xs_device.cuh"

namespace iq4xs {
namespace gemm_tc {

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address >> 4 (bits 0-13),
// leading byte offset (unused for swizzled K-major, encoded 1), stride byte offset 1024 >> 4 (8-row
// core groups are 1024 bytes apart, bits 32-45), fixed version bits 46-47 = 1, swizzle mode 2 at
// bits 61-63.  Advancing K by 32 bytes (16 fp16 or 32 int8) inside the swizzle atom adds 2 to the encoded start address.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_3d_nohint(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                   uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrives once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void sts_u4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Packed fp32 pair arithmetic (sm_100): d = a * b and d = a * b + d, two lanes per instruction.
// (The float2 builtins let the register allocator place the pairs; inline asm that packs two
// scalars into a .b64 operand costs register moves when the scalars are not an aligned pair.)
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    const float2 r = __fmul2_rn(make_float2(a0, a1), make_float2(b0, b1));
    d0 = r.x;
    d1 = r.y;
}

__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(d0, d1));
    d0 = r.x;
    d1 = r.y;
}

// Bounded sleeping wait on one phase parity; gives up (error word + abort flag) after ~20 s or
// when another role raised the abort flag.
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag, uint32_t* err,
                                      uint32_t code) {
    for (uint32_t i = 0; i < 20000u; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (*abort_flag) return false;
    }
    record_error(err, code);
    *abort_flag = 1u;
    return false;
}

// Bounded wait used while draining after an abort (no abort check: the copy must land first).
__device__ __forceinline__ void gdrain(uint64_t* bar, uint32_t parity, uint32_t* err) {
    for (uint32_t i = 0; i < 20000u; ++i)
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return;
    record_error(err, kDevErrDrainWait);
}

// d = a * b + c, two lanes per instruction.
__device__ __forceinline__ void fma2c(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
    const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(c0, c1));
    d0 = r.x;
    d1 = r.y;
}

// Two phases in turn, each with the sleeping wait: a waiting thread issues (almost) nothing until the
// phase completes, so the warps that wait leave the issue slots to the warps that compute.
__device__ __forceinline__ bool gwait_seq(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2,
                                          volatile uint32_t* abort_flag, uint32_t* err, uint32_t code) {
    return gwait(b1, p1, abort_flag, err, code) && gwait(b2, p2, abort_flag, err, code);
}

// Bounded wait without a suspend hint (prompt wake-up), giving up on abort.
__device__ __forceinline__ bool gwait_fast(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag, uint32_t* err,
                                           uint32_t code) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 15u && *abort_flag) return false;
    }
    record_error(err, code);
    *abort_flag = 1u;
    return false;
}

// Host side: cuTensorMapEncodeTiled through the runtime's driver entry point.
typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn2 encode_fn2() {
    // Function-local static: initialised once, thread-safe when several host threads launch at once.
    static const EncodeTiledFn2 fn = []() -> EncodeTiledFn2 {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn2>(p);
        return nullptr;
    }();
    return fn;
}

}  // namespace gemm_tc
}  // namespace iq4xs
