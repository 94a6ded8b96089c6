// weights.cu -- synthetic data and the IQ4_XS weight format on the device.
//
//  * fill_normal: counter-based N(mean, stddev) draws (Philox4x32-10, Salmon et al. SC'11, then the
//    Box-Muller transform), deterministic per (seed, index), for the seeded synthetic workloads.
//  * quantize_iq4_xs: the IQ4_XS weight quantizer.  The reference quantises its test matrices with
//    upstream ggml's quantize_row_iq4_xs (llama.cpp bb4caa75), which it does not vendor; this is the
//    same published algorithm (per-sub-block least-squares scale search over 15 trial scales, 6-bit
//    sub-block scales relative to an fp16 super-block scale, codes from the fixed 16-value codebook),
//    one warp per 256-weight super-block, lane j = element j of the current 32-weight sub-block.
//    Every float operation is an explicitly rounded _rn intrinsic and the two per-trial sums use the
//    xor-butterfly order, so the result is identical, bit for bit, to the C restatement used by the
//    tests as the checker.
//  * dequantize: fp32 expansion (ref_cpu.cpp:115-139 semantics) for tests and tools.
#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

__constant__ int8_t c_kvalues[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

// ------------------------------------------------------------------------------ Philox + Box-Muller
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
        const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += W0;
        k.y += W1;
    }
    return c;
}

__global__ void fill_normal_kernel(float* __restrict__ dst, int64_t n, uint64_t seed, float mean, float stddev) {
    const uint2 key = make_uint2((uint32_t)seed, (uint32_t)(seed >> 32));
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i * 4 < n; i += nthreads) {
        const uint4 r = philox4x32_10(make_uint4((uint32_t)i, (uint32_t)((uint64_t)i >> 32), 0x1234567u, 0u), key);
        const float k = 2.3283064365386963e-10f;  // 2^-32
        const float u1 = ((float)r.x + 0.5f) * k, u2 = ((float)r.y + 0.5f) * k;
        const float u3 = ((float)r.z + 0.5f) * k, u4 = ((float)r.w + 0.5f) * k;
        const float ra = sqrtf(-2.0f * logf(u1)), rb = sqrtf(-2.0f * logf(u3));
        float s1, c1, s2, c2;
        sincospif(2.0f * u2, &s1, &c1);
        sincospif(2.0f * u4, &s2, &c2);
        const float z[4] = {ra * c1, ra * s1, rb * c2, rb * s2};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (i * 4 + j < n) dst[i * 4 + j] = mean + stddev * z[j];
    }
}

cudaError_t launch_fill_normal(float* dst, int64_t n, uint64_t seed, float mean, float stddev, cudaStream_t stream) {
    const int64_t threads = (n + 3) / 4;
    const int64_t grid = std::min<int64_t>((threads + 255) / 256, 148 * 64);
    fill_normal_kernel<<<(unsigned)std::max<int64_t>(grid, 1), 256, 0, stream>>>(dst, n, seed, mean, stddev);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------ IQ4_XS quantizer
__device__ __forceinline__ int nearest_code(float v) {
    if (v <= (float)c_kvalues[0]) return 0;
    if (v >= (float)c_kvalues[15]) return 15;
    int lo = 0, hi = 15;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (v < (float)c_kvalues[mid]) hi = mid; else lo = mid;
    }
    return (__fsub_rn(v, (float)c_kvalues[hi - 1]) < __fsub_rn((float)c_kvalues[hi], v)) ? hi - 1 : hi;
}

__device__ __forceinline__ float warp_butterfly_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    return v;
}

__global__ void __launch_bounds__(256) quantize_iq4_xs_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                              int64_t nblocks, int64_t n_per_row) {
    const int lane = threadIdx.x & 31;
    const int64_t kb = n_per_row / kQK;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < nblocks; blk += nwarps) {
        const int64_t row = blk / kb, b = blk - row * kb;
        const float* x = src + row * n_per_row + b * kQK;
        float scales[8];
        float max_scale = 0.0f, amax_scale = 0.0f;
#pragma unroll 1
        for (int ib = 0; ib < 8; ++ib) {
            const float xv = x[32 * ib + lane];
            const float w = __fmul_rn(xv, xv);
            // first index of the largest |x|
            float ax = fabsf(xv);
            int idx = lane;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float oa = __shfl_xor_sync(0xFFFFFFFFu, ax, off);
                const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, off);
                if (oa > ax || (oa == ax && oi < idx)) { ax = oa; idx = oi; }
            }
            const float amax = ax;
            const float xmax = __shfl_sync(0xFFFFFFFFu, xv, idx);
            if (amax < 1e-15f) { scales[ib] = 0.0f; continue; }
            float d = __fdiv_rn(-xmax, (float)c_kvalues[0]);
            float id = __fdiv_rn(1.0f, d);
            int l = nearest_code(__fmul_rn(id, xv));
            float q = (float)c_kvalues[l];
            float wq = __fmul_rn(w, q);
            float sumqx = warp_butterfly_sum(__fmul_rn(wq, xv));
            float sumq2 = warp_butterfly_sum(__fmul_rn(wq, q));
            d = __fdiv_rn(sumqx, sumq2);
            float best = __fmul_rn(d, sumqx);
#pragma unroll 1
            for (int t = -7; t <= 7; ++t) {
                id = __fdiv_rn(__fadd_rn((float)t, (float)c_kvalues[0]), xmax);
                l = nearest_code(__fmul_rn(id, xv));
                q = (float)c_kvalues[l];
                wq = __fmul_rn(w, q);
                sumqx = warp_butterfly_sum(__fmul_rn(wq, xv));
                sumq2 = warp_butterfly_sum(__fmul_rn(wq, q));
                if (sumq2 > 0.0f && __fmul_rn(sumqx, sumqx) > __fmul_rn(best, sumq2)) {
                    d = __fdiv_rn(sumqx, sumq2);
                    best = __fmul_rn(d, sumqx);
                }
            }
            scales[ib] = d;
            const float ad = fabsf(d);
            if (ad > amax_scale) { amax_scale = ad; max_scale = d; }
        }
        uint8_t* out = dst + blk * kBlockBytes;
        const float d = __fdiv_rn(-max_scale, 32.0f);
        const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
        uint32_t scales_h = 0, scales_l = 0;
#pragma unroll 1
        for (int ib = 0; ib < 8; ++ib) {
            int l = __float2int_rn(__fmul_rn(id, scales[ib]));
            l = max(-32, min(31, l));
            const float dl = __fmul_rn(d, (float)l);
            const float idl = (dl != 0.0f) ? __fdiv_rn(1.0f, dl) : 0.0f;
            const int code = nearest_code(__fmul_rn(idl, x[32 * ib + lane]));
            const int code_hi = __shfl_down_sync(0xFFFFFFFFu, code, 16);
            if (lane < 16) out[8 + 16 * ib + lane] = (uint8_t)(code | (code_hi << 4));
            l += 32;
            scales_l |= (uint32_t)(l & 0xF) << (4 * ib);
            scales_h |= (uint32_t)(l >> 4) << (2 * ib);
        }
        if (lane == 0) {
            const uint16_t dh = __half_as_ushort(__float2half_rn(d));
            *reinterpret_cast<uint16_t*>(out) = dh;
            *reinterpret_cast<uint16_t*>(out + 2) = (uint16_t)scales_h;
            *reinterpret_cast<uint32_t*>(out + 4) = scales_l;
        }
    }
}

cudaError_t launch_quantize_iq4_xs(const float* src, uint8_t* dst, int64_t nrows, int64_t n_per_row, cudaStream_t stream) {
    const int64_t nblocks = nrows * (n_per_row / kQK);
    const int64_t grid = std::min<int64_t>((nblocks + 7) / 8, 148 * 32);
    quantize_iq4_xs_kernel<<<(unsigned)std::max<int64_t>(grid, 1), 256, 0, stream>>>(src, dst, nblocks, n_per_row);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------ dequantize
__global__ void dequantize_kernel(const uint8_t* __restrict__ W, float* __restrict__ out, int64_t K, int64_t N) {
    const int64_t nsb = N * (K / kQK8);
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nsb; i += nthreads) {
        const int64_t row = i / (K / kQK8), sb = i - row * (K / kQK8);
        const uint8_t* blk = W + row * (K / kQK) * kBlockBytes + (sb >> 3) * kBlockBytes;
        const int ib = (int)(sb & 7);
        const uint32_t h0 = *reinterpret_cast<const uint16_t*>(blk) | ((uint32_t)*reinterpret_cast<const uint16_t*>(blk + 2) << 16);
        const uint32_t h1 = *reinterpret_cast<const uint32_t*>(blk + 4);
        const float dl = __fmul_rn(f16_bits_to_f32(h0), (float)(subblock_scale(h0, h1, ib) - 32));
        float* o = out + row * K + sb * 32;
        for (int j = 0; j < 16; ++j) {
            const uint8_t v = blk[8 + 16 * ib + j];
            o[j] = __fmul_rn(dl, (float)c_kvalues[v & 0xF]);
            o[j + 16] = __fmul_rn(dl, (float)c_kvalues[v >> 4]);
        }
    }
}

cudaError_t launch_dequantize(const uint8_t* W, float* out, int64_t K, int64_t N, cudaStream_t stream) {
    const int64_t nsb = N * (K / kQK8);
    const int64_t grid = std::min<int64_t>((nsb + 255) / 256, 148 * 32);
    dequantize_kernel<<<(unsigned)std::max<int64_t>(grid, 1), 256, 0, stream>>>(W, out, K, N);
    return cudaGetLastError();
}

}  // namespace iq4xs
