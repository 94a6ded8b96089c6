// decode_ops.cu -- the per-token operations of the decoder step around the IQ4_XS GEMVs, fused so
// that one decoder layer at batch 1 is four GEMVs and three small kernels:
//
//   residual_rmsnorm_q8   x += delta (all-reduced o_proj / down_proj output), RMSNorm, Q8_1
//   attention_decode_q8   RoPE of q and the new k, KV-cache append (f16), causal attention of every
//                         query head over the cache, Q8_1 of the head outputs (the o_proj input)
//   swiglu_q8             silu(gate) * up, Q8_1 (the down_proj input)
//
// Each produces the quantised activations of the next GEMV directly (through q8_1_block_store, the
// same code as the standalone quantizer, so the bytes equal iq4xs_q8_1_quantize of the fp32 values).
// All three trigger their dependents first and wait for the preceding grid before reading, so a
// GEMV launched after them with programmatic dependent launch streams its weights while they run.
// The arithmetic follows the decoder's torch formulation op for op (separately rounded multiplies
// and adds where torch rounds), the reductions are in a different order.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "iq4xs_device.cuh"
#include "iq4xs_kernels.h"

namespace iq4xs {

namespace {
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kHeadDim = 128;

__device__ __forceinline__ void half4_to_float(uint2 u, float f[4]) {
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    f[0] = fa.x; f[1] = fa.y; f[2] = fb.x; f[3] = fb.y;
}
}  // namespace

// One cluster of kNormCtas CTAs per token row t: x[t] += delta[t] (when delta is given; written
// back), then h = (x * rsqrt(mean(x^2) + eps)) * w, stored as Q8_1 blocks q8[t][D/32] and/or fp32
// h_out[t][D].  CTA c owns the 32-element blocks [nb*c/kNormCtas, nb*(c+1)/kNormCtas), a warp every
// kNormWarps-th of them (one element per lane); the CTAs' partial sums of squares are exchanged
// through distributed shared memory and added in rank order, so every CTA gets the same total.
constexpr int kNormCtas = 8;
constexpr int kNormWarps = 4;
constexpr int kNormMaxPer = 8;  // blocks per warp: D <= 8192

// kPeer: delta is the fused all-reduce of `peer`'s slots instead of a vector (T = 1).
template <bool kPeer>
__global__ void __cluster_dims__(kNormCtas, 1, 1) __launch_bounds__(kNormWarps * 32) residual_rmsnorm_q8_kernel(
    float* __restrict__ x, const float* __restrict__ delta, const float* __restrict__ w, int D, float eps,
    uint8_t* __restrict__ q8, float* __restrict__ h_out, const iq4xs_peer_slots* peer, uint32_t* err) {
    namespace cg = cooperative_groups;
    grid_launch_dependents();
    grid_dependency_wait();
    const uint32_t ep = kPeer ? peer_slots_epoch(peer) : 0u;
    __shared__ float red[kNormWarps];
    __shared__ float css;
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int t = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = D / kQK8;
    const int b0 = nb * crank / kNormCtas, b1 = nb * (crank + 1) / kNormCtas;
    float* xr = x + (int64_t)t * D;
    const float* dr = delta ? delta + (int64_t)t * D : nullptr;
    float v[kNormMaxPer], wv[kNormMaxPer], dv[kNormMaxPer];
    int idx[kNormMaxPer];
    bool ok[kNormMaxPer];
#pragma unroll
    for (int j = 0; j < kNormMaxPer; ++j) {
        const int b = b0 + warp + j * kNormWarps;
        ok[j] = b < b1;
        idx[j] = b * kQK8 + lane;
        v[j] = wv[j] = dv[j] = 0.f;
        if (ok[j]) {
            wv[j] = w[idx[j]];
            v[j] = xr[idx[j]];
            if (dr) dv[j] = dr[idx[j]];
        }
    }
    if constexpr (kPeer) peer_slots_sum1_batch<kNormMaxPer>(peer, D, idx, ok, ep, err, dv);  // a slot's loads together
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormMaxPer; ++j) {
        if (ok[j]) {
            if (kPeer || dr) {
                v[j] = __fadd_rn(v[j], dv[j]);
                xr[idx[j]] = v[j];
            }
            ss = fmaf(v[j], v[j], ss);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float c = 0.f;
#pragma unroll
        for (int i = 0; i < kNormWarps; ++i) c += red[i];
        css = c;
    }
    cluster.sync();
    float tot = 0.f;
#pragma unroll
    for (int c = 0; c < kNormCtas; ++c) tot += *cluster.map_shared_rank(&css, c);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, (float)D), eps));
#pragma unroll
    for (int j = 0; j < kNormMaxPer; ++j) {
        const int b = b0 + warp + j * kNormWarps;
        if (b < b1) {  // warp-uniform
            const int e = b * kQK8 + lane;
            const float h = __fmul_rn(__fmul_rn(v[j], r), wv[j]);
            if (h_out) h_out[(int64_t)t * D + e] = h;
            if (q8) q8_1_block_store(h, q8 + ((int64_t)t * nb + b) * kQ8Bytes, lane);
        }
    }
    cluster.sync();  // keep css alive until every CTA of the cluster has read it
}

// Decode attention for one token at position p = *pos.  One cluster of kChunks CTAs per kv head;
// CTA c of the cluster takes the positions [c0, c1) = [(p+1)*c/kChunks, (p+1)*(c+1)/kChunks) for all
// G = q_heads/kv_heads query heads of the group, so every K/V row is read once per group.  Each CTA
// keeps its own softmax max m_c and sum l_c per head and an unnormalised output o_c, and pushes those
// of head r into CTA r's shared memory (distributed shared memory stores); after one cluster barrier
// CTA r merges head r from its own shared memory:
//   M = max_c m_c,  o = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c.
// qkv: fp32 [hq + 2*hkv][128] (q heads, then k heads, then v heads) of this token;
// k_cache / v_cache: f16 [hkv][max_seq][128]; cos/sin: fp32 [max_seq][64].
// The new k (after RoPE) and v are rounded to f16 and appended at position p by CTA 0 of each
// cluster; the CTA whose range holds p uses its own copy of them instead of reading row p.
// Output: Q8_1 blocks q8[h*4 .. h*4+3] for query head h, optionally fp32 o_out[h*128 .. +127].
constexpr int kChunks = 8;

// Sum of 8 per-lane values over the warp, transposed: lanes 4j..4j+3 end with the total of v[j].
__device__ __forceinline__ float warp_sum8_transposed(const float v[8], int lane) {
    const unsigned full = 0xFFFFFFFFu;
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
    float w[4], x[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b4 ? v[i] : v[i + 4];
        const float keep = b4 ? v[i + 4] : v[i];
        w[i] = keep + __shfl_xor_sync(full, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b3 ? w[i] : w[i + 2];
        const float keep = b3 ? w[i + 2] : w[i];
        x[i] = keep + __shfl_xor_sync(full, send, 8);
    }
    float y = (b2 ? x[1] : x[0]) + __shfl_xor_sync(full, b2 ? x[0] : x[1], 4);
    y += __shfl_xor_sync(full, y, 2);
    y += __shfl_xor_sync(full, y, 1);
    return y;
}

template <int G>
__global__ void __cluster_dims__(kChunks, 1, 1) __launch_bounds__(kAttnThreads, 1) attention_decode_q8_kernel(
    const float* __restrict__ qkv, __half* __restrict__ kc, __half* __restrict__ vc,
    const float* __restrict__ cosb, const float* __restrict__ sinb, const int64_t* __restrict__ pos_p, int hq,
    int hkv, int max_seq, int lmax, uint8_t* __restrict__ q8, float* __restrict__ o_out, uint32_t* err,
    bool early_state) {
    namespace cg = cooperative_groups;
    grid_launch_dependents();
    // early_state: the position, the cache rows before it and the RoPE tables are not written by the
    // preceding kernel, so they are read (and the K/V rows requested) before waiting for it; only qkv is
    if (!early_state) grid_dependency_wait();
    extern __shared__ __align__(16) float dyn[];
    float* sc = dyn;                                   // [G][lmax] scores, then exp(s - m_c)
    float* stage = dyn + G * lmax;                     // [kAttnWarps][G][128] per-warp partial outputs
    __shared__ __align__(16) float qs[G][kHeadDim];
    __shared__ __align__(16) float kn[kHeadDim];
    __shared__ __align__(16) float vn[kHeadDim];
    __shared__ float mc[G], lc[G];                      // this CTA's softmax max and sum per head
    // CTA r < G owns head r of the group: every CTA c pushes its (m_c, l_c, o_c) of head r here
    __shared__ float rm[kChunks], rl[kChunks];
    __shared__ __align__(16) float ro[kChunks][kHeadDim];
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int kvh = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t p64 = *pos_p;
    if (p64 < 0 || p64 >= max_seq) {  // uniform over the grid: no CTA reaches a cluster barrier
        if (tid == 0 && crank == 0 && kvh == 0) record_error(err, kDevErrPosition);
        return;
    }
    const int p = (int)p64;
    // first phase of a cluster barrier: this CTA has started (its shared memory may receive the other
    // CTAs' pushes once every CTA has arrived; the wait comes just before the first push)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int c0 = (int)((int64_t)(p + 1) * crank / kChunks), c1 = (int)((int64_t)(p + 1) * (crank + 1) / kChunks);
    constexpr int kHalf = kHeadDim / 2;
    // warp w takes positions c0 + w + 8k, kU at a time; lane holds dims 4*lane .. 4*lane+3.  The
    // first batch of K and V rows is requested before the RoPE work so the loads overlap it.
    constexpr int kU = 10;
    const __half* kbase = kc + (int64_t)kvh * max_seq * kHeadDim + 4 * lane;
    const __half* vbase = vc + (int64_t)kvh * max_seq * kHeadDim + 4 * lane;
    uint2 kraw[kU], vraw[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
        const int t = c0 + warp + u * kAttnWarps;
        kraw[u] = vraw[u] = make_uint2(0u, 0u);
        if (t < c1 && t != p) {
            kraw[u] = *reinterpret_cast<const uint2*>(kbase + (int64_t)t * kHeadDim);
            vraw[u] = *reinterpret_cast<const uint2*>(vbase + (int64_t)t * kHeadDim);
        }
    }
    if (early_state) grid_dependency_wait();  // qkv comes from the preceding kernel
    // RoPE (rotate-half) of the group's q heads and the new k; the new k and v rounded to f16
    for (int it = tid; it < G * kHalf + kHalf + kHeadDim; it += kAttnThreads) {
        if (it < G * kHalf) {
            const int j = it / kHalf, i = it - j * kHalf;
            const float c = cosb[(int64_t)p * kHalf + i], s = sinb[(int64_t)p * kHalf + i];
            const float* qh = qkv + (int64_t)(kvh * G + j) * kHeadDim;
            const float x1 = qh[i], x2 = qh[i + kHalf];
            qs[j][i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
            qs[j][i + kHalf] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
        } else if (it < G * kHalf + kHalf) {
            const int i = it - G * kHalf;
            const float c = cosb[(int64_t)p * kHalf + i], s = sinb[(int64_t)p * kHalf + i];
            const float* kh = qkv + (int64_t)(hq + kvh) * kHeadDim;
            const float x1 = kh[i], x2 = kh[i + kHalf];
            const __half k1 = __float2half_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
            const __half k2 = __float2half_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
            kn[i] = __half2float(k1);
            kn[i + kHalf] = __half2float(k2);
            if (crank == 0) {
                __half* dst = kc + ((int64_t)kvh * max_seq + p) * kHeadDim;
                dst[i] = k1;
                dst[i + kHalf] = k2;
            }
        } else {
            const int i = it - G * kHalf - kHalf;
            const __half v = __float2half_rn(qkv[(int64_t)(hq + hkv + kvh) * kHeadDim + i]);
            vn[i] = __half2float(v);
            if (crank == 0) vc[((int64_t)kvh * max_seq + p) * kHeadDim + i] = v;
        }
    }
    __syncthreads();

    // scores
    float q[G][4];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const float4 t4 = *reinterpret_cast<const float4*>(&qs[j][4 * lane]);
        q[j][0] = t4.x; q[j][1] = t4.y; q[j][2] = t4.z; q[j][3] = t4.w;
    }
    const float4 kn4 = *reinterpret_cast<const float4*>(kn + 4 * lane);
    const float scale = 11.3137084989847604f;  // sqrt(128), divided by as the torch model does
    for (int t0 = c0 + warp; t0 < c1; t0 += kAttnWarps * kU) {
        if (t0 != c0 + warp) {  // later batches
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int t = t0 + u * kAttnWarps;
                kraw[u] = make_uint2(0u, 0u);
                if (t < c1 && t != p) kraw[u] = *reinterpret_cast<const uint2*>(kbase + (int64_t)t * kHeadDim);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = t0 + u * kAttnWarps;
            if (t >= c1) break;  // warp-uniform
            float k[4];
            if (t == p) {
                k[0] = kn4.x; k[1] = kn4.y; k[2] = kn4.z; k[3] = kn4.w;
            } else {
                half4_to_float(kraw[u], k);
            }
            float d[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                d[j] = 0.f;
                if (j < G) d[j] = fmaf(q[j][0], k[0], fmaf(q[j][1], k[1], fmaf(q[j][2], k[2], q[j][3] * k[3])));
            }
            float s;
            if constexpr (G == 8) {
                s = warp_sum8_transposed(d, lane);
                if ((lane & 3) == 0) sc[(lane >> 2) * lmax + (t - c0)] = __fdiv_rn(s, scale);
            } else {
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    s = d[j];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
                    if (lane == 0) sc[j * lmax + (t - c0)] = __fdiv_rn(s, scale);
                }
            }
        }
    }
    __syncthreads();
    // per-head softmax statistics of this CTA's positions: warp j < G takes head j
    if (warp < G) {
        float* row = sc + warp * lmax;
        float m = -INFINITY;
        for (int t = lane; t < c1 - c0; t += 32) m = fmaxf(m, row[t]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
        float l = 0.f;
        for (int t = lane; t < c1 - c0; t += 32) {
            const float e = expf(__fsub_rn(row[t], m));
            row[t] = e;
            l += e;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, off);
        if (lane == 0) {
            mc[warp] = m;
            lc[warp] = l;
        }
    }
    __syncthreads();
    // o_c = sum_t exp(s_t - m_c) v_t
    float acc[G][4];
#pragma unroll
    for (int j = 0; j < G; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const float4 vn4 = *reinterpret_cast<const float4*>(vn + 4 * lane);
    for (int t0 = c0 + warp; t0 < c1; t0 += kAttnWarps * kU) {
        if (t0 != c0 + warp) {
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int t = t0 + u * kAttnWarps;
                vraw[u] = make_uint2(0u, 0u);
                if (t < c1 && t != p) vraw[u] = *reinterpret_cast<const uint2*>(vbase + (int64_t)t * kHeadDim);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = t0 + u * kAttnWarps;
            if (t >= c1) break;
            float v[4];
            if (t == p) {
                v[0] = vn4.x; v[1] = vn4.y; v[2] = vn4.z; v[3] = vn4.w;
            } else {
                half4_to_float(vraw[u], v);
            }
#pragma unroll
            for (int j = 0; j < G; ++j) {
                const float pj = sc[j * lmax + (t - c0)];
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[j][i] = fmaf(pj, v[i], acc[j][i]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < G; ++j)
        *reinterpret_cast<float4*>(stage + ((size_t)warp * G + j) * kHeadDim + 4 * lane) =
            make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    __syncthreads();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA of the cluster has started
    // push this CTA's unnormalised output of head j, and its m_c / l_c, into the owner CTA j
    for (int it = tid; it < G * kHeadDim; it += kAttnThreads) {
        float o = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kAttnWarps; ++w2) o += stage[(size_t)w2 * G * kHeadDim + it];
        const int j = it / kHeadDim;
        cluster.map_shared_rank(&ro[0][0], j)[crank * kHeadDim + it % kHeadDim] = o;
    }
    if (tid < G) {
        cluster.map_shared_rank(&rm[0], tid)[crank] = mc[tid];
        cluster.map_shared_rank(&rl[0], tid)[crank] = lc[tid];
    }
    cluster.sync();  // every push has landed; from here on each CTA reads only its own shared memory
    if (crank < G && tid < kHeadDim) {
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) M = fmaxf(M, rm[c]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
            const float m = rm[c];
            if (m == -INFINITY) continue;  // an empty range
            const float w = expf(__fsub_rn(m, M));
            L = fmaf(w, rl[c], L);
            o = fmaf(w, ro[c][tid], o);
        }
        o = __fdiv_rn(o, L);
        const int h = kvh * G + crank;
        if (o_out) o_out[(int64_t)h * kHeadDim + tid] = o;
        q8_1_block_store(o, q8 + ((int64_t)h * (kHeadDim / kQK8) + warp) * kQ8Bytes, lane);
    }
}

// act = silu(gate) * up for gu [T][2F] (gate columns [0, F), up columns [F, 2F)); Q8_1 blocks
// q8[T][F/32], one warp per block.
__global__ void __launch_bounds__(256) swiglu_q8_kernel(const float* __restrict__ gu, int64_t F, int64_t T,
                                                        uint8_t* __restrict__ q8) {
    grid_launch_dependents();
    grid_dependency_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nb = F / kQK8, total = nb * T;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t blk = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); blk < total; blk += nwarps) {
        const int64_t t = blk / nb, b = blk - t * nb;
        const float* row = gu + t * 2 * F + b * kQK8 + lane;
        const float g = row[0], u = row[F];
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        q8_1_block_store(__fmul_rn(silu, u), q8 + blk * kQ8Bytes, lane);
    }
}

// x[0..D) = the fp32 value of row *tok of the f16 embedding table emb [vocab][D] (the token is a
// device int64, so a captured decode step reads the token the previous step chose).  A token
// outside [0, vocab) records kDevErrToken and writes nothing.  D % 8 == 0, emb 16-byte aligned:
// one 16-byte load of 8 halves per thread.
__global__ void __launch_bounds__(256) embed_f16_kernel(const __half* __restrict__ emb, const int64_t* tok,
                                                        int64_t vocab, int64_t D, float* __restrict__ x,
                                                        uint32_t* err) {
    grid_launch_dependents();
    grid_dependency_wait();
    const int64_t t = *tok;
    if (t < 0 || t >= vocab) {
        if (blockIdx.x == 0 && threadIdx.x == 0) record_error(err, kDevErrToken);
        return;
    }
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (8 * i >= D) return;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(emb + t * D) + i);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    float4 lo, hi;
    float2 f = __half22float2(h[0]);
    lo.x = f.x;
    lo.y = f.y;
    f = __half22float2(h[1]);
    lo.z = f.x;
    lo.w = f.y;
    f = __half22float2(h[2]);
    hi.x = f.x;
    hi.y = f.y;
    f = __half22float2(h[3]);
    hi.z = f.x;
    hi.w = f.y;
    reinterpret_cast<float4*>(x)[2 * i] = lo;
    reinterpret_cast<float4*>(x)[2 * i + 1] = hi;
}

// Greedy sampling of one token: *tok = the index of the largest of v[0..n) (the first one on ties,
// NaN above every number: torch.argmax's result), then *pos += 1 when pos is not null.  One cluster
// of kArgCtas CTAs: CTA c scans [n*c/kArgCtas, n*(c+1)/kArgCtas) with coalesced loads, the CTAs'
// winners meet in CTA 0 through distributed shared memory.
constexpr int kArgCtas = 8;
constexpr int kArgThreads = 512;

// (a, ia) wins over (b, ib)
__device__ __forceinline__ bool argmax_better(float a, int64_t ia, float b, int64_t ib) {
    const bool na = a != a, nb = b != b;
    if (na != nb) return na;
    if (!na && a != b) return a > b;
    return ia < ib;
}

__global__ void __cluster_dims__(kArgCtas, 1, 1) __launch_bounds__(kArgThreads)
    argmax_kernel(const float* __restrict__ v, int64_t n, int64_t* tok, int64_t* pos) {
    namespace cg = cooperative_groups;
    grid_launch_dependents();
    grid_dependency_wait();
    __shared__ float wv[kArgThreads / 32];
    __shared__ int64_t wi[kArgThreads / 32];
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int64_t r0 = n * crank / kArgCtas, r1 = n * (crank + 1) / kArgCtas;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // four independent running winners per thread (loads in flight together), merged in index order
    float bv[4];
    int64_t bi[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        bv[k] = -INFINITY;
        bi[k] = INT64_MAX;
    }
    for (int64_t i0 = r0 + threadIdx.x; i0 < r1; i0 += 4 * kArgThreads) {
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t i = i0 + (int64_t)k * kArgThreads;
            x[k] = i < r1 ? __ldg(v + i) : -INFINITY;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t i = i0 + (int64_t)k * kArgThreads;
            if (i < r1 && argmax_better(x[k], i, bv[k], bi[k])) {
                bv[k] = x[k];
                bi[k] = i;
            }
        }
    }
#pragma unroll
    for (int k = 1; k < 4; ++k)
        if (argmax_better(bv[k], bi[k], bv[0], bi[0])) {
            bv[0] = bv[k];
            bi[0] = bi[k];
        }
    float b = bv[0];
    int64_t ib = bi[0];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xFFFFFFFFu, b, off);
        const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, ib, off);
        if (argmax_better(ob, oi, b, ib)) {
            b = ob;
            ib = oi;
        }
    }
    if (lane == 0) {
        wv[warp] = b;
        wi[warp] = ib;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgThreads / 32; ++w)
            if (argmax_better(wv[w], wi[w], wv[0], wi[0])) {
                wv[0] = wv[w];
                wi[0] = wi[w];
            }
    }
    cluster.sync();
    if (crank == 0 && threadIdx.x == 0) {
        float best = wv[0];
        int64_t bidx = wi[0];
        for (int c = 1; c < kArgCtas; ++c) {
            const float cv = *cluster.map_shared_rank(&wv[0], c);
            const int64_t ci = *cluster.map_shared_rank(&wi[0], c);
            if (argmax_better(cv, ci, best, bidx)) {
                best = cv;
                bidx = ci;
            }
        }
        *tok = bidx;
        if (pos) *pos += 1;
    }
    cluster.sync();  // keep the CTAs' winners alive until CTA 0 has read them
}

namespace {
cudaLaunchConfig_t launch_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                              cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}
}  // namespace

cudaError_t launch_residual_rmsnorm_q8(float* x, const float* delta, const float* w, int D, int T, float eps,
                                       uint8_t* q8, float* h_out, cudaStream_t stream, bool pdl,
                                       const iq4xs_peer_slots* peer) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_cfg(dim3(kNormCtas, (unsigned)T), dim3(kNormWarps * 32), 0, stream, pdl, attr);
    if (peer)
        return cudaLaunchKernelEx(&cfg, residual_rmsnorm_q8_kernel<true>, x, delta, w, D, eps, q8, h_out, peer,
                                  device_error_word());
    return cudaLaunchKernelEx(&cfg, residual_rmsnorm_q8_kernel<false>, x, delta, w, D, eps, q8, h_out, peer,
                              device_error_word());
}

// score row length per head: the longest position range of a CTA, rounded up to 4 floats so that
// the stage area after the rows stays 16-byte aligned
int attention_lmax(int max_seq) { return ((max_seq + kChunks - 1) / kChunks + 3) & ~3; }

size_t attention_decode_smem(int max_seq, int g) {
    return ((size_t)g * attention_lmax(max_seq) + (size_t)kAttnWarps * g * kHeadDim) * sizeof(float);
}

template <int G>
cudaError_t launch_attention_g(const float* qkv, __half* kc, __half* vc, const float* cosb, const float* sinb,
                               const int64_t* pos, int hq, int hkv, int max_seq, uint8_t* q8, float* o_out,
                               uint32_t* err, cudaStream_t stream, bool pdl, bool early_state) {
    const size_t smem = attention_decode_smem(max_seq, G);
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(attention_decode_q8_kernel<G>), (int)smem);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_cfg(dim3(kChunks, (unsigned)hkv), dim3(kAttnThreads), smem, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, attention_decode_q8_kernel<G>, qkv, kc, vc, cosb, sinb, pos, hq, hkv, max_seq,
                              attention_lmax(max_seq), q8, o_out, err, early_state && pdl);
}

cudaError_t launch_attention_decode_q8(const float* qkv, __half* kc, __half* vc, const float* cosb,
                                       const float* sinb, const int64_t* pos, int hq, int hkv, int max_seq,
                                       uint8_t* q8, float* o_out, uint32_t* err, cudaStream_t stream, bool pdl,
                                       bool early_state) {
    switch (hq / hkv) {
        case 1: return launch_attention_g<1>(qkv, kc, vc, cosb, sinb, pos, hq, hkv, max_seq, q8, o_out, err, stream, pdl, early_state);
        case 2: return launch_attention_g<2>(qkv, kc, vc, cosb, sinb, pos, hq, hkv, max_seq, q8, o_out, err, stream, pdl, early_state);
        case 4: return launch_attention_g<4>(qkv, kc, vc, cosb, sinb, pos, hq, hkv, max_seq, q8, o_out, err, stream, pdl, early_state);
        case 8: return launch_attention_g<8>(qkv, kc, vc, cosb, sinb, pos, hq, hkv, max_seq, q8, o_out, err, stream, pdl, early_state);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_swiglu_q8(const float* gu, int64_t F, int64_t T, uint8_t* q8, cudaStream_t stream, bool pdl) {
    const int64_t total = (F / kQK8) * T;
    const int64_t grid = std::min<int64_t>((total + 7) / 8, (int64_t)device_sm_count() * 8);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_cfg(dim3((unsigned)grid), dim3(256), 0, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, swiglu_q8_kernel, gu, F, T, q8);
}

cudaError_t launch_embed_f16(const __half* emb, const int64_t* tok, int64_t vocab, int64_t D, float* x,
                             cudaStream_t stream, bool pdl) {
    const int64_t grid = (D / 8 + 255) / 256;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_cfg(dim3((unsigned)grid), dim3(256), 0, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, embed_f16_kernel, emb, tok, vocab, D, x, device_error_word());
}

cudaError_t launch_argmax(const float* v, int64_t n, int64_t* tok, int64_t* pos, cudaStream_t stream, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_cfg(dim3(kArgCtas), dim3(kArgThreads), 0, stream, pdl, attr);
    return cudaLaunchKernelEx(&cfg, argmax_kernel, v, n, tok, pos);
}

}  // namespace iq4xs
