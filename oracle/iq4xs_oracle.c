/*
 * iq4xs_oracle.c -- CPU restatement of the reference IQ4_XS x Q8_1 pipeline.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  Compiled with
 * -ffp-contract=off so every float operation rounds exactly once, in source order.
 * File paths in citations are relative to the reference project root.
 */
#include "iq4xs_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* kernels/common/block_iq4_xs.h:22-24 */
const int8_t or_kvalues_iq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                     1,    13,   25,  38,  53,  69,  89,  113};

static float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* Exact half -> float.  kernels/common/block_iq4_xs.h:34-68 (subnormals renormalised). */
float or_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1F;
    uint32_t m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return bits_to_f32(sign);
        /* subnormal: value = m * 2^-24 exactly representable in fp32 */
        float v = (float)m * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (e == 31) return bits_to_f32(sign | 0x7F800000u | (m << 13));
    return bits_to_f32(sign | ((uint32_t)(e + 112) << 23) | (m << 13));
}

/* Truncating float -> half used for the Q8_1 ds pair.
 * kernels/common/block_iq4_xs.h:71-86 and real_stock_dp4a_comparator.hip:45-58:
 * the mantissa is cut to 10 bits (no rounding); exponents below the half range
 * shift the (already cut) mantissa into a subnormal; overflow and NaN both give inf. */
uint16_t or_fp32_to_fp16_trunc(float f) {
    uint32_t x = f32_to_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t m = (x >> 13) & 0x3FFu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m = (m | 0x400u) >> (1 - e);
        return (uint16_t)(sign | m);
    }
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

/* Round-to-nearest-even float -> half (used for the weight super-block scale d). */
uint16_t or_fp32_to_fp16_rne(float f) {
    uint32_t x = f32_to_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to >= 65520 -> inf */
    if (ax < 0x38800000u) {                                      /* below 2^-14: subnormal half */
        /* value / 2^-24, rounded to nearest even integer */
        float v = bits_to_f32(ax) * 16777216.0f;
        float r = nearbyintf(v);
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = ((ax >> 23) - 112) << 10;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t h = e | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

/* Scale decode, ref_cpu.cpp:30-34 / real_stock_dp4a_comparator.hip:162. */
int or_iq4xs_scale(const or_block_iq4_xs* b, int ib) {
    int lo = (b->scales_l[ib / 2] >> (4 * (ib & 1))) & 0x0F;
    int hi = (b->scales_h >> (2 * ib)) & 0x03;
    return lo | (hi << 4);
}

/* Q8_1 quantizer, device form of real_stock_dp4a_comparator.hip:230-264.
 * amax and sum are reduced with the 32-lane xor butterfly (offsets 16,8,4,2,1);
 * every lane ends with the same value, reproduced here lane by lane in fp32.
 * d = amax/127 (IEEE division); q = (int8)roundf(x/d) (half away from zero); amax==0 -> q=0.
 * ds = {trunc16(d), trunc16(sum)}. */
void or_quantize_q8_1(const float* X, or_block_q8_1* Y, int64_t K, int64_t M) {
    const int64_t nb = K / OR_QK8_1;
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t ib = 0; ib < nb; ++ib) {
            const float* x = X + m * K + ib * OR_QK8_1;
            float amax[32], sum[32];
            for (int l = 0; l < 32; ++l) { amax[l] = fabsf(x[l]); sum[l] = x[l]; }
            for (int off = 16; off > 0; off >>= 1) {
                float na[32], ns[32];
                for (int l = 0; l < 32; ++l) {
                    na[l] = fmaxf(amax[l], amax[l ^ off]);
                    ns[l] = sum[l] + sum[l ^ off];
                }
                memcpy(amax, na, sizeof na);
                memcpy(sum, ns, sizeof ns);
            }
            const float a = amax[0];
            const float d = a / 127.0f;
            or_block_q8_1* y = Y + m * nb + ib;
            for (int l = 0; l < 32; ++l) {
                int8_t q = 0;
                if (a != 0.0f) q = (int8_t)roundf(x[l] / d);
                y->qs[l] = q;
            }
            y->d = or_fp32_to_fp16_trunc(d);
            y->s = or_fp32_to_fp16_trunc(sum[0]);
        }
    }
}

/* Raw sub-block dot.  vec_dot_iq4_xs_q8_1 (real_stock_dp4a_comparator.hip:145-160):
 * qs byte j (0..15) of sub-block ib holds element j in its low nibble and element j+16
 * in its high nibble (codebook gather :105-131); int8 x int8 products summed in int32. */
int32_t or_subblock_dot(const or_block_iq4_xs* b, int ib, const or_block_q8_1* q) {
    const uint8_t* qs = b->qs + 16 * ib;
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        s += (int32_t)or_kvalues_iq4nl[qs[j] & 0x0F] * (int32_t)q->qs[j];
        s += (int32_t)or_kvalues_iq4nl[qs[j] >> 4] * (int32_t)q->qs[j + 16];
    }
    return s;
}

void or_subblock_dots(const or_block_iq4_xs* W, const or_block_q8_1* Q, int32_t* S,
                      int64_t K, int64_t N, int64_t M) {
    const int64_t kb = K / OR_QK_K, nb = K / OR_QK8_1;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            for (int64_t sb = 0; sb < nb; ++sb)
                S[(m * N + n) * nb + sb] =
                    or_subblock_dot(W + n * kb + sb / 8, (int)(sb % 8), Q + m * nb + sb);
}

/* real_stock_dp4a_comparator.hip:162-165: sumi *= ls-32; d = f32(w.d)*f32(ds.lo); d*(float)sumi. */
float or_term_f32(const or_block_iq4_xs* b, int ib, const or_block_q8_1* q) {
    const int32_t sumi = or_subblock_dot(b, ib, q) * (or_iq4xs_scale(b, ib) - 32);
    const float d = or_fp16_to_fp32(b->d) * or_fp16_to_fp32(q->d);
    return d * (float)sumi;
}

void or_matmul_q8(const or_block_iq4_xs* W, const or_block_q8_1* Q, double* Y, double* A,
                  int64_t K, int64_t N, int64_t M) {
    const int64_t kb = K / OR_QK_K, nb = K / OR_QK8_1;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0, aabs = 0.0;
            for (int64_t sb = 0; sb < nb; ++sb) {
                const double t = (double)or_term_f32(W + n * kb + sb / 8, (int)(sb % 8), Q + m * nb + sb);
                acc += t;
                aabs += fabs(t);
            }
            Y[m * N + n] = acc;
            if (A) A[m * N + n] = aabs;
        }
}

/* fp32 accumulation in the order of gemv_iq4xs_stock_dp4a_kernel
 * (real_stock_dp4a_comparator.hip:325-360): lane t sums super-blocks kbx = t/8 + 4i at
 * sub-block (t%8), then the 32 lanes reduce with the xor butterfly. */
void or_matmul_q8_f32(const or_block_iq4_xs* W, const or_block_q8_1* Q, float* Y,
                      int64_t K, int64_t N, int64_t M) {
    const int64_t kb = K / OR_QK_K, nb = K / OR_QK8_1;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float lane[32];
            for (int t = 0; t < 32; ++t) {
                float tmp = 0.0f;
                for (int64_t kbx = t / 8; kbx < kb; kbx += 4)
                    tmp += or_term_f32(W + n * kb + kbx, t % 8, Q + m * nb + kbx * 8 + t % 8);
                lane[t] = tmp;
            }
            for (int off = 16; off > 0; off >>= 1) {
                float nl[32];
                for (int t = 0; t < 32; ++t) nl[t] = lane[t] + lane[t ^ off];
                memcpy(lane, nl, sizeof nl);
            }
            Y[m * N + n] = lane[0];
        }
}

/* ref_cpu.cpp:12-52 restated for token-major X [M][K] and Y [M][N]. */
void or_matmul_f64(const or_block_iq4_xs* W, const float* X, float* Y, int64_t K, int64_t N, int64_t M) {
    const int64_t kb = K / OR_QK_K;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t b = 0; b < kb; ++b) {
                const or_block_iq4_xs* blk = W + n * kb + b;
                const float d = or_fp16_to_fp32(blk->d);
                for (int ib = 0; ib < 8; ++ib) {
                    const double dl = (double)d * (double)((float)or_iq4xs_scale(blk, ib) - 32.0f);
                    const float* x = X + m * K + b * OR_QK_K + ib * 32;
                    for (int j = 0; j < 16; ++j) {
                        const uint8_t v = blk->qs[16 * ib + j];
                        acc += dl * (double)or_kvalues_iq4nl[v & 0x0F] * (double)x[j];
                        acc += dl * (double)or_kvalues_iq4nl[v >> 4] * (double)x[j + 16];
                    }
                }
            }
            Y[m * N + n] = (float)acc;
        }
}

/* ref_cpu.cpp:115-139. */
void or_dequantize(const or_block_iq4_xs* W, float* out, int64_t K, int64_t N) {
    const int64_t kb = K / OR_QK_K;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t b = 0; b < kb; ++b) {
            const or_block_iq4_xs* blk = W + n * kb + b;
            const float d = or_fp16_to_fp32(blk->d);
            for (int ib = 0; ib < 8; ++ib) {
                const float dl = d * ((float)or_iq4xs_scale(blk, ib) - 32.0f);
                float* y = out + n * K + b * OR_QK_K + ib * 32;
                for (int j = 0; j < 16; ++j) {
                    const uint8_t v = blk->qs[16 * ib + j];
                    y[j] = dl * (float)or_kvalues_iq4nl[v & 0x0F];
                    y[j + 16] = dl * (float)or_kvalues_iq4nl[v >> 4];
                }
            }
        }
}

/* ------------------------------------------------------------------------------------------
 * IQ4_XS weight quantizer.  The reference calls upstream ggml's quantize_row_iq4_xs
 * (llama.cpp bb4caa75, benchmarks/environment/llamacpp-pin.txt) which is not vendored.
 * Restated algorithm, no importance matrix:
 *   per 32-weight sub-block: weights w_j = x_j^2; take the signed extreme xmax; start from
 *   scale xmax/127 and refine the least-squares scale sum(w q x)/sum(w q q) over 15 trial
 *   inverse scales (t + kv[0])/xmax, t = -7..7, keeping the one maximising (sum w q x)^2/sum w q q;
 *   per super-block: d = -max_scale/32 (the scale of largest magnitude maps to -32), each
 *   sub-block scale rounded to an integer l in [-32,31], codes re-chosen with scale d*l,
 *   stored ls = l+32 (4 low bits in scales_l, 2 high bits in scales_h), d stored as fp16 (RNE).
 * Float expressions are evaluated one rounding at a time in the order written here, and the
 * two 32-term sums of each trial use the warp xor-butterfly order, so that a warp-per-super-block
 * GPU quantizer can reproduce every bit.
 * ------------------------------------------------------------------------------------------ */
static int nearest_code(float v) {
    const int8_t* kv = or_kvalues_iq4nl;
    if (v <= (float)kv[0]) return 0;
    if (v >= (float)kv[15]) return 15;
    int lo = 0, hi = 15;
    while (hi - lo > 1) {
        const int mid = (lo + hi) / 2;
        if (v < (float)kv[mid]) hi = mid; else lo = mid;
    }
    return (v - (float)kv[hi - 1] < (float)kv[hi] - v) ? hi - 1 : hi;
}

static int round_half_even(float v) { return (int)nearbyintf(v); }

/* 32-lane xor-butterfly sum (offsets 16,8,4,2,1), the order a warp reduction produces. */
static float butterfly_sum32(const float* v) {
    float a[32];
    memcpy(a, v, sizeof a);
    for (int off = 16; off > 0; off >>= 1) {
        float n[32];
        for (int l = 0; l < 32; ++l) n[l] = a[l] + a[l ^ off];
        memcpy(a, n, sizeof a);
    }
    return a[0];
}

/* sum_j w_j q_j x_j and sum_j w_j q_j^2 for the codes chosen with inverse scale id. */
static void trial_sums(const float* xb, const float* w, float id, uint8_t* L, float* sumqx, float* sumq2) {
    float t1[32], t2[32];
    for (int j = 0; j < 32; ++j) {
        const int l = nearest_code(id * xb[j]);
        if (L) L[j] = (uint8_t)l;
        const float q = (float)or_kvalues_iq4nl[l];
        const float wq = w[j] * q;
        t1[j] = wq * xb[j];
        t2[j] = wq * q;
    }
    *sumqx = butterfly_sum32(t1);
    *sumq2 = butterfly_sum32(t2);
}

static void quantize_superblock(const float* x, or_block_iq4_xs* out) {
    float scales[8];
    uint8_t L[256];
    float max_scale = 0.0f, amax_scale = 0.0f;
    memset(L, 0, sizeof L);
    for (int ib = 0; ib < 8; ++ib) {
        const float* xb = x + 32 * ib;
        float w[32];
        float amax = 0.0f, xmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            w[j] = xb[j] * xb[j];
            const float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; xmax = xb[j]; }  /* first index of the largest |x| */
        }
        if (amax < 1e-15f) { scales[ib] = 0.0f; continue; }
        float d = -xmax / (float)or_kvalues_iq4nl[0];
        float sumqx, sumq2;
        trial_sums(xb, w, 1.0f / d, L + 32 * ib, &sumqx, &sumq2);
        d = sumqx / sumq2;
        float best = d * sumqx;
        for (int t = -7; t <= 7; ++t) {
            const float id = ((float)t + (float)or_kvalues_iq4nl[0]) / xmax;
            trial_sums(xb, w, id, NULL, &sumqx, &sumq2);
            if (sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                d = sumqx / sumq2;
                best = d * sumqx;
            }
        }
        scales[ib] = d;
        const float ad = fabsf(d);
        if (ad > amax_scale) { amax_scale = ad; max_scale = d; }
    }
    memset(out, 0, sizeof *out);
    const float d = -max_scale / 32.0f;
    out->d = or_fp32_to_fp16_rne(d);
    const float id = (d != 0.0f) ? 1.0f / d : 0.0f;
    for (int ib = 0; ib < 8; ++ib) {
        int l = round_half_even(id * scales[ib]);
        if (l < -32) l = -32;
        if (l > 31) l = 31;
        const float dl = d * (float)l;
        const float idl = (dl != 0.0f) ? 1.0f / dl : 0.0f;
        for (int j = 0; j < 32; ++j) L[32 * ib + j] = (uint8_t)nearest_code(idl * x[32 * ib + j]);
        l += 32;
        if (ib % 2 == 0) out->scales_l[ib / 2] = (uint8_t)(l & 0xF);
        else out->scales_l[ib / 2] |= (uint8_t)((l & 0xF) << 4);
        out->scales_h |= (uint16_t)((l >> 4) << (2 * ib));
    }
    for (int ib = 0; ib < 8; ++ib)
        for (int j = 0; j < 16; ++j)
            out->qs[16 * ib + j] = (uint8_t)(L[32 * ib + j] | (L[32 * ib + 16 + j] << 4));
}

void or_quantize_iq4_xs(const float* src, or_block_iq4_xs* dst, int64_t nrows, int64_t n_per_row) {
    const int64_t kb = n_per_row / OR_QK_K;
    for (int64_t r = 0; r < nrows; ++r)
        for (int64_t b = 0; b < kb; ++b)
            quantize_superblock(src + r * n_per_row + b * OR_QK_K, dst + r * kb + b);
}
