// ref_inputs.cpp -- the reference tests' synthetic inputs, regenerated bit for bit.
//
// TEST INFRASTRUCTURE ONLY.  Restates gen_iq4xs_weights (kernels/common/matmul_test_util.h:49-67:
// std::mt19937(seed); d ~ U(0.008,0.6) stored through the truncating fp32->fp16; scales_h, scales_l
// and qs uniform random) and the activation draw used by every reference test
// (std::mt19937 + std::normal_distribution<float>(0,1), e.g. test_gemv_dp4a_compare.cpp:124-126),
// with the same standard-library engines, so the parity tests run on the reference's own inputs.
#include <cstdint>
#include <random>

#include "iq4xs_oracle.h"

extern "C" {

void or_gen_iq4xs_random_blocks(or_block_iq4_xs* W, int64_t K, int64_t N, uint32_t seed) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> d_dist(0.008f, 0.6f);
    std::uniform_int_distribution<int> sh_dist(0, 65535), b_dist(0, 255);
    const int64_t total = N * (K / OR_QK_K);
    for (int64_t i = 0; i < total; ++i) {
        const float dv = d_dist(rng);
        W[i].d = or_fp32_to_fp16_trunc(dv);
        W[i].scales_h = static_cast<uint16_t>(sh_dist(rng));
        for (int k = 0; k < 4; ++k) W[i].scales_l[k] = static_cast<uint8_t>(b_dist(rng));
        for (int k = 0; k < 128; ++k) W[i].qs[k] = static_cast<uint8_t>(b_dist(rng));
    }
}

// Draws n N(0,1) floats from one engine; state continues across calls through *state_out
// only when the caller keeps using the same seed sequence, so tests simply draw all values
// of one case in a single call, matching a reference loop over a fresh engine.
void or_gen_normal(float* x, int64_t n, uint32_t seed, float mean, float stddev) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> g(mean, stddev);
    for (int64_t i = 0; i < n; ++i) x[i] = g(rng);
}

}  // extern "C"

extern "C" {

// Sequential draws of several test cases from ONE std::mt19937(seed) with a fresh
// std::normal_distribution<float>(0,1) per case: the pattern of the reference tests, which
// keep a single engine in main() and construct the distribution inside each per-shape
// function (e.g. test_gemv_dp4a_compare.cpp:124-126,180).  counts[i] values go to out in order.
void or_gen_normal_seq(float* out, const int64_t* counts, int ncounts, uint32_t seed) {
    std::mt19937 rng(seed);
    for (int c = 0; c < ncounts; ++c) {
        std::normal_distribution<float> g(0.0f, 1.0f);
        for (int64_t i = 0; i < counts[c]; ++i) *out++ = g(rng);
    }
}

}  // extern "C"
