"""The CPU oracle pinned against the reference's own code and the committed golden vectors.

tests/golden/golden_v1.npz holds outputs of the reference's kernels/matmul_iq4xs/ref_cpu.cpp
(compiled unchanged into oracle/_ref/) on the reference tests' own inputs, plus the oracle's
quantised-pipeline outputs; tests/golden/make_golden.py regenerates them.
"""
import numpy as np
import pytest


def cases(golden):
    return [str(c) for c in golden["cases"]]


def test_fp16_truncation_matches_reference(O, golden):
    # block_iq4_xs.h:71-86 (the ds conversion of the Q8_1 quantizer, comparator.hip:45-58)
    x, want = golden["fp16/x"], golden["fp16/trunc"]
    got = np.array([O.lib().or_fp32_to_fp16_trunc(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(got, want)


def test_fp16_to_fp32_exact_all_bit_patterns(O):
    L = O.lib()
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([L.or_fp16_to_fp32(int(v)) for v in h], dtype=np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(got[finite], want[finite])
    assert np.array_equal(np.isinf(got), np.isinf(want))


@pytest.mark.parametrize("i", range(5))
def test_oracle_vs_reference_ref_cpu(O, golden, i):
    name = cases(golden)[i]
    K, N, M = (int(v) for v in golden[f"{name}/shape"])
    W, X = golden[f"{name}/W"], golden[f"{name}/X"]
    # Dequantisation: bit-exact with the reference's dequant_mat_iq4xs_cpu (ref_cpu.cpp:115-139).
    rows = golden[f"{name}/deq"].shape[0]
    assert np.array_equal(O.dequantize(W[:rows], K, rows), golden[f"{name}/deq"])
    # FP64 dequant-and-dot: bit-exact with gemv_iq4xs_cpu_ref (ref_cpu.cpp:12-52), same op order.
    assert np.array_equal(O.matmul_f64(W, X, K, N, M), golden[f"{name}/Yref"])
    # gemm_iq4xs_cpu_ref (X [K][M], Y [N][M]) computes the same sums.
    assert np.array_equal(golden[f"{name}/Yref_gemm"].T, golden[f"{name}/Yref"])


@pytest.mark.parametrize("i", range(5))
def test_quantised_pipeline_regression_and_accuracy(O, golden, i):
    name = cases(golden)[i]
    K, N, M = (int(v) for v in golden[f"{name}/shape"])
    W, X = golden[f"{name}/W"], golden[f"{name}/X"]
    Q = O.quantize_q8_1(X)
    assert np.array_equal(Q, golden[f"{name}/Q"])
    S = O.subblock_dots(W, Q, K, N, M)
    assert np.array_equal(S, golden[f"{name}/S"])
    Y64, A = O.matmul_q8(W, Q, K, N, M)
    assert np.array_equal(Y64, golden[f"{name}/Y64"])
    assert np.array_equal(A, golden[f"{name}/A"])
    # The quantised pipeline against the reference's unquantised FP64 oracle: the reference gates
    # its DP4A path at cosine >= 0.99 and measured 0.999985 (BASELINE_DP4A.md:28-32).
    cos = O.cosine(Y64, golden[f"{name}/Yref"])
    assert cos >= 0.9999, cos


def test_fp32_reference_order_close_to_fp64(O, golden):
    name = "attn_q_trunc"
    K, N, M = (int(v) for v in golden[f"{name}/shape"])
    Y32 = O.matmul_q8_f32(golden[f"{name}/W"], golden[f"{name}/Q"], K, N, M)
    Y64, A = golden[f"{name}/Y64"], golden[f"{name}/A"]
    assert np.all(np.abs(Y32 - Y64) <= O.tolerance(Y64, A, K // 32))


@pytest.mark.parametrize("kind", ["port", "reference"])
def test_threaded_cpu_gemv_matches_reference_outputs(O, golden, kind):
    # The CPU baseline's row-sliced GEMV (bench.py's reference arm) with either implementation
    # reproduces gemv_iq4xs_cpu_ref's outputs bit for bit, whatever the slicing.
    if kind == "reference" and not O.ref_available():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    name = cases(golden)[0]
    K, N, M = (int(v) for v in golden[f"{name}/shape"])
    W, X, Yref = golden[f"{name}/W"], golden[f"{name}/X"].reshape(M, K), golden[f"{name}/Yref"]
    for threads in (1, 3):
        for m in range(M):
            y = O.ref_gemv_threaded(W, X[m], K, N, threads, kind=kind)
            assert np.array_equal(y, Yref[m])
