"""GPU parity of the tensor-core prefill GEMM (tcgen05 + TMEM), called through the C ABI.

Same bar as the GEMV: the activation quants bit-exact with the Q8_1 oracle; fp32 outputs within
|y - y64| <= 1e-5 * max(|y64|, sum|terms|/sqrt(n_terms)) of the FP64 oracle of the quantised
pipeline and cosine >= 0.999999.  The reference's own GEMM tests (test_real_stock_compare.cpp,
test_gemm_wmma_compare.cpp) gate cosine >= 0.99 / 0.999 against its unquantised FP64 oracle;
their inputs are replayed here as well.
"""
import numpy as np
import pytest
import torch

import torch_ref

pytestmark = pytest.mark.gpu

REL = 1e-5
COS = 0.999999


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check_close(O, Y, Y64, A, K, what=""):
    Y = np.asarray(Y, dtype=np.float64)
    tol = O.tolerance(Y64, A, K // 32, REL)
    err = np.abs(Y - Y64)
    bad = err > tol
    assert not bad.any(), f"{what}: {bad.sum()} outside tolerance, worst ratio {np.max(err / tol):.3g}"
    assert O.cosine(Y, Y64) >= COS, f"{what}: cosine {O.cosine(Y, Y64)}"


def no_device_error(pkg):
    torch.cuda.synchronize()
    assert pkg.device_error() == 0


def lookup_positions():
    """Element e = 4w+i+16j of a 32-block sits at position 8w+2i+j in the GEMM's fp16 quants."""
    e = np.arange(32)
    return 8 * ((e & 15) >> 2) + 2 * (e & 3) + (e >> 4)


# ----------------------------------------------------------------------------- activation quantiser
@pytest.mark.parametrize("K,M,scale", [(512, 1, 1.0), (5120, 37, 1.0), (17408, 16, 1e-3), (1024, 130, 1e4)])
def test_gemm_quantize_bitexact(pkg, O, K, M, scale):
    X = (np.random.default_rng(K + M).standard_normal((M, K)) * scale).astype(np.float32)
    X[0, :32] = 0.0
    X[-1, 64:96] = 0.0
    X[-1, 64], X[-1, 65], X[-1, 66] = 127.0, 2.5, -2.5   # d = 1: exact .5 ties round away from zero
    xq, xs = pkg.debug_gemm_quantize(dev(X))
    Q = O.quantize_q8_1(X).reshape(M, K // 32, 36)
    q = Q[:, :, 4:].view(np.int8).astype(np.float32)          # [M][K/32][32] by element
    d = Q[:, :, 0:2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    got = xq.cpu().numpy().astype(np.float32).reshape(M, K // 32, 32)
    assert np.array_equal(got[:, :, lookup_positions()], q)
    assert np.array_equal(xs.cpu().numpy().T, d)


@pytest.mark.parametrize("K,M,scale", [(512, 1, 1.0), (5120, 37, 1.0), (17408, 16, 1e-3), (1024, 130, 1e4)])
def test_gemm_i8_quantize_bitexact(pkg, O, K, M, scale):
    """The int8 GEMM's quantiser: the Q8_1 quants as int8 and the fp32 value of each block's fp16 d."""
    X = (np.random.default_rng(K + M + 1).standard_normal((M, K)) * scale).astype(np.float32)
    X[0, :32] = 0.0
    X[-1, 64], X[-1, 65], X[-1, 66] = 127.0, 2.5, -2.5
    xq, xs = pkg.debug_gemm_i8_quantize(dev(X))
    Q = O.quantize_q8_1(X).reshape(M, K // 32, 36)
    q = Q[:, :, 4:].view(np.int8)
    d = Q[:, :, 0:2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    got = xq.cpu().numpy().reshape(M, K // 32, 32)
    assert np.array_equal(got[:, :, lookup_positions()], q)
    assert np.array_equal(xs.cpu().numpy().T, d)


# ----------------------------------------------------------------------------- small shapes vs C oracle
SMALL = [(512, 128, 128), (512, 100, 37), (1024, 256, 16), (2048, 384, 300), (5120, 200, 130),
         (17408, 130, 20), (8192, 64, 256), (512, 1, 1), (1024, 129, 129), (512, 256, 640)]


KINDS = ["i8", "f16"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("K,N,M", SMALL)
def test_gemm_small_vs_oracle(pkg, O, K, N, M, kind):
    W = O.random_blocks(K, N, 777 + K * 31 + N)
    X = O.normal(M * K, 11 + M).reshape(M, K)
    Q = O.quantize_q8_1(X)
    Y64, A = O.matmul_q8(W, Q, K, N, M)
    Y = pkg.gemm(dev(W), dev(X), N, kind=kind).cpu().numpy()
    check_close(O, Y, Y64, A, K, f"gemm {kind} K={K} N={N} M={M}")
    no_device_error(pkg)


def test_gemm_kinds_agree_and_default(pkg, O):
    """int8 and fp16 operands give the same integer dots; their outputs differ only by the order of
    the fp32 scale products (a few ulp), and the default call is the fp16 kernel bit for bit."""
    K, N, M = 5120, 768, 200
    W = dev(O.random_blocks(K, N, 55))
    X = dev(O.normal(M * K, 56).reshape(M, K))
    Yi = pkg.gemm(W, X, N, kind="i8")
    Yf = pkg.gemm(W, X, N, kind="f16")
    assert torch.equal(pkg.gemm(W, X, N), Yf)
    Y64, A = torch_ref.matmul_q8(W, pkg.q8_1_quantize(X), K)
    tol = O.tolerance(Y64.cpu().numpy(), A.cpu().numpy(), K // 32, REL)
    assert np.all(np.abs(Yi.cpu().numpy() - Yf.cpu().numpy()) <= tol)
    no_device_error(pkg)


def test_gemm_deterministic_and_matches_gemv(pkg, O):
    K, N, M = 5120, 1000, 8
    W = dev(O.random_blocks(K, N, 31))
    X = dev(O.normal(M * K, 32).reshape(M, K))
    Y1 = pkg.gemm(W, X, N)
    Y2 = pkg.gemm(W, X, N)
    assert torch.equal(Y1, Y2)
    Yv = pkg.gemv(W, X, N)
    Y64, A = torch_ref.matmul_q8(W, pkg.q8_1_quantize(X), K)
    tol = O.tolerance(Y64.cpu().numpy(), A.cpu().numpy(), K // 32, REL)
    assert np.all(np.abs(Y1.cpu().numpy() - Yv.cpu().numpy()) <= 2 * tol)
    no_device_error(pkg)


# ----------------------------------------------------------------------------- full C3 shapes
def torch_ref_chunked(W, q8, K, rows=4096, toks=256):
    N, M = W.shape[0], q8.shape[0]
    Y = torch.empty((M, N), dtype=torch.float64, device=W.device)
    A = torch.empty((M, N), dtype=torch.float64, device=W.device)
    for r0 in range(0, N, rows):
        r1 = min(N, r0 + rows)
        for t0 in range(0, M, toks):
            t1 = min(M, t0 + toks)
            y, a = torch_ref.matmul_q8(W[r0:r1], q8[t0:t1], K)
            Y[t0:t1, r0:r1] = y
            A[t0:t1, r0:r1] = a
    return Y, A


C3 = [("q_proj", 8192, 5120), ("k_proj", 1024, 5120), ("o_proj", 5120, 8192), ("gate_up", 34816, 5120),
      ("down", 5120, 17408)]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("M", [512, 2048])
@pytest.mark.parametrize("name,N,K", C3)
def test_gemm_full_shapes(pkg, O, name, N, K, M, kind):
    W = pkg.random_weights(N, K, seed=4242 + N + K)
    X = pkg.fill_normal(M * K, seed=99 + M).view(M, K)
    Y = pkg.gemm(W, X, N, kind=kind)
    q8 = pkg.q8_1_quantize(X)
    if M == 2048 and N * M > 2048 * 8192:
        # full torch check on a slab of rows, C oracle on sampled rows
        rs = slice(N // 2, N // 2 + 2048)
        Y64, A = torch_ref_chunked(W[rs], q8, K)
        Yc = Y[:, rs]
    else:
        Y64, A = torch_ref_chunked(W, q8, K)
        Yc = Y
    tol = O.tolerance(Y64.cpu().numpy(), A.cpu().numpy(), K // 32, REL)
    err = np.abs(Yc.cpu().numpy().astype(np.float64) - Y64.cpu().numpy())
    assert np.all(err <= tol), f"{name} M={M}: {np.sum(err > tol)} outside, worst {np.max(err / tol):.3g}"
    rows = np.unique(np.linspace(0, N - 1, 24).astype(np.int64))
    Wn = W.cpu().numpy()
    Qn = q8.cpu().numpy()
    Y64c, Ac = O.matmul_q8(Wn[rows], Qn, K, len(rows), M)
    check_close(O, Y.cpu().numpy()[:, rows], Y64c, Ac, K, f"{name} M={M} sampled rows")
    no_device_error(pkg)


# ----------------------------------------------------------------------------- reference entry points
def test_reference_named_gemm_layouts(pkg, O):
    K, N, M = 5120, 640, 96
    W = dev(O.random_blocks(K, N, 8))
    X = O.normal(M * K, 9).reshape(M, K)
    Xd = dev(X)
    ref = pkg.gemm(W, Xd, N)
    Xkm = dev(np.ascontiguousarray(X.T))        # playground layout X[k*M+m]
    for fn in (pkg.gemm_iq4xs_stock_dp4a_gpu, pkg.gemm_iq4xs_wmma_stream_gpu):
        Ynm = torch.empty((N, M), dtype=torch.float32, device="cuda")
        fn(W, Xkm, Ynm, K, N, M)
        assert torch.equal(Ynm.t(), ref)
    Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    assert pkg.custom_gemm_iq4xs_dispatch(W, Xd, Y, K, N, M) == 0
    assert torch.equal(Y, ref)
    assert pkg.custom_gemm_iq4xs_can_handle(K, N, M)
    assert not pkg.custom_gemm_iq4xs_can_handle(K, N, 8)       # small batches stay on the GEMV
    assert pkg.custom_gemm_iq4xs_can_handle(768, N, M)         # odd super-block count (patch:150)
    assert not pkg.custom_gemm_iq4xs_can_handle(1000, N, M)    # not whole super-blocks
    assert not pkg.custom_gemm_iq4xs_can_handle(K, N, M, 2)    # not IQ4_XS
    no_device_error(pkg)


def test_reference_gemm_test_inputs(pkg, O):
    """test_real_stock_compare.cpp: GEMV shapes then six GEMM cases from one mt19937(42); weights
    from gen_iq4xs_weights(54321 + K*31 + N); X in the playground layout [K][M].  Gate here: cosine
    >= 0.999 vs the reference's FP64 oracle on a row slice (the reference gates 0.99), plus the
    quantised FP64 oracle's tolerance."""
    canon = [(5120, 5120), (5120, 5120), (5120, 5120), (5120, 6144), (5120, 5120), (5120, 17408),
             (5120, 17408), (17408, 5120)]
    gemm = [(5120, 5120, 16), (5120, 5120, 128), (5120, 17408, 16), (5120, 17408, 128), (17408, 5120, 16),
            (17408, 5120, 128)]
    counts = [K for K, _ in canon] + [512] + [K * M for K, _, M in gemm]
    draws = O.normal_seq(counts, 42)[len(canon) + 1:]
    for (K, N, M), x in zip(gemm, draws):
        W = O.random_blocks(K, N, (54321 + K * 31 + N) & 0xFFFFFFFF)
        Xkm = x.reshape(K, M)
        Ynm = torch.empty((N, M), dtype=torch.float32, device="cuda")
        pkg.gemm_iq4xs_stock_dp4a_gpu(dev(W), dev(Xkm), Ynm, K, N, M)
        Ynm = Ynm.cpu().numpy()
        rows = 192
        y_ref = O.ref_gemm(W[:rows], Xkm, K, rows, M)             # reference FP64 oracle, [rows][M]
        assert O.cosine(Ynm[:rows], y_ref) >= 0.999
        Q = O.quantize_q8_1(np.ascontiguousarray(Xkm.T))
        Y64, A = O.matmul_q8(W[:rows], Q, K, rows, M)
        check_close(O, Ynm[:rows].T, Y64, A, K, f"ref-input K={K} N={N} M={M}")
    no_device_error(pkg)


def test_gemm_invalid_arguments(pkg, O):
    L = pkg.lib()
    K, N, M = 1024, 64, 32
    W = dev(O.random_blocks(K, N, 1))
    X = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ws = torch.zeros(pkg.gemm_workspace_bytes(K, M), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nb = ws.numel()
    assert L.iq4xs_gemm(W.data_ptr(), X.data_ptr(), Y.data_ptr(), 1000, N, M, ws.data_ptr(), nb, s) == 2
    # odd K/256 runs in the ggml output layout only
    assert L.iq4xs_gemm_strided(W.data_ptr(), X.data_ptr(), 768, 1, Y.data_ptr(), 1, M, 768, N, M, ws.data_ptr(),
                                nb, s) == 2
    assert L.iq4xs_gemm(W.data_ptr(), X.data_ptr(), Y.data_ptr(), K, N, 0, ws.data_ptr(), nb, s) == 1
    assert L.iq4xs_gemm(None, X.data_ptr(), Y.data_ptr(), K, N, M, ws.data_ptr(), nb, s) == 1
    assert L.iq4xs_gemm(W.data_ptr(), X.data_ptr(), Y.data_ptr(), K, N, M, ws.data_ptr(), nb - 1, s) == 4
    assert L.iq4xs_gemm(W.data_ptr() + 8, X.data_ptr(), Y.data_ptr(), K, N - 1, M, ws.data_ptr(), nb, s) == 3
    assert L.iq4xs_gemm(W.data_ptr(), X.data_ptr(), Y.data_ptr(), K, N, M, ws.data_ptr(), nb, s) == 0
    for bad_flags in (0x30, 0x1, 0x40):   # both kinds, or an unknown bit
        assert L.iq4xs_gemm_ex(W.data_ptr(), X.data_ptr(), K, 1, Y.data_ptr(), N, 1, K, N, M, ws.data_ptr(), nb,
                               bad_flags, s) == 1
    for kind in (0x10, 0x20):
        assert L.iq4xs_gemm_ex(W.data_ptr(), X.data_ptr(), K, 1, Y.data_ptr(), N, 1, K, N, M, ws.data_ptr(), nb,
                               kind, s) == 0
    no_device_error(pkg)


@pytest.mark.parametrize("K,N,M", [(768, 640, 16), (2304, 1000, 100), (1280, 272, 37)])
def test_gemm_odd_superblock_count(pkg, O, K, N, M):
    """K/256 odd (the patch's hook takes any K % 256 == 0, patch:148-151): the ggml dispatch and
    iq4xs_gemm quantise to Q8_1 and run the direct-load kernel 8 tokens at a time; checked against
    the C oracle of the quantised pipeline (tolerance) and the batched GEMV on the same tokens (bits)."""
    W = dev(O.random_blocks(K, N, 777 + K))
    X = O.normal(M * K, 31 + M).reshape(M, K)
    Xd = dev(X)
    assert pkg.custom_gemm_iq4xs_can_handle(K, N, M)
    Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    assert pkg.custom_gemm_iq4xs_dispatch(W, Xd, Y, K, N, M) == 0
    Y2 = pkg.gemm(W, Xd, N)
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)
    Q = O.quantize_q8_1(X)
    Y64, A = O.matmul_q8(W.cpu().numpy(), Q, K, N, M)
    check_close(O, Y.cpu().numpy(), Y64, A, K, f"odd K={K} N={N} M={M}")
    for m0 in range(0, M, 8):  # the same bits as the GEMV entry point on each chunk of tokens
        Yg = pkg.gemv(W, Xd[m0:m0 + 8].contiguous(), N)
        assert torch.equal(Yg, Y[m0:m0 + 8])
    no_device_error(pkg)


@pytest.mark.parametrize("kind", KINDS)
def test_gemm_deterministic_and_row_independent(pkg, kind):
    """The same GEMM repeated gives the same bits, in both output layouts, and a row slice of W gives
    the same rows (each output element's sum order depends on K only): what the row-sharded GEMM
    across GPUs relies on.  The transposed-layout calls take the default kind."""
    N, K, M = 34816, 5120, 256
    W = pkg.random_weights(N, K, seed=901)
    X = pkg.fill_normal(M * K, seed=902).view(M, K)
    ref = pkg.gemm(W, X, N, kind=kind)
    for _ in range(6):
        Y = pkg.gemm(W, X, N, kind=kind)
        bad = (Y != ref).sum().item()
        assert bad == 0, f"repeat differs in {bad} elements, max {float((Y - ref).abs().max())}"
    if kind != "f16":
        no_device_error(pkg)
        return
    h = N // 2
    halves = torch.cat([pkg.gemm_nm(W[:h].contiguous(), X, h), pkg.gemm_nm(W[h:].contiguous(), X, N - h)])
    bad = (halves != ref.t()).sum().item()
    assert bad == 0, f"row halves differ in {bad} elements, max {float((halves - ref.t()).abs().max())}"
    no_device_error(pkg)
