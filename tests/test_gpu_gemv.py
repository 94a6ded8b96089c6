"""GPU parity of the Q8_1 quantizer and the decode GEMV, called through the C ABI.

Bar: Q8_1 bytes and int32 sub-block dots bit-exact with the oracle; fp32
outputs within |y - y64| <= 1e-5 * max(|y64|, sum|terms|/sqrt(n_terms)) of the FP64 oracle of the
quantised pipeline, and cosine >= 0.999999.  The reference's own gate against its unquantised FP64
oracle (cosine >= 0.99 for the DP4A path, test_real_stock_compare.cpp:41; >= 0.999 for the coop
GEMV, test_gemv_dp4a_compare.cpp:157) is checked as well on the reference tests' own inputs.
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


# ----------------------------------------------------------------------------- Q8_1 quantizer
@pytest.mark.parametrize("K,M,scale", [(256, 1, 1.0), (5120, 3, 1.0), (17408, 8, 0.01), (4096, 2, 1e4), (1024, 5, 1e-6)])
def test_q8_1_bitexact(pkg, O, K, M, scale):
    X = (np.random.default_rng(K + M).standard_normal((M, K)) * scale).astype(np.float32)
    X[0, :32] = 0.0                                   # all-zero block
    X[-1, 32:64] = np.arange(32, dtype=np.float32) - 15.5  # x/d ties: amax 16.5 is not a tie maker,
    X[-1, 64:96] = 0.0
    X[-1, 64], X[-1, 65], X[-1, 66] = 127.0, 2.5, -2.5    # amax 127 -> d = 1, exact .5 ties
    got = pkg.q8_1_quantize(dev(X)).cpu().numpy()
    assert np.array_equal(got, O.quantize_q8_1(X))


def test_q8_1_reference_batched_layout(pkg, O):
    K, M = 1024, 6
    X = np.random.default_rng(5).standard_normal((M, K)).astype(np.float32)
    Xkm = dev(np.ascontiguousarray(X.T))             # reference playground layout X[k*M+m]
    Y = torch.empty((M, K // 32 * 36), dtype=torch.uint8, device="cuda")
    pkg.quantize_row_q8_1_batched_gpu(Xkm, Y, K, M)
    assert np.array_equal(Y.cpu().numpy(), O.quantize_q8_1(X))
    y1 = torch.empty(K // 32 * 36, dtype=torch.uint8, device="cuda")
    pkg.quantize_row_q8_1_gpu(dev(X[2]), y1, K)
    assert np.array_equal(y1.cpu().numpy(), O.quantize_q8_1(X[2:3])[0])


# ----------------------------------------------------------------------------- small shapes vs C oracle
SMALL = [(512, 64, b) for b in range(1, 9)] + [
    (5120, 100, 3), (17408, 40, 8), (4096, 131, 2), (256, 33, 8), (768, 17, 2), (8192, 9, 5), (1024, 1, 1)]


@pytest.mark.parametrize("K,N,B", SMALL)
def test_gemv_small_vs_oracle(pkg, O, K, N, B):
    W = O.random_blocks(K, N, 9000 + K * 7919 + N)
    X = O.normal(B * K, 42 + B).reshape(B, K)
    Q = O.quantize_q8_1(X)
    Wd, Qd = dev(W), dev(Q)
    S = pkg.debug_subblock_dots(Wd, Qd, K, N, B).cpu().numpy()
    assert np.array_equal(S, O.subblock_dots(W, Q, K, N, B))
    Y64, A = O.matmul_q8(W, Q, K, N, B)
    Y = pkg.gemv_q8(Wd, Qd, K, N, B).cpu().numpy()
    check_close(O, Y, Y64, A, K, f"bulk K={K} N={N} B={B}")
    Yg = pkg.gemv_q8(Wd, Qd, K, N, B, generic=True).cpu().numpy()
    check_close(O, Yg, Y64, A, K, f"generic K={K} N={N} B={B}")
    Yf = pkg.gemv(Wd, dev(X), N).cpu().numpy()       # fp32 entry point: quantize + GEMV (PDL)
    assert np.array_equal(Yf, Y)
    no_device_error(pkg)


def test_golden_vectors_on_gpu(pkg, O, golden):
    for name in golden["cases"]:
        name = str(name)
        K, N, M = (int(v) for v in golden[f"{name}/shape"])
        W, X = golden[f"{name}/W"], golden[f"{name}/X"]
        q8 = pkg.q8_1_quantize(dev(X))
        assert np.array_equal(q8.cpu().numpy(), golden[f"{name}/Q"])
        S = pkg.debug_subblock_dots(dev(W), q8, K, N, M).cpu().numpy()
        assert np.array_equal(S, golden[f"{name}/S"])
        Y = pkg.gemv_q8(dev(W), q8, K, N, M).cpu().numpy()
        check_close(O, Y, golden[f"{name}/Y64"], golden[f"{name}/A"], K, name)
        # against the reference's own FP64 CPU oracle (unquantised activations)
        assert O.cosine(Y, golden[f"{name}/Yref"]) >= 0.9999


def test_torch_reference_matches_c_oracle(pkg, O):
    K, N, B = 2048, 96, 3
    W = O.random_blocks(K, N, 11)
    X = O.normal(B * K, 12).reshape(B, K)
    Q = O.quantize_q8_1(X)
    Y64, A = O.matmul_q8(W, Q, K, N, B)
    T64, TA = torch_ref.matmul_q8(dev(W), dev(Q), K)
    assert np.allclose(T64.cpu().numpy(), Y64, rtol=1e-12, atol=1e-12)
    assert np.allclose(TA.cpu().numpy(), A, rtol=1e-12, atol=0)
    assert np.array_equal(torch_ref.subblock_dots(dev(W), dev(Q), K).cpu().numpy().astype(np.int64),
                          O.subblock_dots(W, Q, K, N, B).astype(np.int64))


# ----------------------------------------------------------------------------- BASELINE shapes, full size
SHAPES = {  # name: (N out, K in)
    "c1_4096": (4096, 4096),
    "q_proj": (8192, 5120), "k_proj": (1024, 5120), "o_proj": (5120, 8192),
    "gate": (17408, 5120), "gate_up": (34816, 5120), "down": (5120, 17408),
    "lm_head": (152064, 5120),  # the row-sharded matrix of the multi-GPU config, whole
}


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("B", [1, 2, 4, 8])
def test_gemv_full_size(pkg, O, name, B):
    N, K = SHAPES[name]
    W = pkg.random_weights(N, K, seed=1000 + list(SHAPES).index(name))
    X = pkg.fill_normal(B * K, seed=42 + B).view(B, K)
    q8 = pkg.q8_1_quantize(X)
    Y = pkg.gemv_q8(W, q8, K, N, B)
    T64, TA = torch_ref.matmul_q8(W, q8, K)
    check_close(O, Y.cpu().numpy(), T64.cpu().numpy(), TA.cpu().numpy(), K, f"{name} B={B}")
    # sampled rows against the C oracle (bytes copied back), and raw dots bit-exact
    rows = np.random.default_rng(B).choice(N, size=6, replace=False)
    Wr = W[torch.as_tensor(rows, device="cuda")].contiguous()
    Qh = q8.cpu().numpy()
    Y64, A = O.matmul_q8(Wr.cpu().numpy(), Qh, K, len(rows), B)
    check_close(O, Y.cpu().numpy()[:, rows], Y64, A, K, f"{name} B={B} sampled")
    S = pkg.debug_subblock_dots(Wr, q8, K, len(rows), B).cpu().numpy()
    assert np.array_equal(S, O.subblock_dots(Wr.cpu().numpy(), Qh, K, len(rows), B))
    # row-range independence: a sub-matrix gives the same rows (bit for bit with the batch-1 kernel,
    # whose per-row order does not depend on N; within tolerance for the tensor-core kernel, whose
    # K-part grouping is chosen per shape)
    r0 = N // 3
    r1 = min(N, r0 + 777)
    Ys = pkg.gemv_q8(W[r0:r1].contiguous(), q8, K, r1 - r0, B)
    if B == 1:
        assert torch.equal(Ys, Y[:, r0:r1])
    else:
        check_close(O, Ys.cpu().numpy(), T64.cpu().numpy()[:, r0:r1], TA.cpu().numpy()[:, r0:r1], K, f"{name} slice")
    no_device_error(pkg)


# ----------------------------------------------------------------------------- reference tests' inputs
def test_reference_gemv_dp4a_compare_inputs(pkg, O):
    """test_gemv_dp4a_compare.cpp: 8 canonical shapes + syn_512 + syn_1024 with its seeds, one
    mt19937(42) across shapes; gate cosine >= 0.999 vs the reference's FP64 CPU oracle."""
    shapes = [(5120, 5120), (5120, 5120), (5120, 5120), (5120, 6144), (5120, 5120), (5120, 17408),
              (5120, 17408), (17408, 5120), (512, 512), (1024, 2048)]
    xs = O.normal_seq([K for K, _ in shapes], 42)
    for (K, N), x in zip(shapes, xs):
        W = O.random_blocks(K, N, 9000 + K * 7919 + N)
        y_ref = O.ref_gemv_threaded(W, x, K, N, O.host_threads())   # the reference's own oracle
        Wd, xd = dev(W), dev(x)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        pkg.gemv_iq4xs_dp4a_coop_gpu(Wd, xd, y, K, N)
        y = y.cpu().numpy()
        assert O.cosine(y, y_ref) >= 0.999
        Q = O.quantize_q8_1(x[None])
        rows = np.arange(0, N, max(1, N // 64))
        Y64, A = O.matmul_q8(W[rows], Q, K, len(rows), 1)
        check_close(O, y[None, rows], Y64, A, K, f"ref-input K={K} N={N}")


def test_reference_named_entry_points_agree(pkg, O):
    K, N = 5120, 6144
    W = O.random_blocks(K, N, 4)
    x = O.normal(K, 5)
    Wd, xd = dev(W), dev(x)
    outs = []
    for fn in (pkg.gemv_iq4xs_dp4a_coop_gpu, pkg.gemv_iq4xs_stock_dp4a_gpu):
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        fn(Wd, xd, y, K, N)
        outs.append(y)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    assert pkg.custom_gemv_iq4xs_dispatch(Wd, xd, y, K, N) == 0
    outs.append(y)
    ref = pkg.gemv(Wd, xd[None], N)[0]
    for o in outs:
        assert torch.equal(o, ref)
    Xb = dev(O.normal(3 * K, 6).reshape(3, K))
    yb = torch.empty((3, N), dtype=torch.float32, device="cuda")
    assert pkg.custom_gemv_iq4xs_dispatch_batched(Wd, Xb, yb, K, N, 3) == 0
    assert torch.equal(yb, pkg.gemv(Wd, Xb, N))
    no_device_error(pkg)


def test_invalid_arguments_on_device(pkg, O):
    L = pkg.lib()
    K, N = 512, 16
    W = dev(O.random_blocks(K, N, 1))
    q8 = pkg.q8_1_quantize(dev(O.normal(K, 2)[None]))
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(pkg.gemv_q8_workspace_bytes(K, N, 1), dtype=torch.uint8, device="cuda")
    wsb = ws.numel()
    assert L.iq4xs_gemv_q8(W.data_ptr() + 4, q8.data_ptr(), y.data_ptr(), K, N, 1, ws.data_ptr(), wsb, s) == 3
    assert L.iq4xs_gemv_q8(W.data_ptr(), q8.data_ptr(), y.data_ptr(), K, N, 9, ws.data_ptr(), wsb, s) == 2
    # 8-byte aligned but not 16: served by the direct-load kernel, same result
    buf = torch.empty(W.numel() + 8, dtype=torch.uint8, device="cuda")
    buf[8:] = W.view(-1)
    y8 = torch.empty(N, dtype=torch.float32, device="cuda")
    assert L.iq4xs_gemv_q8(buf.data_ptr() + 8, q8.data_ptr(), y8.data_ptr(), K, N, 1, ws.data_ptr(), wsb, s) == 0
    yg = pkg.gemv_q8(W, q8, K, N, 1, generic=True)
    assert torch.equal(y8, yg[0])
    no_device_error(pkg)


def test_cuda_graph_capture_replays_bit_exact(pkg, O):
    K, N, B = 5120, 8192, 2
    W = pkg.random_weights(N, K, seed=9)
    X = pkg.fill_normal(B * K, seed=10).view(B, K)
    ws = torch.zeros(pkg.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    pkg.gemv(W, X, N, workspace=ws, out=Y)
    ref = Y.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            pkg.gemv(W, X, N, workspace=ws, out=Y, stream=s)
    Y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(Y, ref)
    del g
    no_device_error(pkg)


# ----------------------------------------------------------------------------- weight format
def test_weight_quantizer_gpu_bitexact(pkg, O):
    src = pkg.fill_normal(48 * 1024, seed=77, std=0.02).view(48, 1024)
    src[3, :256] = 0.0
    src[5, 256:288] = 1e-20
    W = pkg.quantize_weights(src).cpu().numpy()
    assert np.array_equal(W, O.quantize_iq4_xs(src.cpu().numpy()))
    deq = pkg.dequantize(dev(W), 1024, 48).cpu().numpy()
    assert np.array_equal(deq, O.dequantize(W, 1024, 48))


def test_fill_normal_statistics(pkg):
    x = pkg.fill_normal(1 << 22, seed=3, mean=0.0, std=0.02)
    assert abs(x.mean().item()) < 1e-4
    assert abs(x.std().item() - 0.02) < 2e-4
    y = pkg.fill_normal(1 << 22, seed=3, mean=0.0, std=0.02)
    assert torch.equal(x, y)
