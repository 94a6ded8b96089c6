"""iq4xs_gemv_grouped: independent GEMVs of one batch size in one launch sequence.

Every problem's output is checked against the FP64 restatement of the quantised pipeline (the
tolerance of the other GEMV tests) and against the single-matrix entry point iq4xs_gemv_f32 on the
same inputs: bit for bit at batch 1 (the row kernel's per-row order does not depend on the CTA
count), within tolerance at batch 2..8 (the grouped launch may split K into parts differently).
Groups: the six 27B-class layer shapes of the benchmark (the row and tensor-core grouped kernels,
with and without K parts), a q/k/v group sharing one activation, and groups the grouped kernels do
not take (odd K/256, an unaligned W) that run as one call per problem."""
import numpy as np
import pytest
import torch

import torch_ref

pytestmark = pytest.mark.gpu

REL = 1e-5
LAYER = [(8192, 5120), (1024, 5120), (1024, 5120), (5120, 8192), (34816, 5120), (5120, 17408)]


def check(pkg, O, W, X, Y, what):
    K = X.shape[1]
    q8 = pkg.q8_1_quantize(X)
    T64, TA = torch_ref.matmul_q8(W, q8, K)
    tol = O.tolerance(T64.cpu().numpy(), TA.cpu().numpy(), K // 32, REL)
    err = np.abs(Y.cpu().numpy().astype(np.float64) - T64.cpu().numpy())
    assert np.all(err <= tol), f"{what}: {np.sum(err > tol)} outside tolerance, worst {np.max(err / tol):.3g}"
    assert O.cosine(Y.cpu().numpy(), T64.cpu().numpy()) >= 0.999999


def run_group(pkg, shapes, B, seed):
    Ws = [pkg.random_weights(N, K, seed=seed + i) for i, (N, K) in enumerate(shapes)]
    Xs = [pkg.fill_normal(B * K, seed=seed + 100 + i).view(B, K) for i, (N, K) in enumerate(shapes)]
    Ys = [torch.full((B, N), float("nan"), dtype=torch.float32, device="cuda") for N, K in shapes]
    pkg.gemv_grouped(list(zip(Ws, Xs, Ys)))
    torch.cuda.synchronize()
    return Ws, Xs, Ys


@pytest.mark.parametrize("B", [1, 2, 4, 8])
def test_grouped_layer_shapes(pkg, O, B):
    Ws, Xs, Ys = run_group(pkg, LAYER, B, 7000 + 10 * B)
    for i, ((N, K), W, X, Y) in enumerate(zip(LAYER, Ws, Xs, Ys)):
        single = pkg.gemv(W, X, N)
        torch.cuda.synchronize()
        if B == 1:
            assert torch.equal(Y, single), f"problem {i} ({N}x{K})"
        check(pkg, O, W, X, Y, f"grouped B={B} problem {i} ({N}x{K})")
    assert pkg.device_error() == 0


def test_grouped_qkv_one_activation_twice(pkg, O):
    """q, k, v of one token (the same X for the three matrices), two calls in a row on one workspace:
    the second call's results do not depend on what the first left behind."""
    shapes = [(8192, 5120), (1024, 5120), (1024, 5120)]
    Ws = [pkg.random_weights(N, K, seed=7300 + i) for i, (N, K) in enumerate(shapes)]
    need = pkg.gemv_grouped_workspace_bytes([(K, N) for N, K in shapes], 3)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    for call in range(2):
        X = pkg.fill_normal(3 * 5120, seed=7310 + call).view(3, 5120)
        Ys = [torch.empty((3, N), dtype=torch.float32, device="cuda") for N, K in shapes]
        pkg.gemv_grouped([(W, X, Y) for W, Y in zip(Ws, Ys)], workspace=ws)
        torch.cuda.synchronize()
        for W, Y, (N, K) in zip(Ws, Ys, shapes):
            check(pkg, O, W, X, Y, f"qkv call {call} N={N}")
    assert pkg.device_error() == 0


@pytest.mark.parametrize("B", [1, 3])
def test_grouped_fallback_per_problem(pkg, O, B):
    """Odd K/256 and a W that is only 8-byte aligned: one iq4xs_gemv_f32_ex per problem, the same bits
    as the single-matrix entry point."""
    shapes = [(1000, 768), (640, 2304), (512, 5120)]
    Ws = [pkg.random_weights(N, K, seed=7400 + i) for i, (N, K) in enumerate(shapes)]
    rb = 5120 // 256 * 136
    buf = torch.empty(512 * rb + 8, dtype=torch.uint8, device="cuda")
    Wu = buf[8:8 + 512 * rb].view(512, rb)          # 8 mod 16: the direct-load kernel
    Wu.copy_(Ws[2])
    Ws[2] = Wu
    Xs = [pkg.fill_normal(B * K, seed=7410 + i).view(B, K) for i, (N, K) in enumerate(shapes)]
    Ys = [torch.empty((B, N), dtype=torch.float32, device="cuda") for N, K in shapes]
    pkg.gemv_grouped(list(zip(Ws, Xs, Ys)))
    torch.cuda.synchronize()
    for W, X, Y, (N, K) in zip(Ws, Xs, Ys, shapes):
        assert torch.equal(Y, pkg.gemv(W, X, N))
        check(pkg, O, W, X, Y, f"fallback B={B} {N}x{K}")
    assert pkg.device_error() == 0


def test_grouped_validation(pkg):
    L = pkg.lib()
    K, N, B = 5120, 256, 2
    W = pkg.random_weights(N, K, seed=1)
    X = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    arr = pkg.api._problems([(W, X, Y)])
    need = int(L.iq4xs_gemv_grouped_workspace_bytes(arr, 1, B))
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert L.iq4xs_gemv_grouped(arr, 1, B, ws.data_ptr(), need - 1, 0, s) == 4      # workspace too small
    assert L.iq4xs_gemv_grouped(arr, 1, 9, ws.data_ptr(), need, 0, s) == 2          # batch
    assert L.iq4xs_gemv_grouped(arr, 9, B, ws.data_ptr(), need, 0, s) == 2          # group size
    assert L.iq4xs_gemv_grouped(arr, 0, B, ws.data_ptr(), need, 0, s) == 1
    assert L.iq4xs_gemv_grouped(arr, 1, B, ws.data_ptr() + 128, need, 0, s) == 3    # workspace alignment
    bad = pkg.api._problems([(W, X, Y)])
    bad[0].K = 1000
    assert L.iq4xs_gemv_grouped(bad, 1, B, ws.data_ptr(), need, 0, s) == 2
    assert L.iq4xs_gemv_grouped(arr, 1, B, ws.data_ptr(), need, 0, s) == 0
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
