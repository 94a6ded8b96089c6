"""iq4xs_gemv_f32_noalloc: the fp32 GEMV for callers that cannot allocate device memory.

Such callers (a ggml hook inside a graph whose memory is planned ahead, a runtime that forbids
cudaMalloc once serving because it synchronises the device) pass only inputs and outputs; the
entry point keeps its scratch in a static 4 MiB device array.  Checked here through the C ABI
against the workspace entry point iq4xs_gemv_f32 (bit for bit) and the FP64 restatement (with the
tolerance the other GEMV tests use), on two calls in a row.  This file is named to run last.
"""
import numpy as np
import pytest
import torch

import torch_ref

pytestmark = pytest.mark.gpu

REL = 1e-5


def call_noalloc(pkg, W, X, N):
    B, K = X.shape
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    st = pkg.lib().iq4xs_gemv_f32_noalloc(W.data_ptr(), X.data_ptr(), Y.data_ptr(), K, N, B,
                                          torch.cuda.current_stream().cuda_stream)
    return st, Y


@pytest.mark.parametrize("N,K,B", [(8192, 5120, 1), (34816, 5120, 8), (5120, 17408, 4), (4096, 4096, 2)])
def test_noalloc_matches_workspace_entry_point(pkg, O, N, K, B):
    W = pkg.random_weights(N, K, seed=5150 + B)
    for call in range(2):  # two calls in a row, different inputs
        X = pkg.fill_normal(B * K, seed=100 * call + B).view(B, K)
        st, Y = call_noalloc(pkg, W, X, N)
        assert st == 0, pkg.STATUS.get(st)
        ws = torch.zeros(pkg.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
        Yref = pkg.gemv(W, X, N, workspace=ws)
        torch.cuda.synchronize()
        q8 = pkg.q8_1_quantize(X)
        T64, TA = torch_ref.matmul_q8(W, q8, K)
        tol = O.tolerance(T64.cpu().numpy(), TA.cpu().numpy(), K // 32, REL)
        y, yr = Y.cpu().numpy().astype(np.float64), Yref.cpu().numpy().astype(np.float64)
        assert np.array_equal(y, yr)  # same kernels, same activation policy: the same bits
        assert np.all(np.abs(y - T64.cpu().numpy()) <= tol)
    assert pkg.device_error() == 0


def test_noalloc_batch1_long_rows_need_no_partials(pkg):
    # Batch 1 with K <= 24576 runs the row kernel, which writes no partial sums: only the 18 KiB of
    # Q8_1 activations count against the static scratch, so an lm_head-sized N is accepted.  (The
    # tensor-core path at this shape would want ~4.3 MiB of partial sums.)
    N, K, B = 152064, 16384, 1
    W = pkg.random_weights(N, K, seed=5160)
    ws = torch.zeros(pkg.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
    for call in range(2):
        X = pkg.fill_normal(B * K, seed=300 + call).view(B, K)
        st, Y = call_noalloc(pkg, W, X, N)
        assert st == 0, pkg.STATUS.get(st)
        Yref = pkg.gemv(W, X, N, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(Y, Yref)
    assert pkg.device_error() == 0


@pytest.mark.parametrize("N,K,B,x_offset", [(3000, 4096, 2, 1), (2048, 768, 3, 0), (1000, 2304, 1, 1)])
def test_noalloc_fallback_paths(pkg, N, K, B, x_offset):
    # The standalone quantizer into the static array, then the GEMV on those Q8_1 blocks: taken when X
    # is not 16-byte aligned (x_offset = 1 float) or when K/256 is odd (the direct-load kernel).
    W = pkg.random_weights(N, K, seed=5170 + K)
    ws = torch.zeros(pkg.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
    for call in range(2):
        buf = pkg.fill_normal(B * K + 4, seed=400 + call)
        X = buf[x_offset:x_offset + B * K].view(B, K)
        st, Y = call_noalloc(pkg, W, X, N)
        assert st == 0, pkg.STATUS.get(st)
        Yref = pkg.gemv(W, X, N, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(Y, Yref)
    assert pkg.device_error() == 0


def test_noalloc_rejects_oversized_scratch(pkg):
    # K = 524288 at batch 8 needs 4.5 MiB of Q8_1 activations alone, more than the 4 MiB of static
    # scratch: refused before any launch (W and X are full size all the same).
    N, K, B = 16, 524288, 8
    W = torch.zeros((N, K // 256 * 136), dtype=torch.uint8, device="cuda")
    X = torch.zeros((B, K), dtype=torch.float32, device="cuda")
    st, _ = call_noalloc(pkg, W, X, N)
    assert st == 4  # IQ4XS_ERR_WORKSPACE_TOO_SMALL
    assert pkg.device_error() == 0
