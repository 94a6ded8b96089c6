"""Row-sharded GEMV / GEMM through the CUDA path with NCCL on 2 GPUs (skipped on a box with fewer),
against the single-GPU kernels on the full matrix: the GEMM and the batch-1 GEMV
are per-row identical (bit-exact), batched GEMV partial sums may be split differently (tolerance)."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch.distributed as dist
    import torch_ref
    from conftest import load_pkg
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        P = load_pkg()
        res = []
        for N, K in [(6144, 5120), (1000, 1024)]:
            W = P.random_weights(N, K, seed=77)                       # same full matrix on every rank
            r0, r1 = P.sharded.shard_rows(N, world, rank)
            S = P.sharded.RowShardedIQ4XS(W[r0:r1].contiguous(), N, K)
            for B in (1, 3):
                X = P.fill_normal(B * K, seed=5 + B).view(B, K)
                Y = S.gemv(X)
                Yf = P.gemv(W, X, N)
                if B == 1:
                    res.append(bool(torch.equal(Y, Yf)))
                else:
                    Y64, A = torch_ref.matmul_q8(W, P.q8_1_quantize(X), K)
                    tol = torch.from_numpy(O.tolerance(Y64.cpu().numpy(), A.cpu().numpy(), K // 32, 1e-5))
                    res.append(bool(((Y.cpu().double() - Y64.cpu()).abs() <= tol).all()))
            M = 200
            Xm = P.fill_normal(M * K, seed=9).view(M, K)
            Yt = S.gemm_nm(Xm)
            res.append(bool(torch.equal(Yt, P.gemm(W, Xm, N).t())))
        torch.cuda.synchronize()
        q.put((rank, res, P.device_error()))
    finally:
        dist.destroy_process_group()


def test_row_sharded_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    from conftest import run_ranks
    out, codes = run_ranks(_worker, world, lambda r, port, q: (r, world, port, q), timeout=300)
    assert all(c == 0 for c in codes), codes
    assert len(out) == world
    for rank, res, err in out:
        assert all(res), (rank, res)
        assert err == 0
