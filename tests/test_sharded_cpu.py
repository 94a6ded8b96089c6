"""Host logic of the row-sharded matmuls on CPU ranks (gloo, world size 2 and 3).

The local matmul is the C oracle here (injected), so the test covers the row partition, the
padding of uneven shards and the assembly of the gathered output, not the CUDA kernels (those are
covered on the GPU by test_gpu_sharded.py).
"""
import os

import numpy as np
import pytest
import torch


def _worker(rank, world, port, N, K, B, M, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch.distributed as dist
    from conftest import load_pkg
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = load_pkg().sharded
        W = O.random_blocks(K, N, 1234)
        r0, r1 = sh.shard_rows(N, world, rank)

        def gemv_fn(Wl, X):
            Xn = X.numpy()
            Y64, _ = O.matmul_q8(Wl.numpy(), O.quantize_q8_1(Xn), K, Wl.shape[0], Xn.shape[0])
            return torch.from_numpy(Y64.astype(np.float32))

        def gemm_fn(Wl, X):
            return gemv_fn(Wl, X).t().contiguous()

        S = sh.RowShardedIQ4XS(torch.from_numpy(W[r0:r1].copy()), N, K, local_gemv=gemv_fn, local_gemm=gemm_fn)
        X = torch.from_numpy(O.normal(B * K, 7).reshape(B, K))
        Y = S.gemv(X)
        Xm = torch.from_numpy(O.normal(M * K, 8).reshape(M, K))
        Yt = S.gemm_nm(Xm)
        full, _ = O.matmul_q8(W, O.quantize_q8_1(X.numpy()), K, N, B)
        fullm, _ = O.matmul_q8(W, O.quantize_q8_1(Xm.numpy()), K, N, M)
        ok = (tuple(Y.shape) == (B, N) and np.array_equal(Y.numpy(), full.astype(np.float32)) and
              tuple(Yt.shape) == (N, M) and np.array_equal(Yt.numpy(), fullm.astype(np.float32).T))
        q.put((rank, ok, (r0, r1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 96), (2, 100), (3, 200)])
def test_row_sharded_gather_gloo(world, N):
    K, B, M = 512, 3, 5
    from conftest import run_ranks
    out, codes = run_ranks(_worker, world, lambda r, port, q: (r, world, port, N, K, B, M, q), timeout=240)
    assert all(c == 0 for c in codes), codes
    res = sorted(out)
    assert all(ok for _, ok, _ in res), res
    # the shards tile [0, N) with whole 16-row tiles
    bounds = [b for _, _, b in res]
    assert bounds[0][0] == 0 and bounds[-1][1] == N
    assert all(bounds[i][1] == bounds[i + 1][0] for i in range(world - 1))
    assert all(b[0] % 16 == 0 for b in bounds)


def test_shard_rows_properties():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from conftest import load_pkg
    sh = load_pkg().sharded
    for N in (1, 16, 17, 152064, 34816, 5120, 1000):
        for world in (1, 2, 3, 4, 8):
            rs = [sh.shard_rows(N, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == N
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 16
    assert sh.shard_rows(152064, 8, 3) == (57024, 76032)


class _FakePeers:
    """peer.PeerGroup's interface on CPU ranks: the areas are local tensors and the all-gather is
    gloo's, so the row-sharded GEMV's peer path (area alternation, padded slices, assembly) runs
    here; the NVLink kernel itself is covered on 2 GPUs by test_gpu_peer.py."""

    def __init__(self, area_floats, areas, world):
        self.bufs = [torch.zeros(area_floats) for _ in range(areas)]
        self.world = world
        self.used = []

    def area(self, i, n):
        self.used.append(i)
        return self.bufs[i][:n]

    def allgather(self, i, n, out):
        import torch.distributed as dist
        dist.all_gather_into_tensor(out.view(-1)[:self.world * n], self.bufs[i][:n].contiguous())
        return out


def _peer_worker(rank, world, port, N, K, B, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch.distributed as dist
    from conftest import load_pkg
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = load_pkg().sharded
        W = O.random_blocks(K, N, 4321)
        r0, r1 = sh.shard_rows(N, world, rank)

        def gemv_fn(Wl, X):
            Xn = X.numpy()
            Y64, _ = O.matmul_q8(Wl.numpy(), O.quantize_q8_1(Xn), K, Wl.shape[0], Xn.shape[0])
            return torch.from_numpy(Y64.astype(np.float32))

        peers = _FakePeers(B * sh.max_shard_rows(N, world), 2, world)
        S = sh.RowShardedIQ4XS(torch.from_numpy(W[r0:r1].copy()), N, K, local_gemv=gemv_fn, local_gemm=gemv_fn,
                               peers=peers)
        ok = True
        for it in range(3):
            X = torch.from_numpy(O.normal(B * K, 70 + it).reshape(B, K))
            Y = S.gemv(X)
            full, _ = O.matmul_q8(W, O.quantize_q8_1(X.numpy()), K, N, B)
            ok &= tuple(Y.shape) == (B, N) and np.array_equal(Y.numpy(), full.astype(np.float32))
        q.put((rank, ok, peers.used))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 96), (3, 200)])
def test_row_sharded_peer_path_gloo(world, N):
    K, B = 512, 2
    from conftest import run_ranks
    out, codes = run_ranks(_peer_worker, world, lambda r, port, q: (r, world, port, N, K, B, q), timeout=240)
    assert all(c == 0 for c in codes), codes
    res = sorted(out)
    assert all(ok for _, ok, _ in res), res
    assert all(used == [0, 1, 0] for _, _, used in res)  # consecutive collectives alternate areas
