"""Row-sharded IQ4_XS matmuls over the GPUs of one node (one process per GPU, torch.distributed).

The weight matrix W [N][K] is split by output rows: every row is independent, so each rank owns a
contiguous range of whole 16-row tiles (the GEMV tile height), multiplies it by the full activations
(quantised to Q8_1 locally on every rank) and the only exchange is one all-gather of the output
slices (NCCL over NVLink).  Shapes where N splits evenly (lm_head 152064 and gate|up 34816 at 2, 4
and 8 ranks) gather without padding; otherwise slices are padded to the largest one.

    GEMV (batch B <= 8): local y [B][Nr] -> gathered [P][B][Nr] -> Y [B][N]
    GEMM (M tokens):     local Y^T [Nr][M] (row shard = one contiguous block) -> gathered Y^T [N][M]

The local compute goes through the C ABI (iq4xs_gemv_f32 / iq4xs_gemm_strided).  `local_gemv` /
`local_gemm` replace it only in tests that run the host logic on CPU ranks (gloo).

With a `peers` group (peer.PeerGroup) the GEMV (decode-size outputs) writes its slice straight into
this rank's peer-memory area and the all-gather is the NVLink pull kernel of csrc/peer.cu instead of
NCCL; the GEMM output (tens to hundreds of MB) always goes through NCCL.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

TILE_ROWS = 16


def shard_rows(N: int, world: int, rank: int) -> Tuple[int, int]:
    """Row range [r0, r1) of `rank`: whole 16-row tiles, balanced over `world` ranks."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    tiles = (N + TILE_ROWS - 1) // TILE_ROWS
    t0 = tiles * rank // world
    t1 = tiles * (rank + 1) // world
    return min(N, t0 * TILE_ROWS), min(N, t1 * TILE_ROWS)


def max_shard_rows(N: int, world: int) -> int:
    return max(r1 - r0 for r0, r1 in (shard_rows(N, world, r) for r in range(world)))


class RowShardedIQ4XS:
    """One rank's share of a row-sharded IQ4_XS matrix.

    W_local: this rank's rows [r1 - r0][K/256*136] (uint8, on this rank's GPU), as produced by
    shard_rows(N, world, rank) applied to the full matrix (or quantised there directly).
    """

    def __init__(self, W_local, N: int, K: int, group=None, rank: Optional[int] = None, world: Optional[int] = None,
                 local_gemv: Optional[Callable] = None, local_gemm: Optional[Callable] = None, peers=None,
                 peer_areas=(0, 1)):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.N, self.K = N, K
        self.r0, self.r1 = shard_rows(N, self.world, self.rank)
        self.rows = self.r1 - self.r0
        self.pad = max_shard_rows(N, self.world)
        if W_local.shape[0] != self.rows:
            raise ValueError(f"rank {self.rank}: expected {self.rows} weight rows, got {W_local.shape[0]}")
        self.W = W_local
        self._gemv = local_gemv
        self._gemm = local_gemm
        self._bufs = {}
        self.peers = peers if (peers is not None and self.world > 1) else None
        self.peer_areas = tuple(peer_areas)  # used in turn: consecutive collectives need different areas
        self._area_i = 0
        self._pkg = None
        if local_gemv is None or local_gemm is None:
            from . import api as _api  # the CUDA path; raises if the library is missing
            self._pkg = _api

    # ------------------------------------------------------------------ local compute
    def _local_gemv(self, X, out):
        if self._gemv is not None:
            out.copy_(self._gemv(self.W, X))
            return out
        if self.rows == 0:
            return out
        return self._pkg.gemv(self.W, X, self.rows, out=out)

    def _local_gemm_nm(self, X, out):
        if self._gemm is not None:
            out.copy_(self._gemm(self.W, X))
            return out
        if self.rows == 0:
            return out
        return self._pkg.gemm_nm(self.W, X, self.rows, out=out)

    def _buf(self, key, shape, device):
        """Per-shape output buffers, reused across calls (the result of a call is valid until the
        next call of the same shape)."""
        import torch
        b = self._bufs.get(key)
        if b is None or tuple(b.shape) != tuple(shape) or b.device != device:
            b = torch.zeros(shape, dtype=torch.float32, device=device)
            self._bufs[key] = b
        return b

    # ------------------------------------------------------------------ sharded ops
    def gemv(self, X):
        """Y [B][N] on every rank from X [B][K] (the same on every rank)."""
        import torch
        X = X if X.dim() == 2 else X[None]
        B = X.shape[0]
        if self.peers is not None:
            return self._gemv_peer(X, B)
        loc = self._buf(("gemv_loc", B), (B, self.pad), X.device)
        if self.rows == self.pad:
            self._local_gemv(X, loc)
        else:  # the kernels write a dense [B][rows] block
            tmp = torch.zeros((B, self.rows), dtype=torch.float32, device=X.device)
            loc[:, :self.rows] = self._local_gemv(X, tmp)
        if self.world == 1:
            return loc[:, :self.N]
        gathered = self._buf(("gemv_all", B), (self.world * B, self.pad), X.device)
        self.dist.all_gather_into_tensor(gathered, loc, group=self.group)
        return self._assemble_bn(gathered.view(self.world, B, self.pad), B)

    def _gemv_peer(self, X, B):
        import torch
        area = self.peer_areas[self._area_i % len(self.peer_areas)]
        self._area_i += 1
        loc = self.peers.area(area, B * self.pad).view(B, self.pad)
        if self.rows == self.pad:
            self._local_gemv(X, loc)
        else:
            tmp = self._buf(("gemv_tmp", B), (B, self.rows), X.device)
            loc[:, :self.rows] = self._local_gemv(X, tmp)
        gathered = self._buf(("gemv_all", B), (self.world * B, self.pad), X.device)
        self.peers.allgather(area, B * self.pad, gathered)
        return self._assemble_bn(gathered.view(self.world, B, self.pad), B)

    def gemm_nm(self, X):
        """Y^T [N][M] on every rank from X [M][K]."""
        import torch
        M = X.shape[0]
        loc = self._buf(("gemm_loc", M), (self.pad, M), X.device)
        self._local_gemm_nm(X, loc[:self.rows])
        if self.world == 1:
            return loc[:self.N]
        gathered = self._buf(("gemm_all", M), (self.world * self.pad, M), X.device)
        self.dist.all_gather_into_tensor(gathered, loc, group=self.group)
        if self.pad * self.world == self.N:
            return gathered
        return torch.cat([gathered[r * self.pad: r * self.pad + (b - a)]
                          for r, (a, b) in enumerate(shard_rows(self.N, self.world, q) for q in range(self.world))])

    def _assemble_bn(self, gathered, B):
        import torch
        if self.pad * self.world == self.N:
            return gathered.permute(1, 0, 2).reshape(B, self.N)
        parts = []
        for r in range(self.world):
            a, b = shard_rows(self.N, self.world, r)
            parts.append(gathered[r, :, : b - a])
        return torch.cat(parts, dim=1)
