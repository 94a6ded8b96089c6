"""Collectives over NVLink peer memory for one process group (one rank per GPU), for the message
sizes of decode: the all-gather of a row-sharded GEMV's output slices and the all-reduce of the
tensor-parallel decoder's o_proj / down_proj partial sums.

Each rank allocates one buffer (`iq4xs_peer_alloc`), exports it with CUDA IPC and maps every other
rank's buffer (handles exchanged with torch.distributed.all_gather_object); no multicast object and
no NVLS are involved.  Buffer layout: [flags: world uint32, padded to 256 B][area 0][area 1]...;
a producer kernel writes this rank's contribution into one of its own areas (plain local stores,
e.g. a GEMV's `out=` is `area(i, n)`), then `allreduce` / `allgather` launches the collective kernel
(csrc/peer.cu) on the current stream: signal every peer, wait (bounded) for every peer, pull the
data over NVLink.  Consecutive collectives must use different areas; every rank issues the same
collectives in the same order.  The calls are graph-capture safe (epochs live in device memory).
"""
from __future__ import annotations

from typing import List


class _DevArray:
    """A raw device pointer presented through __cuda_array_interface__ (zero-copy torch view)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGroup:
    FLAG_BYTES = 256

    def __init__(self, area_floats: int, areas: int = 3, group=None, device=None):
        import torch
        import torch.distributed as dist
        from . import api
        self.api, self.torch = api, torch
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > api.MAX_PEERS:
            raise ValueError(f"at most {api.MAX_PEERS} ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.area_floats = int(area_floats)
        self.area_bytes = (self.area_floats * 4 + 255) // 256 * 256
        self.areas = int(areas)
        self.nbytes = self.FLAG_BYTES + self.areas * self.area_bytes
        with torch.cuda.device(self.device):
            self.own = api.peer_alloc(self.nbytes)
            handle = api.ipc_handle(self.own)
        handles: List[bytes] = [b""] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.bases: List[int] = []
        with torch.cuda.device(self.device):
            for q in range(self.world):
                self.bases.append(self.own if q == self.rank else api.ipc_open(handles[q]))
        self.counter = torch.zeros(2, dtype=torch.int32, device=self.device)  # private epoch counter
        self._views = {}

    def _area_addr(self, q: int, i: int) -> int:
        if not 0 <= i < self.areas:
            raise ValueError(f"area {i} of {self.areas}")
        return self.bases[q] + self.FLAG_BYTES + i * self.area_bytes

    def area(self, i: int, n: int):
        """This rank's area i as a float32 tensor of n elements (a producer's output buffer)."""
        if n > self.area_floats:
            raise ValueError(f"{n} floats do not fit an area of {self.area_floats}")
        key = (i, n)
        v = self._views.get(key)
        if v is None:
            v = self.torch.as_tensor(_DevArray(self._area_addr(self.rank, i), (n,)), device=self.device)
            self._views[key] = v
        return v

    def _run(self, i: int, n: int, out, gather: bool):
        src = [self._area_addr(q, i) for q in range(self.world)]
        self.api.peer_collective(src, self.bases, self.own, self.counter.data_ptr(), self.rank, self.world, gather,
                                 n, out.data_ptr())
        return out

    def allreduce(self, i: int, n: int, out):
        """out[:n] = sum over ranks (in rank order) of their area i (fp32)."""
        if out.numel() < n or out.dtype != self.torch.float32 or not out.is_contiguous():
            raise ValueError("out: contiguous float32 with at least n elements")
        return self._run(i, n, out, False)

    def allgather(self, i: int, n: int, out):
        """out[q*n:(q+1)*n] = the first n floats of rank q's area i."""
        if out.numel() < n * self.world or out.dtype != self.torch.float32 or not out.is_contiguous():
            raise ValueError("out: contiguous float32 with at least world*n elements")
        return self._run(i, n, out, True)

    def slots(self, i: int, n: int):
        """Device descriptor (iq4xs_peer_slots) of the fused all-reduce over area i with `world` slots
        of n 64-bit words (value + epoch tag): slot q of every area is rank q's partial output
        (dec_gemv_q8_push writes it, dec_rmsnorm_gemv_peer / dec_residual_rmsnorm_q8_peer sum the
        slots in rank order)."""
        if 2 * n * self.world > self.area_floats:
            raise ValueError(f"{self.world} slots of {n} words do not fit an area of {self.area_floats} floats")
        key = ("slots", i, n)
        v = self._views.get(key)
        if v is None:
            api, torch = self.api, self.torch
            d = api.PeerSlots()
            for q in range(self.world):
                d.dst[q] = self._area_addr(q, i) + 8 * n * self.rank
            d.local = self._area_addr(self.rank, i)
            d.counter = self.counter.data_ptr()
            d.rank, d.world, d.spin_limit = self.rank, self.world, 0
            raw = bytes(memoryview(d))
            v = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.device)
            self._views[key] = v
        return v

    def close(self):
        """Unmap the peers' buffers, then (after every rank has unmapped ours) free this rank's."""
        import torch.distributed as dist
        if self.own is None:
            return
        self.torch.cuda.synchronize(self.device)
        self._views.clear()
        for q, b in enumerate(self.bases):
            if q != self.rank:
                self.api.ipc_close(b)
        dist.barrier(group=self.group)
        self.api.peer_free(self.own)
        self.own = None
        self.bases = []
