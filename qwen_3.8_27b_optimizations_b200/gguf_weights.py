"""IQ4_XS weight matrices from and to GGUF files, the format llama.cpp keeps quantised models in.

A GGUF tensor of type IQ4_XS (ggml type 23) with ggml shape (ne0 = K, ne1 = N) stores N rows of
K/256 super-blocks of 136 bytes back to back -- exactly the layout the GEMV and GEMM kernels read
(`block_iq4_xs`, kernels/common/block_iq4_xs.h:10-24 in the reference), so a tensor goes to the
device as its bytes, with no repacking, and `W.data` feeds `gemv`, `gemm` and the C ABI directly.
Parsing and writing use gguf-py (the Python package of llama.cpp's source tree); this module only
selects the IQ4_XS matrices, checks their geometry and moves their bytes.

    mats = read_iq4xs("model.gguf")                 # every 2-D IQ4_XS tensor, on cuda
    W = mats["blk.0.ffn_down.weight"]               # W.K = 17408, W.N = 5120
    y = api.gemv(W.data, x, W.N)

The reference itself reads no GGUF (its kernels take synthetic blocks); the model files its
benchmarks load come through llama.cpp, whose IQ4_XS tensors this reads the same way.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import numpy as np

IQ4_XS_TYPE = 23        # GGMLQuantizationType.IQ4_XS
QK = 256                # weights per super-block
BLOCK_BYTES = 136       # bytes per super-block
_CHUNK = 64 << 20       # host->device copy granule (bytes)


@dataclass
class IQ4XSMatrix:
    name: str
    K: int              # input features (ggml ne0)
    N: int              # output rows (ggml ne1)
    data: "object"      # torch.uint8 [N][K/256*136]


def _gguf():
    try:
        import gguf
    except ImportError as e:  # pragma: no cover - gguf-py ships with the image
        raise ImportError("reading GGUF files needs the gguf package (llama.cpp's gguf-py)") from e
    return gguf


def _to_device(arr: np.ndarray, device):
    """uint8 [N][rb] (possibly a read-only memory map) -> a contiguous torch tensor on `device`,
    copied in chunks through one pinned buffer when the device is a GPU."""
    import torch
    dev = torch.device(device)
    if dev.type != "cuda":
        return torch.from_numpy(np.array(arr, dtype=np.uint8, copy=True))
    out = torch.empty(arr.shape, dtype=torch.uint8, device=dev)
    flat_out = out.view(-1)
    flat_in = arr.reshape(-1)
    stage = torch.empty(min(_CHUNK, flat_in.size), dtype=torch.uint8).pin_memory()
    stage_np = stage.numpy()
    for o in range(0, flat_in.size, stage.numel()):
        n = min(stage.numel(), flat_in.size - o)
        stage_np[:n] = flat_in[o:o + n]
        flat_out[o:o + n].copy_(stage[:n], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()  # the staging buffer is reused next round
    return out


def read_iq4xs(path, names: Optional[Iterable[str]] = None, device="cuda") -> Dict[str, IQ4XSMatrix]:
    """The IQ4_XS matrices of a GGUF file: every 2-D IQ4_XS tensor, or exactly `names` (a name that
    is missing, not IQ4_XS or not 2-D is an error).  Raises ValueError on a tensor whose byte size
    does not match its shape."""
    gguf = _gguf()
    reader = gguf.GGUFReader(str(path), "r")
    want = None if names is None else list(names)
    by_name = {t.name: t for t in reader.tensors}
    if want is not None:
        missing = [n for n in want if n not in by_name]
        if missing:
            raise ValueError(f"not in {path}: {missing}")
    out: Dict[str, IQ4XSMatrix] = {}
    for name, t in by_name.items():
        if want is not None and name not in want:
            continue
        is_iq4 = int(t.tensor_type) == IQ4_XS_TYPE and len(t.shape) == 2
        if not is_iq4:
            if want is not None:
                raise ValueError(f"{name}: type {t.tensor_type.name}, shape {list(t.shape)}; "
                                 "expected a 2-D IQ4_XS tensor")
            continue
        K, N = int(t.shape[0]), int(t.shape[1])
        if K % QK != 0:
            raise ValueError(f"{name}: K = {K} is not a multiple of {QK}")
        rb = K // QK * BLOCK_BYTES
        raw = np.asarray(t.data)
        if raw.dtype != np.uint8 or raw.size != N * rb:
            raise ValueError(f"{name}: {raw.size} bytes for {N} x {K} IQ4_XS (want {N * rb})")
        out[name] = IQ4XSMatrix(name, K, N, _to_device(raw.reshape(N, rb), device))
    return out


def write_iq4xs(path, mats: Dict[str, object], arch: str = "iq4xs-synthetic", extra=None) -> None:
    """Write IQ4_XS matrices (name -> uint8 [N][K/256*136], numpy or torch on any device) as a GGUF
    file that llama.cpp's loader and `read_iq4xs` accept.  `extra`: name -> float32/float16 numpy
    arrays stored beside them (norm weights and the like)."""
    gguf = _gguf()
    w = gguf.GGUFWriter(str(path), arch)
    for name, m in mats.items():
        a = m.detach().cpu().numpy() if hasattr(m, "detach") else np.asarray(m)
        if a.dtype != np.uint8 or a.ndim != 2 or a.shape[1] % BLOCK_BYTES != 0:
            raise ValueError(f"{name}: expected uint8 [N][K/256*136], got {a.dtype} {a.shape}")
        w.add_tensor(name, np.ascontiguousarray(a), raw_dtype=gguf.GGMLQuantizationType.IQ4_XS)
    for name, a in (extra or {}).items():
        w.add_tensor(name, np.ascontiguousarray(a))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
