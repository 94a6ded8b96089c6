"""Python host side of the C ABI in include/iq4xs.h (ctypes over libiq4xs_b200.so).

The names and argument meanings follow the reference harness (kernels/matmul_iq4xs) and its ggml
hook; torch tensors are only the device-memory / stream plumbing.  There is no CPU fallback:
loading fails loudly when the CUDA library is missing, and every non-zero status raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libiq4xs_b200.so"

QK_K = 256
QK8_1 = 32
BLOCK_BYTES = 136
Q8_1_BYTES = 36
MAX_GEMV_BATCH = 8
GGML_TYPE_IQ4_XS = 23

STATUS = {
    0: "ok", 1: "invalid argument", 2: "unsupported shape", 3: "misaligned pointer",
    4: "workspace too small", 5: "CUDA error", 6: "device wait timed out", 7: "not supported",
}

# Every exported symbol of include/iq4xs.h with (restype, argtypes).
_i64, _vp, _sz, _u64, _f, _i = C.c_int64, C.c_void_p, C.c_size_t, C.c_uint64, C.c_float, C.c_int
SIGNATURES = {
    "iq4xs_status_string": (C.c_char_p, [_i]),
    "iq4xs_version": (_i, []),
    "iq4xs_device_error": (_i, [C.POINTER(C.c_uint32)]),
    "iq4xs_q8_1_quantize": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "iq4xs_q8_1_bytes": (_sz, [_i64, _i64]),
    "iq4xs_gemv_q8": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "iq4xs_gemv_q8_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "iq4xs_gemv_q8_ex": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_gemv_f32": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "iq4xs_gemv_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "iq4xs_gemv_f32_ex": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_gemv_f32_noalloc": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "iq4xs_gemm_workspace_bytes": (_sz, [_i64, _i64]),
    "iq4xs_gemm": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    "iq4xs_gemm_strided": (_i, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp]),
    "iq4xs_gemm_ex": (_i, [_vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_debug_gemm_quantize": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "iq4xs_debug_gemm_i8_quantize": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "iq4xs_debug_subblock_dots": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "iq4xs_gemv_q8_generic": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "iq4xs_fill_normal": (_i, [_vp, _i64, _u64, _f, _f, _vp]),
    "iq4xs_quantize_weights": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "iq4xs_dequantize": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "gemv_iq4xs_dp4a_coop_gpu": (_i, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "gemv_iq4xs_stock_dp4a_gpu": (_i, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "quantize_row_q8_1_gpu": (_i, [_vp, _vp, _i64, _vp]),
    "quantize_row_q8_1_batched_gpu": (_i, [_vp, _vp, _i64, _i64, _vp]),
    "gemm_iq4xs_stock_dp4a_gpu": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "gemm_iq4xs_wmma_stream_gpu": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "custom_gemv_iq4xs_can_handle": (C.c_bool, [_i64, _i64, _i64, _i]),
    "custom_gemv_iq4xs_dispatch": (_i, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "custom_gemv_iq4xs_dispatch_batched": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "custom_gemm_iq4xs_can_handle": (C.c_bool, [_i64, _i64, _i64, _i]),
    "custom_gemm_iq4xs_dispatch": (_i, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "iq4xs_gemv_grouped_workspace_bytes": (_sz, [_vp, _i, _i64]),
    "iq4xs_gemv_grouped": (_i, [_vp, _i, _i64, _vp, _sz, C.c_uint, _vp]),
}
MAX_GROUP = 8


class GemvProblem(C.Structure):
    """iq4xs_gemv_problem (include/iq4xs.h)."""
    _fields_ = [("W", _vp), ("X", _vp), ("Y", _vp), ("K", _i64), ("N", _i64)]
# include/iq4xs_bench.h (measurement driver, not the matmul path)
BENCH_SIGNATURES = {
    "iq4xs_bench_e2e_gemv": (_i, [_vp, _vp, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _i, _vp, C.POINTER(C.c_float)]),
    "iq4xs_bench_e2e_floats": (_i64, [_vp, _i, _vp, _i]),
    "iq4xs_bench_e2e_gemv_grouped": (_i, [_vp, _vp, _vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _sz, _i, _vp,
                                          C.POINTER(C.c_float)]),
}

# include/iq4xs_decoder.h (the decoder-step operations around the GEMVs)
DECODER_SIGNATURES = {
    "iq4xs_dec_residual_rmsnorm_q8": (_i, [_vp, _vp, _vp, _i64, _i64, _f, _vp, _vp, C.c_uint, _vp]),
    "iq4xs_dec_attention_decode_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp,
                                           C.c_uint, _vp]),
    "iq4xs_dec_swiglu_q8": (_i, [_vp, _i64, _i64, _vp, C.c_uint, _vp]),
    "iq4xs_dec_embed": (_i, [_vp, _vp, _i64, _i64, _vp, C.c_uint, _vp]),
    "iq4xs_dec_swiglu_gemv": (_i, [_vp, _vp, _i64, _i64, _vp, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_dec_argmax": (_i, [_vp, _i64, _vp, _vp, C.c_uint, _vp]),
    "iq4xs_dec_rmsnorm_gemv": (_i, [_vp, _vp, _vp, _vp, _f, _vp, _vp, _i64, _i64, _vp, _sz, C.c_uint, _vp]),
}

# include/iq4xs_peer.h (collectives over NVLink peer memory)
PEER_SIGNATURES = {
    "iq4xs_peer_alloc": (_i, [_sz, C.POINTER(_vp)]),
    "iq4xs_peer_free": (_i, [_vp]),
    "iq4xs_ipc_handle": (_i, [_vp, _vp]),
    "iq4xs_ipc_open": (_i, [_vp, C.POINTER(_vp)]),
    "iq4xs_ipc_close": (_i, [_vp]),
    "iq4xs_peer_collective": (_i, [C.POINTER(_vp), C.POINTER(_vp), _vp, _vp, _i, _i, _i, _i64, _vp, C.c_uint32, _vp]),
    "iq4xs_dec_gemv_q8_push": (_i, [_vp, _vp, _i64, _i64, _vp, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_dec_swiglu_gemv_push": (_i, [_vp, _vp, _i64, _i64, _vp, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_dec_rmsnorm_gemv_peer": (_i, [_vp, _vp, _vp, _vp, _f, _vp, _vp, _i64, _i64, _vp, _sz, C.c_uint, _vp]),
    "iq4xs_dec_residual_rmsnorm_q8_peer": (_i, [_vp, _vp, _vp, _i64, _f, _vp, _vp, C.c_uint, _vp]),
}
IPC_HANDLE_BYTES = 64
MAX_PEERS = 8

_lib = None


class IQ4XSError(RuntimeError):
    def __init__(self, fn: str, status: int, cuda: bool = False):
        kind = "cudaError" if cuda else STATUS.get(status, "unknown status")
        super().__init__(f"{fn} failed: {kind} ({status})")
        self.status = status


def lib():
    """Load the CUDA library (raises if it was not built: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with __graft_entry__.build()")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in {**SIGNATURES, **BENCH_SIGNATURES, **DECODER_SIGNATURES, **PEER_SIGNATURES}.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(fn: str, status: int, cuda: bool = False) -> None:
    if status != 0:
        raise IQ4XSError(fn, status, cuda)


# ----------------------------------------------------------------------------- torch helpers
def _torch():
    import torch
    return torch


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> int:
    return t.data_ptr()


def weight_row_bytes(K: int) -> int:
    return K // QK_K * BLOCK_BYTES


def device_error() -> int:
    code = C.c_uint32(0)
    _check("iq4xs_device_error", lib().iq4xs_device_error(C.byref(code)))
    return int(code.value)


def q8_1_quantize(X, stream=None):
    """fp32 [M][K] (cuda) -> uint8 [M][K/32*36] Q8_1 blocks."""
    torch = _torch()
    X = X.contiguous()
    if X.dim() == 1:
        X = X[None]
    M, K = X.shape
    q8 = torch.empty((M, K // QK8_1 * Q8_1_BYTES), dtype=torch.uint8, device=X.device)
    _check("iq4xs_q8_1_quantize", lib().iq4xs_q8_1_quantize(_ptr(X), _ptr(q8), K, M, _stream(stream)))
    return q8


_ws_cache = {}


def _workspace(nbytes: int, device, kind: str = "gemv"):
    """A workspace cached per (device, kind); GEMV and GEMM workspaces have different layouts, so
    the two never share one."""
    torch = _torch()
    key = (str(device), kind)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def gemv_q8_workspace_bytes(K: int, N: int, B: int) -> int:
    return int(lib().iq4xs_gemv_q8_workspace_bytes(K, N, B))


def gemv_q8(W, q8, K: int, N: int, B: int, out=None, stream=None, generic: bool = False, workspace=None):
    """Y [B][N] fp32 from IQ4_XS W and pre-quantised activations q8 [B][K/32] blocks."""
    torch = _torch()
    Y = out if out is not None else torch.empty((B, N), dtype=torch.float32, device=W.device)
    if generic:
        _check("iq4xs_gemv_q8_generic", lib().iq4xs_gemv_q8_generic(_ptr(W), _ptr(q8), _ptr(Y), K, N, B, _stream(stream)))
        return Y
    ws = workspace if workspace is not None else _workspace(gemv_q8_workspace_bytes(K, N, B), W.device)
    _check("iq4xs_gemv_q8", lib().iq4xs_gemv_q8(_ptr(W), _ptr(q8), _ptr(Y), K, N, B, _ptr(ws),
                                                ws.numel() * ws.element_size(), _stream(stream)))
    return Y


def gemv_q8_ex(W, q8, K: int, N: int, B: int, out=None, stream=None, flags: int = 0, workspace=None):
    """gemv_q8 with flags: FLAG_OVERLAP_PRECEDING launches the GEMV as a programmatic dependent of
    the kernel before it (the producer of q8, which must not write W)."""
    torch = _torch()
    Y = out if out is not None else torch.empty((B, N), dtype=torch.float32, device=W.device)
    ws = workspace if workspace is not None else _workspace(gemv_q8_workspace_bytes(K, N, B), W.device)
    _check("iq4xs_gemv_q8_ex", lib().iq4xs_gemv_q8_ex(_ptr(W), _ptr(q8), _ptr(Y), K, N, B, _ptr(ws),
                                                      ws.numel() * ws.element_size(), flags, _stream(stream)))
    return Y


def gemv_workspace_bytes(K: int, N: int, B: int) -> int:
    return int(lib().iq4xs_gemv_workspace_bytes(K, N, B))


FLAG_OVERLAP_PRECEDING = 1


def _problems(items):
    arr = (GemvProblem * len(items))()
    for i, (W, X, Y) in enumerate(items):
        arr[i] = GemvProblem(_ptr(W), _ptr(X), _ptr(Y), X.shape[-1], Y.shape[-1])
    return arr


def gemv_grouped_workspace_bytes(shapes, B: int) -> int:
    """Workspace bytes of iq4xs_gemv_grouped for problems of (K, N) shapes at batch B."""
    arr = (GemvProblem * len(shapes))()
    for i, (K, N) in enumerate(shapes):
        arr[i] = GemvProblem(None, None, None, K, N)
    return int(lib().iq4xs_gemv_grouped_workspace_bytes(arr, len(shapes), B))


def gemv_grouped(items, workspace=None, stream=None, flags: int = 0):
    """Independent GEMVs of one batch size in one launch sequence: items = [(W, X [B][K], Y [B][N])],
    every X fp32 contiguous with the same B; each Y receives W . X^T (iq4xs_gemv_grouped)."""
    B = items[0][1].shape[0]
    for W, X, Y in items:
        if X.dim() != 2 or X.shape[0] != B or not X.is_contiguous() or not Y.is_contiguous() or Y.shape[0] != B:
            raise ValueError("every problem needs contiguous X [B][K] and Y [B][N] with the same B")
    arr = _problems(items)
    need = int(lib().iq4xs_gemv_grouped_workspace_bytes(arr, len(items), B))
    ws = workspace if workspace is not None else _workspace(need, items[0][1].device)
    _check("iq4xs_gemv_grouped", lib().iq4xs_gemv_grouped(arr, len(items), B, _ptr(ws), ws.numel() * ws.element_size(),
                                                          flags, _stream(stream)))
    return [Y for _, _, Y in items]


def gemv(W, X, N: int, workspace=None, out=None, stream=None, flags: int = 0):
    """Y [B][N] = W . X^T for fp32 activations X [B][K] (quantised on the fly into the workspace).
    The workspace needs no initialisation (nothing in it carries over between calls).  flags=FLAG_OVERLAP_PRECEDING
    when W is not written by the preceding kernel on the stream."""
    torch = _torch()
    X = X.contiguous()
    if X.dim() == 1:
        X = X[None]
    B, K = X.shape
    need = gemv_workspace_bytes(K, N, B)
    ws = workspace if workspace is not None else _workspace(need, X.device)
    Y = out if out is not None else torch.empty((B, N), dtype=torch.float32, device=X.device)
    _check("iq4xs_gemv_f32", lib().iq4xs_gemv_f32_ex(_ptr(W), _ptr(X), _ptr(Y), K, N, B, _ptr(ws),
                                                     ws.numel() * ws.element_size(), flags, _stream(stream)))
    return Y


def gemm_workspace_bytes(K: int, M: int) -> int:
    return int(lib().iq4xs_gemm_workspace_bytes(K, M))


GEMM_KIND_F16 = 0x10
GEMM_KIND_I8 = 0x20
_GEMM_KINDS = {None: 0, "f16": GEMM_KIND_F16, "i8": GEMM_KIND_I8}


def gemm(W, X, N: int, workspace=None, out=None, stream=None, kind=None):
    """Y [M][N] = X [M][K] . W^T on the tensor cores (X fp32, quantised per 32-block inside).
    kind: None (the library's default), "i8" or "f16" (tensor-core operand kind)."""
    torch = _torch()
    X = X.contiguous()
    M, K = X.shape
    need = gemm_workspace_bytes(K, M)
    ws = workspace if workspace is not None else _workspace(need, X.device, "gemm")
    Y = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=X.device)
    if kind is None:
        _check("iq4xs_gemm", lib().iq4xs_gemm(_ptr(W), _ptr(X), _ptr(Y), K, N, M, _ptr(ws),
                                              ws.numel() * ws.element_size(), _stream(stream)))
    else:
        _check("iq4xs_gemm_ex", lib().iq4xs_gemm_ex(_ptr(W), _ptr(X), K, 1, _ptr(Y), N, 1, K, N, M, _ptr(ws),
                                                    ws.numel() * ws.element_size(), _GEMM_KINDS[kind],
                                                    _stream(stream)))
    return Y


def gemm_nm(W, X, N: int, workspace=None, out=None, stream=None):
    """Y^T [N][M] = W . X^T for X [M][K] (the transposed output layout: a row shard of W gives one
    contiguous block of Y^T)."""
    torch = _torch()
    X = X.contiguous()
    M, K = X.shape
    need = gemm_workspace_bytes(K, M)
    ws = workspace if workspace is not None else _workspace(need, X.device, "gemm")
    Yt = out if out is not None else torch.empty((N, M), dtype=torch.float32, device=X.device)
    _check("iq4xs_gemm_strided", lib().iq4xs_gemm_strided(_ptr(W), _ptr(X), K, 1, _ptr(Yt), 1, M, K, N, M, _ptr(ws),
                                                          ws.numel() * ws.element_size(), _stream(stream)))
    return Yt


def debug_gemm_quantize(X, stream=None):
    """The GEMM's activation quantiser, unpacked from its stage blocks into
    (fp16 q [M][K] in the lookup order within each 32-block, fp32 d [K/32][M])."""
    torch = _torch()
    X = X.contiguous()
    M, K = X.shape
    ws = torch.zeros(gemm_workspace_bytes(K, M), dtype=torch.uint8, device=X.device)
    _check("iq4xs_debug_gemm_quantize", lib().iq4xs_debug_gemm_quantize(_ptr(X), _ptr(ws), K, M, _stream(stream)))
    T, S = (M + 127) // 128, K // 64
    blocks = ws.view(T, S, 17408)
    r = torch.arange(128, device=X.device)[:, None]
    p = torch.arange(64, device=X.device)[None, :]
    idx = ((r // 8) * 1024 + (r % 8) * 128 + (((p // 8) ^ (r % 8)) * 16) + (p % 8) * 2) // 2   # [128][64]
    q16 = blocks[:, :, :16384].contiguous().view(torch.float16).view(T, S, 8192)
    xq = q16[:, :, idx.reshape(-1)].view(T, S, 128, 64).permute(0, 2, 1, 3).reshape(T * 128, K)[:M]
    xs = blocks[:, :, 16384:].contiguous().view(torch.float32).view(T, S, 2, 128)
    xs = xs.permute(1, 2, 0, 3).reshape(K // 32, T * 128)[:, :M]
    return xq, xs


def debug_gemm_i8_quantize(X, stream=None):
    """The int8 GEMM's activation quantiser, unpacked from its stage blocks into
    (int8 q [M][K] in the lookup order within each 32-block, fp32 d [K/32][M])."""
    torch = _torch()
    X = X.contiguous()
    M, K = X.shape
    ws = torch.zeros(gemm_workspace_bytes(K, M), dtype=torch.uint8, device=X.device)
    _check("iq4xs_debug_gemm_i8_quantize", lib().iq4xs_debug_gemm_i8_quantize(_ptr(X), _ptr(ws), K, M, _stream(stream)))
    T, S = (M + 127) // 128, K // 128
    blocks = ws[:T * S * 18432].view(T, S, 18432)
    r = torch.arange(128, device=X.device)[:, None]
    p = torch.arange(128, device=X.device)[None, :]
    idx = (r // 8) * 1024 + (r % 8) * 128 + (((p // 16) ^ (r % 8)) * 16) + (p % 16)   # [128][128]
    q8 = blocks[:, :, :16384].contiguous().view(torch.int8).view(T, S, 16384)
    xq = q8[:, :, idx.reshape(-1)].view(T, S, 128, 128).permute(0, 2, 1, 3).reshape(T * 128, K)[:M]
    xs = blocks[:, :, 16384:].contiguous().view(torch.float32).view(T, S, 4, 128)
    xs = xs.permute(1, 2, 0, 3).reshape(K // 32, T * 128)[:, :M]
    return xq, xs


def debug_subblock_dots(W, q8, K: int, N: int, B: int, stream=None):
    """Raw int32 sub-block dots [B][N][K/32] from the production GEMV inner loop."""
    torch = _torch()
    S = torch.empty((B, N, K // QK8_1), dtype=torch.int32, device=W.device)
    _check("iq4xs_debug_subblock_dots", lib().iq4xs_debug_subblock_dots(_ptr(W), _ptr(q8), _ptr(S), K, N, B, _stream(stream)))
    return S


def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0, device="cuda", out=None, stream=None):
    torch = _torch()
    t = out if out is not None else torch.empty(n, dtype=torch.float32, device=device)
    _check("iq4xs_fill_normal", lib().iq4xs_fill_normal(_ptr(t), n, seed, mean, std, _stream(stream)))
    return t


def quantize_weights(src, stream=None):
    """fp32 [N][K] (cuda) -> IQ4_XS uint8 [N][K/256*136]."""
    torch = _torch()
    src = src.contiguous()
    N, K = src.shape
    W = torch.empty((N, weight_row_bytes(K)), dtype=torch.uint8, device=src.device)
    _check("iq4xs_quantize_weights", lib().iq4xs_quantize_weights(_ptr(src), _ptr(W), N, K, _stream(stream)))
    return W


def random_weights(N: int, K: int, seed: int, std: float = 0.02, device="cuda", stream=None):
    """fp32 N(0, std) weights drawn from `seed`, quantised to IQ4_XS on the device."""
    torch = _torch()
    src = fill_normal(N * K, seed, 0.0, std, device=device, stream=stream).view(N, K)
    W = quantize_weights(src, stream=stream)
    del src
    return W


def dequantize(W, K: int, N: int, stream=None):
    torch = _torch()
    out = torch.empty((N, K), dtype=torch.float32, device=W.device)
    _check("iq4xs_dequantize", lib().iq4xs_dequantize(_ptr(W), _ptr(out), K, N, _stream(stream)))
    return out


# ----------------------------------------------------------------------------- reference-named
def gemv_iq4xs_dp4a_coop_gpu(W, x, y, K: int, N: int, stream=None) -> None:
    _check("gemv_iq4xs_dp4a_coop_gpu", lib().gemv_iq4xs_dp4a_coop_gpu(_ptr(W), _ptr(x), _ptr(y), K, N, _stream(stream)), True)


def gemv_iq4xs_stock_dp4a_gpu(W, x, y, K: int, N: int, stream=None) -> None:
    _check("gemv_iq4xs_stock_dp4a_gpu", lib().gemv_iq4xs_stock_dp4a_gpu(_ptr(W), _ptr(x), _ptr(y), K, N, _stream(stream)), True)


def quantize_row_q8_1_gpu(x, y, K: int, stream=None) -> None:
    _check("quantize_row_q8_1_gpu", lib().quantize_row_q8_1_gpu(_ptr(x), _ptr(y), K, _stream(stream)), True)


def quantize_row_q8_1_batched_gpu(X_km, Y, K: int, M: int, stream=None) -> None:
    _check("quantize_row_q8_1_batched_gpu", lib().quantize_row_q8_1_batched_gpu(_ptr(X_km), _ptr(Y), K, M, _stream(stream)), True)


def gemm_iq4xs_stock_dp4a_gpu(W, X_km, Y_nm, K: int, N: int, M: int, stream=None) -> None:
    _check("gemm_iq4xs_stock_dp4a_gpu",
           lib().gemm_iq4xs_stock_dp4a_gpu(_ptr(W), _ptr(X_km), _ptr(Y_nm), K, N, M, _stream(stream)), True)


def gemm_iq4xs_wmma_stream_gpu(W, X_km, Y_nm, K: int, N: int, M: int, stream=None) -> None:
    _check("gemm_iq4xs_wmma_stream_gpu",
           lib().gemm_iq4xs_wmma_stream_gpu(_ptr(W), _ptr(X_km), _ptr(Y_nm), K, N, M, _stream(stream)), True)


def custom_gemv_iq4xs_can_handle(K: int, N: int, M: int, type_: int = GGML_TYPE_IQ4_XS) -> bool:
    return bool(lib().custom_gemv_iq4xs_can_handle(K, N, M, type_))


def custom_gemv_iq4xs_dispatch(W, x, y, K: int, N: int, stream=None) -> int:
    """Returns the cudaError_t code (0 = handled), like the ggml hook expects."""
    return int(lib().custom_gemv_iq4xs_dispatch(_ptr(W), _ptr(x), _ptr(y), K, N, _stream(stream)))


def custom_gemv_iq4xs_dispatch_batched(W, x, y, K: int, N: int, M: int, stream=None) -> int:
    return int(lib().custom_gemv_iq4xs_dispatch_batched(_ptr(W), _ptr(x), _ptr(y), K, N, M, _stream(stream)))


def custom_gemm_iq4xs_can_handle(K: int, N: int, M: int, type_: int = GGML_TYPE_IQ4_XS) -> bool:
    return bool(lib().custom_gemm_iq4xs_can_handle(K, N, M, type_))


def custom_gemm_iq4xs_dispatch(W, X, Y, K: int, N: int, M: int, stream=None) -> int:
    return int(lib().custom_gemm_iq4xs_dispatch(_ptr(W), _ptr(X), _ptr(Y), K, N, M, _stream(stream)))


# ----------------------------------------------------------------------------- decoder step (iq4xs_decoder.h)
FLAG_PDL = 1
FLAG_ATTN_EARLY_STATE = 2  # attention: position, cache and RoPE tables not written by the preceding kernel


def _q8_out(rows: int, D: int, device, out):
    torch = _torch()
    if out is not None:
        return out
    return torch.empty((rows, D // QK8_1 * Q8_1_BYTES), dtype=torch.uint8, device=device)


def dec_residual_rmsnorm_q8(x, w, eps: float, delta=None, q8=None, h_out=None, want_q8: bool = True,
                            flags: int = 0, stream=None):
    """x [T][D] fp32 (updated in place to x + delta when delta is given); returns (q8, h_out):
    Q8_1 blocks [T][D/32*36] of rmsnorm(x) * w (when want_q8 or q8 is given) and the fp32 values
    (when h_out is given)."""
    T, D = x.shape
    if want_q8 or q8 is not None:
        q8 = _q8_out(T, D, x.device, q8)
    _check("iq4xs_dec_residual_rmsnorm_q8", lib().iq4xs_dec_residual_rmsnorm_q8(
        _ptr(x), _ptr(delta) if delta is not None else None, _ptr(w), D, T, eps,
        _ptr(q8) if q8 is not None else None, _ptr(h_out) if h_out is not None else None, flags, _stream(stream)))
    return q8, h_out


def dec_attention_decode_q8(qkv, k_cache, v_cache, cos, sin, pos, q_heads: int, kv_heads: int, q8=None,
                            o_out=None, flags: int = 0, stream=None):
    """One decode token: qkv fp32 [(q_heads + 2 kv_heads) * 128], caches f16 [kv_heads][max_seq][128],
    cos/sin fp32 [max_seq][64], pos int64 [1] on the device.  Returns Q8_1 blocks [1][q_heads*128/32*36]
    of the attention output (and fills o_out fp32 [q_heads*128] when given)."""
    hd = k_cache.shape[-1]
    max_seq = k_cache.shape[-2]
    q8 = _q8_out(1, q_heads * hd, qkv.device, q8)
    _check("iq4xs_dec_attention_decode_q8", lib().iq4xs_dec_attention_decode_q8(
        _ptr(qkv), _ptr(k_cache), _ptr(v_cache), _ptr(cos), _ptr(sin), _ptr(pos), q_heads, kv_heads, hd, max_seq,
        _ptr(q8), _ptr(o_out) if o_out is not None else None, flags, _stream(stream)))
    return q8


def dec_swiglu_gemv(W, gu, K: int, N: int, out=None, slots=None, flags: int = 0, stream=None, workspace=None):
    """Y [1][N] = W . q8(silu(gate) * up) for gu [1][2K] (the SwiGLU fused into the down_proj GEMV);
    with `slots` (PeerGroup.slots) the outputs are pushed into every rank's slot instead (returns None)."""
    torch = _torch()
    ws = workspace if workspace is not None else _workspace(gemv_workspace_bytes(K, N, 1), gu.device)
    nbytes = ws.numel() * ws.element_size()
    if slots is not None:
        _check("iq4xs_dec_swiglu_gemv_push", lib().iq4xs_dec_swiglu_gemv_push(
            _ptr(W), _ptr(gu), K, N, _ptr(slots), _ptr(ws), nbytes, flags, _stream(stream)))
        return None
    Y = out if out is not None else torch.empty((1, N), dtype=torch.float32, device=gu.device)
    _check("iq4xs_dec_swiglu_gemv", lib().iq4xs_dec_swiglu_gemv(
        _ptr(W), _ptr(gu), K, N, _ptr(Y), _ptr(ws), nbytes, flags, _stream(stream)))
    return Y


def dec_embed(emb, tok, out=None, flags: int = 0, stream=None):
    """out [1][D] fp32 = emb[tok] for the f16 table emb [vocab][D] and a device int64 token tok [1]."""
    torch = _torch()
    vocab, D = emb.shape
    out = out if out is not None else torch.empty((1, D), dtype=torch.float32, device=emb.device)
    _check("iq4xs_dec_embed", lib().iq4xs_dec_embed(_ptr(emb), _ptr(tok), vocab, D, _ptr(out), flags,
                                                    _stream(stream)))
    return out


def dec_argmax(logits, tok, pos=None, flags: int = 0, stream=None):
    """tok [1] (device int64) = argmax of the fp32 logits (first index on ties); pos [1] += 1 if given."""
    if not logits.is_contiguous():
        raise ValueError("logits must be contiguous")
    _check("iq4xs_dec_argmax", lib().iq4xs_dec_argmax(_ptr(logits), logits.numel(), _ptr(tok),
                                                      _ptr(pos) if pos is not None else None, flags,
                                                      _stream(stream)))
    return tok


def dec_swiglu_q8(gu, F: int, q8=None, flags: int = 0, stream=None):
    """gu [T][2F] fp32 -> Q8_1 blocks [T][F/32*36] of silu(gate) * up."""
    T = gu.shape[0]
    q8 = _q8_out(T, F, gu.device, q8)
    _check("iq4xs_dec_swiglu_q8", lib().iq4xs_dec_swiglu_q8(_ptr(gu), F, T, _ptr(q8), flags, _stream(stream)))
    return q8


def dec_rmsnorm_gemv(W, x, w, eps: float, N: int, delta=None, x_out=None, out=None, flags: int = 0, stream=None,
                     workspace=None):
    """Y [1][N] = W . q8(rmsnorm(x + delta) * w) in one kernel (batch 1); x + delta also goes to x_out
    when given (a buffer other than x and delta)."""
    torch = _torch()
    K = x.shape[-1]
    Y = out if out is not None else torch.empty((1, N), dtype=torch.float32, device=x.device)
    ws = workspace if workspace is not None else _workspace(gemv_q8_workspace_bytes(K, N, 1), x.device)
    _check("iq4xs_dec_rmsnorm_gemv", lib().iq4xs_dec_rmsnorm_gemv(
        _ptr(W), _ptr(x), _ptr(delta) if delta is not None else None, _ptr(w), eps,
        _ptr(x_out) if x_out is not None else None, _ptr(Y), K, N, _ptr(ws), ws.numel() * ws.element_size(), flags,
        _stream(stream)))
    return Y


def dec_gemv_q8_push(W, q8, K: int, N: int, slots, flags: int = 0, stream=None, workspace=None):
    """Batch-1 GEMV of Q8_1 blocks whose N outputs go to slot `rank` of every rank's area of the
    fused all-reduce described by `slots` (a device tensor holding an iq4xs_peer_slots, see
    PeerGroup.slots); the last CTA signals the peers."""
    need = gemv_q8_workspace_bytes(K, N, 1)
    ws = workspace if workspace is not None else (_workspace(need, q8.device) if need else None)
    _check("iq4xs_dec_gemv_q8_push", lib().iq4xs_dec_gemv_q8_push(
        _ptr(W), _ptr(q8), K, N, _ptr(slots), _ptr(ws) if ws is not None else None,
        ws.numel() * ws.element_size() if ws is not None else 0, flags, _stream(stream)))


def dec_rmsnorm_gemv_peer(W, x, slots, w, eps: float, N: int, x_out=None, out=None, flags: int = 0, stream=None,
                          workspace=None):
    """dec_rmsnorm_gemv with delta = the fused all-reduce of `slots` (waits for every peer)."""
    torch = _torch()
    K = x.shape[-1]
    Y = out if out is not None else torch.empty((1, N), dtype=torch.float32, device=x.device)
    ws = workspace if workspace is not None else _workspace(gemv_q8_workspace_bytes(K, N, 1), x.device)
    _check("iq4xs_dec_rmsnorm_gemv_peer", lib().iq4xs_dec_rmsnorm_gemv_peer(
        _ptr(W), _ptr(x), _ptr(slots), _ptr(w), eps, _ptr(x_out) if x_out is not None else None, _ptr(Y), K, N,
        _ptr(ws), ws.numel() * ws.element_size(), flags, _stream(stream)))
    return Y


def dec_residual_rmsnorm_q8_peer(x, slots, w, eps: float, q8=None, h_out=None, want_q8: bool = True, flags: int = 0,
                                 stream=None):
    """dec_residual_rmsnorm_q8 (one token) with delta = the fused all-reduce of `slots`."""
    T, D = x.shape
    if want_q8 or q8 is not None:
        q8 = _q8_out(T, D, x.device, q8)
    _check("iq4xs_dec_residual_rmsnorm_q8_peer", lib().iq4xs_dec_residual_rmsnorm_q8_peer(
        _ptr(x), _ptr(slots), _ptr(w), D, eps, _ptr(q8) if q8 is not None else None,
        _ptr(h_out) if h_out is not None else None, flags, _stream(stream)))
    return q8, h_out


class PeerSlots(C.Structure):
    """iq4xs_peer_slots (include/iq4xs_peer.h)."""
    _fields_ = [("dst", C.c_uint64 * MAX_PEERS), ("local", C.c_uint64), ("counter", C.c_uint64),
                ("rank", C.c_int32), ("world", C.c_int32), ("spin_limit", C.c_uint32), ("reserved", C.c_uint32)]


# ----------------------------------------------------------------------------- peer memory (iq4xs_peer.h)
def peer_alloc(nbytes: int) -> int:
    p = C.c_void_p()
    _check("iq4xs_peer_alloc", lib().iq4xs_peer_alloc(nbytes, C.byref(p)))
    return int(p.value)


def peer_free(ptr: int) -> None:
    _check("iq4xs_peer_free", lib().iq4xs_peer_free(ptr))


def ipc_handle(ptr: int) -> bytes:
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    _check("iq4xs_ipc_handle", lib().iq4xs_ipc_handle(ptr, buf))
    return bytes(buf.raw)


def ipc_open(handle: bytes) -> int:
    p = C.c_void_p()
    buf = C.create_string_buffer(handle, IPC_HANDLE_BYTES)
    _check("iq4xs_ipc_open", lib().iq4xs_ipc_open(buf, C.byref(p)))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _check("iq4xs_ipc_close", lib().iq4xs_ipc_close(ptr))


def peer_collective(src, rflags, flags: int, counter: int, rank: int, world: int, gather: bool, n: int, out: int,
                    spin_limit: int = 0, stream=None) -> None:
    """src / rflags: per-rank device addresses (this rank's view); see include/iq4xs_peer.h."""
    arr = C.c_void_p * world
    _check("iq4xs_peer_collective", lib().iq4xs_peer_collective(
        arr(*src), arr(*rflags), flags, counter, rank, world, 1 if gather else 0, n, out, spin_limit,
        _stream(stream)))
