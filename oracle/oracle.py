"""ctypes front-end of the CPU checker (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline / reference arm import
this module; the product never does.  Two libraries sit behind it:

* ``oracle/liboracle.so`` -- the C restatement of the reference pipeline (iq4xs_oracle.c):
  Q8_1 quantizer, raw sub-block dots, FP64 quantised-pipeline matmul, dequant, IQ4_XS
  weight quantizer, and the reference tests' input generators (ref_inputs.cpp).
* ``oracle/_ref/libref_cpu.so`` -- the reference's own kernels/matmul_iq4xs/ref_cpu.cpp built
  unchanged (oracle/Makefile), i.e. the reference's FP64 CPU oracle and CPU path.

Layouts: weights are raw IQ4_XS bytes [N][K/256][136]; activations are token-major fp32
[M][K]; Q8_1 blocks are 36 bytes [M][K/32]; outputs are [M][N].
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_PATH = HERE / "_ref" / "libref_cpu.so"

QK_K = 256
QK8_1 = 32
BLOCK_BYTES = 136
Q8_BYTES = 36

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        i64, vp, u32, f = C.c_int64, C.c_void_p, C.c_uint32, C.c_float
        L.or_fp16_to_fp32.argtypes = [C.c_uint16]
        L.or_fp16_to_fp32.restype = C.c_float
        L.or_fp32_to_fp16_trunc.argtypes = [C.c_float]
        L.or_fp32_to_fp16_trunc.restype = C.c_uint16
        L.or_fp32_to_fp16_rne.argtypes = [C.c_float]
        L.or_fp32_to_fp16_rne.restype = C.c_uint16
        L.or_quantize_q8_1.argtypes = [vp, vp, i64, i64]
        L.or_subblock_dots.argtypes = [vp, vp, vp, i64, i64, i64]
        L.or_matmul_q8.argtypes = [vp, vp, vp, vp, i64, i64, i64]
        L.or_matmul_q8_f32.argtypes = [vp, vp, vp, i64, i64, i64]
        L.or_matmul_f64.argtypes = [vp, vp, vp, i64, i64, i64]
        L.or_dequantize.argtypes = [vp, vp, i64, i64]
        L.or_quantize_iq4_xs.argtypes = [vp, vp, i64, i64]
        L.or_gen_iq4xs_random_blocks.argtypes = [vp, i64, i64, u32]
        L.or_gen_normal.argtypes = [vp, i64, u32, f, f]
        L.or_gen_normal_seq.argtypes = [vp, vp, C.c_int, u32]
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_PATH.exists()


def ref():
    """The reference's own ref_cpu.cpp (built by oracle/Makefile into _ref/)."""
    global _ref
    if _ref is None:
        if not REF_PATH.exists():
            raise FileNotFoundError(f"{REF_PATH} missing: run `make -C oracle` where the reference tree exists")
        L = C.CDLL(str(REF_PATH))
        i64, vp = C.c_int64, C.c_void_p
        L.ref_gemv_iq4xs_cpu_ref.argtypes = [vp, vp, vp, i64, i64]
        L.ref_gemm_iq4xs_cpu_ref.argtypes = [vp, vp, vp, i64, i64, i64]
        L.ref_dequant_mat_iq4xs_cpu.argtypes = [vp, vp, i64, i64]
        L.ref_fp16_to_fp32.argtypes = [C.c_uint16]
        L.ref_fp16_to_fp32.restype = C.c_float
        L.ref_fp32_to_fp16.argtypes = [C.c_float]
        L.ref_fp32_to_fp16.restype = C.c_uint16
        _ref = L
    return _ref


# ----------------------------------------------------------------------------- inputs
def random_blocks(K: int, N: int, seed: int) -> np.ndarray:
    """gen_iq4xs_weights (matmul_test_util.h:49-67) regenerated: uint8 [N][K/256*136]."""
    W = np.zeros((N, K // QK_K * BLOCK_BYTES), dtype=np.uint8)
    lib().or_gen_iq4xs_random_blocks(_p(W), K, N, seed & 0xFFFFFFFF)
    return W


def normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """std::mt19937(seed) + std::normal_distribution<float>: the reference tests' activations."""
    x = np.empty(n, dtype=np.float32)
    lib().or_gen_normal(_p(x), n, seed & 0xFFFFFFFF, mean, std)
    return x


def normal_seq(counts, seed: int) -> list:
    """Reference-test activation draws: one std::mt19937(seed), a fresh normal distribution per case."""
    counts = np.asarray(counts, dtype=np.int64)
    out = np.empty(int(counts.sum()), dtype=np.float32)
    lib().or_gen_normal_seq(_p(out), _p(counts), len(counts), seed & 0xFFFFFFFF)
    res, o = [], 0
    for c in counts:
        res.append(out[o:o + int(c)].copy())
        o += int(c)
    return res


# ----------------------------------------------------------------------------- pipeline
def quantize_q8_1(X: np.ndarray) -> np.ndarray:
    """fp32 [M][K] -> uint8 [M][K/32*36] Q8_1 blocks (device-form quantizer)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    if X.ndim == 1:
        X = X[None]
    M, K = X.shape
    Q = np.zeros((M, K // QK8_1 * Q8_BYTES), dtype=np.uint8)
    lib().or_quantize_q8_1(_p(X), _p(Q), K, M)
    return Q


def subblock_dots(W: np.ndarray, Q: np.ndarray, K: int, N: int, M: int) -> np.ndarray:
    S = np.zeros((M, N, K // QK8_1), dtype=np.int32)
    lib().or_subblock_dots(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(Q)), _p(S), K, N, M)
    return S


def matmul_q8(W: np.ndarray, Q: np.ndarray, K: int, N: int, M: int):
    """FP64 oracle of the quantised pipeline -> (Y [M][N] f64, sum|terms| [M][N] f64)."""
    Y = np.zeros((M, N), dtype=np.float64)
    A = np.zeros((M, N), dtype=np.float64)
    lib().or_matmul_q8(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(Q)), _p(Y), _p(A), K, N, M)
    return Y, A


def matmul_q8_f32(W: np.ndarray, Q: np.ndarray, K: int, N: int, M: int) -> np.ndarray:
    Y = np.zeros((M, N), dtype=np.float32)
    lib().or_matmul_q8_f32(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(Q)), _p(Y), K, N, M)
    return Y


def matmul_f64(W: np.ndarray, X: np.ndarray, K: int, N: int, M: int) -> np.ndarray:
    X = np.ascontiguousarray(X, dtype=np.float32).reshape(M, K)
    Y = np.zeros((M, N), dtype=np.float32)
    lib().or_matmul_f64(_p(np.ascontiguousarray(W)), _p(X), _p(Y), K, N, M)
    return Y


def dequantize(W: np.ndarray, K: int, N: int) -> np.ndarray:
    out = np.zeros((N, K), dtype=np.float32)
    lib().or_dequantize(_p(np.ascontiguousarray(W)), _p(out), K, N)
    return out


def quantize_iq4_xs(src: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(src, dtype=np.float32)
    N, K = src.shape
    W = np.zeros((N, K // QK_K * BLOCK_BYTES), dtype=np.uint8)
    lib().or_quantize_iq4_xs(_p(src), _p(W), N, K)
    return W


def q8_scales(Q: np.ndarray, M: int, K: int) -> np.ndarray:
    """fp32 value of the truncated fp16 d of every Q8_1 block: [M][K/32]."""
    q = Q.reshape(M, K // QK8_1, Q8_BYTES)
    d16 = q[:, :, 0:2].copy().view(np.uint16).reshape(M, K // QK8_1)
    return d16.astype(np.uint16).view(np.float16).astype(np.float32)


# ----------------------------------------------------------------------------- tolerance
def tolerance(Y64: np.ndarray, A: np.ndarray, n_terms: int, rel: float = 1e-5) -> np.ndarray:
    """Per-element bound |y_gpu - y_oracle| <= rel * max(|y|, tau), tau = sum|terms| / sqrt(n_terms).

    tau is the size the sum would have without cancellation between its n_terms fp32 terms
    (random signs), so near-zero outputs are judged against the magnitude of what was summed.
    """
    tau = A / np.sqrt(max(n_terms, 1))
    return rel * np.maximum(np.abs(Y64), tau)


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na < 1e-300 and nb < 1e-300:
        return 1.0
    return float(a @ b / (na * nb))


# ----------------------------------------------------------------------------- reference CPU
def ref_gemv(W: np.ndarray, x: np.ndarray, K: int, N: int) -> np.ndarray:
    y = np.zeros(N, dtype=np.float32)
    ref().ref_gemv_iq4xs_cpu_ref(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(x, dtype=np.float32)), _p(y), K, N)
    return y


def ref_gemm(W: np.ndarray, X_KM: np.ndarray, K: int, N: int, M: int) -> np.ndarray:
    """The reference's gemm_iq4xs_cpu_ref: X [K][M] -> Y [N][M]."""
    Y = np.zeros((N, M), dtype=np.float32)
    ref().ref_gemm_iq4xs_cpu_ref(_p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(X_KM, dtype=np.float32)), _p(Y), K, N, M)
    return Y


def ref_dequant(W: np.ndarray, K: int, N: int) -> np.ndarray:
    out = np.zeros((N, K), dtype=np.float32)
    ref().ref_dequant_mat_iq4xs_cpu(_p(np.ascontiguousarray(W)), _p(out), K, N)
    return out


_POOLS = {}


def _pool(threads: int):
    from concurrent.futures import ThreadPoolExecutor

    if threads not in _POOLS:
        _POOLS[threads] = ThreadPoolExecutor(max_workers=threads)
    return _POOLS[threads]


def cpu_gemv_kind() -> str:
    """Which CPU GEMV ref_gemv_threaded runs: "reference" (the reference's ref_cpu.cpp, built where
    its tree exists) or "port" (or_matmul_f64, the C restatement of the same FP64 loop)."""
    return "reference" if ref_available() else "port"


def ref_gemv_threaded(W: np.ndarray, x: np.ndarray, K: int, N: int, threads: int, y: np.ndarray = None,
                      kind: str = "reference") -> np.ndarray:
    """The reference's gemv_iq4xs_cpu_ref (kind "reference") or its C restatement or_matmul_f64
    (kind "port", ref_cpu.cpp:12-39) over contiguous row slices on `threads` host threads of a
    persistent pool (ctypes releases the GIL for the duration of each call)."""
    W = np.ascontiguousarray(W)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if y is None:
        y = np.zeros(N, dtype=np.float32)
    rb = K // QK_K * BLOCK_BYTES
    base_w, base_y = W.ctypes.data, y.ctypes.data
    bounds = np.linspace(0, N, threads + 1).astype(np.int64)
    if kind == "reference":
        fn = ref().ref_gemv_iq4xs_cpu_ref
        call = lambda w, yy, n: fn(w, _p(x), yy, K, n)  # noqa: E731
    elif kind == "port":
        fn = lib().or_matmul_f64
        call = lambda w, yy, n: fn(w, _p(x), yy, K, n, 1)  # noqa: E731  (M = 1: y is [1][n])
    else:
        raise ValueError(f"unknown CPU GEMV kind {kind!r}")

    def run(i):
        r0, r1 = int(bounds[i]), int(bounds[i + 1])
        if r1 > r0:
            call(C.c_void_p(base_w + r0 * rb), C.c_void_p(base_y + 4 * r0), r1 - r0)

    list(_pool(threads).map(run, range(threads)))
    return y


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
