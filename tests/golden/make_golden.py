"""Generate the committed golden vectors in tests/golden/ (run where the reference tree exists).

Inputs are the reference tests' own synthetic inputs, regenerated bit for bit (oracle/ref_inputs.cpp:
gen_iq4xs_weights + std::mt19937/std::normal_distribution).  Outputs come from two places:

* the reference itself: kernels/matmul_iq4xs/ref_cpu.cpp compiled unchanged into
  oracle/_ref/libref_cpu.so -- FP64 GEMV/GEMM on unquantised activations, fp32 dequantisation,
  the truncating fp32->fp16 of block_iq4_xs.h;
* the C restatement (oracle/iq4xs_oracle.c) -- Q8_1 bytes, raw int32 sub-block dots and the FP64
  result of the quantised pipeline, recorded so later edits of the oracle are caught.

tests/test_oracle_golden.py checks the oracle against both.  Usage:
    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden_v1.npz"

# (name, K, N, M, weight seed, activation seed): the seeds are the reference tests' formulas
# (test_gemv_dp4a_compare.cpp:123 uses 9000 + K*7919 + N; activations from mt19937(42)).
CASES = [
    ("syn_512", 512, 512, 1, 9000 + 512 * 7919 + 512, 42),
    ("syn_1024x384_b4", 1024, 384, 4, 9000 + 1024 * 7919 + 2048, 43),
    ("attn_q_trunc", 5120, 48, 2, 9000 + 5120 * 7919 + 5120, 44),
    ("ffn_down_trunc", 17408, 16, 1, 9000 + 17408 * 7919 + 5120, 45),
    ("k256_n33_b8", 256, 33, 8, 777, 46),
]


def main() -> None:
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libref_cpu.so missing: run `make -C oracle` with the reference tree present")
    data = {}
    for name, K, N, M, wseed, xseed in CASES:
        W = O.random_blocks(K, N, wseed & 0xFFFFFFFF)
        X = O.normal(M * K, xseed).reshape(M, K)
        Q = O.quantize_q8_1(X)
        S = O.subblock_dots(W, Q, K, N, M)
        Y64, A = O.matmul_q8(W, Q, K, N, M)
        Yref = np.stack([O.ref_gemv(W, X[m], K, N) for m in range(M)])       # reference FP64 GEMV
        Yref_gemm = O.ref_gemm(W, np.ascontiguousarray(X.T), K, N, M)        # reference FP64 GEMM [N][M]
        rows = min(N, 8)
        deq = O.ref_dequant(W[:rows], K, rows)
        for k, v in dict(W=W, X=X, Q=Q, S=S, Y64=Y64, A=A, Yref=Yref, Yref_gemm=Yref_gemm, deq=deq).items():
            data[f"{name}/{k}"] = v
        data[f"{name}/shape"] = np.array([K, N, M], dtype=np.int64)
    # The reference's truncating fp32 -> fp16 on a spread of magnitudes and edge values.
    rng = np.random.default_rng(1234)
    vals = (rng.standard_normal(3000) * 10.0 ** rng.uniform(-9, 6, 3000)).astype(np.float32)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.0, 65520.0, 1e10, -1e10, np.inf, -np.inf,
                     6.1035156e-05, 6.0e-05, 5.96e-08, 2.98e-08, 1e-45, 127.0 / 127.0, 3.0 / 127.0], dtype=np.float32)
    vals = np.concatenate([vals, edge])
    R = O.ref()
    data["fp16/x"] = vals
    data["fp16/trunc"] = np.array([R.ref_fp32_to_fp16(float(v)) for v in vals], dtype=np.uint16)
    data["cases"] = np.array([c[0] for c in CASES])
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
