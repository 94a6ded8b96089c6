"""Run one GEMV (or, with --M, GEMM) shape a few times on cuda:0 -- the small, self-ending case for
ncu captures.

    python qwen_3.8_27b_optimizations_b200/profile_case.py --N 69632 --K 5120 --B 1 --launches 3
    python qwen_3.8_27b_optimizations_b200/profile_case.py --N 17408 --K 5120 --M 2048

Weights are synthetic IQ4_XS (N(0, 0.02) quantised on the device), activations N(0, 1), quantised
to Q8_1 once up front, so the launches of interest are `--launches` GEMV kernels after `--warmup`
untimed ones.  The default N (twice the gate|up projection) keeps the weights above the 126 MB L2.
Prints one line with the event-timed average per launch (meaningless under a profiler).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
from pathlib import Path

import torch


def _load_pkg():
    here = Path(__file__).resolve().parent
    spec = importlib.util.spec_from_file_location("_iq4xs_loader", here / "loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.load()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--N", type=int, default=69632)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--M", type=int, default=0, help="tokens: run the prefill GEMM instead of the GEMV")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args()
    P = _load_pkg()
    N, K, B = args.N, args.K, args.B
    W = P.random_weights(N, K, seed=7)
    if args.M:
        return gemm_case(P, W, N, K, args.M, args.launches, args.warmup)
    X = P.fill_normal(B * K, seed=11).view(B, K)
    q8 = P.q8_1_quantize(X)
    ws = torch.zeros(P.gemv_q8_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        P.gemv_q8(W, q8, K, N, B, out=Y, workspace=ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.launches):
        P.gemv_q8(W, q8, K, N, B, out=Y, workspace=ws)
    e1.record()
    torch.cuda.synchronize()
    if P.device_error():
        raise RuntimeError(f"device error word {P.device_error()}")
    us = e0.elapsed_time(e1) * 1e3 / max(args.launches, 1)
    nbytes = N * K * 17 // 32 + 4 * B * K + 4 * B * N
    print(json.dumps({"N": N, "K": K, "B": B, "us_per_launch": round(us, 2),
                      "algorithmic_bytes": nbytes, "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}))
    return 0


def gemm_case(P, W, N, K, M, launches, warmup):
    X = P.fill_normal(M * K, seed=11).view(M, K)
    ws = torch.zeros(P.gemm_workspace_bytes(K, M), dtype=torch.uint8, device="cuda")
    Y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        P.gemm(W, X, N, workspace=ws, out=Y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(launches):
        P.gemm(W, X, N, workspace=ws, out=Y)
    e1.record()
    torch.cuda.synchronize()
    if P.device_error():
        raise RuntimeError(f"device error word {P.device_error()}")
    us = e0.elapsed_time(e1) * 1e3 / max(launches, 1)
    ops = 2 * M * N * K
    print(json.dumps({"N": N, "K": K, "M": M, "us_per_call": round(us, 2), "tops": round(ops / (us * 1e-6) / 1e12, 1)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
