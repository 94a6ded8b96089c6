"""Run one GEMV (or, with --M, GEMM) shape a few times on cuda:0 -- the small, self-ending case for
ncu captures.

    python qwen_3.8_27b_optimizations_b200/profile_case.py --N 69632 --K 5120 --B 1 --launches 3
    python qwen_3.8_27b_optimizations_b200/profile_case.py --N 69632 --K 5120 --B 2 --act f32
    python qwen_3.8_27b_optimizations_b200/profile_case.py --N 17408 --K 5120 --M 2048
    python qwen_3.8_27b_optimizations_b200/profile_case.py --op attention --pos 512
    python qwen_3.8_27b_optimizations_b200/profile_case.py --op sweep

--op attention: the decoder's decode attention kernel (64 query / 8 KV heads of 128, KV cache of
640 positions, the token at --pos).  --op sweep: one step of the benchmark's decode GEMV sweep
(q, k, v, o, gate|up, down at batch 1, 2, 4, 8 through the fp32 entry point), launched eagerly so
that a profiler lists every kernel.

Weights are synthetic IQ4_XS (N(0, 0.02) quantised on the device), activations N(0, 1), quantised
to Q8_1 once up front (or, with --act f32, passed as fp32 to the fp32 entry point), so the launches
of interest are `--launches` GEMV kernels after `--warmup` untimed ones.  The default N (twice the gate|up projection) keeps the weights above the 126 MB L2.
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
    ap.add_argument("--op", default="gemv", choices=["gemv", "attention", "sweep"])
    ap.add_argument("--pos", type=int, default=512)
    ap.add_argument("--act", default="q8", choices=["q8", "f32"],
                    help="GEMV activations: pre-quantised Q8_1, or fp32 through the fp32 entry point "
                         "(quantised inside the GEMV kernel where the launch policy does that)")
    args = ap.parse_args()
    P = _load_pkg()
    if args.op == "attention":
        return attention_case(P, args.pos, args.launches, args.warmup)
    if args.op == "sweep":
        return sweep_case(P, args.launches, args.warmup)
    N, K, B = args.N, args.K, args.B
    W = P.random_weights(N, K, seed=7)
    if args.M:
        return gemm_case(P, W, N, K, args.M, args.launches, args.warmup)
    X = P.fill_normal(B * K, seed=11).view(B, K)
    q8 = P.q8_1_quantize(X)
    ws = torch.zeros(P.gemv_q8_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    if args.act == "f32":
        ws = torch.zeros(P.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
        run = lambda: P.gemv(W, X, N, workspace=ws, out=Y)
    else:
        run = lambda: P.gemv_q8(W, q8, K, N, B, out=Y, workspace=ws)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.launches):
        run()
    e1.record()
    torch.cuda.synchronize()
    if P.device_error():
        raise RuntimeError(f"device error word {P.device_error()}")
    us = e0.elapsed_time(e1) * 1e3 / max(args.launches, 1)
    nbytes = N * K * 17 // 32 + 4 * B * K + 4 * B * N
    print(json.dumps({"N": N, "K": K, "B": B, "act": args.act, "us_per_launch": round(us, 2),
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


def attention_case(P, pos, launches, warmup):
    hq, hkv, hd, max_seq = 64, 8, 128, 640
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn((1, (hq + 2 * hkv) * hd), generator=g, device="cuda")
    kc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    vc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    inv = 1.0 / (1.0e6 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(max_seq, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang).float().cuda(), torch.sin(ang).float().cuda()
    p = torch.tensor([pos], dtype=torch.long, device="cuda")
    q8 = torch.empty((1, hq * hd // 32 * 36), dtype=torch.uint8, device="cuda")
    run = lambda: P.dec_attention_decode_q8(qkv, kc, vc, cos, sin, p, hq, hkv, q8=q8)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(launches):
        run()
    e1.record()
    torch.cuda.synchronize()
    if P.device_error():
        raise RuntimeError(f"device error word {P.device_error()}")
    kv_bytes = 2 * hkv * (pos + 1) * hd * 2
    print(json.dumps({"op": "attention", "pos": pos, "us_per_launch": round(e0.elapsed_time(e1) * 1e3 / max(launches, 1), 2),
                      "kv_bytes": kv_bytes}))
    return 0


def sweep_case(P, steps, warmup):
    shapes = [(8192, 5120), (1024, 5120), (1024, 5120), (5120, 8192), (34816, 5120), (5120, 17408)]
    Ws = [P.random_weights(N, K, seed=i) for i, (N, K) in enumerate(shapes)]
    Xs = {B: P.fill_normal(B * 17408, seed=B) for B in (1, 2, 4, 8)}
    Ys = {B: torch.empty(B * 34816, dtype=torch.float32, device="cuda") for B in (1, 2, 4, 8)}

    def step():
        for B in (1, 2, 4, 8):
            for W, (N, K) in zip(Ws, shapes):
                P.gemv(W, Xs[B][:B * K].view(B, K), N, out=Ys[B][:B * N].view(B, N), flags=P.FLAG_OVERLAP_PRECEDING)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    if P.device_error():
        raise RuntimeError(f"device error word {P.device_error()}")
    print(json.dumps({"op": "sweep", "us_per_step_eager": round(e0.elapsed_time(e1) * 1e3 / max(steps, 1), 1)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
