#!/usr/bin/env python
"""bench.py -- IQ4_XS decode GEMV sweep on B200 (BASELINE.json metric: IQ4_XS GEMV HBM GB/s).

Workload (one GPU): one step = the decode GEMV of every 27B-class layer
shape -- q_proj 8192x5120, k_proj 1024x5120, v_proj 1024x5120, o_proj 5120x8192, gate|up fused
34816x5120, down 5120x17408 (out x in) -- at batch 1, 2, 4 and 8 (24 GEMVs, each a Q8_1 quantize
plus the GEMV kernel).  Weights: fp32 N(0, 0.02) from fixed seeds quantised to IQ4_XS on the device;
activations fp32 N(0, 1).  Two copies of the layer weights (384 MB, > 3x the 126 MB L2) alternate
between steps and the 24 GEMVs of a step stream 768 MB, so every weight byte comes from HBM.

value  = algorithmic bytes (sum over GEMVs of N*K*17/32 + 4*B*K + 4*B*N) / device time, all ranks
         (each rank runs the full step on its own weights: weak scaling), inputs resident in HBM,
         the step replayed as a CUDA graph.
e2e    = same metric through the reference-facing ggml hook (custom_gemv_iq4xs_dispatch_batched)
         called from a C++ host loop, with the step's activations copied from pinned host memory
         and every output copied back, per GEMV, inside the timed region.
roofline = the GEMV kernel alone (quantizer excluded), timed per launch with CUDA events on its
         stream, against the measured HBM copy bandwidth (MEASURED_PEAKS.json).
gemm   = prefill GEMM: the same layer shapes at M = 512 and 2048 tokens
         (iq4xs_gemm: Q8_1 activation quantisation + the tensor-core GEMM per call), TOPS = 2*M*N*K /
         device time, against the measured dense bf16 tensor peak; reported beside the headline.
--impl reference: the reference's own CPU path (kernels/matmul_iq4xs/ref_cpu.cpp, compiled unchanged
         into oracle/_ref/) on the host cores, same metric on a bounded row sample; where oracle/_ref
         was not built, the oracle's C restatement of that loop (cpu_baseline.kind "port").
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent

SHAPES = [  # (name, N out, K in)
    ("q_proj", 8192, 5120),
    ("k_proj", 1024, 5120),
    ("v_proj", 1024, 5120),
    ("o_proj", 5120, 8192),
    ("gate_up", 34816, 5120),
    ("down", 5120, 17408),
]
BATCHES = [1, 2, 4, 8]
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
GEMM_TOKENS = [512, 2048]


def gemv_bytes(N: int, K: int, B: int) -> int:
    return N * K * 17 // 32 + 4 * B * K + 4 * B * N


def step_bytes() -> int:
    return sum(gemv_bytes(N, K, B) for B in BATCHES for _, N, K in SHAPES)


def load_pkg():
    spec = importlib.util.spec_from_file_location("_iq4xs_loader", ROOT / "qwen_3.8_27b_optimizations_b200" / "loader.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.load()


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def graph_kernel_nodes(g) -> int:
    """Kernel nodes in a captured torch CUDA graph (driver API: cuGraphGetNodes / cuGraphNodeGetType)."""
    try:
        drv = C.CDLL("libcuda.so.1")
        graph = C.c_void_p(g.raw_cuda_graph())
    except Exception:
        return -1
    n = C.c_size_t(0)
    if drv.cuGraphGetNodes(graph, None, C.byref(n)) != 0 or n.value == 0:
        return -1
    nodes = (C.c_void_p * n.value)()
    if drv.cuGraphGetNodes(graph, nodes, C.byref(n)) != 0:
        return -1
    kind = C.c_int(-1)
    count = 0
    for i in range(n.value):
        if drv.cuGraphNodeGetType(C.c_void_p(nodes[i]), C.byref(kind)) == 0 and kind.value == 0:  # kernel
            count += 1
    return count


def bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return FALLBACK_BF16_TFLOPS, "fallback"


def gemm_sweep(P, weights, dev, stream, reps: int = 3, kind=None):
    """Prefill GEMM over the layer shapes at M = 512 and 2048: per shape the median of 3 timed CUDA-graph
    replays of `reps` calls (weights alternate between the two copies).  kind: the tensor-core operand
    kind ("i8", "f16"; None = the library's default)."""
    import torch
    per, tot_flops, tot_ms = [], 0.0, 0.0
    for M in GEMM_TOKENS:
        for i, (name, N, K) in enumerate(SHAPES):
            X = P.fill_normal(M * K, seed=77 + M + i).view(M, K)
            Y = torch.empty((M, N), dtype=torch.float32, device=dev)
            ws = torch.empty(P.gemm_workspace_bytes(K, M), dtype=torch.uint8, device=dev)
            with torch.cuda.stream(stream):
                P.gemm(weights[0][i], X, N, workspace=ws, out=Y, stream=stream, kind=kind)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for r in range(reps):
                        P.gemm(weights[r % 2][i], X, N, workspace=ws, out=Y, stream=stream, kind=kind)
                g.replay()
                stream.synchronize()
                ts = []
                for _ in range(3):
                    a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a0.record(stream)
                    g.replay()
                    b0.record(stream)
                    stream.synchronize()
                    ts.append(a0.elapsed_time(b0) / reps)
            del g
            d = statistics.median(ts)
            fl = 2.0 * M * N * K
            per.append({"shape": name, "M": M, "us": round(d * 1e3, 1), "tops": round(fl / (d * 1e-3) / 1e12, 1)})
            tot_flops += fl
            tot_ms += d
            del X, Y, ws
    return per, tot_flops / (tot_ms * 1e-3) / 1e12


def c1_gemv(P, dev, stream, copies: int = 16):
    """one GEMV 4096 x 4096 at batch 1 through the fp32 entry point (Q8_1 of x
    inside the call).  `copies` weight matrices (16 x 8.9 MB = 143 MB > L2) rotate through a captured
    graph of `copies` calls, so every call streams its weights from HBM; per-call time = median of 3
    replays / copies."""
    import torch
    N = K = 4096
    Ws = [P.random_weights(N, K, seed=9100 + i) for i in range(copies)]
    X = P.fill_normal(K, seed=9099).view(1, K)
    Y = torch.empty((1, N), dtype=torch.float32, device=dev)
    ws = torch.zeros(P.gemv_workspace_bytes(K, N, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        for W in Ws:
            P.gemv(W, X, N, workspace=ws, out=Y, stream=stream, flags=P.FLAG_OVERLAP_PRECEDING)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for W in Ws:
                P.gemv(W, X, N, workspace=ws, out=Y, stream=stream, flags=P.FLAG_OVERLAP_PRECEDING)
        g.replay()
        stream.synchronize()
        ts = []
        for _ in range(3):
            a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            g.replay()
            b0.record(stream)
            stream.synchronize()
            ts.append(a0.elapsed_time(b0) / copies)
    del g
    ms = statistics.median(ts)
    nb = gemv_bytes(N, K, 1)
    peak, peak_kind = hbm_peak()
    gbs = nb / (ms * 1e-3) / 1e9
    return {"config": "single IQ4_XS GEMV 4096 x 4096, batch 1 (BASELINE.json configs[0]), fp32 x quantised "
                      "to Q8_1 inside the call", "us_per_call": round(ms * 1e3, 2), "GBs": round(gbs, 1),
            "roofline": {"bound": "hbm", "peak": peak, "peak_kind": peak_kind, "frac": round(gbs / peak, 4)},
            "l2": f"{copies} weight copies ({copies * nb / 1e6:.0f} MB) rotate"}


def c1_cpu_reference(threads: int, kind: str, calls: int = 5):
    """The reference's CPU GEMV (gemv_iq4xs_cpu_ref, or its C port where oracle/_ref is absent) on the
    full 4096 x 4096 C1 matrix (reference random-byte blocks), all host threads, median of `calls`."""
    import numpy as np
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    N = K = 4096
    W = O.random_blocks(K, N, 4096)
    x = np.random.default_rng(1).standard_normal(K).astype(np.float32)
    O.ref_gemv_threaded(W, x, K, N, threads, kind=kind)
    ts = []
    for _ in range(calls):
        t0 = time.perf_counter()
        O.ref_gemv_threaded(W, x, K, N, threads, kind=kind)
        ts.append(time.perf_counter() - t0)
    dt = statistics.median(ts)
    return {"us_per_call": round(dt * 1e6, 1), "GBs": round(gemv_bytes(N, K, 1) / dt / 1e9, 3), "cores": threads,
            "kind": kind, "sample": f"all 4096 rows, median of {calls} calls"}


SHARDED = [("lm_head", 152064, 5120), ("gate_up", 34816, 5120)]


def sharded_sweep(P, dev, stream, rank: int, world: int, barrier, reps: int = 5):
    """lm_head and gate|up split by output rows over the ranks, GEMV at batch 1
    and GEMM at M = 2048, each call followed by the all-gather of the output slices (GEMV: the NVLink
    peer-memory pull kernel; GEMM: NCCL).  Time per call = max over ranks of the CUDA-event time of
    `reps` calls."""
    import torch
    import torch.distributed as dist
    out = []
    peers = None
    if world > 1:
        peers = P.peer.PeerGroup(max(P.sharded.max_shard_rows(N, world) for _, N, _ in SHARDED), areas=2)
    for name, N, K in SHARDED:
        r0, r1 = P.sharded.shard_rows(N, world, rank)
        W = P.random_weights(r1 - r0, K, seed=5000 + N + rank)
        S = P.sharded.RowShardedIQ4XS(W, N, K, rank=rank, world=world, peers=peers) if world > 1 else \
            P.sharded.RowShardedIQ4XS(W, N, K, rank=0, world=1)
        for op, M in (("gemv", 1), ("gemm", 2048)):
            X = P.fill_normal(M * K, seed=31 + M).view(M, K)
            fn = (lambda: S.gemv(X)) if op == "gemv" else (lambda: S.gemm_nm(X))
            torch.cuda.synchronize()
            barrier()  # the first collective of a call waits for every rank
            with torch.cuda.stream(stream):
                for _ in range(3):
                    fn()
                stream.synchronize()
                barrier()
                a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                for _ in range(reps):
                    fn()
                b0.record(stream)
                stream.synchronize()
            ms = a0.elapsed_time(b0) / reps
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            rec = {"matrix": name, "N": N, "K": K, "op": op, "M": M, "ranks": world, "ms": round(ms, 4)}
            if op == "gemv":
                rec["GBs"] = round((N * K * 17 // 32 + 4 * K + 4 * N) / (ms * 1e-3) / 1e9, 1)
            else:
                rec["TOPS"] = round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1)
            out.append(rec)
            del X
        del S, W
        torch.cuda.empty_cache()
    if peers is not None:
        peers.close()
    return out


DECODER_PROMPT, DECODER_STEPS = 512, 128


PARITY_TOKEN = 12345  # the fixed input token of the decode step compared across TP degrees
PARITY_SEQ = [17, 4242, 99, 150001]  # fixed decode inputs from position 0 (the exact check)


def decoder_parity_logits(m, prompt):
    """Prefill logits of `prompt`, then the logits of one decode step (the fused decode kernels and, at
    TP > 1, the peer collectives) on a fixed token; both flattened to float64 on the device."""
    _, lg_pre = m.prefill(prompt)
    m._tok.fill_(PARITY_TOKEN % m.cfg.vocab)
    m._step()
    return lg_pre.flatten().double(), m._last_logits.flatten().double().clone()


def decoder_seq_logits(m):
    """Logits of fixed decode inputs fed one per step from position 0 (no prompt): every operation is
    one of this library's kernels, so TP-N with peer collectives (rank-order sums) and its single-GPU
    rank emulation must agree bit for bit."""
    import torch
    m.reset_decode(0)
    out = []
    for t in PARITY_SEQ:
        m._tok.fill_(t % m.cfg.vocab)
        m._step()
        out.append(m._last_logits.clone())
    torch.cuda.synchronize()
    return torch.cat(out)


def decoder_run(P, dev, rank: int, world: int, barrier):
    """the synthetic 64-layer decoder, tensor-parallel over the ranks: a
    512-token uniform random prompt (seed 7), then 128 greedy decode steps (CUDA-graph replay per
    token).  Times are CUDA events on each rank, max over ranks.  Also returns the model's prefill
    and fixed-token decode logits (untimed) for the multi-GPU parity check."""
    import torch
    import torch.distributed as dist
    cfg = P.decoder.DecoderConfig()
    t0 = time.time()
    m = P.decoder.TPDecoder(cfg, rank=rank, world=world, seed=1)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    prompt = torch.randint(0, cfg.vocab, (DECODER_PROMPT,), generator=torch.Generator().manual_seed(7)).to(dev)
    logits = decoder_parity_logits(m, prompt) + (decoder_seq_logits(m) if world > 1 else None,)
    m.prefill(prompt)
    m.decode(4)                      # warm-up: eager steps and graph capture
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record()
    m.prefill(prompt)
    ev[1].record()
    ev[2].record()
    toks = m.decode(DECODER_STEPS)
    ev[3].record()
    torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    pre_ms, dec_ms = float(t[0]), float(t[1])
    alt = None
    form = ("fused" if m.fused_allreduce else "collective") if world > 1 and m.peers is not None else None
    # the other form is timed at 2 and 4 ranks; at 8 only the default (the collective kernel: every
    # consumer CTA of the fused form reads world x hidden x 8 bytes of slots, already slower at 4)
    if form is not None and world <= 4:
        # the same model with the other all-reduce form (fused into the GEMVs <-> a separate peer
        # collective kernel after each o_proj / down_proj GEMV)
        m.fused_allreduce = not m.fused_allreduce
        m.graph = None
        m.prefill(prompt)
        m.decode(4)                  # re-capture
        m.prefill(prompt)            # back to position 512: 128 steps fill the 640-slot cache exactly
        barrier()
        ev[0].record()
        m.decode(DECODER_STEPS)
        ev[1].record()
        torch.cuda.synchronize()
        tc = torch.tensor([ev[0].elapsed_time(ev[1])], dtype=torch.float64, device=dev)
        dist.all_reduce(tc, op=dist.ReduceOp.MAX)
        alt = round(DECODER_STEPS / (float(tc[0]) * 1e-3), 1)
    m.release()
    del m
    torch.cuda.empty_cache()
    return {"metric": "decode tok/s (greedy, batch 1)", "value": round(DECODER_STEPS / (dec_ms * 1e-3), 1),
            "unit": "tok/s", "tp": world, "prompt": DECODER_PROMPT, "steps": DECODER_STEPS,
            "prefill_ms": round(pre_ms, 1), "prefill_tok_s": round(DECODER_PROMPT / (pre_ms * 1e-3), 1),
            "decode_ms": round(dec_ms, 1), "build_s": round(build_s, 1), "first_tokens": toks[:8],
            "allreduce": {"fused": "fused into the o_proj / down_proj GEMVs (push epilogue + next kernel's prologue)",
                          "collective": "a peer collective kernel after each o_proj / down_proj GEMV"}.get(form),
            "tok_s_other_allreduce": ({"form": "collective" if form == "fused" else "fused", "value": alt}
                                      if alt is not None else None),
            "model": "64 x (hidden 5120, 64x128 q heads, 8 kv heads, SwiGLU 17408), vocab 152064, IQ4_XS "
                     "linear layers, fp32 norms, f16 embeddings and KV cache, random N(0, 0.02) init"}, logits


def logit_agreement(a, b) -> dict:
    """a against the reference b (flat float64 tensors): cosine, max |a - b| / max |b|, same argmax, and
    how many of b's top 5 are in a's top 5."""
    import torch
    cos = float(torch.dot(a, b) / (a.norm() * b.norm()))
    rel = float((a - b).abs().max() / b.abs().max())
    top_a, top_b = set(torch.topk(a, 5).indices.tolist()), set(torch.topk(b, 5).indices.tolist())
    return {"cosine": round(cos, 9), "max_rel": float(f"{rel:.3g}"), "argmax_same": bool(a.argmax() == b.argmax()),
            "top5_common": len(top_a & top_b)}


def multi_gpu_parity(P, dev, rank: int, world: int, c5_logits) -> dict:
    """N > 1, outside every timed region: multi-GPU results against single-GPU results that every rank
    computes itself on the same inputs.
      * row-sharded GEMV (peer-memory all-gather) and GEMM (NCCL all-gather) of gate|up 34816 x 5120:
        batch 1 and the GEMM bit-exact against the full-matrix kernels (rows are independent, per-row
        arithmetic identical); batch 3 bit-exact against the concatenated per-shard GEMVs and within
        1e-5 (of max |y|) of the full-matrix GEMV (its K parts may be split differently);
      * tensor-parallel decoders (a small 2-layer model, the C5 dimensions at 2 layers, the full
        64-layer C5 model), two checks each:
        - exact: four decode steps on fixed tokens from position 0 through the fused decode kernels
          and the peer collectives, bit for bit against the single-GPU rank emulation of the same TP
          degree (TPDecoder(emulate_ranks=N): the o_proj / down_proj GEMVs run as the ranks' K slices
          and are added in rank order, as the peer all-reduce adds them);
        - against TP 1: prefill logits and one decode step after the prompt, by cosine (gates below).
          The prefill's NCCL all-reduce and TP 1's single GEMV add the K slices in another order, which
          moves single Q8_1 roundings of the next layer's activations; 64 layers amplify that (cosine
          ~0.995 at TP 2), a wrong shard would give a cosine near 0.  The small model also compares
          peer collectives against NCCL all-reduces."""
    import torch
    res, ok = {}, True
    # ---- row-sharded matmuls
    N, K = 34816, 5120
    W = P.random_weights(N, K, seed=777)
    shards = [P.sharded.shard_rows(N, world, r) for r in range(world)]
    r0, r1 = shards[rank]
    peers = P.peer.PeerGroup(3 * P.sharded.max_shard_rows(N, world), areas=2)
    S = P.sharded.RowShardedIQ4XS(W[r0:r1].contiguous(), N, K, peers=peers)
    sh = {}
    for B in (1, 3):
        X = P.fill_normal(B * K, seed=5 + B).view(B, K)
        Y = S.gemv(X).clone()
        Yf = P.gemv(W, X, N)
        if B == 1:
            sh["gemv_b1_bitexact"] = bool(torch.equal(Y, Yf))
        else:
            Ycat = torch.cat([P.gemv(W[a:b].contiguous(), X, b - a) for a, b in shards], 1)
            sh["gemv_b3_bitexact_vs_shards"] = bool(torch.equal(Y, Ycat))
            rel = float((Y - Yf).abs().max() / Yf.abs().max())
            sh["gemv_b3_max_rel_vs_full"] = float(f"{rel:.3g}")
            sh["gemv_b3_within_1e-5"] = rel <= 1e-5
    Xm = P.fill_normal(256 * K, seed=9).view(256, K)
    sh["gemm_m256_bitexact"] = bool(torch.equal(S.gemm_nm(Xm), P.gemm(W, Xm, N).t()))
    torch.cuda.synchronize()
    peers.close()
    del S, W
    torch.cuda.empty_cache()
    ok &= all(v for k, v in sh.items() if isinstance(v, bool))
    res["sharded_gate_up"] = sh

    def run(cfg, w, rk, prompt, seed=4, **kw):
        m = P.decoder.TPDecoder(cfg, rank=rk, world=w, seed=seed, **kw)
        out = decoder_parity_logits(m, prompt)
        seq = decoder_seq_logits(m)
        m.release()
        del m
        torch.cuda.empty_cache()
        return out, seq

    def exact(tag, seq_tp, seq_emu):
        nonlocal ok
        same = bool(torch.equal(seq_tp, seq_emu))
        d = {"bitexact": same, "steps": len(PARITY_SEQ),
             "max_abs_diff": float((seq_tp.double() - seq_emu.double()).abs().max())}
        ok &= same
        res[tag] = d

    def agree(tag, a, b, gate):
        nonlocal ok
        d = {"prefill": logit_agreement(a[0], b[0]), "decode_step": logit_agreement(a[1], b[1]),
             "gate_cosine": gate}
        d["ok"] = d["prefill"]["cosine"] >= gate and d["decode_step"]["cosine"] >= gate
        ok &= d["ok"]
        res[tag] = d

    # ---- small decoder: one KV head and 4 query heads per rank, two FFN super-block pairs per rank
    small = P.decoder.DecoderConfig(layers=2, hidden=1024, heads=4 * world, kv_heads=world, head_dim=128,
                                    ffn=1024 * world, vocab=3072, max_seq=40)
    prompt = torch.randint(0, small.vocab, (12,), generator=torch.Generator().manual_seed(3)).to(dev)
    (peer_l, peer_s) = run(small, world, rank, prompt, peer_collectives=True)
    (nccl_l, _) = run(small, world, rank, prompt, peer_collectives=False)
    (tp1_l, _) = run(small, 1, 0, prompt)
    (_, emu_s) = run(small, 1, 0, prompt, emulate_ranks=world)
    agree("small_2layer_peer_vs_nccl", peer_l, nccl_l, 0.999)
    agree("small_2layer_tp_vs_tp1", peer_l, tp1_l, 0.999)
    exact("small_2layer_decode_vs_emulation", peer_s, emu_s)
    # ---- C5 dimensions, 2 layers
    c5_2 = P.decoder.DecoderConfig(layers=2)
    prompt = torch.randint(0, c5_2.vocab, (DECODER_PROMPT,), generator=torch.Generator().manual_seed(7)).to(dev)
    (tp_l, tp_s) = run(c5_2, world, rank, prompt)
    (tp1_l, _) = run(c5_2, 1, 0, prompt)
    (_, emu_s) = run(c5_2, 1, 0, prompt, emulate_ranks=world)
    agree("c5_2layer_tp_vs_tp1", tp_l, tp1_l, 0.999)
    exact("c5_2layer_decode_vs_emulation", tp_s, emu_s)
    # ---- full C5 (64 layers): the timed model's logits against TP 1 of the same weights (seed 1), and
    # its fixed-input decode steps against the rank emulation
    if c5_logits is not None:
        (tp1_l, _) = run(P.decoder.DecoderConfig(), 1, 0, prompt, seed=1)
        agree("c5_64layer_tp_vs_tp1", c5_logits[:2], tp1_l, 0.98)
        (_, emu_s) = run(P.decoder.DecoderConfig(), 1, 0, prompt, seed=1, emulate_ranks=world)
        exact("c5_64layer_decode_vs_emulation", c5_logits[2], emu_s)
    res["ok"] = bool(ok)
    return res


def ncu_traffic():
    """Per-launch DRAM bytes of the GEMV kernel from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "gemv_ncu_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, max clock and throttle reasons during the timed region: NVML polled from a
    thread every 2 ms (the timed regions are short), nvidia-smi -lms 200 as a fallback."""

    def __init__(self, torch_device_index: int):
        self.idx = torch_device_index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._proc = None

    def _bus_id(self):
        """PCI bus id of the torch device: names the same physical GPU to NVML and nvidia-smi whatever
        CUDA_VISIBLE_DEVICES or the enumeration order is."""
        import torch
        pr = torch.cuda.get_device_properties(self.idx)
        return f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(self._bus_id())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.idx)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            masks = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for name, m in masks.items():
                            if r & m:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    self._stop.wait(0.002)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:
            fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                      "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            try:
                try:
                    gpu = self._bus_id()
                except Exception:
                    gpu = str(self.idx)
                self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                               "-lms", "200", "-i", gpu], stdout=subprocess.PIPE,
                                              stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except Exception:
                self._proc.kill()
                out = ""
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for l in out.splitlines():
                f = [x.strip() for x in l.split(",")]
                if len(f) < 6:
                    continue
                try:
                    self.samples.append(float(f[0]))
                    self.max_mhz = max(self.max_mhz or 0.0, float(f[1]))
                except ValueError:
                    continue
                for n, v in zip(names, f[2:6]):
                    if v.lower() == "active":
                        self.reasons.add(n)

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------- reference arm (CPU)
def cpu_sample_plan(rows_per_shape: int):
    return [(name, min(N, rows_per_shape), K) for name, N, K in SHAPES]


def run_cpu_reference(threads: int, rows_per_shape: int, steps: int, warmup: int, kind: str = "reference"):
    """The reference's gemv_iq4xs_cpu_ref (FP64, unquantised x; kind "reference") or the oracle's C
    restatement of it (kind "port", used where oracle/_ref was not built) over a row sample of every
    shape, every batch size (one call per token, as the reference's CPU path has no batch), row
    slices spread over `threads` host threads.  Returns (GB/s, seconds per step, sample text)."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O

    plan = cpu_sample_plan(rows_per_shape)
    rng = np.random.default_rng(0)
    mats = {}
    for name, n, K in plan:
        W = O.random_blocks(K, n, 1000 + [s[0] for s in SHAPES].index(name))
        xs = [rng.standard_normal(K).astype(np.float32) for _ in range(max(BATCHES))]
        mats[name] = (W, xs, n, K)

    def one_step():
        for B in BATCHES:
            for name, n, K in plan:
                W, xs, _, _ = mats[name]
                for b in range(B):
                    O.ref_gemv_threaded(W, xs[b], K, n, threads, kind=kind)

    for _ in range(warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    dt = (time.perf_counter() - t0) / max(steps, 1)
    nbytes = sum(gemv_bytes(n, K, B) for B in BATCHES for _, n, K in plan)
    fn = "gemv_iq4xs_cpu_ref" if kind == "reference" else "or_matmul_f64 (C port of gemv_iq4xs_cpu_ref)"
    sample = (f"first {rows_per_shape} rows of each of the 6 shapes (all rows of k/v), batch 1/2/4/8 "
              f"(one FP64 {fn} call per token), rows split over {threads} threads")
    return nbytes / dt / 1e9, dt, sample


def reference_arm(args, rank: int, world: int):
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    kind = O.cpu_gemv_kind()
    threads = O.host_threads()
    gbs, dt, sample = run_cpu_reference(threads, args.cpu_rows, args.steps, args.warmup, kind)
    path = ("kernels/matmul_iq4xs/ref_cpu.cpp gemv_iq4xs_cpu_ref (unchanged)" if kind == "reference"
            else "oracle/iq4xs_oracle.c or_matmul_f64 (restatement of ref_cpu.cpp:12-39)")
    line = {
        "impl": "reference",
        "metric": "IQ4_XS decode GEMV sweep HBM GB/s", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (reference random-byte IQ4_XS blocks, N(0,1) activations)",
        "config": {"workload": "decode_gemv_sweep_27b_layers", "shapes": {n: [N, K] for n, N, K in SHAPES},
                   "batches": BATCHES, "path": path},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- single cases (profiling)
def run_case(argv) -> int:
    """`bench.py --case {gemv,gemm,attention,sweep} ...`: one small, self-ending case on cuda:0 for ncu
    captures (never a bench number: it prints the event-timed average of `--launches` launches after
    `--warmup` untimed ones, meaningless under a profiler).

      --case gemv --N 69632 --K 5120 --B 8 [--act f32]   one GEMV shape (Q8_1 quantised once up front,
                                                          or fp32 through the fp32 entry point)
      --case gemm --N 17408 --K 5120 --M 2048             the prefill GEMM
      --case attention --pos 512                          the decoder's decode attention (64 / 8 heads)
      --case sweep                                        one benchmark sweep step, eager launches
      --case grouped --B 8                                one grouped call over the six layer shapes
      --case gsweep                                       one benchmark step (a grouped call per batch), eager
      --case decode --tp 8 --layers 4 [--graph]           decode steps of the C5 decoder with one rank's
                                                          shapes at TP 1/2/4/8 on this GPU alone (no
                                                          communication): eager (for a launch list), or
                                                          --graph: ms per token of the captured step
    The default N (twice the gate|up projection) keeps the weights above the 126 MB L2."""
    import torch
    ap = argparse.ArgumentParser(prog="bench.py --case")
    ap.add_argument("--case", required=True,
                    choices=["gemv", "gemm", "attention", "sweep", "grouped", "gsweep", "decode"])
    ap.add_argument("--tp", type=int, default=1, choices=[1, 2, 4, 8])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--N", type=int, default=69632)
    ap.add_argument("--K", type=int, default=5120)
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--M", type=int, default=2048)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--pos", type=int, default=512)
    ap.add_argument("--act", default="q8", choices=["q8", "f32"])
    ap.add_argument("--kind", default=None, choices=["i8", "f16"], help="GEMM operand kind (default: library's)")
    a = ap.parse_args(argv)
    P = load_pkg()
    torch.cuda.set_device(0)

    def timed(run, launches, warmup):
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
        return e0.elapsed_time(e1) * 1e3 / max(launches, 1)

    if a.case == "attention":
        hq, hkv, hd, max_seq = 64, 8, 128, 640
        g = torch.Generator(device="cuda").manual_seed(3)
        qkv = torch.randn((1, (hq + 2 * hkv) * hd), generator=g, device="cuda")
        kc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
        vc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
        inv = 1.0 / (1.0e6 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
        ang = torch.arange(max_seq, dtype=torch.float64)[:, None] * inv[None, :]
        cos, sin = torch.cos(ang).float().cuda(), torch.sin(ang).float().cuda()
        p = torch.tensor([a.pos], dtype=torch.long, device="cuda")
        q8 = torch.empty((1, hq * hd // 32 * 36), dtype=torch.uint8, device="cuda")
        us = timed(lambda: P.dec_attention_decode_q8(qkv, kc, vc, cos, sin, p, hq, hkv, q8=q8), a.launches, a.warmup)
        print(json.dumps({"case": "attention", "pos": a.pos, "us_per_launch": round(us, 2),
                          "kv_bytes": 2 * hkv * (a.pos + 1) * hd * 2}))
        return 0
    if a.case == "decode":
        # one rank's share of the C5 model at TP tp: tp-th of the heads, the largest rank's FFN pairs,
        # a vocab/tp lm_head shard; the same kernels and shapes a TP rank runs, without its exchanges
        tp = a.tp
        cfg = P.decoder.DecoderConfig(layers=a.layers, heads=64 // tp, kv_heads=max(1, 8 // tp),
                                      ffn=512 * (-(-34 // tp)), vocab=152064 // tp)
        m = P.decoder.TPDecoder(cfg, rank=0, world=1, seed=1)
        prompt = torch.randint(0, cfg.vocab, (16,), generator=torch.Generator().manual_seed(7)).to("cuda")
        m.prefill(prompt)
        torch.cuda.synchronize()
        res = {"case": "decode", "tp_shapes": tp, "layers": a.layers}
        if a.graph:
            m.decode(4)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            m.decode(64)
            e1.record()
            torch.cuda.synchronize()
            res["ms_per_token"] = round(e0.elapsed_time(e1) / 64, 4)
        else:
            res["tokens"] = m.decode(max(a.launches, 1), use_graph=False)
        if P.device_error():
            raise RuntimeError(f"device error word {P.device_error()}")
        m.release()
        print(json.dumps(res))
        return 0
    if a.case == "sweep":
        Ws = [P.random_weights(N, K, seed=i) for i, (_, N, K) in enumerate(SHAPES)]
        Xs = {B: P.fill_normal(B * 17408, seed=B) for B in BATCHES}
        Ys = {B: torch.empty(B * 34816, dtype=torch.float32, device="cuda") for B in BATCHES}

        def step():
            for B in BATCHES:
                for W, (_, N, K) in zip(Ws, SHAPES):
                    P.gemv(W, Xs[B][:B * K].view(B, K), N, out=Ys[B][:B * N].view(B, N), flags=P.FLAG_OVERLAP_PRECEDING)
        us = timed(step, a.launches, a.warmup)
        print(json.dumps({"case": "sweep", "us_per_step_eager": round(us, 1)}))
        return 0
    if a.case == "gsweep":
        Ws = [P.random_weights(N, K, seed=i) for i, (_, N, K) in enumerate(SHAPES)]
        items = {}
        for B in BATCHES:
            Xs = [P.fill_normal(B * K, seed=50 + B + i).view(B, K) for i, (_, N, K) in enumerate(SHAPES)]
            Ys = [torch.empty((B, N), dtype=torch.float32, device="cuda") for _, N, K in SHAPES]
            items[B] = list(zip(Ws, Xs, Ys))
        gws = torch.zeros(max(P.gemv_grouped_workspace_bytes([(K, N) for _, N, K in SHAPES], B) for B in BATCHES),
                          dtype=torch.uint8, device="cuda")

        def gstep():
            for B in BATCHES:
                P.gemv_grouped(items[B], workspace=gws, flags=P.FLAG_OVERLAP_PRECEDING)
        us = timed(gstep, a.launches, a.warmup)
        print(json.dumps({"case": "gsweep", "us_per_step_eager": round(us, 1),
                          "gbs": round(step_bytes() / (us * 1e-6) / 1e9, 1)}))
        return 0
    if a.case == "grouped":
        B = a.B
        Ws = [P.random_weights(N, K, seed=i) for i, (_, N, K) in enumerate(SHAPES)]
        Xs = [P.fill_normal(B * K, seed=50 + i).view(B, K) for i, (_, N, K) in enumerate(SHAPES)]
        Ys = [torch.empty((B, N), dtype=torch.float32, device="cuda") for _, N, K in SHAPES]
        gws = torch.zeros(P.gemv_grouped_workspace_bytes([(K, N) for _, N, K in SHAPES], B), dtype=torch.uint8,
                          device="cuda")
        us = timed(lambda: P.gemv_grouped(list(zip(Ws, Xs, Ys)), workspace=gws), a.launches, a.warmup)
        nb = sum(gemv_bytes(N, K, B) for _, N, K in SHAPES)
        print(json.dumps({"case": "grouped", "B": B, "us_per_call": round(us, 2), "gbs": round(nb / (us * 1e-6) / 1e9, 1)}))
        return 0
    N, K, B = a.N, a.K, a.B
    W = P.random_weights(N, K, seed=7)
    if a.case == "gemm":
        X = P.fill_normal(a.M * K, seed=11).view(a.M, K)
        ws = torch.zeros(P.gemm_workspace_bytes(K, a.M), dtype=torch.uint8, device="cuda")
        Y = torch.empty((a.M, N), dtype=torch.float32, device="cuda")
        us = timed(lambda: P.gemm(W, X, N, workspace=ws, out=Y, kind=a.kind), a.launches, a.warmup)
        print(json.dumps({"case": "gemm", "kind": a.kind or "default", "N": N, "K": K, "M": a.M, "us_per_call": round(us, 2),
                          "tops": round(2.0 * a.M * N * K / (us * 1e-6) / 1e12, 1)}))
        return 0
    X = P.fill_normal(B * K, seed=11).view(B, K)
    Y = torch.empty((B, N), dtype=torch.float32, device="cuda")
    if a.act == "f32":
        ws = torch.zeros(P.gemv_workspace_bytes(K, N, B), dtype=torch.uint8, device="cuda")
        run = lambda: P.gemv(W, X, N, workspace=ws, out=Y)
    else:
        q8 = P.q8_1_quantize(X)
        ws = torch.zeros(max(P.gemv_q8_workspace_bytes(K, N, B), 1), dtype=torch.uint8, device="cuda")
        run = lambda: P.gemv_q8(W, q8, K, N, B, out=Y, workspace=ws)
    us = timed(run, a.launches, a.warmup)
    nb = gemv_bytes(N, K, B)
    print(json.dumps({"case": "gemv", "N": N, "K": K, "B": B, "act": a.act, "us_per_launch": round(us, 2),
                      "algorithmic_bytes": nb, "gbs": round(nb / (us * 1e-6) / 1e9, 1)}))
    return 0


# ----------------------------------------------------------------------------- GPU arm
def main():
    if "--case" in sys.argv[1:]:
        return run_case(sys.argv[1:])
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=256, help="rows per shape in the CPU samples")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=0, help="default: same as --steps")
    ap.add_argument("--extras", default="all", choices=["all", "none"],
                    help="side measurements after the headline (prefill GEMM sweep, row-sharded matmuls, decoder); "
                         "'none' leaves the headline, e2e, roofline and CPU baseline unchanged")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local_rank))
    P = load_pkg()
    L = P.lib()
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.Stream(device=dev)

    # ---- data (2 weight copies alternate between steps)
    weights = [[P.random_weights(N, K, seed=1000 + 97 * c + i + 7919 * rank) for i, (_, N, K) in enumerate(SHAPES)]
               for c in range(2)]
    X = {(B, i): P.fill_normal(B * K, seed=42 + B + 31 * i + 7919 * rank).view(B, K)
         for B in BATCHES for i, (_, N, K) in enumerate(SHAPES)}
    Y = {(B, i): torch.empty((B, N), dtype=torch.float32, device=dev) for B in BATCHES for i, (_, N, K) in enumerate(SHAPES)}
    ws = torch.zeros(max(P.gemv_workspace_bytes(K, N, B) for B in BATCHES for _, N, K in SHAPES), dtype=torch.uint8,
                     device=dev)
    gws = torch.zeros(max(P.gemv_grouped_workspace_bytes([(K, N) for _, N, K in SHAPES], B) for B in BATCHES),
                      dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def step(c: int, s):
        """The measured step: per batch size one grouped call over the six layer GEMVs."""
        for B in BATCHES:
            P.gemv_grouped([(weights[c][i], X[(B, i)], Y[(B, i)]) for i in range(len(SHAPES))], workspace=gws,
                           stream=s, flags=P.FLAG_OVERLAP_PRECEDING)

    def step_single(c: int, s):
        """The same 24 GEMVs as one iq4xs_gemv_f32 call each (reported beside the headline)."""
        for B in BATCHES:
            for i, (_, N, K) in enumerate(SHAPES):
                P.gemv(weights[c][i], X[(B, i)], N, workspace=ws, out=Y[(B, i)], stream=s, flags=P.FLAG_OVERLAP_PRECEDING)

    def capture(fn):
        gs = []
        with torch.cuda.stream(stream):
            fn(0, stream)
            fn(1, stream)
            stream.synchronize()
            for c in range(2):
                g = torch.cuda.CUDAGraph(keep_graph=True)  # keep the cudaGraph_t: its kernel nodes are counted
                with torch.cuda.graph(g, stream=stream):
                    fn(c, stream)
                g.instantiate()
                gs.append(g)
        torch.cuda.synchronize()
        return gs

    # one graph per weight copy
    graphs = capture(step)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # kernels of one step: quantiser + GEMV (+ part reduction) per GEMV call, counted in the graph
    launches_per_step = graph_kernel_nodes(graphs[0])
    if launches_per_step <= 0:
        launches_per_step = len(SHAPES) * len(BATCHES) * 2

    # ---- warmup
    with torch.cuda.stream(stream):
        for w in range(args.warmup):
            graphs[w % 2].replay()
    stream.synchronize()

    # ---- timed region (value)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for k in range(args.steps):
                graphs[k % 2].replay()
            e1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    sb = step_bytes()
    value_gbs = world * sb * args.steps / (ms_max * 1e-3) / 1e9
    clocks = clk.summary()

    # ---- the same sweep as 24 single-matrix calls (graph-replayed; reported beside the headline)
    graphs_single = capture(step_single)
    with torch.cuda.stream(stream):
        for w in range(args.warmup):
            graphs_single[w % 2].replay()
        a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for k in range(args.steps):
            graphs_single[k % 2].replay()
        b0.record(stream)
        stream.synchronize()
    single_ms = a0.elapsed_time(b0) / args.steps
    single = {"what": "the same 24 GEMVs, one iq4xs_gemv_f32 call each (CUDA graph replay)",
              "GBs": round(world * step_bytes() / (single_ms * 1e-3) / 1e9, 1), "ms_per_step": round(single_ms, 4),
              "launches_per_step": graph_kernel_nodes(graphs_single[0])}
    graphs_single.clear()

    # ---- roofline: per grouped launch (quantiser + grouped GEMV kernel + part sums), a CUDA graph of
    # `reps` back-to-back calls over the two weight copies, timed with events on its stream; and the
    # single-matrix GEMV kernel per shape (Q8_1 input, part sums included) for reference
    peak, peak_kind = hbm_peak()
    reps = 10

    def graph_time(call):
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for r in range(reps):
                    call(r % 2)
            g.replay()
            stream.synchronize()
            ts = []
            for _ in range(3):
                a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                g.replay()
                b0.record(stream)
                stream.synchronize()
                ts.append(a0.elapsed_time(b0) / reps)
        del g
        return statistics.median(ts)

    per = []
    tot_bytes, tot_ms = 0, 0.0
    for B in BATCHES:
        d = graph_time(lambda c, B=B: P.gemv_grouped([(weights[c][i], X[(B, i)], Y[(B, i)]) for i in range(len(SHAPES))],
                                                     workspace=gws, stream=stream, flags=P.FLAG_OVERLAP_PRECEDING))
        nb = sum(gemv_bytes(N, K, B) for _, N, K in SHAPES)
        per.append({"B": B, "gemvs": len(SHAPES), "us": round(d * 1e3, 2), "gbs": round(nb / (d * 1e-3) / 1e9, 1),
                    "frac": round(nb / (d * 1e-3) / 1e9 / peak, 4)})
        tot_bytes += nb
        tot_ms += d
    achieved = tot_bytes / (tot_ms * 1e-3) / 1e9
    per_single = []
    q8s = {(B, i): P.q8_1_quantize(X[(B, i)], stream=stream) for B in BATCHES for i in range(len(SHAPES))}
    stream.synchronize()
    for B in BATCHES:
        for i, (name, N, K) in enumerate(SHAPES):
            d = graph_time(lambda c, B=B, i=i, N=N, K=K: P.gemv_q8(weights[c][i], q8s[(B, i)], K, N, B, out=Y[(B, i)],
                                                                  stream=stream, workspace=ws))
            nb = gemv_bytes(N, K, B)
            per_single.append({"shape": name, "B": B, "us": round(d * 1e3, 2), "gbs": round(nb / (d * 1e-3) / 1e9, 1)})
    # DRAM traffic per launch: the dominant kernel's ncu ratio (dram read+write / algorithmic bytes,
    # captured on a smaller case) scaled to the mean algorithmic bytes of the step's launches.
    traffic = ncu_traffic()
    traffic_per_launch, traffic_src = None, None
    if traffic:
        kname, k = next(iter(traffic["kernels"].items()))
        case = k.get("case") or f"{k.get('N')}x{k.get('K')} B={k.get('B')}"
        traffic_per_launch = round(k["traffic_ratio"] * tot_bytes / len(per))
        traffic_src = (f"ncu dram__bytes_read+write of {kname} on {case} (ratio {k['traffic_ratio']} of "
                       f"algorithmic), scaled to the mean grouped launch of the step")

    # ---- e2e through the ggml hook from the C++ host loop, pinned host buffers
    e2e_steps = args.e2e_steps or args.steps
    wptrs = (C.c_void_p * len(SHAPES))(*[w.data_ptr() for w in weights[0]])
    Ks = (C.c_int64 * len(SHAPES))(*[K for _, _, K in SHAPES])
    Ns = (C.c_int64 * len(SHAPES))(*[N for _, N, _ in SHAPES])
    Bs = (C.c_int64 * len(BATCHES))(*BATCHES)
    nx = int(L.iq4xs_bench_e2e_floats(Ks, len(SHAPES), Bs, len(BATCHES)))  # one pass's inputs, concatenated
    ny = int(L.iq4xs_bench_e2e_floats(Ns, len(SHAPES), Bs, len(BATCHES)))  # one pass's results
    hx = torch.empty(nx, dtype=torch.float32).pin_memory()
    hx.normal_()
    hy = torch.empty(ny, dtype=torch.float32).pin_memory()
    dx = torch.empty(nx, dtype=torch.float32, device=dev)
    dy = torch.empty(ny, dtype=torch.float32, device=dev)

    def run_e2e(grouped: bool, steps: int) -> float:
        ems = C.c_float(0.0)
        if grouped:
            rc = L.iq4xs_bench_e2e_gemv_grouped(wptrs, Ks, Ns, len(SHAPES), Bs, len(BATCHES), hx.data_ptr(),
                                                hy.data_ptr(), dx.data_ptr(), dy.data_ptr(), gws.data_ptr(),
                                                gws.numel(), steps, stream.cuda_stream, C.byref(ems))
        else:
            rc = L.iq4xs_bench_e2e_gemv(wptrs, Ks, Ns, len(SHAPES), Bs, len(BATCHES), hx.data_ptr(), hy.data_ptr(),
                                        dx.data_ptr(), dy.data_ptr(), steps, stream.cuda_stream, C.byref(ems))
        if rc != 0:
            raise RuntimeError(f"e2e ({'grouped' if grouped else 'hook'}) failed: cudaError {rc}")
        return float(ems.value)

    e2e_val = {}
    for grouped in (True, False):
        run_e2e(grouped, max(args.warmup, 3))
        barrier()
        t = torch.tensor([run_e2e(grouped, e2e_steps)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_val[grouped] = world * sb * e2e_steps / (float(t.item()) * 1e-3) / 1e9
    e2e_gbs, e2e_hook_gbs = e2e_val[True], e2e_val[False]
    h2d, d2h = 4 * nx, 4 * ny  # the bytes of the two copies of every step

    gemm_per, gemm_tops, sharded, decoder = [], None, [], None
    gemm_per_i8, gemm_tops_i8 = [], None
    bpeak, bpeak_kind = bf16_peak()
    c1 = c1_gemv(P, dev, stream)
    if args.extras == "all":
        # ---- prefill GEMM sweep (reported beside the headline)
        gemm_per, gemm_tops = gemm_sweep(P, weights, dev, stream)
        gemm_per_i8, gemm_tops_i8 = gemm_sweep(P, weights, dev, stream, kind="i8")
        # ---- row-sharded lm_head / gate|up across the ranks (strong scaling, output all-gather)
        sharded = sharded_sweep(P, dev, stream, rank, world, barrier)
        # ---- synthetic decoder, tensor-parallel over the ranks
        del weights
        torch.cuda.empty_cache()
        decoder, c5_logits = decoder_run(P, dev, rank, world, barrier)
    parity = None
    if world > 1:
        # ---- multi-GPU results against single-GPU results (outside every timed region)
        parity = multi_gpu_parity(P, dev, rank, world, c5_logits if args.extras == "all" else None)
        flags = torch.tensor([1.0 if parity["ok"] else 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        parity["ok_all_ranks"] = bool(flags.item() == 1.0)

    torch.cuda.synchronize()
    err = P.device_error()
    if err:
        raise RuntimeError(f"device error word {err}")

    # ---- CPU baseline (rank 0, one GPU only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(ROOT))
        from oracle import oracle as O
        kind = O.cpu_gemv_kind()
        threads = O.host_threads()
        gbs, _, sample = run_cpu_reference(threads, args.cpu_rows, 2, 1, kind)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample}
        c1["cpu_reference"] = c1_cpu_reference(threads, kind)

    for g in graphs:
        del g
    graphs.clear()
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()

    if rank == 0:
        line = {
            "metric": "IQ4_XS decode GEMV sweep HBM GB/s", "value": round(value_gbs, 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic: fp32 N(0,0.02) weights quantised to IQ4_XS on device, fp32 N(0,1) activations",
            "config": {"workload": "decode_gemv_sweep_27b_layers", "shapes": {n: [N, K] for n, N, K in SHAPES},
                       "batches": BATCHES, "gemvs_per_step": len(SHAPES) * len(BATCHES),
                       "bytes_per_step": sb, "l2": "inputs larger than L2: 2 x 192 MB weight sets alternate, 768 MB streamed per step",
                       "api": "iq4xs_gemv_grouped: one call per batch size over the six layer GEMVs",
                       "timing": "CUDA graph replay of the step, CUDA events on the launch stream, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": traffic_per_launch,
                         "algorithmic_bytes_per_launch": round(tot_bytes / len(per)),
                         "traffic_source": traffic_src,
                         "kernel": "gemv_rows_grouped_kernel (B=1) / gemv_mma_grouped_kernel (B=2..8), one grouped "
                                   "launch per batch size (its quantiser and part-sum kernels included in the time)",
                         "per_launch": per,
                         "per_shape_single_kernel": per_single},
            "single_calls": single,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "iq4xs_gemv_grouped (one call per batch size) from a C++ host loop, pinned host x/y: "
                            "each step uploads its activations in one copy and downloads its results in one copy, "
                            "on two copy streams overlapping the neighbouring steps' GEMVs",
                    "hook_value": round(e2e_hook_gbs, 1),
                    "hook_path": "the same loop through the ggml hook custom_gemv_iq4xs_dispatch_batched, one call "
                                 "per GEMV"},
            "gemm": None if gemm_tops is None else {
                "metric": "IQ4_XS prefill GEMM TOPS (2*M*N*K / time, Q8_1 quantisation included)",
                "value": round(gemm_tops, 1), "unit": "TOPS", "tokens": GEMM_TOKENS,
                "roofline": {"bound": "tensor", "achieved": round(gemm_tops, 1), "peak": bpeak,
                             "unit": "TFLOP/s", "frac": round(gemm_tops / bpeak, 4), "peak_kind": bpeak_kind,
                             "kernel": "gemm_iq4xs_tc_kernel (tcgen05.mma kind::f16, fp32 TMEM accumulators)"},
                "per_shape": gemm_per,
                "i8_operands": {"value": round(gemm_tops_i8, 1), "unit": "TOPS",
                                "kernel": "gemm_iq4xs_i8_kernel (tcgen05.mma kind::i8, s32 TMEM accumulators)",
                                "per_shape": gemm_per_i8}},
            "c1": c1,
            "parity": parity,
            "decoder": decoder,
            "sharded": {"what": "row-sharded over the ranks (strong scaling), all-gather of the outputs (GEMV: "
                                "NVLink peer-memory pull kernel, GEMM: NCCL), time = max over ranks",
                        "results": sharded},
            "gpu_launches": args.steps * launches_per_step,
            "gpu_launches_per_step": launches_per_step,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if parity is not None and not parity["ok_all_ranks"]:
        return 3  # a multi-GPU result disagrees with the single-GPU one
    return 0


if __name__ == "__main__":
    sys.exit(main())
