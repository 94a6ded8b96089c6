"""Collectives over NVLink peer memory (csrc/peer.cu, peer.PeerGroup) on 2, 4 and 8 GPUs (each
skipped on a box with fewer): all-reduce and all-gather bit-exact against the rank-order sum and the
concatenation of the ranks' inputs (and within fp32 rounding of NCCL's all-reduce), repeated calls
with alternating areas, the same collectives replayed from a CUDA graph, the row-sharded GEMV with
the peer all-gather against the single-GPU kernel, and the tensor-parallel decoder with peer
collectives against the same model with NCCL all-reduces and, bit for bit, against its single-GPU
rank emulation -- with the all-reduce fused into the row-parallel GEMVs (push epilogue, summed in
the next kernel's prologue) and with the separate collective kernel.  NVLS is off; no multicast memory is
used."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch.distributed as dist
    from conftest import load_pkg
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    res = {}
    try:
        P = load_pkg()
        dev = torch.device("cuda", rank)
        g = P.peer.PeerGroup(1 << 16, areas=3)
        # all-reduce / all-gather against NCCL, several rounds (the epoch counter advances)
        ok_ar, ok_ag = True, True
        for it in range(6):
            n = [5120, 1000, 65536][it % 3]
            area = it % 2
            x = torch.randn(n, generator=torch.Generator(device=dev).manual_seed(100 * it + rank), device=dev)
            g.area(area, n).copy_(x)
            out = torch.empty(n, device=dev)
            g.allreduce(area, n, out)
            parts = torch.empty(world * n, device=dev)
            dist.all_gather_into_tensor(parts, x)
            ref = parts[:n].clone()
            for r in range(1, world):  # rank order, one rounded fp32 add per rank
                ref += parts[r * n:(r + 1) * n]
            nccl = x.clone()
            dist.all_reduce(nccl)  # NCCL's order is its own beyond 2 ranks
            ok_ar &= bool(torch.equal(out, ref)) and bool(torch.allclose(out, nccl, rtol=1e-5, atol=1e-5))
            area = (it + 1) % 2
            g.area(area, n).copy_(x)
            outg = torch.empty(world * n, device=dev)
            g.allgather(area, n, outg)
            refg = torch.empty(world * n, device=dev)
            dist.all_gather_into_tensor(refg, x)
            ok_ag &= bool(torch.equal(outg, refg))
        res["allreduce"], res["allgather"] = ok_ar, ok_ag
        # replayed from a CUDA graph: two collectives per replay, alternating areas
        n = 4096
        out0, out1 = torch.empty(n, device=dev), torch.empty(n, device=dev)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                g.allreduce(0, n, out0)
                g.allreduce(1, n, out1)
        torch.cuda.current_stream().wait_stream(s)
        ok_graph = True
        for it in range(5):
            a0 = torch.full((n,), float(it + 1 + rank), device=dev)
            a1 = torch.full((n,), float(10 * it - rank), device=dev)
            g.area(0, n).copy_(a0)
            g.area(1, n).copy_(a1)
            gr.replay()
            torch.cuda.synchronize()
            exp0 = sum(float(it + 1 + r) for r in range(world))
            exp1 = sum(float(10 * it - r) for r in range(world))
            ok_graph &= bool((out0 == exp0).all()) and bool((out1 == exp1).all())
        del gr
        res["graph"] = ok_graph
        # row-sharded GEMV with the peer all-gather against the full-matrix kernel
        N, K = 6144, 5120
        W = P.random_weights(N, K, seed=77)
        r0, r1 = P.sharded.shard_rows(N, world, rank)
        S = P.sharded.RowShardedIQ4XS(W[r0:r1].contiguous(), N, K, peers=g)
        ok_sh = True
        for B in (1, 1, 3):
            X = P.fill_normal(B * K, seed=5 + B).view(B, K)
            Y = S.gemv(X)
            Yf = P.gemv(W, X, N) if B == 1 else torch.cat([P.gemv(W[a:b].contiguous(), X, b - a) for a, b in
                                                           (P.sharded.shard_rows(N, world, r) for r in range(world))], 1)
            ok_sh &= bool(torch.equal(Y, Yf))
        res["sharded"] = ok_sh
        torch.cuda.synchronize()
        g.close()
        # decoder, tensor parallel: peer collectives vs NCCL all-reduces (same model, same prompt)
        dec = P.decoder
        # one KV head group of 4 query heads and 2 FFN super-block pairs per rank
        cfg = dec.DecoderConfig(layers=2, hidden=1024, heads=4 * world, kv_heads=world, head_dim=128,
                                ffn=1024 * world, vocab=3072, max_seq=40)
        prompt = torch.randint(0, cfg.vocab, (12,), generator=torch.Generator().manual_seed(3)).to(dev)
        lg = {}
        for use_peer in (True, False):
            m = dec.TPDecoder(cfg, rank=rank, world=world, seed=4, peer_collectives=use_peer)
            m.prefill(prompt)
            toks = m.decode(5, use_graph=True)
            lg[use_peer] = (toks, m._last_logits.clone())
            m.release()
            del m
        a, b = lg[True][1].double().flatten(), lg[False][1].double().flatten()
        if world == 2:  # both collectives add the two ranks' partial sums with one rounded add
            res["decoder_tokens"] = lg[True][0] == lg[False][0]
            res["decoder_logits"] = bool(torch.equal(a, b))
        else:  # NCCL's order of the partial sums is its own: compared by cosine
            res["decoder_logits"] = bool(torch.dot(a, b) / (a.norm() * b.norm()) >= 0.999)
        # exact: fixed decode inputs from position 0 with peer collectives (rank-order sums) against
        # the single-GPU emulation of the same ranks (o_proj / down_proj K slices added in rank order)
        # (the fused all-reduce in the GEMV epilogues and the separate collective kernel alike)
        seqs = {}
        for kind in ("fused", "collective", "emu"):
            emu = kind == "emu"
            m = dec.TPDecoder(cfg, rank=0 if emu else rank, world=1 if emu else world, seed=4,
                              peer_collectives=None if emu else True, emulate_ranks=world if emu else 1,
                              fused_allreduce=kind == "fused")
            assert emu or m.fused_allreduce == (kind == "fused")
            m.reset_decode(0)
            out = []
            for t in (5, 1234, 77, 3001):
                m._tok.fill_(t)
                m._step()
                out.append(m._last_logits.clone())
            seqs[kind] = torch.cat(out)
            m.release()
            del m
        res["decoder_exact_vs_emulation"] = bool(torch.equal(seqs["fused"], seqs["emu"]))
        res["decoder_collective_exact_vs_emulation"] = bool(torch.equal(seqs["collective"], seqs["emu"]))
        torch.cuda.synchronize()
        q.put((rank, res, P.device_error(), lg[True][0]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_collectives(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from conftest import run_ranks
    out, codes = run_ranks(_worker, world, lambda r, port, q: (r, world, port, q), timeout=300)
    assert all(c == 0 for c in codes), codes
    assert len(out) == world
    for rank, res, err, toks in out:
        assert all(res.values()), (rank, res)
        assert err == 0
        assert toks == out[0][3]  # every rank holds the same tokens (identical all-reduce bits)
