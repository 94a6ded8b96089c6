"""The tensor-parallel decoder's host logic on CPU ranks (gloo): a tiny config at TP=2 against TP=1.

Matmuls are the FP64 oracle of the quantised pipeline (injected), weights are quantised by the C
oracle; the test covers the head / FFN partition, the K-slicing of the row-parallel layers, the
all-reduces, the KV cache and RoPE/attention indexing, and the sharded lm_head."""
import os

import numpy as np
import torch


def tiny_cfg(dec, heads=8, kv_heads=2, ffn=1024):
    return dec.DecoderConfig(layers=2, hidden=512, heads=heads, kv_heads=kv_heads, head_dim=128, ffn=ffn,
                             vocab=1000, max_seq=40)


def _worker(rank, world, port, q, cfg_kw=None, exact=False):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    import torch.distributed as dist
    from conftest import load_pkg
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dec = load_pkg().decoder

        def matmul(W, X, N):
            Xn = np.ascontiguousarray(X.numpy(), dtype=np.float32)
            K = Xn.shape[1]
            if exact:  # unquantised activations, FP64 sums: no Q8_1 rounding flips between partitions
                return torch.from_numpy(O.matmul_f64(W.numpy(), Xn, K, N, Xn.shape[0]))
            Y, _ = O.matmul_q8(W.numpy(), O.quantize_q8_1(Xn), K, N, Xn.shape[0])
            return torch.from_numpy(Y.astype(np.float32))

        def gen_weights(N, K, s):
            return torch.from_numpy(O.quantize_iq4_xs(O.normal(N * K, s, 0.0, 0.02).reshape(N, K)))

        def gen_normal(n, s, mean, std):
            return torch.from_numpy(O.normal(n, s, mean, std))

        m = dec.TPDecoder(tiny_cfg(dec, **(cfg_kw or {})), rank=rank, world=world, seed=3, device="cpu", matmul=matmul,
                          gen_weights=gen_weights, gen_normal=gen_normal)
        prompt = torch.from_numpy(np.random.default_rng(7).integers(0, 1000, 12)).long()
        first, lg = m.prefill(prompt)
        toks = [int(first)] + m.decode(6, use_graph=False)
        q.put((rank, toks, lg.numpy(), m._last_logits.numpy()))
    finally:
        dist.destroy_process_group()


def _run(world, cfg_kw=None, exact=False):
    from conftest import run_ranks
    out, codes = run_ranks(_worker, world, lambda r, port, q: (r, world, port, q, cfg_kw, exact))
    assert all(c == 0 for c in codes), codes
    return sorted(out, key=lambda r: r[0])


def test_tp2_matches_tp1():
    one = _run(1)[0]
    two = _run(2)
    for rank, toks, lg, last in two:
        # the all-reduce adds the two halves of o_proj / down_proj in another order: tiny differences
        assert np.max(np.abs(lg - one[2])) <= 1e-3 * np.max(np.abs(one[2]))
        assert toks[:4] == one[1][:4], (toks, one[1])
    assert two[0][1] == two[1][1]      # both ranks hold the same tokens


def test_tp4_matches_tp1():
    """Four ranks: one KV head and four query heads each, an FFN of 5 super-block pairs split
    unevenly (2/1/1/1), the lm_head over 4 shards."""
    kw = dict(heads=16, kv_heads=4, ffn=2560)
    one = _run(1, kw)[0]
    four = _run(4, kw)
    for rank, toks, lg, last in four:
        assert np.max(np.abs(lg - one[2])) <= 1e-3 * np.max(np.abs(one[2]))
        assert toks[:4] == one[1][:4]


def test_tp8_matches_tp1():
    """Eight ranks, as on a full 8-GPU box: one KV head and four query heads each, an FFN of 9
    super-block pairs split 2/1/1/1/1/1/1/1, the lm_head over 8 shards.  The matmul is the unquantised
    FP64 one, so the partitioning must reproduce TP=1 up to fp32 rounding of the partial sums (with
    Q8_1 activations a partial sum that lands on the other side of a rounding boundary flips one
    quant, and two layers amplify that to ~1e-2 of the largest logit)."""
    kw = dict(heads=32, kv_heads=8, ffn=4608)
    one = _run(1, kw, exact=True)[0]
    eight = _run(8, kw, exact=True)
    for rank, toks, lg, last in eight:
        assert np.max(np.abs(lg - one[2])) <= 1e-5 * np.max(np.abs(one[2]))
        assert np.max(np.abs(last - one[3])) <= 1e-5 * np.max(np.abs(one[3]))
        assert toks == one[1]
    assert all(r[1] == eight[0][1] for r in eight)
