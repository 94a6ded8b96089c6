"""The decoder on the CUDA kernels (one GPU) against the same model with the FP64 pipeline
reference for every matmul: logits within a small relative bound, identical greedy tokens, the same
tokens with and without the CUDA-graph decode step."""
import torch
import pytest

import torch_ref

pytestmark = pytest.mark.gpu


def test_decoder_kernels_vs_reference(pkg):
    dec = pkg.decoder
    cfg = dec.DecoderConfig(layers=3, hidden=1024, heads=8, kv_heads=2, head_dim=128, ffn=2048, vocab=3000,
                            max_seq=48)

    def ref_matmul(W, X, N):
        q8 = pkg.q8_1_quantize(X.contiguous())
        Y64, _ = torch_ref.matmul_q8(W, q8, X.shape[1])
        return Y64.float()

    prompt = torch.randint(0, cfg.vocab, (20,), generator=torch.Generator().manual_seed(5)).cuda()
    runs = {}
    for name, mm, graph in (("kernels", None, True), ("kernels_eager", None, False), ("reference", ref_matmul, False)):
        m = dec.TPDecoder(cfg, seed=11, matmul=mm)
        first, lg = m.prefill(prompt)
        toks = [int(first)] + m.decode(8, use_graph=graph)
        runs[name] = (toks, lg.clone())
        m.release()
        del m
    assert runs["kernels"][0] == runs["kernels_eager"][0]
    k, r = runs["kernels"][1], runs["reference"][1]
    assert torch.max(torch.abs(k - r)) <= 1e-3 * torch.max(torch.abs(r))
    assert runs["kernels"][0][:6] == runs["reference"][0][:6]
    torch.cuda.synchronize()
    assert pkg.device_error() == 0


def test_fused_decode_layers_vs_torch_ops(pkg):
    """The fused decode layers (RMSNorm/attention/SwiGLU kernels producing Q8_1, GEMVs on Q8_1 input)
    against the same kernels' GEMVs with the torch ops between them: per-step logits agree to the
    level of a Q8_1 rounding flip, and the greedy tokens are the same."""
    dec = pkg.decoder
    cfg = dec.DecoderConfig(layers=3, hidden=1024, heads=8, kv_heads=2, head_dim=128, ffn=2048, vocab=3000,
                            max_seq=48)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=torch.Generator().manual_seed(6)).cuda()
    out = {}
    for fused in (True, False):
        m = dec.TPDecoder(cfg, seed=12, fused_decode=fused)
        m.prefill(prompt)
        toks, lgs = [], []
        for _ in range(6):
            toks.append(int(m._step()))
            lgs.append(m._last_logits.clone())
        out[fused] = (toks, torch.cat(lgs))
        m.release()
        del m
    assert out[True][0] == out[False][0]
    a, b = out[True][1].double(), out[False][1].double()
    cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
    assert cos.min().item() >= 0.9999
    assert torch.max(torch.abs(a - b)) <= 2e-2 * torch.max(torch.abs(b))
    assert pkg.device_error() == 0


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_rank_emulation_on_one_gpu(pkg, ranks):
    """TPDecoder(emulate_ranks=R) on one GPU (the reference a TP-R run is compared with bit for bit on
    several GPUs): the o_proj / down_proj GEMVs of the decode step run as R K slices added in rank
    order.  Against the plain one-GPU model the sums of the slices differ by fp32 rounding only, so
    the logits agree by cosine; the emulated decode is deterministic (two runs, the same bits)."""
    dec = pkg.decoder
    cfg = dec.DecoderConfig(layers=2, hidden=1024, heads=4 * ranks, kv_heads=ranks, head_dim=128, ffn=1024 * ranks,
                            vocab=3072, max_seq=40)
    seqs = {}
    for name, emu in (("plain", 1), ("emulated", ranks), ("emulated_again", ranks)):
        m = dec.TPDecoder(cfg, seed=4, emulate_ranks=emu)
        m.reset_decode(0)
        out = []
        for t in (5, 1234, 77, 3001):
            m._tok.fill_(t)
            m._step()
            out.append(m._last_logits.clone())
        seqs[name] = torch.cat(out).double().flatten()
        m.release()
        del m
    assert torch.equal(seqs["emulated"], seqs["emulated_again"])
    a, b = seqs["emulated"], seqs["plain"]
    assert torch.dot(a, b) / (a.norm() * b.norm()) >= 0.999
    torch.cuda.synchronize()
    assert pkg.device_error() == 0
