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
