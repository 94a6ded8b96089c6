"""IQ4_XS matrices read from a GGUF file straight to the device (chunked through a pinned buffer)
run the GEMV bit for bit like the same bytes uploaded directly."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_gguf_weights_on_device(pkg, O, tmp_path, monkeypatch):
    G = pkg.gguf_weights
    monkeypatch.setattr(G, "_CHUNK", 1 << 20)  # several copy rounds for a 2.8 MB matrix
    N, K = 1024, 5120
    W = O.quantize_iq4_xs(O.normal(N * K, 11, 0.0, 0.02).reshape(N, K))
    path = tmp_path / "kv.gguf"
    G.write_iq4xs(path, {"blk.0.attn_k.weight": W})
    m = G.read_iq4xs(path)["blk.0.attn_k.weight"]
    assert m.data.is_cuda and (m.K, m.N) == (K, N)
    Wd = torch.from_numpy(W).cuda()
    assert torch.equal(m.data, Wd)
    X = pkg.fill_normal(3 * K, seed=4).view(3, K)
    torch.cuda.synchronize()
    assert torch.equal(pkg.gemv(m.data, X, N), pkg.gemv(Wd, X, N))
    assert pkg.device_error() == 0
