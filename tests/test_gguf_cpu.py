"""IQ4_XS matrices through GGUF files (gguf_weights.py): written with gguf-py's writer, read back
byte for byte, non-IQ4_XS tensors skipped or refused by name, and the oracle matmul over the loaded
bytes equal to the one over the originals."""
import numpy as np
import pytest


def _model(O):
    Wq = O.quantize_iq4_xs(O.normal(64 * 512, 1, 0.0, 0.02).reshape(64, 512))
    Wd = O.quantize_iq4_xs(O.normal(48 * 1024, 2, 0.0, 0.02).reshape(48, 1024))
    norm = np.linspace(0.5, 1.5, 512, dtype=np.float32)
    return {"blk.0.attn_q.weight": Wq, "blk.0.ffn_down.weight": Wd}, {"blk.0.attn_norm.weight": norm}


def test_gguf_round_trip(pkg, O, tmp_path):
    G = pkg.gguf_weights
    mats, extra = _model(O)
    path = tmp_path / "m.gguf"
    G.write_iq4xs(path, mats, extra=extra)
    got = G.read_iq4xs(path, device="cpu")
    assert set(got) == set(mats)  # the fp32 norm is not an IQ4_XS matrix
    q, d = got["blk.0.attn_q.weight"], got["blk.0.ffn_down.weight"]
    assert (q.K, q.N, d.K, d.N) == (512, 64, 1024, 48)
    assert np.array_equal(q.data.numpy(), mats["blk.0.attn_q.weight"])
    assert np.array_equal(d.data.numpy(), mats["blk.0.ffn_down.weight"])
    x = O.normal(2 * 1024, 3).reshape(2, 1024)
    Q = O.quantize_q8_1(x)
    y0, _ = O.matmul_q8(mats["blk.0.ffn_down.weight"], Q, 1024, 48, 2)
    y1, _ = O.matmul_q8(d.data.numpy(), Q, 1024, 48, 2)
    assert np.array_equal(y0, y1)


def test_gguf_named_reads(pkg, O, tmp_path):
    G = pkg.gguf_weights
    mats, extra = _model(O)
    path = tmp_path / "m.gguf"
    G.write_iq4xs(path, mats, extra=extra)
    sub = G.read_iq4xs(path, names=["blk.0.ffn_down.weight"], device="cpu")
    assert list(sub) == ["blk.0.ffn_down.weight"]
    with pytest.raises(ValueError):
        G.read_iq4xs(path, names=["blk.0.attn_norm.weight"], device="cpu")  # fp32, not IQ4_XS
    with pytest.raises(ValueError):
        G.read_iq4xs(path, names=["blk.9.attn_q.weight"], device="cpu")     # absent
    with pytest.raises(ValueError):
        G.write_iq4xs(tmp_path / "bad.gguf", {"w": np.zeros((4, 100), dtype=np.uint8)})  # not whole blocks
