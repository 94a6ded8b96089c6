"""bench.py's host arithmetic on CPU: the algorithmic byte count of the decode GEMV sweep (the
numerator of the headline GB/s, the reference's formula N*K*17/32 weight bytes plus fp32 x and y)
and the logit-agreement record of the multi-GPU parity check."""
import sys

import pytest
import torch

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_gemv_bytes_formula():
    # one super-block of 256 weights is 136 bytes; x and y are fp32 per token
    assert bench.gemv_bytes(1, 256, 1) == 136 + 4 * 256 + 4
    assert bench.gemv_bytes(4096, 4096, 1) == 4096 * 4096 * 17 // 32 + 4 * 4096 + 4 * 4096
    assert bench.gemv_bytes(8192, 5120, 8) == 8192 * 5120 * 17 // 32 + 8 * 4 * (5120 + 8192)


def test_step_bytes_is_the_sweep():
    weights = sum(N * K * 17 // 32 for _, N, K in bench.SHAPES)
    acts = sum(4 * B * (K + N) for B in bench.BATCHES for _, N, K in bench.SHAPES)
    assert bench.step_bytes() == len(bench.BATCHES) * weights + acts == 774_819_840
    # the layer shapes of the 27B-class config (out x in)
    assert dict((n, (N, K)) for n, N, K in bench.SHAPES) == {
        "q_proj": (8192, 5120), "k_proj": (1024, 5120), "v_proj": (1024, 5120),
        "o_proj": (5120, 8192), "gate_up": (34816, 5120), "down": (5120, 17408)}


def test_logit_agreement():
    g = torch.Generator().manual_seed(5)
    b = torch.randn(1000, generator=g, dtype=torch.float64)
    same = bench.logit_agreement(b.clone(), b)
    assert same == {"cosine": 1.0, "max_rel": 0.0, "argmax_same": True, "top5_common": 5}
    a = b.clone()
    i = int(b.argmax())
    a[i] = b.min() - 1.0  # the largest logit becomes the smallest
    r = bench.logit_agreement(a, b)
    assert not r["argmax_same"] and r["top5_common"] == 4 and r["cosine"] < 1.0
    assert r["max_rel"] == pytest.approx(float((a - b).abs().max() / b.abs().max()), rel=1e-3)
