"""Known-answer tests of the oracle, derived by reading the reference formulas.

* scale decode ls = (scales_l nibble) | (scales_h 2 bits << 4) (ref_cpu.cpp:30-33)
* nibble order: qs byte j of sub-block ib -> element j (low) and j+16 (high) (ref_cpu.cpp:38-47)
* Q8_1: d = amax/127, q = roundf(x/d) half away from zero, all-zero block -> q = 0 and ds = 0
  (real_stock_dp4a_comparator.hip:252-263)
"""
import numpy as np
import pytest

KV = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int64)


def make_block(d16: int, ls_codes, qs: np.ndarray) -> np.ndarray:
    b = np.zeros(136, dtype=np.uint8)
    b[0:2] = np.array([d16], dtype=np.uint16).view(np.uint8)
    sh = 0
    sl = np.zeros(4, dtype=np.uint8)
    for ib, ls in enumerate(ls_codes):
        sl[ib // 2] |= (ls & 0xF) << (4 * (ib & 1))
        sh |= (ls >> 4) << (2 * ib)
    b[2:4] = np.array([sh], dtype=np.uint16).view(np.uint8)
    b[4:8] = sl
    b[8:] = qs
    return b


def q8_block(values, d16=0x3C00) -> np.ndarray:
    q = np.zeros(36, dtype=np.uint8)
    q[0:2] = np.array([d16], dtype=np.uint16).view(np.uint8)
    q[4:] = np.asarray(values, dtype=np.int8).view(np.uint8)
    return q


def test_every_scale_code_and_nibble(O):
    L = O.lib()
    rng = np.random.default_rng(0)
    for base in range(0, 64, 8):
        codes = list(range(base, base + 8))
        qs = rng.integers(0, 256, 128).astype(np.uint8)
        blk = make_block(0x3C00, codes, qs)  # d = 1.0
        deq = O.dequantize(blk[None], 256, 1)[0]
        for ib in range(8):
            assert L.or_iq4xs_scale(blk.ctypes.data, ib) == codes[ib]
            for j in range(16):
                lo, hi = qs[16 * ib + j] & 15, qs[16 * ib + j] >> 4
                assert deq[32 * ib + j] == (codes[ib] - 32) * KV[lo]
                assert deq[32 * ib + j + 16] == (codes[ib] - 32) * KV[hi]


def test_subblock_dot_one_hot_recovers_codebook(O):
    rng = np.random.default_rng(1)
    qs = rng.integers(0, 256, 128).astype(np.uint8)
    blk = make_block(0x3C00, [40] * 8, qs)
    for ib in (0, 5):
        for e in range(32):
            v = np.zeros(32, dtype=np.int64)
            v[e] = 1
            Q = np.tile(q8_block(v), 8)  # one Q8_1 block per sub-block of the super-block
            S = O.subblock_dots(blk[None], Q[None], 256, 1, 1)[0, 0]
            byte = qs[16 * ib + (e % 16)]
            code = (byte & 15) if e < 16 else (byte >> 4)
            assert S[ib] == KV[code]


def test_q8_1_zero_block(O):
    Q = O.quantize_q8_1(np.zeros((1, 32), dtype=np.float32))
    assert np.all(Q == 0)


def test_q8_1_extremes_and_ties(O):
    # amax = 127 -> d = 1.0 exactly; x/d = x, ties round away from zero.
    x = np.zeros(32, dtype=np.float32)
    x[0], x[1], x[2], x[3], x[4], x[5], x[6] = 127.0, -127.0, 2.5, -2.5, 0.5, -0.5, 1.49999
    Q = O.quantize_q8_1(x[None])[0]
    q = Q[4:].view(np.int8)
    assert list(q[:7]) == [127, -127, 3, -3, 1, -1, 1]
    assert Q[0:2].view(np.uint16)[0] == 0x3C00  # d = 1.0
    s = Q[2:4].view(np.uint16)[0]
    assert s == np.float16(1.49999 + 0.0).view(np.uint16) or s == O.lib().or_fp32_to_fp16_trunc(np.float32(1.49999))


def test_q8_1_scale_truncates(O):
    # amax chosen so amax/127 is not representable in fp16: the stored d is truncated, not rounded.
    x = np.zeros(32, dtype=np.float32)
    x[7] = 1.0
    Q = O.quantize_q8_1(x[None])[0]
    d = np.float32(1.0) / np.float32(127.0)
    assert Q[0:2].view(np.uint16)[0] == O.lib().or_fp32_to_fp16_trunc(d)
    assert np.float16(Q[0:2].view(np.float16)[0]) <= d


@pytest.mark.parametrize("scale", [1e-3, 1.0, 300.0])
def test_q8_1_roundtrip_error(O, scale):
    rng = np.random.default_rng(7)
    X = (rng.standard_normal((3, 256)) * scale).astype(np.float32)
    Q = O.quantize_q8_1(X)
    q = Q.reshape(3, 8, 36)[:, :, 4:].view(np.int8).astype(np.float64)
    d = O.q8_scales(Q, 3, 256).astype(np.float64)[:, :, None]
    amax = np.abs(X.reshape(3, 8, 32)).max(axis=2)[:, :, None]
    err = np.abs(q * (amax / 127.0) - X.reshape(3, 8, 32))
    assert np.all(err <= amax / 127.0 * 0.5 * (1 + 1e-5))
    assert np.all(np.abs(q) <= 127)
    assert np.all(d <= amax / 127.0 + 1e-30)


def test_weight_quantizer_valid_and_accurate(O):
    import gguf
    from gguf import quants
    rng = np.random.default_rng(3)
    src = (rng.standard_normal((16, 1024)) * 0.02).astype(np.float32)
    W = O.quantize_iq4_xs(src)
    dq = O.dequantize(W, 1024, 16)
    # An independent reading of the format (gguf-py's IQ4_XS dequantizer) agrees bit for bit.
    g = quants.dequantize(W, gguf.GGMLQuantizationType.IQ4_XS).reshape(16, 1024)
    assert np.array_equal(g.astype(np.float32), dq)
    rel = np.linalg.norm(dq - src) / np.linalg.norm(src)
    assert rel < 0.09, rel  # 4.25 bpw on Gaussian data
    # all-zero super-block -> zero scale, exact zeros back
    Z = O.quantize_iq4_xs(np.zeros((1, 256), dtype=np.float32))
    assert np.all(O.dequantize(Z, 256, 1) == 0)
