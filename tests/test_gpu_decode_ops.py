"""The fused decoder-step operations (include/iq4xs_decoder.h) against the decoder's torch
formulation of the same ops in fp32, and their Q8_1 output against the library's quantizer applied
to their own fp32 values (bit-exact: both go through the same block routine)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def test_residual_rmsnorm_q8(pkg):
    T, D, eps = 3, 5120, 1e-6
    g = _gen(1)
    x = torch.randn((T, D), generator=g, device="cuda")
    delta = torch.randn((T, D), generator=g, device="cuda") * 0.5
    w = 1.0 + 0.02 * torch.randn(D, generator=g, device="cuda")
    x_ref = x + delta
    h_ref = x_ref * torch.rsqrt(x_ref.pow(2).mean(-1, keepdim=True) + eps) * w
    h = torch.empty_like(x)
    q8, _ = pkg.api.dec_residual_rmsnorm_q8(x, w, eps, delta=delta, h_out=h)
    torch.cuda.synchronize()
    assert torch.equal(x, x_ref)  # the residual add is a single rounded add, as in torch
    assert torch.allclose(h, h_ref, rtol=2e-6, atol=1e-6)
    assert torch.equal(q8, pkg.q8_1_quantize(h))
    # no residual, q8 only (the first layer), and h only (the final norm)
    x2 = torch.randn((1, D), generator=g, device="cuda")
    q8b, _ = pkg.api.dec_residual_rmsnorm_q8(x2, w, eps)
    hb = torch.empty_like(x2)
    pkg.api.dec_residual_rmsnorm_q8(x2, w, eps, h_out=hb, want_q8=False)
    torch.cuda.synchronize()
    assert torch.equal(q8b, pkg.q8_1_quantize(hb))


def _rope_ref(x, c, s):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@pytest.mark.parametrize("hq,hkv,p", [(64, 8, 0), (64, 8, 1), (64, 8, 300), (32, 4, 639), (8, 1, 77), (8, 8, 5)])
def test_attention_decode_q8(pkg, hq, hkv, p):
    hd, max_seq = 128, 640
    g = _gen(100 + p + hq)
    qkv = torch.randn((1, (hq + 2 * hkv) * hd), generator=g, device="cuda")
    kc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    vc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    kc0, vc0 = kc.clone(), vc.clone()
    inv = 1.0 / (1.0e6 ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(max_seq, dtype=torch.float64)[:, None] * inv[None, :]
    cos = torch.cos(ang).float().cuda()
    sin = torch.sin(ang).float().cuda()
    pos = torch.tensor([p], dtype=torch.long, device="cuda")
    o = torch.empty((hq * hd,), dtype=torch.float32, device="cuda")
    q8 = pkg.api.dec_attention_decode_q8(qkv, kc, vc, cos, sin, pos, hq, hkv, o_out=o)
    torch.cuda.synchronize()

    # torch formulation (the decoder's forward for one token)
    c, s = cos[p][None, :], sin[p][None, :]
    q = _rope_ref(qkv[0, :hq * hd].view(hq, hd), c, s)
    k = _rope_ref(qkv[0, hq * hd:(hq + hkv) * hd].view(hkv, hd), c, s)
    v = qkv[0, (hq + hkv) * hd:].view(hkv, hd)
    kc0[:, p] = k.half()
    vc0[:, p] = v.half()
    assert torch.equal(kc, kc0) and torch.equal(vc, vc0)  # appended at p, nothing else touched
    gq = hq // hkv
    K = kc0[:, :p + 1].float()
    V = vc0[:, :p + 1].float()
    qg = q.view(hkv, gq, hd)
    sc = torch.matmul(qg.double(), K.double().transpose(1, 2)) / math.sqrt(hd)
    ref = torch.matmul(torch.softmax(sc, dim=-1), V.double()).reshape(hq * hd)
    err = (o.double() - ref).abs()
    assert err.max().item() <= 2e-5 * max(1.0, ref.abs().max().item())
    assert torch.equal(q8[0], pkg.q8_1_quantize(o)[0])
    assert pkg.device_error() == 0


def test_attention_position_out_of_range_is_an_error(pkg):
    """The kernel's own bounds check: a position at max_seq records device error 5 and writes nothing."""
    hq, hkv, hd, max_seq = 8, 2, 128, 16
    qkv = torch.randn((1, (hq + 2 * hkv) * hd), device="cuda")
    kc = torch.zeros((hkv, max_seq, hd), device="cuda").half()
    vc = torch.zeros_like(kc)
    cs = torch.zeros((max_seq, hd // 2), device="cuda")
    pos = torch.tensor([max_seq], dtype=torch.long, device="cuda")
    q8 = torch.zeros((1, hq * hd // 32 * 36), dtype=torch.uint8, device="cuda")
    pkg.api.dec_attention_decode_q8(qkv, kc, vc, cs, cs, pos, hq, hkv, q8=q8)
    torch.cuda.synchronize()
    assert pkg.device_error() == 5
    assert int(kc.abs().sum()) == 0 and int(q8.sum()) == 0
    assert pkg.device_error() == 0  # read-and-clear


def test_swiglu_q8(pkg):
    T, F = 2, 17408
    g = _gen(9)
    gu = torch.randn((T, 2 * F), generator=g, device="cuda") * 3
    q8 = pkg.api.dec_swiglu_q8(gu, F)
    act = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    ref = pkg.q8_1_quantize(act)
    torch.cuda.synchronize()
    # same op order as torch's silu (x / (1 + exp(-x))) and mul; allow rare last-bit differences of exp
    diff = (q8 != ref).sum().item()
    assert diff <= q8.numel() // 10000, diff
    deq = lambda b: b.view(T, F // 32, 36)[..., 4:].view(torch.int8).float()
    assert (deq(q8) - deq(ref)).abs().max().item() <= 1


def test_gemv_q8_ex_matches_gemv_q8(pkg):
    N, K, B = 4096, 5120, 1
    W = pkg.api.random_weights(N, K, seed=3)
    x = torch.randn((B, K), device="cuda")
    q8 = pkg.q8_1_quantize(x)
    y0 = pkg.api.gemv_q8(W, q8, K, N, B)
    y1 = pkg.api.gemv_q8_ex(W, q8, K, N, B, flags=pkg.api.FLAG_OVERLAP_PRECEDING)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


@pytest.mark.parametrize("N,K", [(4096, 5120), (10240, 5120), (1024, 8192), (5120, 17408), (64, 25600)])
@pytest.mark.parametrize("B", [1, 2, 5, 8])
def test_gemv_f32_entry_equals_quantize_then_gemv(pkg, N, K, B):
    """The fp32 entry quantises inside the GEMV kernel (every CTA into its shared memory): the result
    equals the standalone quantizer followed by the Q8_1 GEMV bit for bit."""
    W = pkg.api.random_weights(N, K, seed=N + K)
    X = torch.randn((B, K), generator=_gen(B + K), device="cuda")
    y_fused = pkg.api.gemv(W, X, N)
    y_ref = pkg.api.gemv_q8(W, pkg.q8_1_quantize(X), K, N, B)
    torch.cuda.synchronize()
    assert torch.equal(y_fused, y_ref)
    assert pkg.device_error() == 0


@pytest.mark.parametrize("N", [10240, 2048])
@pytest.mark.parametrize("with_delta", [True, False])
def test_rmsnorm_gemv(pkg, N, with_delta):
    """Residual + RMSNorm fused into the GEMV against the standalone norm kernel + Q8_1 GEMV: the
    residual output is exact, the GEMV output agrees up to rare Q8_1 rounding flips (the sum of
    squares is reduced in a different order)."""
    K, eps = 5120, 1e-6
    g = _gen(N)
    W = pkg.api.random_weights(N, K, seed=77)
    x = torch.randn((1, K), generator=g, device="cuda")
    delta = torch.randn((1, K), generator=g, device="cuda") * 0.3 if with_delta else None
    w = 1.0 + 0.02 * torch.randn(K, generator=g, device="cuda")
    x_out = torch.full_like(x, float("nan"))
    y = pkg.api.dec_rmsnorm_gemv(W, x, w, eps, N, delta=delta, x_out=x_out if with_delta else None)
    xr = x.clone()
    q8, _ = pkg.api.dec_residual_rmsnorm_q8(xr, w, eps, delta=delta)
    y_ref = pkg.api.gemv_q8(W, q8, K, N, 1)
    torch.cuda.synchronize()
    if with_delta:
        assert torch.equal(x_out, x + delta)
    cos = torch.nn.functional.cosine_similarity(y.double(), y_ref.double(), dim=-1).item()
    assert cos >= 0.999999
    assert (y - y_ref).abs().max().item() <= 2e-3 * y_ref.abs().max().item()
    assert pkg.device_error() == 0


def test_rmsnorm_gemv_rejects_aliased_output(pkg):
    K, N = 5120, 256
    W = pkg.api.random_weights(N, K, seed=1)
    x = torch.randn((1, K), device="cuda")
    w = torch.ones(K, device="cuda")
    with pytest.raises(pkg.IQ4XSError):
        pkg.api.dec_rmsnorm_gemv(W, x, w, 1e-6, N, delta=x.clone(), x_out=x)


def test_embed(pkg):
    vocab, D = 1000, 5120
    g = _gen(7)
    emb = (0.02 * torch.randn((vocab, D), generator=g, device="cuda")).half()
    for t in (0, 1, 517, vocab - 1):
        tok = torch.tensor([t], dtype=torch.long, device="cuda")
        x = pkg.api.dec_embed(emb, tok)
        torch.cuda.synchronize()
        assert torch.equal(x, emb[tok].float())
    assert pkg.device_error() == 0


@pytest.mark.parametrize("n", [152064, 76032, 19008, 1, 4097])
def test_argmax_matches_torch(pkg, n):
    g = _gen(11 + n)
    cases = [torch.randn(n, generator=g, device="cuda")]
    tied = torch.randn(n, generator=g, device="cuda").clamp(max=1.5)  # many copies of the maximum
    cases.append(tied)
    if n > 3:
        with_nan = torch.randn(n, generator=g, device="cuda")
        with_nan[n // 3] = float("nan")
        with_nan[n - 1] = float("nan")
        cases.append(with_nan)
        neg = -torch.rand(n, generator=g, device="cuda") - 1.0
        neg[n - 2] = float("-inf")
        cases.append(neg)
    for v in cases:
        tok = torch.zeros(1, dtype=torch.long, device="cuda")
        pos = torch.tensor([41], dtype=torch.long, device="cuda")
        pkg.api.dec_argmax(v.view(1, n), tok, pos)
        torch.cuda.synchronize()
        assert int(tok) == int(torch.argmax(v)), (n, int(tok), int(torch.argmax(v)))
        assert int(pos) == 42
    tok = torch.zeros(1, dtype=torch.long, device="cuda")
    pkg.api.dec_argmax(cases[0], tok)  # no position
    torch.cuda.synchronize()
    assert int(tok) == int(torch.argmax(cases[0]))


@pytest.mark.parametrize("F,N", [(2560, 5120), (4608, 5120), (6144, 1000), (8704, 5120), (17408, 5120)])
def test_swiglu_gemv_matches_separate_kernels(pkg, F, N):
    # SwiGLU inside the down_proj GEMV (every CTA builds the Q8_1 blocks for F <= 6144, the standalone
    # SwiGLU kernel into the workspace beyond) gives the bits of swiglu_q8 followed by the Q8_1 GEMV
    g = _gen(300 + F)
    W = pkg.random_weights(N, F, seed=700 + F)
    gu = torch.randn((1, 2 * F), generator=g, device="cuda") * 2.0
    q8 = pkg.api.dec_swiglu_q8(gu, F)
    y_ref = pkg.gemv_q8(W, q8, F, N, 1)
    y = pkg.api.dec_swiglu_gemv(W, gu, F, N)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    assert pkg.device_error() == 0


@pytest.mark.parametrize("hq,hkv,p", [(64, 8, 512), (8, 1, 77)])
def test_attention_early_state_same_bits(pkg, hq, hkv, p):
    # IQ4XS_FLAG_ATTN_EARLY_STATE (position, cache and RoPE tables read before waiting for the
    # preceding kernel, as a programmatic dependent): the same cache and outputs as the plain launch
    hd, max_seq = 128, 640
    g = _gen(500 + p)
    qkv = torch.randn((1, (hq + 2 * hkv) * hd), generator=g, device="cuda")
    kc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    vc = torch.randn((hkv, max_seq, hd), generator=g, device="cuda").half()
    cos = torch.randn((max_seq, hd // 2), generator=g, device="cuda")
    sin = torch.randn((max_seq, hd // 2), generator=g, device="cuda")
    pos = torch.tensor([p], dtype=torch.long, device="cuda")
    outs = []
    for flags in (0, pkg.api.FLAG_PDL | pkg.api.FLAG_ATTN_EARLY_STATE):
        k1, v1 = kc.clone(), vc.clone()
        qkv2 = qkv * 1.0  # a kernel right before the launch (its programmatic predecessor)
        o = torch.empty((hq * hd,), dtype=torch.float32, device="cuda")
        q8 = pkg.api.dec_attention_decode_q8(qkv2, k1, v1, cos, sin, pos, hq, hkv, o_out=o, flags=flags)
        torch.cuda.synchronize()
        outs.append((k1, v1, o, q8))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    assert pkg.device_error() == 0
