"""C-ABI checks that need no GPU: the library loads, exports every symbol declared in
include/iq4xs.h, and rejects bad arguments before touching the device."""
import ctypes as C
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "iq4xs.h"
BENCH_HEADER = ROOT / "include" / "iq4xs_bench.h"
DECODER_HEADER = ROOT / "include" / "iq4xs_decoder.h"
PEER_HEADER = ROOT / "include" / "iq4xs_peer.h"


def declared_functions(header=HEADER):
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s+\*?([A-Za-z_][A-Za-z0-9_]*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while", "return")))


def test_header_parses():
    names = declared_functions()
    assert "iq4xs_gemv_f32" in names and "custom_gemv_iq4xs_dispatch" in names
    assert len(names) >= 20


def test_every_declared_symbol_is_exported(pkg):
    L = pkg.lib()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_python_signatures_cover_header(pkg):
    assert set(pkg.SIGNATURES) == set(declared_functions())
    assert set(pkg.api.BENCH_SIGNATURES) == set(declared_functions(BENCH_HEADER))
    assert set(pkg.api.DECODER_SIGNATURES) == set(declared_functions(DECODER_HEADER))
    assert set(pkg.api.PEER_SIGNATURES) == set(declared_functions(PEER_HEADER))


def test_every_header_is_covered():
    assert sorted(p.name for p in (ROOT / "include").glob("*.h")) == sorted(
        p.name for p in (HEADER, BENCH_HEADER, DECODER_HEADER, PEER_HEADER))


def test_bench_header_symbols_exported(pkg):
    L = pkg.lib()
    for name in declared_functions(BENCH_HEADER) + declared_functions(DECODER_HEADER) + declared_functions(PEER_HEADER):
        assert hasattr(L, name), name


def test_decoder_op_validation(pkg):
    L = pkg.lib()
    # rmsnorm: D % 32, D > 8192, neither output, misaligned x
    assert L.iq4xs_dec_residual_rmsnorm_q8(FAKE, None, FAKE, 100, 1, 1e-6, FAKE, None, 0, None) == 2
    assert L.iq4xs_dec_residual_rmsnorm_q8(FAKE, None, FAKE, 8224, 1, 1e-6, FAKE, None, 0, None) == 2
    assert L.iq4xs_dec_residual_rmsnorm_q8(FAKE, None, FAKE, 5120, 1, 1e-6, None, None, 0, None) == 1
    assert L.iq4xs_dec_residual_rmsnorm_q8(FAKE + 2, None, FAKE, 5120, 1, 1e-6, FAKE, None, 0, None) == 3
    # attention: head_dim, GQA divisibility, max_seq, cache alignment, null pos
    args = (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE)
    assert L.iq4xs_dec_attention_decode_q8(*args, 64, 8, 64, 640, FAKE, None, 0, None) == 2
    assert L.iq4xs_dec_attention_decode_q8(*args, 60, 8, 128, 640, FAKE, None, 0, None) == 2
    assert L.iq4xs_dec_attention_decode_q8(*args, 64, 8, 128, 9000, FAKE, None, 0, None) == 2
    assert L.iq4xs_dec_attention_decode_q8(FAKE, FAKE + 8, FAKE, FAKE, FAKE, FAKE, 64, 8, 128, 640, FAKE, None, 0,
                                           None) == 3
    assert L.iq4xs_dec_attention_decode_q8(FAKE, FAKE, FAKE, FAKE, FAKE, None, 64, 8, 128, 640, FAKE, None, 0,
                                           None) == 1
    # swiglu: F % 32
    assert L.iq4xs_dec_swiglu_q8(FAKE, 100, 1, FAKE, 0, None) == 2
    assert L.iq4xs_dec_swiglu_q8(None, 128, 1, FAKE, 0, None) == 1
    # fused norm GEMV: x_out aliasing x, K too long, misaligned W
    assert L.iq4xs_dec_rmsnorm_gemv(FAKE, FAKE, None, FAKE, 1e-6, FAKE, FAKE, 5120, 64, FAKE, 1 << 30, 0, None) == 1
    assert L.iq4xs_dec_rmsnorm_gemv(FAKE, FAKE, None, FAKE, 1e-6, None, FAKE, 25600, 64, FAKE, 1 << 30, 0, None) == 7
    assert L.iq4xs_dec_rmsnorm_gemv(FAKE + 4, FAKE, None, FAKE, 1e-6, None, FAKE, 5120, 64, FAKE, 1 << 30, 0, None) == 3
    # gemv_q8_ex shares gemv_q8's checks
    assert L.iq4xs_gemv_q8_ex(FAKE, FAKE, FAKE, 500, 64, 1, FAKE, 1 << 30, 1, None) == 2
    # embedding: D % 8, null token, misaligned table
    assert L.iq4xs_dec_embed(FAKE, FAKE, 1000, 100, FAKE, 0, None) == 2
    assert L.iq4xs_dec_embed(FAKE, None, 1000, 128, FAKE, 0, None) == 1
    assert L.iq4xs_dec_embed(FAKE + 8, FAKE, 1000, 128, FAKE, 0, None) == 3
    # argmax: empty input, null token, misaligned position
    assert L.iq4xs_dec_argmax(FAKE, 0, FAKE, None, 0, None) == 1
    assert L.iq4xs_dec_argmax(FAKE, 100, None, None, 0, None) == 1
    assert L.iq4xs_dec_argmax(FAKE, 100, FAKE, FAKE + 4, 0, None) == 3
    # SwiGLU GEMV: K % 256, no output, workspace too small, misaligned gu, K past the row kernel
    need = L.iq4xs_gemv_workspace_bytes(5120, 64, 1)
    assert L.iq4xs_dec_swiglu_gemv(FAKE, FAKE, 500, 64, FAKE, FAKE, 1 << 30, 0, None) == 2
    assert L.iq4xs_dec_swiglu_gemv(FAKE, FAKE, 5120, 64, None, FAKE, 1 << 30, 0, None) == 1
    assert L.iq4xs_dec_swiglu_gemv(FAKE, FAKE, 5120, 64, FAKE, FAKE, need - 1, 0, None) == 4
    assert L.iq4xs_dec_swiglu_gemv(FAKE, FAKE + 4, 5120, 64, FAKE, FAKE, 1 << 30, 0, None) == 3
    assert L.iq4xs_dec_swiglu_gemv(FAKE, FAKE, 25600, 64, FAKE, FAKE, 1 << 30, 0, None) == 7
    assert L.iq4xs_dec_swiglu_gemv_push(FAKE, FAKE, 5120, 64, None, FAKE, 1 << 30, 0, None) == 1


def test_status_strings(pkg):
    L = pkg.lib()
    assert L.iq4xs_status_string(0) == b"ok"
    assert L.iq4xs_status_string(2) == b"unsupported shape"
    assert L.iq4xs_version() >= 100


FAKE = 0x10000  # never dereferenced: validation fails first


def test_validation_before_any_launch(pkg):
    L = pkg.lib()
    big = 1 << 30
    assert L.iq4xs_gemv_q8(None, FAKE, FAKE, 512, 64, 1, FAKE, big, None) == 1
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 500, 64, 1, FAKE, big, None) == 2      # K % 256
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 512, 0, 1, FAKE, big, None) == 1       # N <= 0
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 512, 64, 9, FAKE, big, None) == 2      # batch > 8
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 512, 64, 0, FAKE, big, None) == 2      # batch < 1
    assert L.iq4xs_gemv_q8(FAKE + 4, FAKE, FAKE, 512, 64, 1, FAKE, big, None) == 3  # W not 8-byte aligned
    need_q8 = L.iq4xs_gemv_q8_workspace_bytes(5120, 1024, 2)  # K split over CTAs: partial sums
    assert need_q8 > 0
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 5120, 1024, 2, FAKE, need_q8 - 1, None) == 4  # no room
    assert L.iq4xs_gemv_q8(FAKE, FAKE, FAKE, 5120, 1024, 2, None, need_q8, None) == 1      # no workspace
    assert L.iq4xs_q8_1_quantize(None, FAKE, 512, 1, None) == 1
    need = L.iq4xs_gemv_workspace_bytes(512, 64, 2)
    assert need >= 2 * 16 * 36  # the Q8_1 activations at least
    assert L.iq4xs_gemv_f32(FAKE, FAKE, FAKE, 512, 64, 2, FAKE, need - 1, None) == 4
    assert L.iq4xs_q8_1_quantize(FAKE, FAKE, 100, 1, None) == 2
    assert L.iq4xs_q8_1_bytes(5120, 3) == 3 * 160 * 36
    assert L.iq4xs_quantize_weights(FAKE, FAKE, 4, 300, None) == 2


def test_grouped_validation_and_workspace(pkg):
    """iq4xs_gemv_grouped on the host: the workspace covers every problem's Q8_1 activations (each
    slice 256-byte aligned), an invalid group sizes to 0, and bad arguments are rejected before any
    launch (nothing here reaches the device)."""
    L = pkg.lib()
    Prob = pkg.api.GemvProblem

    def group(items):
        a = (Prob * max(len(items), 9))()
        for i, it in enumerate(items):
            a[i] = Prob(*it)
        return C.cast(a, C.c_void_p), a

    layer = [(5120, 8192), (5120, 1024), (5120, 1024), (8192, 5120), (5120, 34816), (17408, 5120)]
    ok, keep = group([(FAKE, FAKE, FAKE, K, N) for K, N in layer])
    for B in range(1, 9):
        need = L.iq4xs_gemv_grouped_workspace_bytes(ok, 6, B)
        q8 = sum((L.iq4xs_q8_1_bytes(K, B) + 255) // 256 * 256 for K, _ in layer)
        assert need >= q8 and need % 256 == 0
    assert L.iq4xs_gemv_grouped_workspace_bytes(ok, 0, 1) == 0
    assert L.iq4xs_gemv_grouped_workspace_bytes(ok, 9, 1) == 0     # more than IQ4XS_MAX_GROUP
    assert L.iq4xs_gemv_grouped_workspace_bytes(ok, 6, 0) == 0
    assert L.iq4xs_gemv_grouped_workspace_bytes(ok, 6, 9) == 0
    odd, k1 = group([(FAKE, FAKE, FAKE, 500, 64)])
    assert L.iq4xs_gemv_grouped_workspace_bytes(odd, 1, 1) == 0

    big = 1 << 40
    need = L.iq4xs_gemv_grouped_workspace_bytes(ok, 6, 2)
    assert L.iq4xs_gemv_grouped(None, 1, 1, FAKE, big, 0, None) == 1
    assert L.iq4xs_gemv_grouped(ok, 0, 1, FAKE, big, 0, None) == 1
    assert L.iq4xs_gemv_grouped(ok, 9, 1, FAKE, big, 0, None) == 2      # more than IQ4XS_MAX_GROUP
    assert L.iq4xs_gemv_grouped(ok, 6, 9, FAKE, big, 0, None) == 2      # batch > 8
    assert L.iq4xs_gemv_grouped(odd, 1, 1, FAKE, big, 0, None) == 2     # K % 256
    null_w, k2 = group([(None, FAKE, FAKE, 5120, 64)])
    assert L.iq4xs_gemv_grouped(null_w, 1, 1, FAKE, big, 0, None) == 1
    mis_w, k3 = group([(FAKE + 4, FAKE, FAKE, 5120, 64)])
    assert L.iq4xs_gemv_grouped(mis_w, 1, 1, FAKE, big, 0, None) == 3   # W not 8-byte aligned
    assert L.iq4xs_gemv_grouped(ok, 6, 2, None, need, 0, None) == 1     # no workspace
    assert L.iq4xs_gemv_grouped(ok, 6, 2, FAKE, need - 1, 0, None) == 4
    assert L.iq4xs_gemv_grouped(ok, 6, 2, FAKE + 16, need, 0, None) == 3  # workspace not 256-byte aligned


def test_ggml_can_handle(pkg):
    assert pkg.custom_gemv_iq4xs_can_handle(5120, 17408, 1)
    assert pkg.custom_gemv_iq4xs_can_handle(4096, 4096, 8)
    assert not pkg.custom_gemv_iq4xs_can_handle(4096, 4096, 9)
    assert not pkg.custom_gemv_iq4xs_can_handle(4000, 4096, 1)
    assert not pkg.custom_gemv_iq4xs_can_handle(4096, 4096, 1, 12)  # another ggml type
    # GEMM hook: the patch's gate (patch:148-151) -- M >= 16 and K % 256 == 0, odd K/256 included
    assert pkg.custom_gemm_iq4xs_can_handle(5120, 17408, 16)
    assert pkg.custom_gemm_iq4xs_can_handle(2304, 5120, 512)
    assert pkg.custom_gemm_iq4xs_can_handle(768, 1000, 64)
    assert not pkg.custom_gemm_iq4xs_can_handle(5120, 17408, 15)
    assert not pkg.custom_gemm_iq4xs_can_handle(1000, 4096, 64)
    assert not pkg.custom_gemm_iq4xs_can_handle(5120, 4096, 64, 12)


def test_peer_validation(pkg):
    import ctypes as C
    L = pkg.lib()
    arr = C.c_void_p * 2
    ok = arr(FAKE, FAKE)
    assert L.iq4xs_peer_collective(ok, ok, FAKE, FAKE, 0, 9, 0, 64, FAKE, 0, None) == 1      # world > 8
    assert L.iq4xs_peer_collective(ok, ok, FAKE, FAKE, 2, 2, 0, 64, FAKE, 0, None) == 1      # rank >= world
    assert L.iq4xs_peer_collective(arr(FAKE, None), ok, FAKE, FAKE, 0, 2, 0, 64, FAKE, 0, None) == 1
    assert L.iq4xs_peer_collective(ok, ok, FAKE, FAKE + 4, 0, 2, 0, 64, FAKE, 0, None) == 3  # counter alignment
    assert L.iq4xs_peer_collective(ok, ok, FAKE, FAKE, 0, 2, 0, 0, FAKE, 0, None) == 1       # n <= 0
    assert L.iq4xs_peer_collective(ok, ok, FAKE, FAKE, 0, 2, 0, 66, FAKE, 0, None) == 2      # n % 4
    assert L.iq4xs_peer_alloc(0, C.byref(C.c_void_p())) == 1
    assert L.iq4xs_ipc_open(None, C.byref(C.c_void_p())) == 1


def test_bench_pass_layout(pkg):
    """The e2e driver's concatenated layout: every call's segment rounded up to 64 floats."""
    import ctypes as C
    L = pkg.lib()
    lens = (C.c_int64 * 3)(5120, 100, 8)
    bs = (C.c_int64 * 2)(1, 3)
    want = sum((b * n + 63) // 64 * 64 for b in (1, 3) for n in (5120, 100, 8))
    assert L.iq4xs_bench_e2e_floats(lens, 3, bs, 2) == want
