"""torch restatement of the oracle's quantised pipeline, for full-size parity on the GPU.

TEST HELPER: elementwise fp32 products exactly as iq4xs_oracle.c's or_term_f32, sums in float64.
Pinned against the C oracle in tests/test_gpu_gemv.py at small sizes.
"""
import torch

KV = torch.tensor([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=torch.float64)


def decode_weights(W: torch.Tensor, K: int):
    """W uint8 [N][K/256*136] -> (codebook values f64 [N][K/32][32], ls-32 int64 [N][K/32], d_w f32 [N][K/256])."""
    N = W.shape[0]
    kb = K // 256
    blk = W.view(N, kb, 136)
    d = blk[:, :, 0:2].contiguous().view(torch.float16).view(N, kb).float()
    sh = blk[:, :, 2:4].contiguous().view(torch.int16).view(N, kb).to(torch.int64) & 0xFFFF
    sl = blk[:, :, 4:8].to(torch.int64)                                     # [N][kb][4]
    ib = torch.arange(8, device=W.device)
    lo = (sl[:, :, ib // 2] >> (4 * (ib & 1))) & 0xF                       # [N][kb][8]
    hi = (sh[:, :, None] >> (2 * ib)) & 3
    ls = (lo | (hi << 4)) - 32
    qs = blk[:, :, 8:].to(torch.int64).view(N, kb, 8, 16)
    codes = torch.cat([qs & 0xF, qs >> 4], dim=3)                            # element j and j+16
    kv = KV.to(W.device)[codes].view(N, kb * 8, 32)
    return kv, ls.view(N, kb * 8), d


def decode_q8(q8: torch.Tensor, K: int):
    B = q8.shape[0]
    nsb = K // 32
    b = q8.view(B, nsb, 36)
    dx = b[:, :, 0:2].contiguous().view(torch.float16).view(B, nsb).float()
    q = b[:, :, 4:].contiguous().view(torch.int8).to(torch.float64)         # [B][nsb][32]
    return q, dx


def subblock_dots(W, q8, K: int):
    kv, _, _ = decode_weights(W, K)
    q, _ = decode_q8(q8, K)
    # [B][N][nsb] exact in float64
    return torch.einsum("nsj,bsj->bns", kv, q)


def matmul_q8(W, q8, K: int):
    """(Y64 [B][N], sum|terms| [B][N]) exactly as the C oracle's or_matmul_q8 (fp64 sum order aside)."""
    kv, ls, dw = decode_weights(W, K)
    q, dx = decode_q8(q8, K)
    sumi = torch.einsum("nsj,bsj->bns", kv, q)                              # exact integers
    scaled = (sumi * ls[None].to(torch.float64)).to(torch.float32)          # |.| < 2^24: exact
    dws = dw.repeat_interleave(8, dim=1)                                    # [N][nsb] f32
    d = dws[None] * dx[:, None, :]                                          # fp32 product
    term = (d * scaled).to(torch.float64)                                   # fp32 product
    return term.sum(dim=2), term.abs().sum(dim=2)
