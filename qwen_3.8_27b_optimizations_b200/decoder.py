"""Synthetic ~25B dense decoder on the IQ4_XS matmuls, tensor-parallel over the ranks of one node.

The model of BASELINE.json configs[4]: 64 layers, hidden 5120, 64 query heads x 128 and 8 KV heads
x 128 (GQA), SwiGLU FFN 17408, RMSNorm, RoPE (theta 1e6), vocab 152064; random N(0, 0.02) linear
weights quantised to IQ4_XS, fp32 norms, f16 embeddings and KV cache.  Every linear layer runs on the
IQ4_XS kernels (GEMV for batch <= 8 tokens, the tensor-core GEMM for the prompt); norms, RoPE,
attention and sampling are plain torch tensor ops around them.

Tensor parallelism (one exchange per block half):
  * q|k|v fused and gate|up fused are column-parallel: each rank owns whole heads (64/P query,
    8/P KV heads) and whole 512-wide FFN slices;
  * o_proj and down_proj are row-parallel: each rank multiplies its K-slice (whole super-block
    pairs) and the partial outputs are summed with an all-reduce;
  * lm_head is row-sharded with an all-gather of the logits (sharded.RowShardedIQ4XS).
The weights are generated identically on every rank from per-matrix seeds and sliced, so the model
does not depend on P.

The decode step (one token) is captured in a CUDA graph and replayed, the position and the token
living in device tensors, so generating N tokens issues no host work per token.  With the CUDA
kernels, a decode layer is six kernels (include/iq4xs_decoder.h): residual + RMSNorm fused into the
q|k|v and gate|up GEMVs (each CTA normalises and quantises the activations in its shared memory),
RoPE + KV-append + attention -> Q8_1, the o_proj GEMV, SwiGLU -> Q8_1 and the down_proj GEMV; each is
launched as a programmatic dependent of the kernel before it, so the GEMVs' weight streams start
while it finishes.  The
prompt (prefill) runs the same model with torch ops around the tensor-core GEMM.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional

PAIR = 512  # weights per super-block pair: the K granule of the tensor-map kernels


@dataclass
class DecoderConfig:
    layers: int = 64
    hidden: int = 5120
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 17408
    vocab: int = 152064
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6
    max_seq: int = 640
    std: float = 0.02


def split_units(n: int, world: int, rank: int):
    """[a, b) of `n` units for `rank`, balanced."""
    return n * rank // world, n * (rank + 1) // world


class _PeerDelta:
    """The o_proj / down_proj output of a fused all-reduce: still spread over the ranks' slots of a
    peer area; the next fused kernel (norm + GEMV, or the final norm) sums it in its prologue."""

    def __init__(self, slots):
        self.slots = slots


class TPDecoder:
    """One rank's share of the decoder.  `matmul(W, X, N) -> Y [M][N]` (fp32 X [M][K]) defaults to the
    CUDA kernels; tests on CPU ranks inject a reference."""

    SLOT_AREAS = (3, 4)  # peer areas of the fused all-reduce's slots for o_proj (0) and down_proj (1)

    def __init__(self, cfg: DecoderConfig, rank: int = 0, world: int = 1, group=None, seed: int = 0,
                 device="cuda", matmul: Optional[Callable] = None, gen_weights: Optional[Callable] = None,
                 gen_normal: Optional[Callable] = None, fused_decode: Optional[bool] = None,
                 peer_collectives: Optional[bool] = None, emulate_ranks: int = 1,
                 fused_allreduce: Optional[bool] = None):
        import torch
        from . import sharded
        self.torch = torch
        # emulate_ranks = R > 1 (single GPU, world 1): the row-parallel GEMVs of the fused decode step
        # run as the R per-rank K slices a tensor-parallel run over R ranks would compute, added in rank
        # order like the peer all-reduce -- the TP-R decode step reproduced on one GPU, bit for bit.
        if emulate_ranks > 1 and (world != 1 or matmul is not None):
            raise ValueError("rank emulation runs on one GPU with the CUDA kernels")
        self.emulate_ranks = int(emulate_ranks)
        self.cfg, self.rank, self.world, self.group = cfg, rank, world, group
        self.device = torch.device(device)
        if cfg.kv_heads % world or cfg.heads % world:
            raise ValueError("the rank count must divide the KV head count")
        if (cfg.heads // world) * cfg.head_dim % PAIR or cfg.hidden % PAIR or cfg.ffn % PAIR:
            raise ValueError("head groups, hidden and FFN must be whole super-block pairs")
        self._api = None
        if matmul is None or gen_weights is None or gen_normal is None:
            from . import api
            self._api = api
        self.matmul = matmul or self._cuda_matmul
        # fused decode layers need the CUDA kernels for every op
        self.fused_decode = (matmul is None) if fused_decode is None else fused_decode
        if self.fused_decode and (matmul is not None or self._api is None):
            raise ValueError("fused decode runs on the CUDA kernels only")
        self._dec = None
        self.gen_weights = gen_weights or (lambda N, K, s: self._api.random_weights(N, K, seed=s, std=cfg.std))
        self.gen_normal = gen_normal or (lambda n, s, mean, std: self._api.fill_normal(n, s, mean, std))

        D, hd = cfg.hidden, cfg.head_dim
        self.hq = cfg.heads // world
        self.hkv = cfg.kv_heads // world
        q0, kv0 = rank * self.hq, rank * self.hkv
        p0, p1 = split_units(cfg.ffn // PAIR, world, rank)
        self.f0, self.f1 = p0 * PAIR, p1 * PAIR
        self.F = self.f1 - self.f0
        self.nqkv = (self.hq + 2 * self.hkv) * hd

        def kslice(W, K, k0, k1):  # columns [k0, k1) of an IQ4_XS matrix, k in whole super-blocks
            N = W.shape[0]
            return W.view(N, K // 256, 136)[:, k0 // 256:k1 // 256, :].contiguous().view(N, -1)

        self.layers = []
        for l in range(cfg.layers):
            s = seed * 100003 + 16 * l
            wq = self.gen_weights(cfg.heads * hd, D, s + 1)
            wk = self.gen_weights(cfg.kv_heads * hd, D, s + 2)
            wv = self.gen_weights(cfg.kv_heads * hd, D, s + 3)
            wqkv = torch.cat([wq[q0 * hd:(q0 + self.hq) * hd], wk[kv0 * hd:(kv0 + self.hkv) * hd],
                              wv[kv0 * hd:(kv0 + self.hkv) * hd]]).contiguous()
            del wq, wk, wv
            wo = kslice(self.gen_weights(D, cfg.heads * hd, s + 4), cfg.heads * hd, q0 * hd, (q0 + self.hq) * hd)
            wg = self.gen_weights(cfg.ffn, D, s + 5)
            wu = self.gen_weights(cfg.ffn, D, s + 6)
            wgu = torch.cat([wg[self.f0:self.f1], wu[self.f0:self.f1]]).contiguous()
            del wg, wu
            wd = kslice(self.gen_weights(D, cfg.ffn, s + 7), cfg.ffn, self.f0, self.f1)
            an = self.gen_normal(D, s + 8, 1.0, cfg.std).to(self.device)
            fn = self.gen_normal(D, s + 9, 1.0, cfg.std).to(self.device)
            L = dict(wqkv=wqkv, wo=wo, wgu=wgu, wd=wd, an=an, fn=fn)
            if self.emulate_ranks > 1:
                # the K slices of rank r of R: whole heads of o_proj, whole FFN pairs of down_proj
                R = self.emulate_ranks
                hqr = cfg.heads // R
                L["wo_parts"] = [(kslice(wo, cfg.heads * hd, r * hqr * hd, (r + 1) * hqr * hd), r * hqr * hd,
                                  (r + 1) * hqr * hd) for r in range(R)]
                L["wd_parts"] = []
                for r in range(R):
                    a, b = split_units(cfg.ffn // PAIR, R, r)
                    L["wd_parts"].append((kslice(wd, cfg.ffn, a * PAIR, b * PAIR), a * PAIR, b * PAIR))
            self.layers.append(L)
        s = seed * 100003 + 16 * cfg.layers
        self.emb = self.gen_normal(cfg.vocab * D, s + 1, 0.0, cfg.std).view(cfg.vocab, D).to(torch.float16)
        self.final_norm = self.gen_normal(D, s + 2, 1.0, cfg.std).to(self.device)
        lm = self.gen_weights(cfg.vocab, D, s + 3)
        r0, r1 = sharded.shard_rows(cfg.vocab, world, rank)
        # decode-step collectives over NVLink peer memory (areas: 0 o_proj, 1 down_proj, 2 lm_head)
        if peer_collectives is None:
            peer_collectives = self.fused_decode and world > 1
        self.peers = None
        if peer_collectives and world > 1:
            from .peer import PeerGroup
            lm_pad = sharded.max_shard_rows(cfg.vocab, world)
            # areas: 0 / 1 the collective kernel's o_proj / down_proj, 2 the lm_head all-gather,
            # 3 / 4 the fused all-reduce's slots (their own areas, so that the two forms can alternate
            # on one model without a slot word left by the other being read as current)
            self.peers = PeerGroup(max(2 * world * D, 8 * lm_pad), areas=5, group=group, device=self.device)
        # fused all-reduce (o_proj / down_proj GEMV epilogues push their rows into every rank's slot,
        # the next kernel's norm prologue sums the slots) instead of a collective kernel per GEMV.
        # Default: fused at 2 ranks, the collective kernel from 4 (measured on B200s, 64-layer C5
        # decoder: TP2 238 vs 220 tok/s, TP4 197 vs 237 -- every consumer CTA reads world x hidden x 8
        # bytes of slots, which outgrows the collective kernel's cost as the rank count grows).
        if fused_allreduce is None:
            fused_allreduce = world <= 2
        self.fused_allreduce = bool(fused_allreduce) and self.peers is not None
        if self.peers is not None:  # the device descriptors exist before any graph capture
            for area in self.SLOT_AREAS:
                self.peers.slots(area, D)
        self.lm_head = sharded.RowShardedIQ4XS(lm[r0:r1].contiguous(), cfg.vocab, D, group=group, rank=rank,
                                               world=world, local_gemv=self._lm_local if matmul else None,
                                               local_gemm=self._lm_local_t if matmul else None, peers=self.peers,
                                               peer_areas=(2,))
        del lm
        self.cache = torch.zeros((cfg.layers, 2, self.hkv, cfg.max_seq, hd), dtype=torch.float16, device=self.device)
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
        ang = torch.arange(cfg.max_seq, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos = torch.cos(ang).to(torch.float32).to(self.device)   # [max_seq][hd/2]
        self.sin = torch.sin(ang).to(torch.float32).to(self.device)
        self.graph = None
        self._pos = self._tok = None

    # ------------------------------------------------------------------ building blocks
    def _cuda_matmul(self, W, X, N):
        if X.shape[0] <= 8:
            return self._api.gemv(W, X, N, flags=self._api.FLAG_OVERLAP_PRECEDING)
        return self._api.gemm(W, X, N)

    def _lm_local(self, W, X):
        return self.matmul(W, X, W.shape[0])

    def _lm_local_t(self, W, X):
        return self.matmul(W, X, W.shape[0]).t()

    def _allreduce(self, t):
        if self.world > 1:
            self.torch.distributed.all_reduce(t, group=self.group)
        return t

    def _rmsnorm(self, x, w):
        return x * self.torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.eps) * w

    def _rope(self, x, pos):
        """x [T][H][hd] at positions pos [T] (rotate-half form)."""
        half = self.cfg.head_dim // 2
        c = self.cos[pos][:, None, :]
        s = self.sin[pos][:, None, :]
        x1, x2 = x[..., :half], x[..., half:]
        return self.torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)

    def _attention(self, q, l, pos, T):
        """q [T][hq][hd] for the T tokens at positions pos, against the f16 KV cache of layer l (keys up
        to each token's own position), in fp32."""
        torch = self.torch
        cfg = self.cfg
        g = self.hq // self.hkv
        K = self.cache[l, 0].float()            # [hkv][max_seq][hd]
        V = self.cache[l, 1].float()
        qg = q.view(T, self.hkv, g, cfg.head_dim).permute(1, 2, 0, 3)          # [hkv][g][T][hd]
        sc = torch.matmul(qg, K.transpose(1, 2)[:, None]) / math.sqrt(cfg.head_dim)  # [hkv][g][T][S]
        keys = torch.arange(cfg.max_seq, device=q.device)
        mask = keys[None, :] > pos[:, None]                                   # [T][S]
        sc = sc.masked_fill(mask[None, None], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        o = torch.matmul(p, V[:, None])                                       # [hkv][g][T][hd]
        return o.permute(2, 0, 1, 3).reshape(T, self.hq * cfg.head_dim)

    def forward(self, x, pos):
        """x [T][hidden] fp32 embeddings of the tokens at positions pos [T]; updates the KV cache and
        returns the final-norm hidden states [T][hidden]."""
        torch = self.torch
        cfg = self.cfg
        T = x.shape[0]
        hd = cfg.head_dim
        for l, L in enumerate(self.layers):
            h = self._rmsnorm(x, L["an"])
            qkv = self.matmul(L["wqkv"], h, self.nqkv)
            q = qkv[:, :self.hq * hd].view(T, self.hq, hd)
            k = qkv[:, self.hq * hd:(self.hq + self.hkv) * hd].view(T, self.hkv, hd)
            v = qkv[:, (self.hq + self.hkv) * hd:].view(T, self.hkv, hd)
            q = self._rope(q, pos)
            k = self._rope(k, pos)
            self.cache[l, 0].index_copy_(1, pos, k.transpose(0, 1).to(torch.float16))
            self.cache[l, 1].index_copy_(1, pos, v.transpose(0, 1).to(torch.float16))
            a = self._attention(q, l, pos, T)
            o = self._allreduce(self.matmul(L["wo"], a.contiguous(), cfg.hidden))
            x = x + o
            h2 = self._rmsnorm(x, L["fn"])
            gu = self.matmul(L["wgu"], h2, 2 * self.F)
            act = torch.nn.functional.silu(gu[:, :self.F]) * gu[:, self.F:]
            d = self._allreduce(self.matmul(L["wd"], act.contiguous(), cfg.hidden))
            x = x + d
        return self._rmsnorm(x, self.final_norm)

    def _decode_buffers(self):
        if self._dec is None:
            torch, cfg = self.torch, self.cfg
            dev = self.device
            D = cfg.hidden
            q8 = lambda K: torch.empty((1, K // 32 * 36), dtype=torch.uint8, device=dev)
            self._dec = dict(x=torch.empty((1, D), dtype=torch.float32, device=dev),
                             x2=torch.empty((1, D), dtype=torch.float32, device=dev),
                             h=torch.empty((1, D), dtype=torch.float32, device=dev),
                             q8d=q8(D), q8a=q8(self.hq * cfg.head_dim), q8f=q8(self.F),
                             qkv=torch.empty((1, self.nqkv), dtype=torch.float32, device=dev),
                             o=torch.empty((1, D), dtype=torch.float32, device=dev),
                             gu=torch.empty((1, 2 * self.F), dtype=torch.float32, device=dev),
                             d=torch.empty((1, D), dtype=torch.float32, device=dev))
        return self._dec

    def forward_decode(self, x):
        """One token through the fused decode layers: x [1][hidden] fp32 embedding at position
        self._pos, or None to embed the token in self._tok on the device; returns the final-norm
        hidden state [1][hidden] (a reused buffer)."""
        api, cfg = self._api, self.cfg
        b = self._decode_buffers()
        D, hd = cfg.hidden, cfg.head_dim
        OV, PDL = api.FLAG_OVERLAP_PRECEDING, api.FLAG_PDL
        cur, nxt = b["x"], b["x2"]  # the residual stream: the fused GEMVs write x + delta to the other one
        if x is None:
            api.dec_embed(self.emb, self._tok, out=cur, flags=PDL)
        else:
            cur.copy_(x)
        delta = None

        def norm_gemv(W, w, N, out):
            nonlocal cur, nxt
            if isinstance(delta, _PeerDelta):
                api.dec_rmsnorm_gemv_peer(W, cur, delta.slots, w, cfg.eps, N, x_out=nxt, out=out, flags=PDL)
            else:
                api.dec_rmsnorm_gemv(W, cur, w, cfg.eps, N, delta=delta, x_out=nxt if delta is not None else None,
                                     out=out, flags=PDL)
            if delta is not None:
                cur, nxt = nxt, cur

        for l, L in enumerate(self.layers):
            norm_gemv(L["wqkv"], L["an"], self.nqkv, b["qkv"])
            # the position and the cache rows before it were written by earlier tokens' kernels
            api.dec_attention_decode_q8(b["qkv"], self.cache[l, 0], self.cache[l, 1], self.cos, self.sin, self._pos,
                                        self.hq, self.hkv, q8=b["q8a"], flags=PDL | api.FLAG_ATTN_EARLY_STATE)
            delta = self._reduce_gemv(L["wo"], b["q8a"], self.hq * hd, b["o"], 0, L.get("wo_parts"))
            norm_gemv(L["wgu"], L["fn"], 2 * self.F, b["gu"])
            if "wd_parts" in L:
                api.dec_swiglu_q8(b["gu"], self.F, q8=b["q8f"], flags=PDL)
                delta = self._reduce_gemv(L["wd"], b["q8f"], self.F, b["d"], 1, L["wd_parts"])
            else:
                delta = self._swiglu_down(L["wd"], b["gu"], b["d"])
        if isinstance(delta, _PeerDelta):
            api.dec_residual_rmsnorm_q8_peer(cur, delta.slots, self.final_norm, cfg.eps, h_out=b["h"], want_q8=False,
                                             flags=PDL)
        else:
            api.dec_residual_rmsnorm_q8(cur, self.final_norm, cfg.eps, delta=delta, h_out=b["h"], want_q8=False,
                                        flags=PDL)
        return b["h"]

    def _reduce_gemv(self, W, q8, K, out, area, parts=None):
        """out [1][hidden] = the row-parallel GEMV's partial sums, summed over the ranks: over NVLink
        peer memory (the GEMV writes into this rank's area, the pull kernel sums in rank order) or
        with an NCCL all-reduce.  With rank emulation (`parts`: the ranks' K slices of W) the slices'
        GEMVs run here and their outputs are added in rank order, as the peer all-reduce adds them."""
        api, D = self._api, self.cfg.hidden
        if parts is not None:
            torch = self.torch
            bufs = self._emu_buffers(len(parts))
            q8v = q8.view(-1)
            for r, (Wr, k0, k1) in enumerate(parts):
                api.gemv_q8_ex(Wr, q8v[k0 // 32 * 36:k1 // 32 * 36], k1 - k0, D, 1, out=bufs[r],
                               flags=api.FLAG_OVERLAP_PRECEDING)
            out.copy_(bufs[0])
            for r in range(1, len(parts)):
                out.add_(bufs[r])
            return out
        if self.peers is None:
            return self._allreduce(api.gemv_q8_ex(W, q8, K, D, 1, out=out, flags=api.FLAG_OVERLAP_PRECEDING))
        if self.fused_allreduce:
            slots = self.peers.slots(self.SLOT_AREAS[area], D)
            api.dec_gemv_q8_push(W, q8, K, D, slots, flags=api.FLAG_PDL)
            return _PeerDelta(slots)
        api.gemv_q8_ex(W, q8, K, D, 1, out=self.peers.area(area, D).view(1, D), flags=api.FLAG_OVERLAP_PRECEDING)
        self.peers.allreduce(area, D, out)
        return out

    def _swiglu_down(self, W, gu, out):
        """The down_proj GEMV with the SwiGLU fused in (iq4xs_dec_swiglu_gemv: the Q8_1 blocks of
        silu(gate) * up are built by the GEMV's CTAs, or by the standalone SwiGLU kernel for long K),
        then the all-reduce as in _reduce_gemv."""
        api, D = self._api, self.cfg.hidden
        if self.peers is None:
            return self._allreduce(api.dec_swiglu_gemv(W, gu, self.F, D, out=out, flags=api.FLAG_PDL))
        if self.fused_allreduce:
            slots = self.peers.slots(self.SLOT_AREAS[1], D)
            api.dec_swiglu_gemv(W, gu, self.F, D, slots=slots, flags=api.FLAG_PDL)
            return _PeerDelta(slots)
        api.dec_swiglu_gemv(W, gu, self.F, D, out=self.peers.area(1, D).view(1, D), flags=api.FLAG_PDL)
        self.peers.allreduce(1, D, out)
        return out

    def _emu_buffers(self, n):
        if getattr(self, "_emu", None) is None or len(self._emu) != n:
            self._emu = [self.torch.empty((1, self.cfg.hidden), dtype=self.torch.float32, device=self.device)
                         for _ in range(n)]
        return self._emu

    def reset_decode(self, pos: int = 0):
        """Start decoding at position `pos` without a prompt (the cache before `pos` is whatever it
        holds); the next decode step reads the token set in self._tok."""
        torch = self.torch
        if self._pos is None:
            self._pos = torch.empty((1,), dtype=torch.long, device=self.device)
            self._tok = torch.empty((1,), dtype=torch.long, device=self.device)
        self._pos.fill_(pos)
        self._tok.fill_(0)

    def logits(self, h):
        """h [T][hidden] -> logits [T][vocab] (row-sharded lm_head + all-gather); the result may be a
        view of the lm_head's output buffer, valid until its next call."""
        if h.shape[0] <= 8:
            return self.lm_head.gemv(h.contiguous())
        return self.lm_head.gemm_nm(h.contiguous()).t()

    # ------------------------------------------------------------------ generation
    def prefill(self, tokens):
        """Run the prompt (token ids [T] on the device); returns the greedy next token [1]."""
        torch = self.torch
        T = tokens.shape[0]
        pos = torch.arange(T, device=self.device)
        h = self.forward(self.emb[tokens].float(), pos)
        lg = self.logits(h[-1:]).clone()  # the sharded lm_head reuses its output buffer
        if self._pos is None:  # the decode graph reads these two tensors: keep them, refill them
            self._pos = torch.empty((1,), dtype=torch.long, device=self.device)
            self._tok = torch.empty((1,), dtype=torch.long, device=self.device)
        self._pos.fill_(T)
        self._tok.copy_(torch.argmax(lg, dim=-1))
        return self._tok.clone(), lg

    def _step(self):
        """One decode step: the token in self._tok at position self._pos -> the next token (greedy) in
        self._tok, the position advanced.  self._last_logits: the step's logits [1][vocab] (with the
        CUDA kernels a view of the lm_head's output buffer, valid until the next step)."""
        torch = self.torch
        if self.fused_decode:
            h = self.forward_decode(None)  # embeds self._tok itself
            lg = self.logits(h)
            self._last_logits = lg
            self._api.dec_argmax(lg, self._tok, self._pos, flags=self._api.FLAG_PDL)
            return self._tok
        x = self.emb[self._tok].float()
        h = self.forward(x, self._pos)
        lg = self.logits(h)
        self._last_logits = lg.clone()
        self._tok.copy_(torch.argmax(lg, dim=-1))
        self._pos.add_(1)
        return self._tok

    def decode(self, steps: int, use_graph: bool = True) -> List[int]:
        """Greedy decode `steps` tokens after prefill(); returns the generated token ids.  With
        use_graph the step is captured once (the first call runs two eager steps, then captures) and
        every later token, in this and later calls, is one graph replay."""
        torch = self.torch
        out = torch.empty(steps, dtype=torch.long, device=self.device)
        if steps <= 0:
            return []
        i = 0
        if not use_graph:
            for i in range(steps):
                out[i:i + 1].copy_(self._step())
            return out.tolist()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            if self.graph is None:
                out[0:1].copy_(self._step())      # eager: allocates the per-shape buffers
                i = 1
                if i < steps:
                    out[1:2].copy_(self._step())  # second eager step on the capture stream
                    i = 2
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=s):
                        self._step()
                    self.graph = g
            for j in range(i, steps):
                self.graph.replay()
                out[j:j + 1].copy_(self._tok)
        torch.cuda.current_stream(self.device).wait_stream(s)
        return out.tolist()

    def release(self):
        """Drop the captured graph and the peer-memory buffers (before destroying the process group)."""
        self.graph = None
        if self.peers is not None:
            self.peers.close()
            self.peers = None
            self.lm_head.peers = None
