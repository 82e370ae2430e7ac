"""CPU oracle for the Audio8 decode tick -- TEST INFRASTRUCTURE ONLY.

A plain torch-on-CPU restatement of the reference engine's per-frame path (serve/fast_engine.py,
serve/fast_kernels.py). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it,
and only as the checker or the timed CPU baseline: the product (audio8-turbo-engine_b200/) never
imports it.

Arithmetic is fp32 on values rounded to bf16 (transformers, upsample stages) or fp16 (conv decoder) at
exactly the points where the reference stores bf16 / fp16 tensors; every function cites the reference
lines it restates. Where the reference's numerics depend on its kernel's blocking (bf16 rounding of the
softmax weights inside flash attention, fp16 accumulation per BK slice in conv_cl), the oracle takes
the exact value (fp32 softmax, fp32 accumulation); tests compare within tolerances that cover those.

Sampling noise is explicit: the exponential-race draw (serve/fast_engine.py:159-166) takes E ~ Exp(1)
from a counter-based Philox4x32-10 stream (``philox_exp``) that the CUDA sampler reproduces bit for
bit, so sampled tokens can be compared exactly rather than only in distribution.

Parity is pinned against the reference itself: tests/golden/make_golden.py runs the reference's own
Triton kernels and engine pieces (Triton interpreter, CPU) on seeded inputs and commits the outputs;
tests/test_oracle_golden.py checks this module against them.
"""
from __future__ import annotations

from types import SimpleNamespace
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.nn.functional as F

BF16, F16, F32 = torch.bfloat16, torch.float16, torch.float32


def bf(x: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and back to fp32 (a bf16 store in the reference)."""
    return x.to(BF16).to(F32)


def hf(x: torch.Tensor) -> torch.Tensor:
    """Round to fp16 and back to fp32 (an fp16 store in the reference's conv decoder)."""
    return x.to(F16).to(F32)


# ------------------------------------------------------------------------------------------------
# load-time weight transforms
# ------------------------------------------------------------------------------------------------
def permute_qk(w: torch.Tensor, nq: int, nkv: int, hd: int) -> torch.Tensor:
    """Rows of the fused [q | k | v] projection with each q / k head's dims reordered from interleaved RoPE pairs
    (2i, 2i+1) to rotate_half halves (i, i + hd/2). serve/fast_engine.py:60-67."""
    p = torch.cat([torch.arange(0, hd, 2), torch.arange(1, hd, 2)])
    rest = w.shape[1:]
    q = w[:nq * hd].reshape(nq, hd, *rest)[:, p].reshape(nq * hd, *rest)
    k = w[nq * hd:(nq + nkv) * hd].reshape(nkv, hd, *rest)[:, p].reshape(nkv * hd, *rest)
    return torch.cat([q, k, w[(nq + nkv) * hd:]], 0).contiguous()


def rope_tables(base: float, hd: int, n: int):
    """cos / sin [n, hd] (bf16 values as fp32) for rotate_half: fp32 phases rounded to bf16.
    serve/fast_engine.py:70-75."""
    fr = 1.0 / (base ** (torch.arange(0, hd, 2).float()[: hd // 2] / hd))
    ph = torch.outer(torch.arange(n).float(), fr)
    c, s = bf(ph.cos()), bf(ph.sin())
    return torch.cat([c, c], -1).contiguous(), torch.cat([s, s], -1).contiguous()


# ------------------------------------------------------------------------------------------------
# kernels (serve/fast_kernels.py)
# ------------------------------------------------------------------------------------------------
def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 GEMM with fp32 accumulation, result rounded to bf16 once (GemmDispatch / cuBLAS,
    serve/fast_kernels.py:364-392, :510-520). Inputs are bf16-valued fp32."""
    y = x @ w.t()
    if b is not None:
        y = y + b
    return bf(y)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None):
    """HF RMSNorm with the reference's rounding points, optionally fused with the residual add.
    serve/fast_kernels.py:30-46: h = bf16(x + res); var = mean(h^2) (fp32); y = bf16(w * bf16(h * rsqrt(var+eps)))."""
    if residual is not None:
        x = bf(x + residual)
    var = (x * x).mean(-1, keepdim=True)
    xn = bf(x * torch.rsqrt(var + eps))
    y = bf(w * xn)
    return (y, x) if residual is not None else y


def bias_rope_store(qkv, bias, cos, sin, pos, slot, kc, vc, nq, nkv, hd, ring=1 << 30):
    """(qkv + bias) in fp32, RoPE (rotate_half) on q / k rounded once to bf16, k / v stored at
    [slot, head, pos % ring]. serve/fast_kernels.py:139-176. qkv: [R, (nq+2nkv)*hd] bf16-valued;
    kc / vc: [rows, nkv, len, hd]. Returns q [R, nq, hd]."""
    R = qkv.shape[0]
    x = qkv.float() + (bias.float() if bias is not None else 0.0)
    x = x.view(R, nq + 2 * nkv, hd)
    half = hd // 2
    c = cos[pos.long()].unsqueeze(1)                 # [R, 1, hd]
    s = sin[pos.long()].unsqueeze(1)
    qk = x[:, :nq + nkv]
    partner = torch.cat([qk[..., half:], qk[..., :half]], -1)
    sign = torch.cat([-torch.ones(half), torch.ones(half)])
    rot = bf(qk * c + sign * partner * s)
    q = rot[:, :nq]
    k = rot[:, nq:]
    v = bf(x[:, nq + nkv:])
    sl = slot.long()
    col = (pos.long() % ring)
    kc[sl, :, col] = k
    vc[sl, :, col] = v
    return q


def _softmax_pv(s, v, eq):
    """softmax(s) V with the reference's rounding point: the unnormalised weights exp(s - max) are rounded to bf16 for
    the P.V product, the normaliser sums them unrounded (serve/fast_kernels.py:225-230, :253). The reference takes the
    max per 64-key block and rescales; the oracle takes the row max (identical for rows of up to 64 keys)."""
    e = torch.exp(s - s.max(-1, keepdim=True).values)
    return torch.einsum(eq, bf(e), v) / e.sum(-1, keepdim=True)


def decode_attention(q, kc, vc, lens, rowmap=None, scale=None):
    """One query per row, GQA: out[r, h] = softmax(q . K[crow, h//group, :L] * scale) V in fp32 (weights rounded to
    bf16 for P.V), rounded to bf16. serve/fast_kernels.py:193-253 (split-K flash decoding; the split merge is exact up
    to rounding)."""
    b, nq, hd = q.shape
    nkv = kc.shape[1]
    g = nq // nkv
    scale = scale if scale is not None else hd ** -0.5
    out = torch.empty(b, nq, hd)
    for r in range(b):
        L = int(lens[r])
        cr = int(rowmap[r]) if rowmap is not None else r
        k = kc[cr, :, :L].float()                      # [nkv, L, hd]
        v = vc[cr, :, :L].float()
        qq = q[r].float().view(nkv, g, hd)
        s = torch.einsum("hgd,hnd->hgn", qq, k) * scale
        out[r] = _softmax_pv(s, v, "hgn,hnd->hgd").reshape(nq, hd)
    return bf(out)


def prefill_attention(q, kc, vc, blocks, scale=None):
    """Packed causal attention over KV already in cache rows. blocks: list of (q0, n, slot, pos0): query rows
    [q0, q0+n) at positions [pos0, pos0+n) of cache row `slot` attend keys [0, pos] of that row.
    serve/fast_kernels.py:296-332."""
    R, nq, hd = q.shape
    nkv = kc.shape[1]
    g = nq // nkv
    scale = scale if scale is not None else hd ** -0.5
    out = torch.zeros(R, nq, hd)
    for q0, n, sl, p0 in blocks:
        if n <= 0:
            continue
        hi = p0 + n
        k = kc[sl, :, :hi].float()
        v = vc[sl, :, :hi].float()
        qq = q[q0:q0 + n].float().view(n, nkv, g, hd)
        s = torch.einsum("nhgd,hkd->nhgk", qq, k) * scale
        qpos = torch.arange(p0, p0 + n).view(n, 1, 1, 1)
        s = s.masked_fill(torch.arange(hi).view(1, 1, 1, hi) > qpos, float("-inf"))
        out[q0:q0 + n] = _softmax_pv(s, v, "nhgk,hkd->nhgd").reshape(n, nq, hd)
    return bf(out)


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """silu(g) rounded to bf16, times u, rounded. serve/fast_kernels.py:526-534."""
    I = gu.shape[-1] // 2
    g, u = gu[..., :I], gu[..., I:]
    gs = bf(g / (1.0 + torch.exp(-g)))
    return bf(gs * u)


# ------------------------------------------------------------------------------------------------
# sampling (serve/fast_engine.py:141-172, :726-735) with explicit noise
# ------------------------------------------------------------------------------------------------
_PHILOX_M0, _PHILOX_M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_PHILOX_W0, _PHILOX_W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)


def philox4x32(c0, c1, c2, c3, k0, k1, rounds=10):
    """Philox4x32-10 (Salmon et al., SC'11) over numpy uint32 arrays: returns 4 uint32 words per counter."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint32).copy() for c in (c0, c1, c2, c3))
    k0 = np.uint32(k0)
    k1 = np.uint32(k1)
    for r in range(rounds):
        p0 = c0.astype(np.uint64) * _PHILOX_M0
        p1 = c2.astype(np.uint64) * _PHILOX_M1
        hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
        if r + 1 < rounds:
            k0 = np.uint32((int(k0) + int(_PHILOX_W0)) & 0xFFFFFFFF)
            k1 = np.uint32((int(k1) + int(_PHILOX_W1)) & 0xFFFFFFFF)
    return c0, c1, c2, c3


def philox_exp(seed: int, stream: int, tick: int, rows: Sequence[int], n: int) -> torch.Tensor:
    """E ~ Exp(1) noise [len(rows), n] for draw `stream` of tick `tick`: counter (i // 4, row, tick, stream),
    key = seed; word i % 4; u = (w >> 8 + 0.5) * 2^-24; E = -log(u) in fp32.
    The CUDA sampler (csrc/sample.cu) computes the same words."""
    rows = np.asarray(rows, dtype=np.uint32)
    i = np.arange(n, dtype=np.uint32)
    C0 = np.broadcast_to(i[None, :] // 4, (len(rows), n))
    C1 = np.broadcast_to(rows[:, None], (len(rows), n))
    C2 = np.full((len(rows), n), tick & 0xFFFFFFFF, dtype=np.uint32)
    C3 = np.full((len(rows), n), stream & 0xFFFFFFFF, dtype=np.uint32)
    w = philox4x32(C0, C1, C2, C3, seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    words = np.stack(w, -1)                                      # [rows, n, 4]
    sel = np.take_along_axis(words, (i % 4)[None, :, None].astype(np.int64).repeat(len(rows), 0), -1)[..., 0]
    u = ((sel >> np.uint32(8)).astype(np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24)
    return torch.from_numpy(-np.log(u).astype(np.float32))


def topk_filter(logits: torch.Tensor, k: int):
    """_Sampler.filt (serve/fast_engine.py:153-156): the k largest logits sorted (ties: lower index first) and
    the cumulative probability of each under the UNTEMPERED full softmax."""
    L = logits.float()
    V = L.shape[-1]
    k = min(k, V)
    idx = torch.stack([torch.from_numpy(np.lexsort((np.arange(V), -row.numpy()))[:k]) for row in L])
    v = torch.gather(L, -1, idx)
    lse = torch.logsumexp(L, -1, keepdim=True)
    cum = torch.exp(v - lse).cumsum(-1)
    return v, idx, cum


def draw(v, idx, cum, p: float, t: float, E: torch.Tensor) -> torch.Tensor:
    """_Sampler.draw (serve/fast_engine.py:159-166): drop candidates whose cumulative probability passes p (the best
    one stays), softmax(v / t), exponential race argmax(p / E)."""
    if p < 1.0:
        drop = cum > p
        drop[:, 0] = False
        v = v.masked_fill(drop, float("-inf"))
    pr = torch.softmax(v / t, -1)
    c = (pr / E).argmax(-1, keepdim=True)
    return idx.gather(-1, c).squeeze(-1)


class Sampler:
    """_Sampler (serve/fast_engine.py:141-172) with explicit noise."""

    def __init__(self, do_sample, temperature, top_k, top_p, vocab):
        self.do_sample = bool(do_sample)
        self.t = max(float(temperature or 1.0), 1e-5)
        self.k = min(int(top_k) if top_k and int(top_k) > 0 else int(vocab), int(vocab))
        self.p = float(top_p) if top_p is not None else 1.0

    def __call__(self, logits, E=None):
        if not self.do_sample:
            return logits.float().argmax(-1)
        v, idx, cum = topk_filter(logits, self.k)
        return draw(v, idx, cum, self.p, self.t, E[:, :self.k])


# ------------------------------------------------------------------------------------------------
# transformer stack (serve/fast_engine.py:82-138)
# ------------------------------------------------------------------------------------------------
class Stack:
    """_Stack on bf16-valued fp32 weights. KV caches [layers, rows, nkv, len, hd] (fp32 holding bf16 values)."""

    def __init__(self, layers, norm, nq, nkv, hd, eps, rope_base, cache_rows, cache_len, max_pos, ring=None,
                 layer_scale=False):
        self.nq, self.nkv, self.hd, self.eps = nq, nkv, hd, float(eps)
        self.layers = []
        for L in layers:
            a, f = L.attention, L.feed_forward
            wo, w2 = a.wo.weight.detach().float(), f.w2.weight.detach().float()
            if layer_scale:        # LayerScale folded into the output projections (serve/fast_engine.py:96-98)
                wo = wo * L.attention_layer_scale.gamma.detach().float()[:, None]
                w2 = w2 * L.ffn_layer_scale.gamma.detach().float()[:, None]
            wqkv = a.wqkv.weight.detach().float()
            self.layers.append(SimpleNamespace(
                wqkv=bf(permute_qk(wqkv, nq, nkv, hd)),
                bqkv=bf(permute_qk(a.wqkv.bias.detach().float(), nq, nkv, hd)) if a.wqkv.bias is not None else None,
                wo=bf(wo), w13=bf(torch.cat([f.w1.weight.detach().float(), f.w3.weight.detach().float()], 0)),
                w2=bf(w2), ln1=bf(L.attention_norm.weight.detach().float()),
                ln2=bf(L.ffn_norm.weight.detach().float())))
        self.norm = bf(norm.weight.detach().float())
        self.cos, self.sin = rope_tables(rope_base, hd, max_pos)
        self.ring = int(ring) if ring else 1 << 30
        self.kc = torch.zeros(len(self.layers), cache_rows, nkv, cache_len, hd)
        self.vc = torch.zeros_like(self.kc)

    def forward(self, x, pos, slot, lens=None, rowmap=True, blocks=None, trace=None):
        """x: [R, H] bf16-valued. Decode (blocks None): row r attends [0, lens[r]) of cache row slot[r] (rowmap) or
        row r. Prefill: `blocks` as in prefill_attention. Returns the final-normed hidden [R, H]. trace (tests): a
        list that receives the residual stream after every layer."""
        R = x.shape[0]
        nl = len(self.layers)
        h = rmsnorm(x, self.layers[0].ln1, self.eps)
        res = x
        for i, L in enumerate(self.layers):
            qkv = linear(h, L.wqkv)
            q = bias_rope_store(qkv, L.bqkv, self.cos, self.sin, pos, slot, self.kc[i], self.vc[i], self.nq, self.nkv,
                                self.hd, self.ring)
            if blocks is not None:
                o = prefill_attention(q, self.kc[i], self.vc[i], blocks)
            else:
                o = decode_attention(q, self.kc[i], self.vc[i], lens, rowmap=slot if rowmap else None)
            a = linear(o.view(R, -1), L.wo)
            h, res = rmsnorm(a, L.ln2, self.eps, residual=res)
            m = linear(silu_mul(linear(h, L.w13)), L.w2)
            nxt = self.layers[i + 1].ln1 if i + 1 < nl else self.norm
            h, res = rmsnorm(m, nxt, self.eps, residual=res)
            if trace is not None:
                trace.append(res.clone())
        return h


# ------------------------------------------------------------------------------------------------
# streaming codec decoder (serve/fast_engine.py:178-494)
# ------------------------------------------------------------------------------------------------
def snake(x, alpha, ib):
    """ArkttsSnake1d as the reference applies it: x + 1/(alpha+1e-9) * sin(alpha x)^2 in fp32
    (serve/fast_kernels.py:578-583, :709-713)."""
    s = torch.sin(x * alpha)
    return x + ib * s * s


class Conv:
    """_CLConv (serve/fast_engine.py:178-232): channels-last causal conv or polyphase transposed conv on fp16
    values, with its activated left context carried per row. `Conv.f16acc_bk` (class switch, default 0): emulate the
    reference kernel's fp16 accumulation of each BK-channel slice instead of the exact fp32 sum."""

    f16acc_bk = 0

    def __init__(self, m, Bmax, snake_mod=None, trans=False):
        c = m.conv
        w = c.weight.detach().float()
        if trans:                                        # ConvTranspose1d [Cin, Cout, 2s], right crop s
            Cin, Cout, K = w.shape
            s = c.stride[0]
            W = torch.zeros(s, 2, Cin, Cout)
            for p in range(s):
                W[p, 0] = w[:, :, p + s]                 # tap 0: previous input frame
                W[p, 1] = w[:, :, p]                     # tap 1: current
            self.taps, self.dil, self.ph, self.ctx = 2, 1, s, 1
        else:
            Cout, Cin, K = w.shape
            self.taps, self.dil, self.ph = K, c.dilation[0], 1
            self.ctx = (K - 1) * self.dil
            W = w.permute(2, 1, 0).unsqueeze(0)          # [1, K, Cin, Cout]
        self.W = hf(W)
        self.bias = hf(c.bias.detach().float()) if c.bias is not None else None
        self.Cin, self.Cout = Cin, Cout
        self.a = self.ib = None
        if snake_mod is not None:
            al = snake_mod.alpha.detach().float().reshape(-1)
            self.a, self.ib = al, 1.0 / (al + 1e-9)
        self.state = torch.zeros(Bmax, self.ctx, Cin) if self.ctx > 0 else None

    def __call__(self, x, b, res=None):
        """x: [b, T, Cin] fp16-valued (pre-activation) -> [b, T*ph, Cout] fp16-valued."""
        T = x.shape[1]
        xa = hf(snake(x, self.a, self.ib)) if self.a is not None else x
        xin = torch.cat([self.state[:b], xa], 1) if self.state is not None else xa
        y = torch.zeros(b, T, self.ph, self.Cout)
        for p in range(self.ph):
            acc = torch.zeros(b, T, self.Cout)
            for j in range(self.taps):
                xs = xin[:, j * self.dil:j * self.dil + T]
                if Conv.f16acc_bk:
                    # the reference's F16ACC: each BK-channel slice's dot product rounded to fp16 before the fp32
                    # accumulation (serve/fast_kernels.py:585-586); off by default (the exact decode)
                    for c0 in range(0, self.Cin, Conv.f16acc_bk):
                        acc = acc + hf(xs[..., c0:c0 + Conv.f16acc_bk] @ self.W[p, j, c0:c0 + Conv.f16acc_bk])
                else:
                    acc = acc + xs @ self.W[p, j]
            y[:, :, p] = acc
        y = y.reshape(b, T * self.ph, self.Cout)
        if self.bias is not None:
            y = y + self.bias
        if res is not None:
            y = y + res
        if self.state is not None:
            self.state[:b] = xin[:, T:]
        return hf(y)


class Vocoder:
    """StreamingVocoder (serve/fast_engine.py:312-494): one codec frame per call, state carried per row."""

    WINDOW = 128

    def __init__(self, codec, Bmax, max_pos=8192):
        q = codec.quantizer
        self.up = 4 * 512

        def table(vq):   # codebook -> 1x1 out_proj (bias included): [V, 1024] (serve/fast_engine.py:326-328)
            with torch.no_grad():
                W = vq.out_proj.weight.detach().float()[:, :, 0]
                return (vq.codebook.weight.detach().float() @ W.t() + vq.out_proj.bias.detach().float()).contiguous()

        self.t_sem = table(q.semantic_quantizer.quantizers[0])
        self.t_res = torch.stack([table(v) for v in q.quantizer.quantizers])
        self.v_sem, self.v_res = self.t_sem.shape[0], self.t_res.shape[1]
        pm = q.post_module
        a0 = pm.layers[0].attention
        self.post = Stack(pm.layers, pm.norm, a0.n_head, a0.n_local_heads, a0.head_dim,
                          getattr(pm.layers[0].attention_norm, "eps", 1e-6), pm.rope_base, cache_rows=Bmax,
                          cache_len=self.WINDOW, max_pos=max_pos, ring=self.WINDOW, layer_scale=True)
        self.pos = torch.zeros(Bmax, dtype=torch.int32)
        self.max_pos = max_pos
        self.ups = []
        for blocks in q.upsample:
            tc, cnx = blocks[0], blocks[1]
            w = tc.conv.weight.detach().float()                      # [Cin, Cout, 2]
            dw = cnx.dwconv
            self.ups.append(SimpleNamespace(
                tw=bf(torch.cat([w[:, :, 0].t(), w[:, :, 1].t()], 0)),
                tb=bf(torch.cat([tc.conv.bias.detach().float()] * 2)),
                dww=bf(dw.conv.weight.detach().float()[:, 0, :].t()), dwb=bf(dw.conv.bias.detach().float()),
                st=torch.zeros(Bmax, dw.kernel_size - 1, w.shape[1]), k=dw.kernel_size,
                ln_w=bf(cnx.norm.weight.detach().float()), ln_b=bf(cnx.norm.bias.detach().float()),
                ln_eps=cnx.norm.eps,
                w1=bf(cnx.pwconv1.weight.detach().float()), b1=bf(cnx.pwconv1.bias.detach().float()),
                w2=bf(cnx.pwconv2.weight.detach().float()), b2=bf(cnx.pwconv2.bias.detach().float()),
                gamma=bf(cnx.gamma.detach().float())))
        mods = list(codec.decoder.model)
        self.dec_in = Conv(mods[0], Bmax)
        self.blocks = []
        for blk in mods[1:5]:
            bm = list(blk.block)
            tc = Conv(bm[1], Bmax, snake_mod=bm[0], trans=True)
            units = [(Conv(ru.block[1], Bmax, snake_mod=ru.block[0]), Conv(ru.block[3], Bmax, snake_mod=ru.block[2]))
                     for ru in bm[2:]]
            self.blocks.append((tc, units))
        self.final = Conv(mods[6], Bmax, snake_mod=mods[5])

    def convs(self):
        out = [self.dec_in]
        for tc, units in self.blocks:
            out.append(tc)
            for c1, c2 in units:
                out += [c1, c2]
        out.append(self.final)
        return out

    def clear(self, rows):
        for c in self.convs():
            if c.state is not None:
                c.state[rows] = 0
        for u in self.ups:
            u.st[rows] = 0
        self.post.kc[:, rows] = 0
        self.post.vc[:, rows] = 0
        self.pos[rows] = 0

    def embed(self, codes):
        """Code tables: t_sem[c0] + sum_k t_res[k, c_k] (fp32), clamped like the codec (serve/fast_engine.py:472-474)."""
        c0 = codes[:, 0].clamp(0, self.v_sem - 1)
        cr = codes[:, 1:].clamp(0, self.v_res - 1)
        ar = torch.arange(self.t_res.shape[0])
        return self.t_sem[c0] + self.t_res[ar, cr].sum(1)

    def upsample(self, x, b):
        """Two [transposed conv k2 s2, causal ConvNeXt] stages in bf16 (serve/fast_engine.py:479-491)."""
        for u in self.ups:
            T = x.shape[1]
            x = linear(x.reshape(b * T, -1), u.tw, u.tb).view(b, 2 * T, -1)
            T = 2 * T
            r = x
            xin = torch.cat([u.st[:b], x], 1)
            y = bf(u.dwb + bf(xin[:, 0:T] * u.dww[0]))
            for j in range(1, u.k):
                y = bf(y + bf(xin[:, j:j + T] * u.dww[j]))
            u.st[:b] = xin[:, T:]
            y = bf(F.layer_norm(y, (y.shape[-1],), u.ln_w, u.ln_b, u.ln_eps))
            y = bf(F.gelu(linear(y.reshape(b * T, -1), u.w1, u.b1)))
            y = linear(y, u.w2, u.b2).view(b, T, -1)
            x = bf(r + bf(u.gamma * y))
        return x

    def decode(self, x, b):
        """_CLDecoder.__call__ (serve/fast_engine.py:301-309): [b, T, 1024] -> [b, T*512] fp32 (tanh)."""
        x = self.dec_in(hf(x), b)
        for tc, units in self.blocks:
            x = tc(x, b)
            for c1, c2 in units:
                x = c2(c1(x, b), b, res=x)
        y = self.final(x, b)
        return torch.tanh(y[..., 0])

    def step(self, codes, b):
        """StreamingVocoder.step (serve/fast_engine.py:470-494): codes [b, 10] -> [b, 2048] fp32."""
        x = self.embed(codes)
        pos = self.pos[:b]
        h = self.post.forward(bf(x), pos.clamp(max=self.max_pos - 1), torch.arange(b, dtype=torch.int32),
                              (pos + 1).clamp(max=self.WINDOW), rowmap=False)
        x = self.upsample(h.unsqueeze(1), b)
        wav = self.decode(x, b)
        self.pos[:b] += 1
        return wav


# ------------------------------------------------------------------------------------------------
# engine (serve/fast_engine.py:570-1156)
# ------------------------------------------------------------------------------------------------
def pf_meta_host(NT, NR, BM, SCR, nt, slots, ns, starts):
    """pf_meta's int32 layout pos[NT] | slot[NT] | q0[NB] | n[NB] | bslot[NB] | pos0[NB] | last[NR] | st[NR] |
    cpos[NR], NB = NT // BM + NR, padding -> SCR. FastEngine._pf_meta_host, serve/fast_engine.py:837-853 and
    :682-691."""
    NB = NT // BM + NR
    o = np.cumsum([0, NT, NT, NB, NB, NB, NB, NR, NR, NR])
    m = np.zeros(int(o[-1]), np.int32)
    pos, slot, q0, n, bslot, p0, last, st, cpos = (m[o[i]:o[i + 1]] for i in range(9))
    slot[:], bslot[:], st[:] = SCR, SCR, SCR
    r0 = bi = 0
    for k, (s, cnt, a) in enumerate(zip(slots, ns, starts)):
        pos[r0:r0 + cnt] = np.arange(a, a + cnt)
        slot[r0:r0 + cnt] = s
        for off in range(0, cnt, BM):
            q0[bi], n[bi], bslot[bi], p0[bi] = r0 + off, min(BM, cnt - off), s, a + off
            bi += 1
        last[k], st[k], cpos[k] = r0 + cnt - 1, s, a + cnt
        r0 += cnt
    assert r0 <= nt and bi <= nt // BM + NR and len(slots) <= NR
    return m


def bucket_for(buckets, n_rows):
    """FastEngine.bucket_for (serve/fast_engine.py:872-876)."""
    for b in buckets:
        if b >= n_rows:
            return b
    return buckets[-1]


def default_buckets(B, env=None):
    """FastEngine's bucket list (serve/fast_engine.py:665-671)."""
    buckets = [int(x) for x in env.split(",") if x.strip()] if env else None
    if not buckets:
        buckets = [1, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32, 40, 48, 56, 64, 72, 80, 88, 96, 104, 112, 120, 128,
                   144, 160, 176, 192]
    return sorted({b for b in buckets if 1 <= b <= B} | {B})


def ref_nsplit(b, nkv=2):
    """The reference's split count per bucket, sized for 84 SMs (serve/fast_engine.py:775-776)."""
    return max(1, min(16, -(-2 * 84 // (b * nkv))))


class OracleEngine:
    """FastEngine's per-frame semantics on the CPU: slot state, the tick (serve/fast_engine.py:737-769), the fast AR
    (:702-713), semantic draw with RAS (:726-735), eager packed prefill (:1089-1156) and prompt building
    (:903-983). Noise for sampled draws comes from philox_exp(seed, stream, tick, rows)."""

    STREAM_CB = 0          # + codebook index 1..9
    STREAM_SEM = 16        # regular semantic draw
    STREAM_RAS = 17        # RAS redraw
    STREAM_PF = 18         # prefill first token

    def __init__(self, model, tokenizer, gen_params: dict, max_slots=4, max_seq=2048, seed=1234, with_voc=True):
        c = self.cfg = model.config
        self.tokz = tokenizer
        self.B = int(max_slots)
        self.S = min(int(max_seq), int(c.max_seq_len))
        gp = dict(gen_params or {})
        self.eos, self.sb, self.se = int(c.eos_token_id), int(c.semantic_begin_id), int(c.semantic_end_id)
        self.ncg, self.cbk = int(c.num_codebooks), int(c.codebook_size)
        self.nsem = self.se - self.sb + 1
        self.samp = Sampler(gp.get("do_sample", True), gp.get("temperature", 0.8), gp.get("top_k", 50),
                            gp.get("top_p", 0.95), self.nsem + 1)
        self.cb_samp = Sampler(gp.get("do_sample", True), gp.get("temperature", 0.8), gp.get("top_k", 50),
                               gp.get("top_p", 0.95), self.cbk)
        self.ras_p, self.ras_t, self.ras_w = float(c.ras_top_p), max(float(c.ras_temperature), 1e-5), \
            int(c.ras_window_size)
        self.seed = int(seed)
        self.tick_no = 0
        H = self.H = int(c.dim)
        B = self.B
        self.SCR = B
        self.slow = Stack(model.layers, model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps, c.rope_base,
                          cache_rows=B + 1, cache_len=self.S, max_pos=self.S)
        self.fast = Stack(model.fast_layers, model.fast_norm, c.fast_n_head, c.fast_n_local_heads, c.fast_head_dim,
                          c.norm_eps, c.rope_base, cache_rows=B, cache_len=self.ncg, max_pos=self.ncg)
        self.emb = bf(model.embeddings.weight.detach().float())
        self.cbemb = bf(model.codebook_embeddings.weight.detach().float())
        self.cb_off = (torch.arange(self.ncg) * self.cbk).view(1, -1)
        nh = self.nh = self.nsem + 1
        W = torch.zeros(nh, H)
        W[:self.nsem] = self.emb[self.sb:self.se + 1]
        W[self.nsem] = self.emb[self.eos]
        self.head = W
        self.fast_emb = bf(model.fast_embeddings.weight.detach().float())
        self.fast_out = bf(model.fast_output.weight.detach().float())
        self.voc = None
        if with_voc:
            codec = model.load_codec(device="cpu", dtype=torch.float32)
            self.voc = Vocoder(codec, B)
            self.up = self.voc.up
        else:
            self.up = 2048
        codes, _ = model.encode_audio(torch.zeros(1, 1, int(c.codec_sample_rate)))
        self.sil_frame = codes[0, :, codes.shape[-1] // 2].long().clamp(min=0)
        self.tok = torch.zeros(B + 1, dtype=torch.long)
        self.hid = torch.zeros(B + 1, H)
        self.cpos = torch.zeros(B + 1, dtype=torch.int32)
        self.prev = torch.zeros(B + 1, self.ras_w, dtype=torch.long)
        self.nstep = torch.zeros(B + 1, dtype=torch.int32)
        self.tok_in = torch.zeros(B, dtype=torch.long)
        self.audio = torch.zeros(B, self.up)
        self.frame_prev = torch.zeros(B, self.ncg, dtype=torch.long)
        self._parts = None
        self._spk_cache: Dict[str, tuple] = {}
        self.record = None              # optional dict: logits per tick

    # ---- draws ----
    def _noise(self, stream, rows, n):
        return philox_exp(self.seed, stream, self.tick_no, rows, n)

    def _to_token(self, j):
        return torch.where(j == self.nsem, torch.full_like(j, self.eos), j + self.sb)

    def _head(self, h):
        """Semantic + EOS logits: bf16 GEMM output as fp32 (serve/fast_engine.py:719-721)."""
        return linear(h, self.head)

    def _sample_sem(self, logits, b):
        """serve/fast_engine.py:726-735."""
        if not self.samp.do_sample:
            return self._to_token(logits.argmax(-1))
        v, idx, cum = topk_filter(logits, self.samp.k)
        rows = list(range(b))
        nrm = self._to_token(draw(v, idx, cum, self.samp.p, self.samp.t, self._noise(self.STREAM_SEM, rows,
                                                                                     self.samp.k)))
        high = self._to_token(draw(v, idx, cum, self.ras_p, self.ras_t, self._noise(self.STREAM_RAS, rows,
                                                                                    self.samp.k)))
        rep = (self.prev[:b] == nrm[:, None]).any(1) & (nrm != self.eos)
        return torch.where(rep, high, nrm)

    def _cb_draw(self, logits, i, b):
        if not self.cb_samp.do_sample:
            return logits.argmax(-1)
        return self.cb_samp(logits, self._noise(self.STREAM_CB + i, list(range(b)), self.cb_samp.k))

    def fast_codes(self, hid, code0, b, forced=None):
        """serve/fast_engine.py:702-713: one 2-token pass (positions 0, 1; cache row = row) then one pass per
        codebook. forced [b, ncg] (tests): each pass takes forced[:, i - 1] as its input code instead of the oracle's
        own draw (teacher forcing of the fast AR; the returned codes are still the oracle's draws)."""
        x = torch.stack([hid, self.fast_emb[code0]], 1).view(2 * b, self.H)
        pos0 = torch.arange(2 * b, dtype=torch.int32) % 2
        slot0 = torch.arange(2 * b, dtype=torch.int32) // 2
        h = self.fast.forward(x, pos0, slot0, pos0 + 1)
        lg = linear(h.view(b, 2, self.H)[:, 1], self.fast_out)
        if self.record is not None:
            self.record.setdefault("fast_logits", []).append(lg.clone())
        c = self._cb_draw(lg, 1, b)
        cs = [code0, c]
        ar = torch.arange(b, dtype=torch.int32)
        for i in range(2, self.ncg):
            pos = torch.full((b,), i, dtype=torch.int32)
            cin = forced[:, i - 1] if forced is not None else c
            h = self.fast.forward(self.fast_emb[cin], pos, ar, pos + 1, rowmap=False)
            lg = linear(h, self.fast_out)
            if self.record is not None:
                self.record.setdefault("fast_logits", []).append(lg.clone())
            c = self._cb_draw(lg, i, b)
            cs.append(c)
        return torch.stack(cs, 1)

    def embed(self, sem, codes):
        """emb[sem] + the 10 codebook embeddings (serve/fast_engine.py:715-717): bf16 sum over codebooks (fp32
        accumulate, one rounding), then a bf16 add."""
        return bf(self.emb[sem] + bf(self.cbemb[codes + self.cb_off].sum(1)))

    def tick(self, b, forced=None):
        """serve/fast_engine.py:737-769. forced [b, ncg] (tests): teacher-forced fast AR (see fast_codes); the slow
        step then embeds the forced codes and the frame queued is the forced one."""
        t_in = self.tok[:b].clone()
        self.tok_in[:b] = t_in
        if self.voc is not None:
            self.audio[:b] = self.voc.step(self.frame_prev[:b], b)
        code0 = (t_in - self.sb).clamp(0, self.cbk - 1)
        codes = self.fast_codes(self.hid[:b], code0, b, forced)
        if forced is not None:
            self.record_codes = codes
            codes = forced.clone()
        pos = self.cpos[:b].clone()
        h = self.slow.forward(self.embed(t_in, codes), pos, torch.arange(b, dtype=torch.int32), pos + 1, rowmap=False)
        logits = self._head(h)
        if self.record is not None:
            self.record.setdefault("logits", []).append(logits.clone())
        upd = torch.cat([self.prev[:b, 1:], t_in.unsqueeze(1)], 1)
        self.prev[:b] = torch.where((self.nstep[:b] > 0).unsqueeze(1), upd, self.prev[:b])
        nt = torch.where(t_in == self.eos, t_in, self._sample_sem(logits, b))
        self.tok[:b] = nt
        self.hid[:b] = h
        self.cpos[:b] = (pos + 1).clamp(max=self.S - 1)
        self.nstep[:b] += 1
        frame = torch.where((t_in == self.eos).unsqueeze(1), self.sil_frame, codes)
        self.frame_prev[:b] = frame
        self.tick_no += 1
        return codes

    # ---- prompts (serve/fast_engine.py:903-983) ----
    def _enc(self, s):
        return self.tokz.encode(s, add_special_tokens=False)

    def _parts_init(self):
        e = self._enc
        self._parts = SimpleNamespace(
            ref_head=e("<|im_start|>system\n") + e("convert the provided text to speech reference to the following:"
                                                  "\n\nText:\n"),
            speech=e("\n\nSpeech:\n"),
            user=e("<|im_end|>\n") + e("<|im_start|>user\n"),
            tail=e("<|im_end|>\n") + e("<|im_start|>assistant\n<|voice|>"),
            noref=e("<|im_start|>system\n") + e("convert the provided text to speech") + e("<|im_end|>\n")
            + e("<|im_start|>user\n"))

    @staticmethod
    def _clean(text):
        return " ".join(str(text).strip().split())

    def prompt_ids(self, item):
        """serve/fast_engine.py:922-939: (semantic ids, codes, is_audio) of the voice prefix."""
        import re
        P = self._parts
        rc = getattr(item, "ref_code", None) if item is not None else None
        if rc is None or not getattr(item, "ref_text", ""):
            ids = torch.tensor(P.noref, dtype=torch.long)
            return ids, torch.zeros(len(ids), self.ncg, dtype=torch.long), torch.zeros(len(ids), dtype=torch.bool)
        t = self._clean(item.ref_text)
        t = t if re.search(r"<\|speaker:\d+\|>", t) else f"<|speaker:0|>{t}"
        head = P.ref_head + self._enc(t) + P.speech
        codes = rc.long().cpu()
        T = codes.shape[0]
        sem = torch.cat([torch.tensor(head, dtype=torch.long), codes[:, 0] + self.sb,
                         torch.tensor(P.user, dtype=torch.long)])
        cb = torch.zeros(len(sem), self.ncg, dtype=torch.long)
        cb[len(head):len(head) + T] = codes
        aud = torch.zeros(len(sem), dtype=torch.bool)
        aud[len(head):len(head) + T] = True
        return sem, cb, aud

    def prompt_embeds(self, sem, cb, aud):
        """serve/fast_engine.py:941-945."""
        e = self.emb[sem]
        return torch.where(aud.unsqueeze(1), bf(e + bf(self.cbemb[cb + self.cb_off].sum(1))), e)

    def rest_ids(self, r):
        """serve/fast_engine.py:970-980: user text + tail (+ continuation codes)."""
        P = self._parts
        ctx_t = (r.get("ctx_text") or "").strip()
        ids = torch.tensor(self._enc(self._clean((ctx_t + " " if ctx_t else "") + r["text"]) or ".") + P.tail,
                           dtype=torch.long)
        cb = torch.zeros(len(ids), self.ncg, dtype=torch.long)
        aud = torch.zeros(len(ids), dtype=torch.bool)
        if r.get("ctx_codes") is not None:
            cc = torch.as_tensor(r["ctx_codes"]).long().reshape(-1, self.ncg)
            ids = torch.cat([ids, cc[:, 0] + self.sb])
            cb = torch.cat([cb, cc])
            aud = torch.cat([aud, torch.ones(len(cc), dtype=torch.bool)])
        return ids, cb, aud

    def admit(self, slots: List[int], reqs: List[dict]) -> List[int]:
        """serve/fast_engine.py:1050-1071 and :1089-1156 (no prefill token cap: the oracle prefills each request
        whole). Each request's prompt = its voice prefix + its rest, prefilled causally into its slot."""
        if self._parts is None:
            self._parts_init()
        lens, ok = [], []
        for s, r in zip(slots, reqs):
            key = r["key"]
            if key not in self._spk_cache:
                self._spk_cache[key] = self.prompt_embeds(*self.prompt_ids(r["item"]))
            pre = self._spk_cache[key]
            rest = self.prompt_embeds(*self.rest_ids(r))
            L = pre.shape[0] + rest.shape[0]
            lens.append(L)
            if L <= min(self.S - 32, 8192):
                ok.append((s, r, pre, rest))
        if ok:
            self._prefill(ok)
        return [L if L <= min(self.S - 32, 8192) else -1 for L in lens]

    def _prefill(self, items):
        hs = []
        for s, r, pre, rest in items:
            x = torch.cat([pre, rest], 0)
            n = x.shape[0]
            pos = torch.arange(n, dtype=torch.int32)
            slot = torch.full((n,), s, dtype=torch.int32)
            blocks = [(q0, min(64, n - q0), s, q0) for q0 in range(0, n, 64)]
            h = self.slow.forward(x, pos, slot, blocks=blocks)
            hs.append(h[-1])
        hl = torch.stack(hs)
        logits = self._head(hl)
        if self.record is not None:
            self.record.setdefault("prefill_logits", []).append(logits.clone())
        st = [s for s, *_ in items]
        if self.samp.do_sample:
            j = self.samp(logits, self._noise(self.STREAM_PF, st, self.samp.k))
        else:
            j = logits.argmax(-1)
        t0 = self._to_token(j)
        for i, (s, r, pre, rest) in enumerate(items):
            self.tok[s] = t0[i]
            self.hid[s] = hl[i]
            self.cpos[s] = pre.shape[0] + rest.shape[0]
            self.prev[s] = 0
            self.nstep[s] = 0
        keep = [s for s, r, *_ in items if r.get("keep_voc")]
        fresh = [s for s, r, *_ in items if not r.get("keep_voc")]
        for s in keep:
            self.frame_prev[s] = self.sil_frame
        if fresh and self.voc is not None:
            self.voc.clear(fresh)
        for s in fresh:
            self.frame_prev[s] = self.sil_frame
