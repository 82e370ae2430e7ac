"""StreamingVocoder on sm_100a kernels: the frame-at-a-time, batched, stateful codec decoder of
serve/fast_engine.py:312-494, same constructor, ``step``, ``snapshot`` / ``load_many`` / ``clear`` / ``clear_many``.

The step is ONE C-ABI call (``a8_voc_step``) over an ``A8Vocoder`` descriptor built here: code tables, the window-128
transformer (a ``PackedStack`` with a 128-entry ring cache), two upsample stages (GEMMs + depthwise conv / LayerNorm
kernel), then the decoder as a program of implicit-GEMM convs (fp16 channels-last, fp32 tensor-core accumulation).
Each conv owns its input rows ``xin`` [B, ctx + T, Cin]: rows [0, ctx) are its carried (activated) context, the rest
is written by the previous conv's epilogue, already activated with this conv's snake; one kernel at the end of the
step moves every context forward a frame. A row's carried state (conv contexts, upsample tails, ring KV, frame count)
is listed in a segment table so that clearing, loading or snapshotting a row is one kernel (``a8_state_rows``).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import List

import torch

from . import _lib as L
from .engine import PackedStack, Scratch

BF16, F16, F32 = torch.bfloat16, torch.float16, torch.float32


class _Conv:
    """One decoder conv packed for a8_conv: W2d[p * Cout + c, j * Cin + ci] fp16 (serve/fast_engine.py:182-216)."""

    def __init__(self, m, Bmax, dev, snake_mod=None, trans=False):
        c = m.conv
        w = c.weight.detach().float().cpu()
        if trans:                                   # ConvTranspose1d [Cin, Cout, 2s], right crop s: a 2-tap conv
            Cin, Cout, K = w.shape
            s = c.stride[0]
            assert K == 2 * s
            W = torch.zeros(s, 2, Cin, Cout)
            for p in range(s):
                W[p, 0] = w[:, :, p + s]            # tap 0: the previous input frame
                W[p, 1] = w[:, :, p]                # tap 1: the current one
            self.taps, self.dil, self.ph, self.ctx = 2, 1, s, 1
        else:                                       # causal Conv1d [Cout, Cin, K]
            Cout, Cin, K = w.shape
            assert c.stride[0] == 1 and c.groups == 1
            self.taps, self.dil, self.ph = K, c.dilation[0], 1
            self.ctx = (K - 1) * self.dil
            W = w.permute(2, 1, 0).unsqueeze(0)     # [1, K, Cin, Cout]
        self.Cin, self.Cout = Cin, Cout
        self.N = self.ph * Cout
        self.w = W.permute(0, 3, 1, 2).reshape(self.N, self.taps * Cin).to(F16).to(dev).contiguous()
        self.bias = c.bias.detach().float().cpu().repeat(self.ph).to(F16).float().to(dev) \
            if c.bias is not None else None                       # the fp16 bias, held as fp32
        self.alpha = self.inv = None
        if snake_mod is not None:
            al = snake_mod.alpha.detach().float().cpu().reshape(-1)
            self.alpha, self.inv = al.to(dev).contiguous(), (1.0 / (al + 1e-9)).to(dev).contiguous()
        self.T, self.xin = 0, None                  # input timesteps a frame and input rows: set by the program


class StreamingVocoder:
    """serve/fast_engine.py:312 StreamingVocoder: one codec frame per ``step`` for rows [0, b)."""

    WINDOW = 128

    def __init__(self, codec, Bmax, dev, max_pos=8192, mm=None):
        self.dev, self.Bmax = dev, int(Bmax)
        B = self.Bmax
        q = codec.quantizer
        self.up = 4 * 512

        def table(vq):      # codebook -> its 1x1 out_proj (bias included): [V, C] fp32 (serve/fast_engine.py:326-328)
            with torch.no_grad():
                W = vq.out_proj.weight.detach().float().cpu()[:, :, 0]
                return vq.codebook.weight.detach().float().cpu() @ W.t() + vq.out_proj.bias.detach().float().cpu()

        self.t_sem = table(q.semantic_quantizer.quantizers[0]).to(dev).contiguous()
        self.t_res = torch.stack([table(v) for v in q.quantizer.quantizers]).to(dev).contiguous()
        self.v_sem, self.v_res = self.t_sem.shape[0], self.t_res.shape[1]
        self.ncb = 1 + self.t_res.shape[0]
        self.C = C_ = self.t_sem.shape[1]
        pm = q.post_module
        a0 = pm.layers[0].attention
        self.post = PackedStack(pm.layers, pm.norm, a0.n_head, a0.n_local_heads, a0.head_dim,
                                getattr(pm.layers[0].attention_norm, "eps", 1e-6), pm.rope_base, cache_rows=B,
                                cache_len=self.WINDOW, max_pos=max_pos, dev=dev, ring=self.WINDOW, layer_scale=True)
        self.scratch = Scratch(B, self.post.dim, self.post.nq * self.post.hd, self.post.inter, self.post.nkv,
                               self.post.hd, self.WINDOW, dev)
        self.max_pos = int(max_pos)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos_c = torch.zeros(B, dtype=torch.int32, device=dev)
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.x = torch.zeros(B, C_, dtype=BF16, device=dev)

        # upsample stages ([transposed conv k = s = 2, ConvNeXt] each)
        self.ups = []
        bf = lambda t: t.detach().float().cpu().to(BF16).to(dev).contiguous()
        for blocks in q.upsample:
            tc, cnx = blocks[0], blocks[1]
            w = tc.conv.weight.detach().float().cpu()                      # [Cin, Cout, 2]
            assert w.shape[-1] == tc.conv.stride[0] == 2
            dw = cnx.dwconv
            u = dict(tw=bf(torch.cat([w[:, :, 0].t(), w[:, :, 1].t()], 0)),
                     tb=bf(torch.cat([tc.conv.bias.detach().float().cpu()] * 2)),
                     dww=bf(dw.conv.weight.detach().float()[:, 0, :].t()), dwb=bf(dw.conv.bias),
                     st=torch.zeros(B, dw.kernel_size - 1, w.shape[1], dtype=BF16, device=dev), K=dw.kernel_size,
                     lnw=bf(cnx.norm.weight), lnb=bf(cnx.norm.bias), eps=float(cnx.norm.eps),
                     w1=bf(cnx.pwconv1.weight), b1=bf(cnx.pwconv1.bias), w2=bf(cnx.pwconv2.weight),
                     b2=bf(cnx.pwconv2.bias), gamma=bf(cnx.gamma))
            u["mlp"] = u["w1"].shape[0]
            self.ups.append(u)
        Tup = 2 ** len(self.ups)
        mlp = max(u["mlp"] for u in self.ups)
        self.ubuf = [torch.zeros(B * Tup, n, dtype=BF16, device=dev) for n in (C_, C_, mlp, C_)]

        # decoder: conv_in, 4 x [snake, transposed conv, 3 residual units], snake, conv_out, tanh
        mods = list(codec.decoder.model)
        self.dec_in = _Conv(mods[0], B, dev)
        self.blocks = []
        for blk in mods[1:5]:
            bm = list(blk.block)
            tc = _Conv(bm[1], B, dev, snake_mod=bm[0], trans=True)
            units = [(_Conv(ru.block[1], B, dev, snake_mod=ru.block[0]), _Conv(ru.block[3], B, dev, snake_mod=ru.block[2]))
                     for ru in bm[2:]]
            self.blocks.append((tc, units))
        self.final = _Conv(mods[6], B, dev, snake_mod=mods[5])
        self.ops = self._program(Tup)
        for c, T, *_ in self.ops:                        # each conv's input rows, its carried context first
            c.T = T
            c.xin = torch.zeros(B, c.ctx + T, c.Cin, dtype=F16, device=dev)
        act = max([c.N * T for c, T, raw, _ in self.ops if raw >= 0] + [16])
        self.act = [torch.zeros(B * act, dtype=F16, device=dev) for _ in range(2)]
        self.audio = torch.zeros(B, self.up, dtype=F32, device=dev)
        ctx = [L.A8CtxShift(xin=c.xin.data_ptr(), ctx=c.ctx, T=c.T, Cin=c.Cin) for c in self.convs() if c.ctx > 0]
        raw = bytes((L.A8CtxShift * len(ctx))(*ctx))
        self.ctx_table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        self.n_ctx = len(ctx)
        self.desc = self._describe()
        self._arena_init()

    # ---- the descriptor ----
    def _program(self, T):
        """[(conv, T_in, raw, res)]: raw = the act buffer (0 / 1) that keeps the conv's raw output for a later
        residual (a unit's input), res = the buffer added to its output (the unit's input, at the unit's 1x1 conv)."""
        ops = [(self.dec_in, T, -1, -1)]
        for tc, units in self.blocks:
            ops.append((tc, T, 0, -1))
            T, cur = T * tc.ph, 0
            for k, (c1, c2) in enumerate(units):
                keep = 1 - cur if k + 1 < len(units) else -1
                ops += [(c1, T, -1, -1), (c2, T, keep, cur)]
                cur = 1 - cur
        ops.append((self.final, T, -1, -1))
        assert T == self.up, T
        return ops

    def _describe(self):
        d = L.A8Vocoder()
        d.B, d.ncb, d.C, d.v_sem, d.v_res = self.Bmax, self.ncb, self.C, self.v_sem, self.v_res
        d.max_pos, d.window, d.up = self.max_pos, self.WINDOW, self.up
        d.t_sem, d.t_res = L.ptr(self.t_sem), L.ptr(self.t_res)
        d.pos, d.pos_c, d.lens, d.x = L.ptr(self.pos), L.ptr(self.pos_c), L.ptr(self.lens), L.ptr(self.x)
        d.post, d.scratch = self.post.desc, self.scratch.desc
        assert len(self.ups) <= L.MAX_UPS and len(self.ops) <= L.MAX_CONV_OPS
        d.n_ups = len(self.ups)
        for i, u in enumerate(self.ups):
            e = d.ups[i]
            for k in ("tw", "tb", "dww", "dwb", "st", "lnw", "lnb", "w1", "b1", "w2", "b2", "gamma"):
                setattr(e, k, L.ptr(u[k]))
            e.st_bs = u["st"][0].numel()
            e.K, e.eps, e.mlp = u["K"], u["eps"], u["mlp"]
        for i, t in enumerate(self.ubuf):
            d.ubuf[i] = t.data_ptr()
        d.n_ops = len(self.ops)
        for i, (c, T, raw, res) in enumerate(self.ops):
            o = d.ops[i]
            o.w, o.bias, o.alpha, o.inv = L.ptr(c.w), L.ptr(c.bias), L.ptr(c.alpha), L.ptr(c.inv)
            o.xin = L.ptr(c.xin)
            o.Cin, o.N, o.taps, o.dil, o.ctx, o.T = c.Cin, c.N, c.taps, c.dil, c.ctx, T
            o.raw, o.res = raw, res
        for i, t in enumerate(self.act):
            d.act[i] = t.data_ptr()
        d.ctx_table, d.n_ctx = L.ptr(self.ctx_table), self.n_ctx
        d.conv_ctas = int(os.environ.get("A8_CONV_CTAS", "0"))
        d.audio = L.ptr(self.audio)
        return d

    def convs(self):
        """Every decoder conv, in order (serve/fast_engine.py:394-404, without the tuning metadata)."""
        return [op[0] for op in self.ops]

    def conv_run(self, i, b):
        """The a8_conv launch of program op i at b rows, as a8_voc_step makes it (to time one conv alone)."""
        c, T, raw, res = self.ops[i]
        r = L.A8ConvRun(xin=L.ptr(c.xin), rows=b, T=T, Cin=c.Cin, ctx=c.ctx, w=L.ptr(c.w), N=c.N, taps=c.taps,
                        dil=c.dil, bias=L.ptr(c.bias))
        if res >= 0:
            r.res, r.res_bs, r.res_ts = self.act[res].data_ptr(), T * c.N, c.N
        if raw >= 0:
            r.raw, r.raw_bs, r.raw_ts = self.act[raw].data_ptr(), T * c.N, c.N
        if i + 1 < len(self.ops):
            nx = self.ops[i + 1][0]
            r.nxt, r.nxt_bs, r.nxt_off, r.cout = nx.xin.data_ptr(), (nx.ctx + nx.T) * nx.Cin, nx.ctx * nx.Cin, nx.Cin
            r.alpha, r.inv = L.ptr(nx.alpha), L.ptr(nx.inv)
        else:
            r.audio, r.audio_bs = self.audio.data_ptr(), self.up
        return r

    def tune(self, b, log=print, cache_path=None):
        """The reference tunes Triton tile configs per conv; these kernels size their tiles from the shapes."""
        return None

    # ---- per-row state (serve/fast_engine.py:368-393, :453-468) ----
    def _states(self):
        """(tensor, chunks a slot, chunk elements, chunk stride elements, slot stride elements) of every state."""
        out = []
        for c in self.convs():
            if c.ctx > 0:                               # the context rows at the head of each slot's input rows
                out.append((c.xin, 1, c.ctx * c.Cin, 0, c.xin[0].numel()))
        for u in self.ups:
            n = u["st"][0].numel()
            out.append((u["st"], 1, n, n, n))
        P = self.post
        per = P.nkv * P.cache_len * P.hd              # one layer of one slot: [nkv, cache_len, hd]
        for cache in (P.kc, P.vc):
            out.append((cache, P.layers, per, P.cache_rows * per, per))
        out.append((self.pos, 1, 1, 1, 1))
        return out

    def _arena_init(self):
        segs, off = [], 0
        for t, nch, n, cs, ss in self._states():
            es = t.element_size()
            segs.append(L.A8StateSeg(base=t.data_ptr(), slot_stride=ss * es, chunk_bytes=n * es,
                                     chunk_stride=cs * es, nchunks=nch, blob_off=off))
            off += (nch * n * es + 15) // 16 * 16
        self.snap_bytes = off
        raw = bytes((L.A8StateSeg * len(segs))(*segs))
        self.seg_table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.dev)
        self.nseg = len(segs)
        self.blob = torch.zeros(1, off, dtype=torch.uint8, device=self.dev)

    def _rows(self, slots, op, blob=None):
        idx = torch.tensor(list(slots), dtype=torch.int32).to(self.dev, non_blocking=True)
        L.call("a8_state_rows", L.ptr(self.seg_table), self.nseg, L.ptr(idx), len(slots), op, L.ptr(blob),
               L.stream_handle())
        return idx

    def snapshot(self, row=0) -> List[torch.Tensor]:
        blob = torch.zeros(1, self.snap_bytes, dtype=torch.uint8, device=self.dev)
        self._rows([row], L.STATE_SNAPSHOT, blob)
        return [blob]

    def load_many(self, slots, snap):
        """Load one snapshot (device or pinned host memory) into several rows."""
        if not slots:
            return
        v = snap[0].to(self.dev, non_blocking=True).view(1, -1)
        assert v.shape[1] == self.snap_bytes, (v.shape, self.snap_bytes)
        self.blob.copy_(v)
        self._rows(slots, L.STATE_LOAD, self.blob)

    def clear(self, slot):
        self._rows([slot], L.STATE_CLEAR)

    def clear_many(self, slots):
        if slots:
            self._rows(slots, L.STATE_CLEAR)

    # ---- one frame for rows [0, b) ----
    def step(self, codes, b):
        """codes [b, ncb] long (the LLM's codes; clamped like the codec) -> audio [b, 2048] fp32 (a view of the
        vocoder's output rows, overwritten by the next step)."""
        codes = codes.contiguous()
        assert codes.dtype == torch.int64 and codes.shape[1] == self.ncb
        L.call("a8_voc_step", C.byref(self.desc), L.ptr(codes), int(b), L.stream_handle())
        return self.audio[:b]

    def decode(self, u, b):
        """The conv decoder alone (serve/fast_engine.py:301-309): u [b, 4, C] bf16 -> audio [b, 2048] fp32."""
        u = u.to(BF16).contiguous()
        L.call("a8_voc_decode", C.byref(self.desc), L.ptr(u), int(b), L.stream_handle())
        return self.audio[:b]
