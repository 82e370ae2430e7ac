"""FastEngine: the drop-in for serve/fast_engine.py's FastEngine on a B200.

Same constructor, attributes and methods as the reference (serve/fast_engine.py:570-1156); the worker
(serve/engine_worker.py) drives it unchanged: ``capture()``, ``admit(slots, reqs)``, ``bucket_for(n)``,
``replay(b)``, then reads ``tok_in[:b]``, ``audio[:b]`` and ``frame_prev[:b]``.

PyTorch only allocates device memory and provides streams and CUDA graphs here. Every kernel of the tick and of
admission is a hand-written sm_100a kernel in libaudio8_b200.so, reached through its C ABI (include/audio8_b200.h):
``a8_tick`` launches one whole frame (fast AR, slow AR, sampling, state update), recorded once per bucket into a
CUDA graph; an admission chunk is one copy of int32 metadata and one replay of a prefill graph per token bucket
(``a8_embed_prompt`` -> ``a8_stack_forward`` with the tensor-core packed attention -> ``a8_gather_rows`` ->
``a8_prefill_finish``), after the voices' cached prefix K/V and codec state are loaded with ``a8_state_rows``.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import time
from types import SimpleNamespace
from typing import Dict, List

import numpy as np
import torch

from . import _lib as L
from .snapstore import SnapStore, ref_fp

BF16 = torch.bfloat16


def permute_qk(w, nq, nkv, hd):
    """Rows of the fused [q | k | v] projection with every q / k head's dims reordered from interleaved RoPE pairs
    (2i, 2i+1) to rotate_half halves (i, i + hd/2); q.k is unchanged (serve/fast_engine.py:60-67)."""
    p = torch.cat([torch.arange(0, hd, 2), torch.arange(1, hd, 2)]).to(w.device)
    rest = w.shape[1:]
    q = w[:nq * hd].reshape(nq, hd, *rest)[:, p].reshape(nq * hd, *rest)
    k = w[nq * hd:(nq + nkv) * hd].reshape(nkv, hd, *rest)[:, p].reshape(nkv * hd, *rest)
    return torch.cat([q, k, w[(nq + nkv) * hd:]], 0).contiguous()


def rope_tables(base, hd, n):
    """cos / sin [n, hd] (bf16) for rotate_half: fp32 phases rounded to bf16 (serve/fast_engine.py:70-75)."""
    fr = 1.0 / (base ** (torch.arange(0, hd, 2).float()[: hd // 2] / hd))
    ph = torch.outer(torch.arange(n).float(), fr)
    c, s = ph.cos().to(BF16), ph.sin().to(BF16)
    return torch.cat([c, c], -1).contiguous(), torch.cat([s, s], -1).contiguous()


def interleave_w13(w1, w3):
    """[w1; w3] reordered so each 128-row tile holds 64 gate rows then the 64 matching up rows (the GEMM's SiLU-mul
    epilogue pairs them inside one tile)."""
    I, D = w1.shape
    assert I % 64 == 0
    return torch.cat([w1.reshape(I // 64, 64, D), w3.reshape(I // 64, 64, D)], 1).reshape(2 * I, D).contiguous()


def _clean_text(text: str) -> str:
    return " ".join(str(text).strip().split())


class PackedStack:
    """One transformer stack's packed weights, caches and RoPE tables on the device + its A8StackDesc."""

    def __init__(self, layers, norm, nq, nkv, hd, eps, rope_base, cache_rows, cache_len, max_pos, dev, ring=0,
                 layer_scale=False):
        def w(t):
            return t.detach().to(torch.float32)
        wq, bq, wo, w13, w2, l1, l2 = [], [], [], [], [], [], []
        for Ly in layers:
            a, f = Ly.attention, Ly.feed_forward
            o_, d_ = w(a.wo.weight), w(f.w2.weight)
            if layer_scale:                 # LayerScale folded into the output projections (serve/fast_engine.py:96-98)
                o_ = o_ * w(Ly.attention_layer_scale.gamma)[:, None]
                d_ = d_ * w(Ly.ffn_layer_scale.gamma)[:, None]
            wq.append(permute_qk(w(a.wqkv.weight), nq, nkv, hd).to(BF16))
            if a.wqkv.bias is not None:
                bq.append(permute_qk(w(a.wqkv.bias), nq, nkv, hd).to(BF16))
            wo.append(o_.to(BF16))
            w13.append(interleave_w13(w(f.w1.weight).to(BF16), w(f.w3.weight).to(BF16)))
            w2.append(d_.to(BF16))
            l1.append(w(Ly.attention_norm.weight).to(BF16))
            l2.append(w(Ly.ffn_norm.weight).to(BF16))
        st = lambda xs: torch.stack(xs).to(dev).contiguous()
        self.wqkv, self.wo, self.w13, self.w2 = st(wq), st(wo), st(w13), st(w2)
        self.bqkv = st(bq) if bq else None
        self.ln1, self.ln2 = st(l1), st(l2)
        self.norm = w(norm.weight).to(BF16).to(dev)
        c, s = rope_tables(rope_base, hd, max_pos)
        self.cos, self.sin = c.to(dev), s.to(dev)
        nl = len(layers)
        self.kc = torch.zeros(nl, cache_rows, nkv, cache_len, hd, dtype=BF16, device=dev)
        self.vc = torch.zeros_like(self.kc)
        self.nq, self.nkv, self.hd, self.eps = nq, nkv, hd, float(eps)
        self.dim = self.wo.shape[1]
        self.inter = self.w2.shape[2]
        self.layers, self.cache_rows, self.cache_len, self.ring = nl, cache_rows, cache_len, int(ring or 0)
        self.desc = L.A8StackDesc(
            layers=nl, dim=self.dim, nq=nq, nkv=nkv, hd=hd, inter=self.inter, eps=self.eps, wqkv=L.ptr(self.wqkv),
            bqkv=L.ptr(self.bqkv), wo=L.ptr(self.wo), w13=L.ptr(self.w13), w2=L.ptr(self.w2), ln1=L.ptr(self.ln1),
            ln2=L.ptr(self.ln2), norm=L.ptr(self.norm), cos=L.ptr(self.cos), sin=L.ptr(self.sin), kc=L.ptr(self.kc),
            vc=L.ptr(self.vc), cache_rows=cache_rows, cache_len=cache_len, ring=self.ring)


class Scratch:
    """Activation buffers and the attention's split workspace for up to `rows` token rows of stacks up to `dim` /
    `inter` wide."""

    def __init__(self, rows, dim, qdim, inter, nkv, hd, max_len, dev):
        mk = lambda n: torch.zeros(rows, n, dtype=BF16, device=dev)
        self.h, self.q, self.o, self.a, self.mlp = mk(dim), mk(qdim), mk(qdim), mk(dim), mk(inter)
        n = C.c_longlong()
        L.check(L.load().a8_attention_workspace(rows, nkv, hd, max_len, C.byref(n), None), "attention workspace")
        self.attn_ws = torch.zeros(max(1, n.value), dtype=torch.float32, device=dev)
        self.attn_counters = torch.zeros(rows * nkv, dtype=torch.int32, device=dev)
        self.ssq = torch.zeros(8, rows, dtype=torch.float32, device=dev)
        self.desc = L.A8Scratch(
            h=L.ptr(self.h), q=L.ptr(self.q), o=L.ptr(self.o), a=L.ptr(self.a), mlp=L.ptr(self.mlp),
            attn_ws=L.ptr(self.attn_ws), attn_ws_floats=self.attn_ws.numel(), attn_counters=L.ptr(self.attn_counters),
            n_attn_counters=self.attn_counters.numel(), ssq=L.ptr(self.ssq), ssq_ld=rows)
        self.rows = rows


class FastEngine:
    """serve/fast_engine.py:570 on sm_100a kernels. Sampling noise: Philox keyed by `seed` (default from
    TTS_SEED, else 1234), counted by the engine's tick number."""

    def __init__(self, model, tokenizer, gen_params: dict, max_slots: int = 32, max_seq: int = 2048, buckets=None,
                 seq_from_env=True, seed=None):
        if not torch.cuda.is_available():
            raise L.A8Error("FastEngine needs a CUDA device (B200); there is no CPU fallback")
        L.load()
        dev = torch.device("cuda", torch.cuda.current_device())
        if not L.load().a8_device_ok():
            raise L.A8Error("libaudio8_b200 kernels need a compute-capability 10.0 GPU (B200)")
        self.m, self.tokz = model, tokenizer
        c = self.cfg = model.config
        self.dev = dev
        self.dt = BF16
        self.B = int(max_slots)
        S = int(os.environ.get("TTS_MAX_SEQ", str(max_seq))) if seq_from_env else int(max_seq)
        self.S = min(S, int(c.max_seq_len))
        gp = dict(gen_params or {})
        self.gp = gp
        self.eos, self.sb, self.se = int(c.eos_token_id), int(c.semantic_begin_id), int(c.semantic_end_id)
        self.ncg, self.cbk = int(c.num_codebooks), int(c.codebook_size)
        self.nsem = self.se - self.sb + 1
        self.do_sample = bool(gp.get("do_sample", True))
        self.temperature = max(float(gp.get("temperature", 0.8) or 1.0), 1e-5)
        tk = gp.get("top_k", 50)
        self.top_k = int(tk) if tk and int(tk) > 0 else 0
        self.top_p = float(gp.get("top_p", 0.95)) if gp.get("top_p", 0.95) is not None else 1.0
        self.ras_p, self.ras_t, self.ras_w = float(c.ras_top_p), max(float(c.ras_temperature), 1e-5), \
            int(c.ras_window_size)
        self.max_new = int(gp.get("max_new_tokens", 2048))
        self.seed = int(seed if seed is not None else os.environ.get("TTS_SEED", "1234"))
        B, H = self.B, int(c.dim)
        self.H = H
        assert int(c.fast_dim) == H and bool(c.norm_fastlayer_input), "fast_project_in / unnormed fast input"
        self.prefill_tokens = int(os.environ.get("TTS_PREFILL_TOKENS", "8192"))
        self.pf_rows = min(self.prefill_tokens, int(os.environ.get("TTS_PREFILL_ROWS", "2048")))
        self.SCR = B
        self.slow = PackedStack(model.layers, model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps,
                                c.rope_base, cache_rows=B + 1, cache_len=self.S, max_pos=self.S, dev=dev)
        self.fast = PackedStack(model.fast_layers, model.fast_norm, c.fast_n_head, c.fast_n_local_heads,
                                c.fast_head_dim, c.norm_eps, c.rope_base, cache_rows=B, cache_len=self.ncg,
                                max_pos=self.ncg, dev=dev)
        f32 = lambda t: t.detach().to(torch.float32)
        emb = f32(model.embeddings.weight)
        self.emb = emb.to(BF16).to(dev)
        self.cbemb = f32(model.codebook_embeddings.weight).to(BF16).to(dev)
        self.cb_off = (torch.arange(self.ncg, device=dev) * self.cbk).view(1, -1)
        nh = self.nh = self.nsem + 1
        head = torch.zeros(nh, H, dtype=BF16)
        head[:self.nsem] = emb[self.sb:self.se + 1].to(BF16)
        head[self.nsem] = emb[self.eos].to(BF16)
        self.head = head.to(dev)
        self.fast_emb = f32(model.fast_embeddings.weight).to(BF16).to(dev)
        self.fast_out = f32(model.fast_output.weight).to(BF16).to(dev)
        # codec: built from an fp32 copy of the model's codec (serve/fast_engine.py:625-633)
        from .codec import StreamingVocoder
        with torch.no_grad():                             # (not inference tensors: callers may write the state)
            codec = model.load_codec(device=dev, dtype=torch.float32)
            self.sr = int(getattr(codec, "sample_rate", getattr(c, "codec_sample_rate", 44100)))
            self.voc = StreamingVocoder(codec, B, dev, max_pos=int(os.environ.get("TTS_VOC_MAX_POS", "8192")))
            del codec
        self.up = self.voc.up
        self.fps = self.sr / self.up
        codes, _ = model.encode_audio(torch.zeros(1, 1, self.sr, device=model.device))
        self.sil_frame = codes[0, :, codes.shape[-1] // 2].long().clamp(min=0).to(dev)
        # TTS_VOC_PRIME=0 (default): a row's codec starts clean and decodes a silence frame first; 1: from a snapshot
        # of its voice's reference decoded (prime_speakers)
        self.voc_prime = os.environ.get("TTS_VOC_PRIME", "0").strip().lower() not in ("0", "false", "no", "off")
        self.prime_frames = max(2, int(os.environ.get("TTS_VOC_PRIME_FRAMES", "160")))
        self.voc_snaps = SnapStore()                # memory only; a worker may install one with a disk cache
        self.side = torch.cuda.Stream(device=dev)

        # persistent per-slot state (fixed addresses; row B = SCR, prefill padding)
        i64, i32 = torch.int64, torch.int32
        self.tok = torch.zeros(B + 1, dtype=i64, device=dev)
        self.hid = torch.zeros(B + 1, H, dtype=BF16, device=dev)
        self.cpos = torch.zeros(B + 1, dtype=i32, device=dev)
        self.prev = torch.zeros(B + 1, self.ras_w, dtype=i64, device=dev)
        self.nstep = torch.zeros(B + 1, dtype=i32, device=dev)
        self.tok_in = torch.zeros(B, dtype=i64, device=dev)
        self.audio = self.voc.audio                       # [B, up] fp32: the codec writes it in the tick
        self.frame_prev = torch.zeros(B, self.ncg, dtype=i64, device=dev)
        self.tick_ctr = torch.zeros(1, dtype=i64, device=dev)
        self.tick_id = torch.zeros(1, dtype=i64, device=dev)
        # tick scratch
        self.x_fast2 = torch.zeros(2 * B, H, dtype=BF16, device=dev)
        self.x_fast = torch.zeros(B, H, dtype=BF16, device=dev)
        self.x_slow = torch.zeros(B, H, dtype=BF16, device=dev)
        self.codes = torch.zeros(B, self.ncg, dtype=i64, device=dev)
        self.ld_logits = (max(self.nh, self.cbk) + 3) // 4 * 4
        self.logits = torch.zeros(max(B, 64), self.ld_logits, dtype=torch.float32, device=dev)
        self.f_pos = torch.arange(self.ncg, dtype=i32, device=dev).view(-1, 1).repeat(1, 2 * B).contiguous()
        self.f_pos0 = (torch.arange(2 * B, dtype=i32, device=dev) % 2).contiguous()
        self.f_slot0 = (torch.arange(2 * B, dtype=i32, device=dev) // 2).contiguous()
        rows = max(2 * B, self.pf_rows)
        self.scratch = Scratch(rows, H, self.slow.nq * self.slow.hd, self.slow.inter, self.slow.nkv, self.slow.hd,
                               self.S, dev)
        self.pf_pos = torch.zeros(self.pf_rows, dtype=i32, device=dev)
        self.pf_slot = torch.zeros(self.pf_rows, dtype=i32, device=dev)
        self.pf_last = torch.zeros(self.pf_rows, dtype=i32, device=dev)
        self.pf_st = torch.zeros(self.pf_rows, dtype=i32, device=dev)
        self.pf_cpos = torch.zeros(self.pf_rows, dtype=i32, device=dev)
        self.pf_hl = torch.zeros(max(B, 64), H, dtype=BF16, device=dev)
        self.pf_blocks = torch.zeros(self.pf_rows // 64 + B + 2, 4, dtype=i32, device=dev)
        # prefill graphs: one per token bucket (64, 128, ... up to pf_rows), up to pf_NR requests a chunk, fed by one
        # int32 metadata buffer (serve/fast_engine.py:682-691 pf_meta, :797-812); TTS_PREFILL_GRAPHS=0: the same
        # launches eagerly
        self.pf_buckets = sorted({64 << k for k in range(16) if (64 << k) <= self.pf_rows} | {self.pf_rows})
        self.pf_NT, self.pf_NR = self.pf_buckets[-1], 64
        self.pf_graph_on = os.environ.get("TTS_PREFILL_GRAPHS", "1").strip().lower() not in ("0", "false", "no", "off")
        self.pf_graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.pf_off = self._pf_layout()
        self.pf_meta = torch.zeros(int(self.pf_off[-1]), dtype=i32, device=dev)
        self.pf_meta_h = torch.zeros(int(self.pf_off[-1]), dtype=i32).pin_memory()
        self.pf_x = torch.zeros(self.pf_rows, H, dtype=BF16, device=dev)

        self.desc = L.A8Engine(
            B=B, S=self.S, H=H, ncb=self.ncg, cbk=self.cbk, nsem=self.nsem, vocab=self.emb.shape[0], ras_w=self.ras_w,
            eos=self.eos, sb=self.sb, do_sample=int(self.do_sample), top_k=self.top_k, top_p=self.top_p,
            temperature=self.temperature, ras_top_p=self.ras_p, ras_temperature=self.ras_t, seed=self.seed,
            slow=self.slow.desc, fast=self.fast.desc, emb=L.ptr(self.emb), cbemb=L.ptr(self.cbemb),
            head=L.ptr(self.head), fast_emb=L.ptr(self.fast_emb), fast_out=L.ptr(self.fast_out), tok=L.ptr(self.tok),
            hid=L.ptr(self.hid), cpos=L.ptr(self.cpos), prev=L.ptr(self.prev), nstep=L.ptr(self.nstep),
            tok_in=L.ptr(self.tok_in), frame_prev=L.ptr(self.frame_prev), sil_frame=L.ptr(self.sil_frame),
            tick_ctr=L.ptr(self.tick_ctr), tick_id=L.ptr(self.tick_id), x_fast2=L.ptr(self.x_fast2),
            x_fast=L.ptr(self.x_fast), x_slow=L.ptr(self.x_slow), codes=L.ptr(self.codes), logits=L.ptr(self.logits),
            ld_logits=self.ld_logits, f_pos=L.ptr(self.f_pos), f_pos0=L.ptr(self.f_pos0),
            f_slot0=L.ptr(self.f_slot0), scratch=self.scratch.desc, voc=C.pointer(self.voc.desc),
            side=C.c_void_p(self.side.cuda_stream))

        env_b = os.environ.get("TTS_BATCH_BUCKETS", "").strip()
        if env_b:
            buckets = [int(x) for x in env_b.split(",") if x.strip()]
        if not buckets:
            buckets = [1, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32, 40, 48, 56, 64, 72, 80, 88, 96, 104, 112, 120, 128,
                       144, 160, 176, 192]
        self.buckets = sorted({b for b in buckets if 1 <= b <= B} | {B})
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self._parts = None
        self._spk_cache: Dict[str, torch.Tensor] = {}
        self._pkv: Dict[str, tuple] = {}
        self.dir = None
        self.guide = False

    # ------------------------------------------------------------------ the tick
    def tick(self, b):
        """One frame for rows [0, b) launched eagerly on the current stream (capture() records it per bucket)."""
        L.call("a8_tick", C.byref(self.desc), int(b), L.stream_handle())

    def slow_step(self, b):
        L.call("a8_slow_step", C.byref(self.desc), int(b), L.stream_handle())

    def record_fast_logits(self, on=True):
        """Keep every codebook's fast-head logits readable after a tick: `rec_logits[i - 1, r, :cbk]` (fp32) for
        codebook i of row r (a diagnostic for tests; the head GEMM writes there instead of the shared logits buffer,
        no extra work). A graph recorded by capture() keeps the choice it was recorded with."""
        self.rec_logits = (torch.zeros(self.ncg - 1, self.B, self.ld_logits, dtype=torch.float32, device=self.dev)
                           if on else None)
        self.desc.rec_logits = L.ptr(self.rec_logits) if on else None

    @torch.inference_mode()
    def capture(self, log=print):
        """Warm up and record one CUDA graph per bucket (largest first)."""
        t0 = time.perf_counter()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        order = sorted(self.buckets, reverse=True)
        with torch.cuda.stream(s):
            for b in order:
                for _ in range(2):
                    self.tick(b)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        for b in order:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.tick(b)
            self.graphs[b] = g
        torch.cuda.synchronize()
        self.capture_prefill(log)
        self.reset_state()
        log(f"[a8] captured {len(self.graphs)} tick graphs {self.buckets} + {len(self.pf_graphs)} prefill graphs "
            f"{sorted(self.pf_graphs)} in {time.perf_counter() - t0:.1f}s")

    def reset_state(self):
        for t in (self.tok, self.cpos, self.hid, self.prev, self.nstep, self.tick_ctr, self.frame_prev, self.audio):
            t.zero_()
        self.voc.clear_many(list(range(self.B)))

    def bucket_for(self, n_rows):
        for b in self.buckets:
            if b >= n_rows:
                return b
        return self.buckets[-1]

    @torch.inference_mode()
    def replay(self, b, bd=0):
        self.graphs[b].replay()

    # ---- guidance / director: not on this model (the worker calls these unconditionally) ----
    def dir_bucket(self):
        return 0

    def pairs_free(self):
        return 0

    def clear_groups(self, slots):
        return None

    def guide_groups(self, groups):
        if groups:
            raise NotImplementedError("guided groups (TTS_INSTRUCT_MODE=guide) are not supported by the Audio8 engine")

    def guide_cross(self, entries):
        return {}

    def attach_director(self, *a, **k):
        raise NotImplementedError("a guidance director (TTS_GUIDE_DIRECTOR) is not supported by the Audio8 engine")

    # ------------------------------------------------------------------ prompts (serve/fast_engine.py:903-983)
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
    def _ref_text(text):
        t = _clean_text(text)
        return t if re.search(r"<\|speaker:\d+\|>", t) else f"<|speaker:0|>{t}"

    def _prompt_ids(self, item):
        P = self._parts
        rc = getattr(item, "ref_code", None) if item is not None else None
        if rc is None or not getattr(item, "ref_text", ""):
            ids = torch.tensor(P.noref, dtype=torch.long)
            return ids, torch.zeros(len(ids), self.ncg, dtype=torch.long), torch.zeros(len(ids), dtype=torch.bool)
        head = P.ref_head + self._enc(self._ref_text(item.ref_text)) + P.speech
        codes = rc.long().cpu()
        T = codes.shape[0]
        sem = torch.cat([torch.tensor(head, dtype=torch.long), codes[:, 0] + self.sb,
                         torch.tensor(P.user, dtype=torch.long)])
        cb = torch.zeros(len(sem), self.ncg, dtype=torch.long)
        cb[len(head):len(head) + T] = codes
        aud = torch.zeros(len(sem), dtype=torch.bool)
        aud[len(head):len(head) + T] = True
        return sem, cb, aud

    def _prompt_rows(self, sem, cb, aud):
        """Prompt positions as the int32 rows a8_embed_prompt reads: (sem, audio, code_0 .. code_{ncg-1}) -- the
        codebook sum is added on audio positions only (serve/fast_engine.py:941-945)."""
        rows = np.zeros((len(sem), 2 + self.ncg), dtype=np.int32)
        rows[:, 0] = np.asarray(sem, dtype=np.int64)
        rows[:, 1] = np.asarray(aud, dtype=np.int64)
        rows[:, 2:] = np.asarray(cb, dtype=np.int64).reshape(len(sem), self.ncg)
        return rows

    def _speaker_prefix(self, key, item):
        hit = self._spk_cache.get(key)
        if hit is None:
            sem, cb, aud = self._prompt_ids(item)
            hit = self._prompt_rows(sem.numpy(), cb.numpy(), aud.numpy())
            self._spk_cache[key] = hit
        return hit

    @torch.inference_mode()
    def build_prompts(self, reqs):
        """(key, voice-prefix rows, rest rows) per request; rows as _prompt_rows (host int32)."""
        if not reqs:
            return []
        if self._parts is None:
            self._parts_init()
        P = self._parts
        out = []
        for r in reqs:
            ctx_t = (r.get("ctx_text") or "").strip()
            ids = torch.tensor(self._enc(_clean_text((ctx_t + " " if ctx_t else "") + r["text"]) or ".") + P.tail,
                               dtype=torch.long)
            cb = torch.zeros(len(ids), self.ncg, dtype=torch.long)
            aud = torch.zeros(len(ids), dtype=torch.bool)
            if r.get("ctx_codes") is not None:
                cc = torch.as_tensor(r["ctx_codes"]).long().reshape(-1, self.ncg)
                ids = torch.cat([ids, cc[:, 0] + self.sb])
                cb = torch.cat([cb, cc])
                aud = torch.cat([aud, torch.ones(len(cc), dtype=torch.bool)])
            rest = self._prompt_rows(ids.numpy(), cb.numpy(), aud.numpy())
            out.append((r["key"], self._speaker_prefix(r["key"], r["item"]), rest))
        return out

    # ------------------------------------------------------------------ admission (serve/fast_engine.py:1035-1156)
    def evict_voices(self, keys) -> int:
        ks, n = set(keys), 0
        for d in (self._pkv, self._spk_cache):
            for k in [k for k in d if k in ks]:
                del d[k]
                n += 1
        return n

    def voice_state_bytes(self) -> int:
        n = sum(e.blob.numel() + e.segs.numel() for e in self._pkv.values())
        return n + sum(t.nbytes for t in self._spk_cache.values())

    def prime_speaker(self, key, item):
        self.prime_speakers([(key, item)])

    @torch.inference_mode()
    def prime_speakers(self, pairs):
        """serve/fast_engine.py:994-1033: up to B voice references decode side by side through the codec (rows
        [0, B), only while nothing runs), each row snapshotted after its own second-to-last frame; the snapshot (host,
        pinned) and the last frame are kept per key. TTS_VOC_PRIME=0 (default): nothing to do."""
        if not self.voc_prime:
            return
        todo, seen = [], set()
        for key, item in pairs:
            if getattr(self.voc_snaps, "path", None):   # its file is named by the codes it is made from
                self.voc_snaps.set_fp(key, ref_fp(item))
            if key not in self.voc_snaps and key not in seen:
                seen.add(key)
                todo.append((key, item))
        for g in range(0, len(todo), self.B):
            grp = todo[g:g + self.B]
            n = len(grp)
            codes = []
            for _, item in grp:
                rc = getattr(item, "ref_code", None)
                if rc is not None:
                    rc = rc[-self.prime_frames:]
                codes.append(rc.to(self.dev).long() if rc is not None and rc.shape[0] > 0
                             else torch.zeros(0, self.ncg, dtype=torch.long, device=self.dev))
            lens = [int(c.shape[0]) for c in codes]
            T = max(lens)
            pad = torch.zeros(n, max(T, 1), self.ncg, dtype=torch.long, device=self.dev)
            for r, c in enumerate(codes):
                pad[r, :lens[r]] = c
            self.voc.clear_many(list(range(n)))
            snaps = [self.voc.snapshot(r) if lens[r] <= 1 else None for r in range(n)]
            for t in range(T - 1):
                self.voc.step(pad[:, t], n)
                for r in range(n):
                    if lens[r] - 2 == t:
                        snaps[r] = self.voc.snapshot(r)
            for r, (key, _) in enumerate(grp):
                last = codes[r][-1].clone() if lens[r] else self.sil_frame.clone()
                self.voc_snaps[key] = ([t.cpu().pin_memory() for t in snaps[r]], last.cpu())
            self.voc.clear_many(list(range(n)))

    @staticmethod
    def query_blocks(pos, slot, bm=64):
        """The packed-prefill query blocks (q0, n, slot, pos0) of rows at host positions `pos` in cache rows `slot`:
        runs of consecutive positions of one cache row, at most `bm` rows each (PrefillPlan's blocks,
        serve/fast_kernels.py:335-347)."""
        pos, slot = np.asarray(pos, dtype=np.int64), np.asarray(slot, dtype=np.int64)
        out, i, n = [], 0, len(pos)
        while i < n:
            j = i + 1
            while j < n and j - i < bm and slot[j] == slot[i] and pos[j] == pos[j - 1] + 1:
                j += 1
            out.append((i, j - i, int(slot[i]), int(pos[i])))
            i = j
        return np.array(out, dtype=np.int32).reshape(-1, 4)

    def _forward_rows(self, x, pos, slot, max_len, pos_h=None, slot_h=None):
        """Packed causal prefill of rows x [n, H] (bf16, consumed) at positions pos into cache rows slot; with the
        positions and cache rows on the host too, attention runs on query blocks (the tensor-core prefill kernel)."""
        n = x.shape[0]
        assert n <= self.pf_rows
        self.pf_pos[:n].copy_(pos, non_blocking=True)
        self.pf_slot[:n].copy_(slot, non_blocking=True)
        nb = 0
        if pos_h is not None:
            blk = self.query_blocks(pos_h, slot_h)
            nb = blk.shape[0]
            assert nb <= self.pf_blocks.shape[0]
            self.pf_blocks[:nb].copy_(torch.from_numpy(blk))
        run = L.A8StackRun(x=L.ptr(x), ldx=self.H, rows=n, pos=L.ptr(self.pf_pos), slot=L.ptr(self.pf_slot),
                           lens=None, lens_max=0, rowmap=L.ptr(self.pf_slot), max_len=int(max_len),
                           scratch=self.scratch.desc, blocks=L.ptr(self.pf_blocks) if nb else None, nblocks=nb)
        L.call("a8_stack_forward", C.byref(self.slow.desc), C.byref(run), L.stream_handle())
        return self.scratch.h[:n]

    def _embed_rows(self, rows, out):
        """Prompt rows (host int32, as _prompt_rows) -> their input embeddings in `out` [n, H] (bf16, device)."""
        n = rows.shape[0]
        dev_rows = torch.from_numpy(np.ascontiguousarray(rows)).to(self.dev)
        L.call("a8_embed_prompt", L.ptr(dev_rows), self.ncg, self.cbk, L.ptr(self.emb), L.ptr(self.cbemb),
               L.ptr(out), self.H, n, self.H, self.emb.shape[0], L.stream_handle())
        return out[:n]

    def _kv_segments(self, Lp):
        """A8StateSeg table (device) of a cache row's first Lp positions of every slow layer's K and V: a prefix's K/V
        as one blob [K / V, kv head, layer, Lp, hd] that a8_state_rows snapshots from the scratch row and loads into
        slots."""
        st = self.slow
        es = 2
        per_pos = st.hd * es
        segs, off = [], 0
        for cache in (st.kc, st.vc):
            for h in range(st.nkv):
                segs.append(L.A8StateSeg(base=cache.data_ptr() + h * st.cache_len * per_pos,
                                         slot_stride=st.nkv * st.cache_len * per_pos, chunk_bytes=Lp * per_pos,
                                         chunk_stride=st.cache_rows * st.nkv * st.cache_len * per_pos,
                                         nchunks=st.layers, blob_off=off))
                off += st.layers * Lp * per_pos
        raw = bytes((L.A8StateSeg * len(segs))(*segs))
        return torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.dev), len(segs), off

    def _prefix_kv(self, pkey, prefix):
        """A voice prefix's K/V for every slow layer, computed once into the scratch row and kept as one blob
        (serve/fast_engine.py:1073-1087); admission loads it into the slots of that voice with one a8_state_rows."""
        hit = self._pkv.get(pkey)
        if hit is not None:
            return hit
        Lp = prefix.shape[0]
        for a in range(0, Lp, self.pf_rows):
            e = min(Lp, a + self.pf_rows)
            x = self._embed_rows(prefix[a:e], self.pf_x)
            pos = torch.arange(a, e, dtype=torch.int32, device=self.dev)
            slot = torch.full((e - a,), self.SCR, dtype=torch.int32, device=self.dev)
            self._forward_rows(x, pos, slot, e, np.arange(a, e), np.full(e - a, self.SCR))
        segs, nseg, nbytes = self._kv_segments(Lp)
        blob = torch.empty(nbytes, dtype=torch.uint8, device=self.dev)
        scr = torch.tensor([self.SCR], dtype=torch.int32, device=self.dev)
        L.call("a8_state_rows", L.ptr(segs), nseg, L.ptr(scr), 1, L.STATE_SNAPSHOT, L.ptr(blob), L.stream_handle())
        hit = SimpleNamespace(Lp=Lp, blob=blob, segs=segs, nseg=nseg)
        self._pkv[pkey] = hit
        return hit

    # ---- packed prefill in a captured graph per token bucket (serve/fast_engine.py:797-853, :1108-1116)
    def _pf_layout(self):
        """Offsets (int32 words) of the prefill metadata: ids [NT, 2 + ncg] | pos [NT] | slot [NT] | blocks [NB, 4] |
        last [NR] | st [NR] | cpos [NR] | frame0 [NR, ncg], NT = the largest token bucket, NB = NT / 64 + NR."""
        NT, NR = self.pf_NT, self.pf_NR
        sizes = [NT * (2 + self.ncg), NT, NT, 4 * (NT // 64 + NR), NR, NR, NR, NR * self.ncg]
        return np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)

    def _pf_views(self, nt):
        o, m = self.pf_off, self.pf_meta
        NR = self.pf_NR
        v = SimpleNamespace()
        v.ids = m[o[0]:o[0] + nt * (2 + self.ncg)]
        v.pos, v.slot = m[o[1]:o[1] + nt], m[o[2]:o[2] + nt]
        v.nb = nt // 64 + NR
        v.blocks = m[o[3]:o[3] + 4 * v.nb]
        v.last, v.st, v.cpos = m[o[4]:o[5]], m[o[5]:o[6]], m[o[6]:o[7]]
        v.frame0 = m[o[7]:o[8]]
        return v

    def _pf_body(self, nt):
        """The prefill of nt packed rows (bucket size) from the static metadata: embeddings, the slow stack with
        packed causal attention on query blocks, each request's last row, its first token / hidden / position /
        first codec frame (serve/fast_engine.py:820-835). Padding rows, blocks and requests point at the scratch row;
        padding blocks are empty."""
        v = self._pf_views(nt)
        st = L.stream_handle()
        L.call("a8_embed_prompt", L.ptr(v.ids), self.ncg, self.cbk, L.ptr(self.emb), L.ptr(self.cbemb),
               L.ptr(self.pf_x), self.H, nt, self.H, self.emb.shape[0], st)
        run = L.A8StackRun(x=L.ptr(self.pf_x), ldx=self.H, rows=nt, pos=L.ptr(v.pos), slot=L.ptr(v.slot), lens=None,
                           lens_max=0, rowmap=L.ptr(v.slot), max_len=self.S, scratch=self.scratch.desc,
                           blocks=L.ptr(v.blocks), nblocks=v.nb)
        L.call("a8_stack_forward", C.byref(self.slow.desc), C.byref(run), st)
        L.call("a8_gather_rows", L.ptr(self.scratch.h), self.H, L.ptr(v.last), L.ptr(self.pf_hl), self.H, self.pf_NR,
               self.H, st)
        L.call("a8_prefill_finish", C.byref(self.desc), L.ptr(self.pf_hl), self.pf_NR, L.ptr(v.st), L.ptr(v.cpos),
               L.ptr(v.frame0), st)

    def _pf_fill(self, nt, slots, parts, starts, frames):
        """The host metadata of one chunk (padded to bucket nt) into the pinned buffer, then one copy to the device."""
        h, o = self.pf_meta_h.numpy(), self.pf_off
        NR, SCR, k = self.pf_NR, self.SCR, len(slots)
        h[:] = 0
        ids = h[o[0]:o[0] + nt * (2 + self.ncg)].reshape(nt, 2 + self.ncg)
        pos, slot = h[o[1]:o[1] + nt], h[o[2]:o[2] + nt]
        slot[:] = SCR
        r0 = 0
        pos_l, slot_l = [], []
        for s, (_, _, rest), a in zip(slots, parts, starts):
            n = rest.shape[0]
            ids[r0:r0 + n] = rest
            pos[r0:r0 + n] = np.arange(a, a + n)
            slot[r0:r0 + n] = s
            r0 += n
        blk = self.query_blocks(pos[:r0], slot[:r0])
        nb = nt // 64 + NR
        assert blk.shape[0] <= nb and k <= NR
        h[o[3]:o[3] + 4 * blk.shape[0]] = blk.reshape(-1)
        last, st, cpos = h[o[4]:o[5]], h[o[5]:o[6]], h[o[6]:o[7]]
        st[:] = SCR
        ends = np.cumsum([p[2].shape[0] for p in parts]) - 1
        last[:k] = ends
        st[:k] = slots
        cpos[:k] = [a + p[2].shape[0] for a, p in zip(starts, parts)]
        h[o[7]:o[8]].reshape(NR, self.ncg)[:k] = np.stack([f.cpu().numpy() for f in frames]) if k else 0
        self.pf_meta[:o[8]].copy_(self.pf_meta_h[:o[8]], non_blocking=True)

    def capture_prefill(self, log=print):
        """Warm up and record one prefill graph per token bucket (largest first), all padding."""
        if not self.pf_graph_on:
            return
        self._pf_fill(self.pf_NT, [], [], [], [])
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for nt in reversed(self.pf_buckets):
                for _ in range(2):
                    self._pf_body(nt)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        for nt in reversed(self.pf_buckets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._pf_body(nt)
            self.pf_graphs[nt] = g
        torch.cuda.synchronize()

    @torch.inference_mode()
    def admit(self, slots: List[int], reqs: List[dict]):
        """Packed prefill of reqs into free slots. Returns each prompt's length, or -1 for one that can't fit."""
        if not reqs:
            return []
        parts = self.build_prompts(reqs)
        lens = [p.shape[0] + r.shape[0] for _, p, r in parts]
        limit = min(self.S - 32, self.prefill_tokens)
        ok = [i for i, n in enumerate(lens) if n <= limit]
        # chunks a prefill graph takes (tokens <= the largest bucket, requests <= NR); a request whose rest exceeds
        # the largest bucket goes through pieces of pf_rows rows on its own
        chunk, tot = [], 0
        for i in ok:
            n = parts[i][2].shape[0]
            if n > self.pf_NT:
                self._prefill_pieces([slots[i]], [reqs[i]], [parts[i]])
                continue
            if chunk and (tot + n > self.pf_NT or len(chunk) >= self.pf_NR):
                self._prefill([slots[k] for k in chunk], [reqs[k] for k in chunk], [parts[k] for k in chunk])
                chunk, tot = [], 0
            chunk.append(i)
            tot += n
        if chunk:
            self._prefill([slots[k] for k in chunk], [reqs[k] for k in chunk], [parts[k] for k in chunk])
        return [n if n <= limit else -1 for n in lens]

    def _load_prefixes(self, slots, parts):
        """Each voice prefix's cached K/V into its requests' slots (one a8_state_rows per voice); returns the start
        position of each request's rest."""
        p0, groups = {}, {}
        for s, (pkey, prefix, _) in zip(slots, parts):
            if pkey is not None:
                groups.setdefault(pkey, []).append(s)
        for pkey, gslots in groups.items():
            prefix = next(p for (k, p, _) in parts if k == pkey)
            kv = self._prefix_kv(pkey, prefix)
            idx = torch.tensor(gslots, dtype=torch.int32).to(self.dev, non_blocking=True)
            L.call("a8_state_rows", L.ptr(kv.segs), kv.nseg, L.ptr(idx), len(gslots), L.STATE_LOAD, L.ptr(kv.blob),
                   L.stream_handle())
            for s in gslots:
                p0[s] = kv.Lp
        return [p0.get(s, 0) for s in slots]

    def _codec_rows(self, slots, reqs):
        """The codec state of admitted rows (serve/fast_engine.py:1134-1156) and the frame each decodes first:
        keep_voc rows keep their state and decode a silence frame first; the others start clean (silence frame first)
        or, primed (TTS_VOC_PRIME=1), from their voice's snapshot with its last reference frame."""
        frames = {}
        vgroups = {}
        for s, r in zip(slots, reqs):
            if r.get("keep_voc"):
                frames[s] = self.sil_frame
            else:
                vgroups.setdefault(r["key"] if self.voc_prime else None, []).append(s)
        for key, gslots in vgroups.items():
            snap = self.voc_snaps.get(key) if key is not None else None
            if snap is None:
                self.voc.clear_many(gslots)
                first = self.sil_frame
            else:
                self.voc.load_many(gslots, snap[0])
                first = snap[1].long()
            for s in gslots:
                frames[s] = first
        return [frames[s] for s in slots]

    def _prefill(self, slots, reqs, parts):
        """One chunk: prefix K/V into the slots, then the packed prefill of the rests in the graph of the smallest
        token bucket that holds them (eager launches of the same body before capture_prefill)."""
        starts = self._load_prefixes(slots, parts)
        frames = self._codec_rows(slots, reqs)
        n = sum(p[2].shape[0] for p in parts)
        nt = next(b for b in self.pf_buckets if b >= n)
        self._pf_fill(nt, slots, parts, starts, frames)
        g = self.pf_graphs.get(nt)
        if g is not None:
            g.replay()
        else:
            self._pf_body(nt)

    def _prefill_pieces(self, slots, reqs, parts):
        """A request whose rest exceeds the largest token bucket: its packed rows in pieces of pf_rows rows (later
        rows attend to the keys earlier pieces stored), its last row gathered from the piece it ends in."""
        starts = self._load_prefixes(slots, parts)
        frames = self._codec_rows(slots, reqs)
        dev = self.dev
        rows = np.concatenate([r for _, _, r in parts], 0)
        ns = [int(r.shape[0]) for _, _, r in parts]
        pos_h = np.concatenate([np.arange(a, a + n) for a, n in zip(starts, ns)]).astype(np.int32)
        slot_h = np.concatenate([np.full(n, s) for n, s in zip(ns, slots)]).astype(np.int32)
        pos, slot_t = torch.from_numpy(pos_h).to(dev), torch.from_numpy(slot_h).to(dev)
        ends = np.cumsum(ns) - 1
        k, T = len(slots), rows.shape[0]
        i0 = 0
        for a in range(0, T, self.pf_rows):
            e = min(T, a + self.pf_rows)
            x = self._embed_rows(rows[a:e], self.pf_x)
            h = self._forward_rows(x, pos[a:e], slot_t[a:e], int(pos_h[a:e].max()) + 1, pos_h[a:e], slot_h[a:e])
            i1 = i0
            while i1 < k and ends[i1] < e:
                i1 += 1
            if i1 > i0:
                self.pf_last[i0:i1].copy_(torch.tensor(ends[i0:i1] - a, dtype=torch.int32))
                L.call("a8_gather_rows", L.ptr(h), self.H, L.ptr(self.pf_last[i0:]), L.ptr(self.pf_hl[i0]), self.H,
                       i1 - i0, self.H, L.stream_handle())
            i0 = i1
        self.pf_st[:k].copy_(torch.tensor(slots, dtype=torch.int32))
        self.pf_cpos[:k].copy_(torch.tensor([a + n for a, n in zip(starts, ns)], dtype=torch.int32))
        fr = torch.stack([f.to(torch.int32).cpu() for f in frames]).to(dev)
        L.call("a8_prefill_finish", C.byref(self.desc), L.ptr(self.pf_hl), k, L.ptr(self.pf_st), L.ptr(self.pf_cpos),
               L.ptr(fr), L.stream_handle())
