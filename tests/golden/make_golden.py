"""Generate the golden fixtures in this folder by running the REFERENCE itself on the CPU.

Run (only where the reference checkout exists; nothing at test time reads it):
    python tests/golden/make_golden.py /path/to/reference [--only kernels,sampler,host,stack,vocoder,engine]

The reference (serve/fast_kernels.py, serve/fast_engine.py) is Triton + torch. Its Triton kernels run here
under the Triton interpreter (TRITON_INTERPRET=1) on CPU tensors, and FastEngine runs with its CUDA-only
calls replaced by no-ops (pinned copies, side stream, graph capture are scheduling, not arithmetic).
Two interpreter defects are patched so that it computes what the GPU computes:
  * the interpreter multiplies bf16 operands of tl.dot as raw uint16 bits; they are widened to fp32
    first (a bf16 MMA with fp32 accumulation);
  * the interpreter converts fp32 -> bf16 by truncation; the GPU (cvt.rn.bf16.f32) rounds to nearest even.
tl.dot's input_precision is ignored by the interpreter (bf16 operands are exact in either mode).
Weights come from oracle/standin.py (seeded), so only inputs and outputs are stored.
"""
from __future__ import annotations

import os
import sys
import time
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"
os.environ["TTS_TRITON_GEMM"] = "0"          # GEMMs through torch.matmul (the reference's cuBLAS path)
os.environ["TTS_PREFILL_GRAPHS"] = "0"       # eager packed prefill (no graphs on a CPU)
os.environ.setdefault("TTS_VOC_FUSED_RU", "")

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np
import torch

BF16, F16 = torch.bfloat16, torch.float16


def _patch_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as I
    orig = I.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        def widen(h):
            if h.dtype.scalar == tl.bfloat16:
                return (h.data.astype(np.uint32) << 16).view(np.float32)
            return h.data
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            out = np.matmul(widen(a), widen(b), dtype=np.float32).astype(d.data.dtype) + d.data
            return I.TensorHandle(out, d.dtype.scalar)
        return orig(self, a, b, d, input_precision, max_num_imprecise_acc)

    I.InterpreterBuilder.create_dot = create_dot
    orig_conv = I._convert_float

    def convert_float(inp, src, dst, rounding_mode):
        if src == tl.float32 and dst == tl.bfloat16 and rounding_mode is None:
            u = np.ascontiguousarray(inp).view(np.uint32).astype(np.uint64)
            r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
            nan = (u & 0x7FFFFFFF) > 0x7F800000
            return np.where(nan, np.uint16(0x7FC0), r)
        return orig_conv(inp, src, dst, rounding_mode)

    I._convert_float = convert_float


class _NoStream:
    def __init__(self, *a, **k):
        pass

    def wait_stream(self, *a, **k):
        pass


class _NoCtx:
    def __init__(self, *a, **k):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _patch_cuda():
    torch.Tensor.pin_memory = lambda self, *a, **k: self
    torch.cuda.Stream = _NoStream
    torch.cuda.current_stream = lambda *a, **k: _NoStream()
    torch.cuda.stream = _NoCtx


def gen(seed):
    return torch.Generator().manual_seed(seed)


def randn(shape, g, scale=1.0, dtype=torch.float32):
    return (torch.randn(shape, generator=g) * scale).to(dtype)


# ------------------------------------------------------------------------------------------------
def make_kernels(fk):
    g = gen(100)
    out = {}
    # rmsnorm (serve/fast_kernels.py:30-69)
    for N in (896, 1024):
        x = randn((5, N), g, 2.0, BF16)
        r = randn((5, N), g, 3.0, BF16)
        w = (torch.rand(N, generator=g) + 0.5).to(BF16)
        y = fk.rmsnorm(x, w, 1e-6)
        r2 = r.clone()
        y2, ro = fk.rmsnorm(x, w, 1e-6, residual=r2)
        out[f"rmsnorm{N}"] = dict(x=x, r=r, w=w, y=y, y_res=y2, res_out=ro.clone())
    # bias_rope_store: slow dims and codec dims with a ring (serve/fast_kernels.py:139-187)
    import fast_engine as fe
    for name, nq, nkv, hd, ring, has_b, npos in (("slow", 14, 2, 64, 1 << 30, True, 64),
                                                  ("codec", 8, 8, 128, 128, False, 400)):
        R, rows, L = 5, 4, (64 if ring > 1000 else 128)
        qkv = randn((R, (nq + 2 * nkv) * hd), g, 2.0, BF16)
        bias = randn(((nq + 2 * nkv) * hd,), g, 0.5, BF16) if has_b else None
        cos, sin = fe._rope_tables(1e6 if name == "slow" else 1e4, hd, npos, torch.device("cpu"))
        pos = torch.randint(0, npos, (R,), generator=g, dtype=torch.int32)
        slot = torch.tensor([0, 3, 1, 2, 0][:R], dtype=torch.int32)
        pos[4] = (pos[0] + 7) % npos                         # same slot, another column
        kc = torch.zeros(rows, nkv, L, hd, dtype=BF16)
        vc = torch.zeros_like(kc)
        q = torch.empty(R, nq, hd, dtype=BF16)
        fk.bias_rope_store(qkv, bias, cos, sin, pos, slot, q, kc, vc, nq, nkv, hd, ring=ring)
        out[f"rope_{name}"] = dict(qkv=qkv, bias=bias, cos=cos, sin=sin, pos=pos, slot=slot, q=q, kc=kc, vc=vc,
                                   nq=nq, nkv=nkv, hd=hd, ring=ring)
    # split-K decode attention, GQA 14/2 (serve/fast_kernels.py:193-290)
    nq, nkv, hd, S = 14, 2, 64, 256
    b = 4
    q = randn((b, nq, hd), g, 1.0, BF16)
    kc = randn((b + 1, nkv, S, hd), g, 1.0, BF16)
    vc = randn((b + 1, nkv, S, hd), g, 1.0, BF16)
    lens = torch.tensor([1, 63, 65, 200], dtype=torch.int32)
    rowmap = torch.tensor([4, 0, 2, 1], dtype=torch.int32)
    att = fk.DecodeAttention(64, nq, nkv, hd, 16, torch.device("cpu"))
    res = {}
    for ns in (1, 3):
        o = torch.empty(b, nq, hd, dtype=BF16)
        att(q, kc, vc, lens, o, nsplit=ns)
        res[f"out_ns{ns}"] = o
    o = torch.empty(b, nq, hd, dtype=BF16)
    att(q, kc, vc, lens, o, nsplit=2, rowmap=rowmap)
    res["out_map"] = o
    out["decode_attn"] = dict(q=q, kc=kc, vc=vc, lens=lens, rowmap=rowmap, **res)
    # MHA, hd 128 (the codec transformer's shape)
    q2 = randn((3, 8, 128), g, 1.0, BF16)
    kc2 = randn((3, 8, 128, 128), g, 1.0, BF16)
    vc2 = randn((3, 8, 128, 128), g, 1.0, BF16)
    lens2 = torch.tensor([1, 77, 128], dtype=torch.int32)
    att2 = fk.DecodeAttention(16, 8, 8, 128, 1, torch.device("cpu"))
    o2 = torch.empty(3, 8, 128, dtype=BF16)
    att2(q2, kc2, vc2, lens2, o2, nsplit=1)
    out["decode_attn_mha"] = dict(q=q2, kc=kc2, vc=vc2, lens=lens2, out=o2)
    # packed causal prefill (serve/fast_kernels.py:296-358): two requests, the first after a stored prefix
    ns_, starts, slots_ = [70, 5], [30, 0], [2, 0]
    R = sum(ns_)
    qp = randn((R, nq, hd), g, 1.0, BF16)
    kcp = randn((3, nkv, 128, hd), g, 1.0, BF16)
    vcp = randn((3, nkv, 128, hd), g, 1.0, BF16)
    plan = fk.PrefillPlan([0, 70], ns_, slots_, starts, torch.device("cpu"))
    op = torch.empty(R, nq, hd, dtype=BF16)
    fk.prefill_attention(qp, kcp, vcp, plan, op, nq // nkv)
    blocks = [(int(a), int(n), int(s), int(p)) for a, n, s, p in zip(plan.q0, plan.n, plan.slot, plan.pos0)]
    out["prefill_attn"] = dict(q=qp, kc=kcp, vc=vcp, blocks=blocks, out=op)
    # silu * mul (serve/fast_kernels.py:526-545)
    gu = randn((3, 2 * 4864), g, 3.0, BF16)
    out["silu_mul"] = dict(gu=gu, y=fk.silu_mul(gu))
    # conv_cl / snake_cat (serve/fast_kernels.py:551-729)
    convs = {}
    for name, Cin, Cout, taps, dil, ph, T, ctx, bias, resid, snake_mode in (
            ("k7d3", 96, 96, 7, 3, 1, 16, 18, True, True, "cat"),
            ("trans4", 64, 32, 2, 1, 4, 3, 1, True, False, "cat"),
            ("pw_snake", 192, 192, 1, 1, 1, 9, 0, True, True, "load"),
            ("k7_out", 96, 1, 7, 1, 1, 20, 6, True, False, "cat")):
        b = 2
        x = randn((b, T, Cin), g, 1.0, F16)
        st = randn((b, ctx, Cin), g, 1.0, F16) if ctx else None
        a = (torch.rand(Cin, generator=g) + 0.5).float()
        ib = 1.0 / (a + 1e-9)
        cp = max(16, Cout)
        W = torch.zeros(ph, taps, Cin, cp)
        W[..., :Cout] = randn((ph, taps, Cin, Cout), g, 1.0 / np.sqrt(Cin * taps))
        W = W.to(F16)
        bb = randn((Cout,), g, 0.1, F16) if bias else None
        res = randn((b, T * ph, Cout), g, 1.0, F16) if resid else None
        y = torch.empty(b, T * ph, Cout, dtype=F16)
        if snake_mode == "load":
            fk.conv_cl(x.contiguous(), W, bb, T, taps, dil, ph, y, res=res, snake=(a, ib))
            xin = None
        else:
            xin = torch.empty(b, ctx + T, Cin, dtype=F16)
            fk.snake_cat(x, st, a, ib, xin)
            fk.conv_cl(xin, W, bb, T, taps, dil, ph, y, res=res)
        convs[name] = dict(x=x, st=st, a=a, W=W[..., :Cout].contiguous(), bias=bb, res=res, taps=taps, dil=dil, ph=ph,
                           T=T, ctx=ctx, xin=xin, y=y, snake_mode=snake_mode)
    out["conv"] = convs
    return out


def make_sampler(fe):
    g = gen(200)
    out = {}
    for V, name in ((4097, "sem"), (4096, "cb")):
        logits = randn((4, V), g, 3.0, BF16).float()         # bf16-valued like the engine's head output
        s = fe._Sampler(True, 0.8, 50, 0.95, V)
        v, idx, cum = s.filt(logits)
        E = torch.empty(4, 50).exponential_(generator=g)
        draws = {}
        for p, t in ((0.95, 0.8), (1.0, 1.0), (0.5, 0.3)):
            noise = E.clone()
            orig = torch.Tensor.exponential_
            torch.Tensor.exponential_ = lambda self, *a, **k: self.copy_(noise)
            try:
                draws[f"p{p}_t{t}"] = fe._Sampler.draw(v, idx, cum, p, t)
            finally:
                torch.Tensor.exponential_ = orig
        out[name] = dict(logits=logits, v=v, idx=idx, cum=cum, E=E, draws=draws, k=50, greedy=logits.argmax(-1))
    return out


def make_host(fe):
    out = {}
    NT, NR, BM = 256, 4, 64
    NB = NT // BM + NR
    o = np.cumsum([0, NT, NT, NB, NB, NB, NB, NR, NR, NR])
    ns_obj = SimpleNamespace(pf_off=o, SCR=9, pf_NR=NR)
    cases = [([3, 1, 7], [70, 5, 130], [30, 0, 12]), ([], [], []), ([0], [64], [100]), ([2, 4, 6, 8], [1, 1, 1, 1],
                                                                                          [0, 1, 2, 3])]
    metas = []
    for slots, ns, starts in cases:
        nt = max(64, sum(ns))
        metas.append(dict(slots=slots, ns=ns, starts=starts, nt=nt,
                          meta=torch.from_numpy(fe.FastEngine._pf_meta_host(ns_obj, nt, slots, ns, starts).copy())))
    out["pf_meta"] = dict(NT=NT, NR=NR, BM=BM, SCR=9, cases=metas)
    g = gen(300)
    w = randn((1152, 8), g)
    bvec = randn((1152,), g)
    out["permute"] = dict(w=w, b=bvec, pw=fe._permute_qk(w, 14, 2, 64), pb=fe._permute_qk(bvec, 14, 2, 64))
    c, s = fe._rope_tables(1e6, 64, 2048, torch.device("cpu"))
    c2, s2 = fe._rope_tables(1e4, 128, 300, torch.device("cpu"))
    out["rope"] = dict(cos=c, sin=s, cos_codec=c2, sin_codec=s2)
    return out


def _small_model():
    from oracle.standin import build_standin, tiny_config
    return build_standin(0, tiny_config())


def make_stack(fe, fk, model):
    """_Stack.forward on the tiny stand-in's 2 slow layers: a packed prefill of two requests then decode steps."""
    c = model.config
    with torch.inference_mode():
        st = fe._Stack(model.layers, model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps, c.rope_base,
                       max_rows=256, cache_rows=4, cache_len=256, max_pos=256, dev=torch.device("cpu"),
                       dt=torch.bfloat16)
        g = gen(400)
        ns_, slots_ = [70, 20], [1, 3]
        R = sum(ns_)
        x = randn((R, c.dim), g, 0.1, BF16)
        pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in ns_])
        slot = torch.cat([torch.full((n,), s, dtype=torch.int32) for n, s in zip(ns_, slots_)])
        plan = fk.PrefillPlan([0, 70], ns_, slots_, [0, 0], torch.device("cpu"))
        h_pf = st.forward(x.clone(), pos, slot, None, plan=plan)
        blocks = [(int(a), int(n), int(s), int(p)) for a, n, s, p in zip(plan.q0, plan.n, plan.slot, plan.pos0)]
        xd = randn((4, c.dim), g, 0.1, BF16)
        dpos = torch.tensor([70, 5, 0, 20], dtype=torch.int32)       # row 1 / 3 continue their prefill
        dslot = torch.tensor([1, 2, 0, 3], dtype=torch.int32)
        h_dec = st.forward(xd.clone(), dpos, dslot, dpos + 1, nsplit=2, rowmap=True)
        kc, vc = st.kc_all.clone(), st.vc_all.clone()
    return dict(x=x, pos=pos, slot=slot, blocks=blocks, h_pf=h_pf, xd=xd, dpos=dpos, dslot=dslot, h_dec=h_dec,
                kc=kc, vc=vc)


def make_vocoder(fe, model, frames=2):
    """StreamingVocoder.step on the tiny stand-in's codec (full-size conv decoder): b=2, a few frames."""
    with torch.inference_mode():
        codec = model.load_codec(torch.device("cpu"), torch.float32)
        v = fe.StreamingVocoder(codec, 2, torch.device("cpu"))
        for c, T, _ in v.convs():          # larger interpreter tiles (a tune result the reference could pick)
            c.cfg = (128, 128, 32, 4, 3)
        g = gen(500)
        codes = torch.randint(0, 4096, (frames, 2, 10), generator=g)
        wavs, hs = [], []
        for t in range(frames):
            t0 = time.time()
            wavs.append(v.step(codes[t], 2).clone())
            print(f"  vocoder frame {t}: {time.time() - t0:.0f}s", flush=True)
    return dict(codes=codes, wav=torch.stack(wavs), pos=v.pos.clone())


def make_engine(fe, model, ticks=3):
    """FastEngine (tiny stand-in, greedy) on the CPU: admit two requests, then `ticks` ticks."""
    from oracle.standin import StubTokenizer
    from tts_engine import voice_item
    tok = StubTokenizer()
    gp = dict(do_sample=False, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    model = model.to(torch.bfloat16)         # the serving stack loads the checkpoint in bf16 (serve/tts_engine.py:38)
    with torch.inference_mode():
        eng = fe.FastEngine(model, tok, gp, max_slots=3, max_seq=512, buckets=[1, 2, 3], seq_from_env=False)
        for c, T, _ in eng.voc.convs():
            c.cfg = (128, 128, 32, 4, 3)
        rec = {"logits": [], "prefill_logits": []}
        head = eng._head

        def _head(h):
            lg = head(h)
            (rec["prefill_logits"] if rec.get("_pf") else rec["logits"]).append(lg.clone())
            return lg
        eng._head = _head
        g = gen(600)
        ref_code = torch.randint(0, 4096, (20, 10), generator=g)
        text = " ".join(str(int(t)) for t in torch.randint(0, 151643, (16,), generator=g))
        text2 = " ".join(str(int(t)) for t in torch.randint(0, 151643, (9,), generator=g))
        item = voice_item(ref_code, "12 34 56 78")
        reqs = [dict(text=text, item=item, key="v0"), dict(text=text2, item=item, key="v0")]
        rec["_pf"] = True
        lens = eng.admit([0, 2], reqs)
        rec["_pf"] = False
        state0 = dict(tok=eng.tok.clone(), cpos=eng.cpos.clone(), hid=eng.hid.clone())
        out = dict(tok_in=[], frame_prev=[], audio=[], tok=[], cpos=[], nstep=[], prev=[])
        for t in range(ticks):
            t0 = time.time()
            eng._tick(3)
            print(f"  engine tick {t}: {time.time() - t0:.0f}s", flush=True)
            for k in ("tok_in", "frame_prev", "audio", "tok", "cpos", "nstep", "prev"):
                out[k].append(getattr(eng, k).clone())
    rec.pop("_pf")
    return dict(text=text, text2=text2, ref_code=ref_code, ref_text="12 34 56 78", lens=lens, state0=state0,
                logits=rec["logits"], prefill_logits=rec["prefill_logits"],
                **{k: torch.stack(v) for k, v in out.items()})


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("--") else None
    if ref is None:
        raise SystemExit("usage: make_golden.py /path/to/reference [--only a,b]")
    only = None
    if "--only" in sys.argv:
        only = set(sys.argv[sys.argv.index("--only") + 1].split(","))
    sys.path.insert(0, os.path.join(ref, "serve"))
    _patch_interpreter()
    _patch_cuda()
    import fast_engine as fe
    import fast_kernels as fk
    torch.manual_seed(0)
    todo = ["kernels", "sampler", "host", "stack", "vocoder", "engine"]
    model = None
    for name in todo:
        if only and name not in only:
            continue
        t0 = time.time()
        if name == "kernels":
            d = make_kernels(fk)
        elif name == "sampler":
            d = make_sampler(fe)
        elif name == "host":
            d = make_host(fe)
        else:
            model = model or _small_model()
            if name == "stack":
                d = make_stack(fe, fk, model)
            elif name == "vocoder":
                d = make_vocoder(fe, model)
            else:
                d = make_engine(fe, model)
        torch.save(d, os.path.join(HERE, f"{name}.pt"))
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
