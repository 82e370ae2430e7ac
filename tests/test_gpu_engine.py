"""The FastEngine drop-in on the GPU against the CPU oracle engine, on the tiny stand-in (real widths, 2 slow layers,
1 fast layer): stack forward (packed prefill + decode), admission, and ticks, greedy and sampled.

Greedy: identical tokens, codes and bookkeeping (tok_in, frame_prev, cpos, nstep, prev) for every tick, semantic
logits within 2e-2 of the oracle's. Sampled: identical draws (same Philox noise) while the logits agree.
"""
import ctypes as C
from types import SimpleNamespace

import pytest
import torch

from oracle import ref_cpu as R
from oracle.standin import StubTokenizer

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.fixture(scope="module")
def dev(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return torch.device("cuda", 0)


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp(min=1e-6))


def test_stack_prefill_then_decode(a8, dev, tiny_model):
    from audio8_b200.engine import PackedStack, Scratch
    L = a8._lib
    c = tiny_model.config
    st = PackedStack(tiny_model.layers, tiny_model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps,
                     c.rope_base, cache_rows=4, cache_len=256, max_pos=256, dev=dev)
    sc = Scratch(256, c.dim, c.n_head * c.head_dim, c.intermediate_size, c.n_local_heads, c.head_dim, 256, dev)
    ost = R.Stack(tiny_model.layers, tiny_model.norm, c.n_head, c.n_local_heads, c.head_dim, c.norm_eps, c.rope_base,
                  cache_rows=4, cache_len=256, max_pos=256)
    g = torch.Generator().manual_seed(1)
    ns, slots = [70, 20, 133], [1, 3, 0]
    x = (torch.randn(sum(ns), c.dim, generator=g) * 0.1).to(BF)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in ns])
    slot = torch.cat([torch.full((n,), s, dtype=torch.int32) for n, s in zip(ns, slots)])
    X, P, S = x.to(dev), pos.to(dev), slot.to(dev)
    run = L.A8StackRun(x=L.ptr(X), ldx=c.dim, rows=X.shape[0], pos=L.ptr(P), slot=L.ptr(S), lens=None, lens_max=0,
                       rowmap=L.ptr(S), max_len=int(pos.max()) + 1, scratch=sc.desc)
    L.call("a8_stack_forward", C.byref(st.desc), C.byref(run), L.stream_handle())
    torch.cuda.synchronize()
    blocks, r0 = [], 0
    for n, s in zip(ns, slots):
        blocks += [(r0 + a, min(64, n - a), s, a) for a in range(0, n, 64)]
        r0 += n
    h_o = ost.forward(x.float(), pos, slot, blocks=blocks)
    assert rel(sc.h[:X.shape[0]], h_o) < 2e-2
    assert rel(st.kc, ost.kc) < 2e-2 and rel(st.vc, ost.vc) < 2e-2
    # decode: rows continue their prefills (rowmap), plus a fresh row in slot 2
    xd = (torch.randn(4, c.dim, generator=g) * 0.1).to(BF)
    dpos = torch.tensor([70, 20, 133, 0], dtype=torch.int32)
    dslot = torch.tensor([1, 3, 0, 2], dtype=torch.int32)
    XD, DP, DS = xd.to(dev), dpos.to(dev), dslot.to(dev)
    run = L.A8StackRun(x=L.ptr(XD), ldx=c.dim, rows=4, pos=L.ptr(DP), slot=L.ptr(DS), lens=None, lens_max=0,
                       rowmap=L.ptr(DS), max_len=256, scratch=sc.desc)
    L.call("a8_stack_forward", C.byref(st.desc), C.byref(run), L.stream_handle())
    torch.cuda.synchronize()
    hd_o = ost.forward(xd.float(), dpos, dslot, dpos + 1, rowmap=True)
    assert rel(sc.h[:4], hd_o) < 2e-2
    assert a8.device_error()[0] == 0


def _requests(seed=0):
    g = torch.Generator().manual_seed(seed)
    ref_code = torch.randint(0, 4096, (20, 10), generator=g)
    item = SimpleNamespace(ref_code=ref_code, ref_text="12 34 56 78")
    t1 = " ".join(str(int(t)) for t in torch.randint(0, 151643, (16,), generator=g))
    t2 = " ".join(str(int(t)) for t in torch.randint(0, 151643, (9,), generator=g))
    return [dict(text=t1, item=item, key="v0"), dict(text=t2, item=item, key="v0")]


@pytest.mark.parametrize("do_sample", [False, True])
def test_engine_ticks_match_oracle(a8, dev, tiny_model, do_sample):
    gp = dict(do_sample=do_sample, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, buckets=[1, 2, 3],
                        seq_from_env=False, seed=77)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, seed=77, with_voc=False)
    ora.record = {}
    reqs = _requests()
    assert eng.admit([0, 2], reqs) == ora.admit([0, 2], reqs)
    torch.cuda.synchronize()
    assert torch.equal(eng.tok.cpu(), ora.tok) and torch.equal(eng.cpos.cpu(), ora.cpos)
    assert rel(eng.hid, ora.hid) < 2e-2
    agree = 0
    for t in range(6):
        eng.tick(3)
        ora.tick(3)
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        lg = eng.logits[:3, :eng.nh]
        assert rel(lg, ora.record["logits"][-1]) < 2e-2, t
        same = torch.equal(eng.tok_in.cpu(), ora.tok_in) and torch.equal(eng.frame_prev.cpu(), ora.frame_prev)
        if not same:
            break
        assert torch.equal(eng.cpos.cpu(), ora.cpos) and torch.equal(eng.nstep.cpu(), ora.nstep)
        assert torch.equal(eng.prev.cpu(), ora.prev) and torch.equal(eng.tok.cpu(), ora.tok)
        agree += 1
    assert agree == 6, f"streams diverged at tick {agree}"


def test_engine_graph_replay_equals_eager(a8, dev, tiny_model):
    """A captured tick graph replays exactly what the eager launches compute."""
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=4, max_seq=512, buckets=[2, 4],
                        seq_from_env=False, seed=5)
    eng.capture(log=lambda *a: None)
    reqs = _requests(1)
    eng.admit([0, 1], reqs)
    snap = [t.clone() for t in (eng.tok, eng.hid, eng.cpos, eng.prev, eng.nstep, eng.tick_ctr, eng.frame_prev,
                                 eng.slow.kc, eng.slow.vc)]
    outs = []
    for _ in range(3):
        eng.replay(2)
        outs.append((eng.tok_in[:2].clone(), eng.frame_prev[:2].clone(), eng.tok[:2].clone()))
    for t, s in zip((eng.tok, eng.hid, eng.cpos, eng.prev, eng.nstep, eng.tick_ctr, eng.frame_prev, eng.slow.kc,
                     eng.slow.vc), snap):
        t.copy_(s)
    for i in range(3):
        eng.tick(2)
        assert torch.equal(eng.tok_in[:2], outs[i][0]) and torch.equal(eng.frame_prev[:2], outs[i][1])
        assert torch.equal(eng.tok[:2], outs[i][2])
    assert a8.device_error()[0] == 0
