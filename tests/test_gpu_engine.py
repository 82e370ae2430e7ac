"""The FastEngine drop-in on the GPU against the CPU oracle engine, on the tiny stand-in (real widths, 2 slow layers,
1 fast layer): stack forward (packed prefill + decode), admission, and ticks, greedy and sampled.

Ticks are compared teacher-forced (each tick starts from the engine's state): codes, tokens and bookkeeping (cpos,
nstep, RAS window, frame_prev) equal the oracle's, semantic logits within 2e-2; with random weights the logits are
nearly flat and bf16-quantized, so a pick may differ where the oracle's own logits (greedy) or race scores (sampled,
same Philox noise) tie to within 2 bf16 ulps -- each such near-tie is checked and reported.
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


def _ulp(v):
    """bf16 spacing at |v|."""
    v = abs(float(v))
    e = max(-126, int(torch.floor(torch.log2(torch.tensor(max(v, 1e-30))))))
    return 2.0 ** (e - 7)


def _near_tie(logits, j_e, j_o, draw=None):
    """The engine's pick j_e and the oracle's j_o are equivalent up to bf16 rounding of the logits. Greedy: the logits
    are within 2 ulps. Sampled (draw = (k, p, t, E)): j_e would win the oracle's race once the logits move by 2 ulps --
    its race score log p - log E is within 2 ulps / t of the winner's, its logit is within 2 ulps of the winner's (their
    sorted places, and so their noise draws, may swap), or it sits on the top-p boundary (cumulative
    probability within 2e-3 of p) or on the top-k boundary (logit within 2 ulps of the k-th). Returns (ok, detail)."""
    lg = logits.float()
    if draw is None:
        gap = float(lg[j_o] - lg[j_e])
        return gap <= 2 * _ulp(lg[j_o]), dict(gap=gap, ulp=_ulp(lg[j_o]))
    k, p, t, E = draw
    v, idx, cum = R.topk_filter(lg[None], k)
    v, idx, cum = v[0], idx[0], cum[0]
    pos = {int(i): n for n, i in enumerate(idx)}
    tol = 2 * _ulp(v[0]) / t
    keep = ~(cum > p) if p < 1.0 else torch.ones(k, dtype=torch.bool)
    keep[0] = True
    po = pos[j_o]
    sc_o = float(v[po]) / t - float(torch.log(E[po]))
    if j_e in pos:
        pe = pos[j_e]
        sc_e = float(v[pe]) / t - float(torch.log(E[pe]))
        at_p = pe > 0 and abs(float(cum[pe]) - p) <= 2e-3
        # the noise is indexed by sorted position: two candidates whose logits are within 2 ulps may swap places
        a, z = min(pe, po), max(pe, po)
        swapped = float(v[a] - v[z]) <= 2 * _ulp(v[a])
        ok = swapped or (sc_e >= sc_o - tol and (bool(keep[pe]) or at_p))
        return ok, dict(pe=pe, po=po, sc_e=sc_e, sc_o=sc_o, cum_e=float(cum[pe]), keep_e=bool(keep[pe]), tol=tol)
    at_k = float(v[-1] - lg[j_e]) <= 2 * _ulp(v[-1])
    return at_k, dict(po=po, outside_topk=True, l_e=float(lg[j_e]), v_k=float(v[-1]))


def _resync(ora, eng):
    """Oracle state := engine state (bf16 values), so the next tick starts from identical inputs."""
    for name in ("tok", "cpos", "prev", "nstep", "tok_in", "frame_prev"):
        getattr(ora, name).copy_(getattr(eng, name).cpu())
    ora.hid.copy_(eng.hid.float().cpu())
    ora.slow.kc.copy_(eng.slow.kc.float().cpu())
    ora.slow.vc.copy_(eng.slow.vc.float().cpu())


def _kept(logits, j, k=50, p=0.95):
    """j is a candidate of the oracle's top-k / top-p filter, boundaries taken within 2 bf16 ulps / 2e-3."""
    v, idx, cum = R.topk_filter(logits.float()[None], k)
    v, idx, cum = v[0], idx[0], cum[0]
    where = (idx == j).nonzero()
    if len(where) == 0:
        return float(v[-1] - logits[j]) <= 2 * _ulp(v[-1])
    n = int(where[0])
    return n == 0 or float(cum[n]) <= p + 2e-3


def _sem_draw(eng, lg, prev_row, t_in, tick, r):
    """_sample_sem (serve/fast_engine.py:726-735) + sticky EOS (:762) on the engine's own logits and noise."""
    v, idx, cum = R.topk_filter(lg.float()[None], 50)
    tok = lambda j: eng.eos if int(j) == eng.nsem else int(j) + eng.sb
    nrm = tok(R.draw(v, idx, cum, 0.95, 0.8, R.philox_exp(eng.seed, 16, tick, [r], 50))[0])
    high = tok(R.draw(v, idx, cum, eng.ras_p, eng.ras_t, R.philox_exp(eng.seed, 17, tick, [r], 50))[0])
    rep = bool((prev_row == nrm).any()) and nrm != eng.eos
    return t_in if t_in == eng.eos else (high if rep else nrm)


@pytest.mark.parametrize("do_sample", [False, True])
def test_engine_ticks_match_oracle(a8, dev, tiny_model, do_sample):
    """Teacher-forced parity: every tick starts from the engine's state. Greedy: all codes and tokens equal the
    oracle's up to the first difference in a row, and every difference is a bf16 near-tie of the oracle's own logits.
    Sampled: every code is a candidate of the oracle's filter, most draws are identical, and each semantic token is
    exactly the draw (with RAS and sticky EOS) of the engine's own logits under the shared Philox noise."""
    gp = dict(do_sample=do_sample, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, buckets=[1, 2, 3],
                        seq_from_env=False, seed=77)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, seed=77, with_voc=False)
    reqs = _requests()
    assert eng.admit([0, 2], reqs) == ora.admit([0, 2], reqs)
    torch.cuda.synchronize()
    assert torch.equal(eng.cpos.cpu(), ora.cpos) and rel(eng.hid, ora.hid) < 2e-2
    ties, b, exact_rows, same_draws, draws = [], 3, 0, 0, 0
    for t in range(8):
        _resync(ora, eng)
        ora.record = {}
        t_in = eng.tok[:b].cpu().clone()
        eng.tick(b)
        codes_o = ora.tick(b)
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        codes_e = eng.codes[:b].cpu()
        for r in range(b):
            if do_sample:
                k0 = next((k for k in range(1, 10) if codes_e[r, k] != codes_o[r, k]), 10)
                for k in range(1, k0 + 1 if k0 < 10 else 10):
                    assert _kept(ora.record["fast_logits"][k - 1][r], int(codes_e[r, k])), (t, r, k)
                draws += 9
                same_draws += k0 - 1
                got = int(eng.tok[r])
                want = _sem_draw(eng, eng.logits[r, :eng.nh].cpu(), eng.prev[r].cpu(), int(t_in[r]), t, r)
                assert got == want, (t, r, got, want)
                assert torch.equal(eng.frame_prev[r].cpu(), codes_e[r] if int(t_in[r]) != eng.eos
                                   else eng.sil_frame.cpu())
                if k0 == 10:
                    assert rel(eng.logits[r, :eng.nh], ora.record["logits"][-1][r]) < 2e-2, (t, r)
                    exact_rows += 1
                continue
            diff = (codes_e[r] != codes_o[r]).nonzero()
            if len(diff):
                k = int(diff[0])                         # first codebook that differs (k >= 1)
                ok, why = _near_tie(ora.record["fast_logits"][k - 1][r], int(codes_e[r, k]), int(codes_o[r, k]))
                assert ok, (t, r, k, int(codes_e[r, k]), int(codes_o[r, k]), why)
                ties.append((t, r, "cb", k))
                continue
            assert rel(eng.logits[r, :eng.nh], ora.record["logits"][-1][r]) < 2e-2, (t, r)
            te, to = int(eng.tok[r]), int(ora.tok[r])
            if te != to:
                j = lambda tok: eng.nsem if tok == eng.eos else tok - eng.sb
                assert _near_tie(ora.record["logits"][-1][r], j(te), j(to))[0], (t, r, te, to)
                ties.append((t, r, "sem", 0))
            else:
                exact_rows += 1
            assert int(eng.cpos[r]) == int(ora.cpos[r]) and int(eng.nstep[r]) == int(ora.nstep[r])
            assert torch.equal(eng.frame_prev[r].cpu(), ora.frame_prev[r])
            assert torch.equal(eng.prev[r].cpu(), ora.prev[r])
    if do_sample:
        assert same_draws >= 0.5 * draws, (same_draws, draws)
        print(f"identical codebook draws {same_draws}/{draws}, rows fully identical {exact_rows}/{8 * b}")
    else:
        assert exact_rows >= 12, (exact_rows, ties)
        print(f"near-ties (tick, row, where, codebook): {ties}")


def test_engine_graph_replay_equals_eager(a8, dev, tiny_model):
    """A captured tick graph (codec on its side stream included) replays exactly what the eager launches compute."""
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=4, max_seq=512, buckets=[2, 4],
                        seq_from_env=False, seed=5)
    eng.capture(log=lambda *a: None)
    reqs = _requests(1)
    eng.admit([0, 1], reqs)
    state = [eng.tok, eng.hid, eng.cpos, eng.prev, eng.nstep, eng.tick_ctr, eng.frame_prev, eng.slow.kc,
             eng.slow.vc] + [s[0] for s in eng.voc._states()]
    snap = [t.clone() for t in state]
    outs = []
    for _ in range(3):
        eng.replay(2)
        outs.append((eng.tok_in[:2].clone(), eng.frame_prev[:2].clone(), eng.tok[:2].clone(), eng.audio[:2].clone()))
    for t, s in zip(state, snap):
        t.copy_(s)
    for i in range(3):
        eng.tick(2)
        assert torch.equal(eng.tok_in[:2], outs[i][0]) and torch.equal(eng.frame_prev[:2], outs[i][1])
        assert torch.equal(eng.tok[:2], outs[i][2]) and torch.equal(eng.audio[:2], outs[i][3])
    assert a8.device_error()[0] == 0


def test_engine_tick_audio_is_codec_of_previous_frame(a8, dev, tiny_model):
    """Each tick's audio is the codec step of the frame the previous tick chose (frame_prev as the tick starts):
    bit-identical to a standalone StreamingVocoder fed those frames -- the side stream reads frame_prev before the
    tick's draw rewrites it. A fresh row's first frame is the silence frame."""
    from audio8_b200.codec import StreamingVocoder
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, buckets=[3],
                        seq_from_env=False, seed=9)
    voc = StreamingVocoder(tiny_model.load_codec(device="cpu"), 3, dev)
    reqs = _requests(2)
    reqs.append(dict(reqs[0], text="11 22 33 44"))
    eng.admit([0, 1, 2], reqs)
    assert torch.equal(eng.frame_prev[:3].cpu(), eng.sil_frame.cpu().expand(3, -1))
    for t in range(4):
        fp = eng.frame_prev[:3].clone()
        eng.tick(3)
        want = voc.step(fp, 3)
        torch.cuda.synchronize()
        assert torch.equal(eng.audio[:3], want), t
    assert a8.device_error()[0] == 0


def test_admission_graph_equals_eager_and_launches_only_library_kernels(a8, dev, tiny_model):
    """An admission chunk is one metadata copy and one replay of the prefill graph of its token bucket: the state it
    leaves (first tokens, hidden, positions, K/V, first codec frames) is bit-identical to the same launches made
    eagerly, and every kernel it runs is this library's (the prompt embedding, the prefix K/V copy and the codec
    state included: no PyTorch kernel)."""
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95)
    mk = lambda: a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=4, max_seq=512, buckets=[4],
                               seq_from_env=False, seed=21)
    eager, graphed = mk(), mk()
    graphed.capture(log=lambda *a: None)
    assert sorted(graphed.pf_graphs) == graphed.pf_buckets
    reqs = _requests(4) + [dict(_requests(5)[0], key="v1")]
    for eng in (eager, graphed):                 # a first admission caches the voices' prefix K/V
        eng.admit([0, 1, 2], reqs)
    torch.cuda.synchronize()
    names = None
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            graphed.admit([3, 1], [reqs[1], reqs[2]])
            torch.cuda.synchronize()
        names = {e.name for e in prof.events() if str(e.device_type).endswith("CUDA")}
    except Exception as exc:                      # no CUPTI on this box: the equality checks below still run
        print("profiler unavailable:", exc)
    eager.admit([3, 1], [reqs[1], reqs[2]])
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    for name in ("tok", "hid", "cpos", "prev", "nstep", "frame_prev"):
        assert torch.equal(getattr(eager, name), getattr(graphed, name)), name
    for s in (0, 1, 2, 3):                        # what admission wrote: each slot's first cpos positions
        n = int(eager.cpos[s])
        assert torch.equal(eager.slow.kc[:, s, :, :n], graphed.slow.kc[:, s, :, :n]), s
        assert torch.equal(eager.slow.vc[:, s, :, :n], graphed.slow.vc[:, s, :, :n]), s
    if names:
        kernels = {n for n in names if not n.lower().startswith("memcpy") and not n.lower().startswith("memset")}
        print("admission kernels:", sorted(kernels))
        assert kernels and all(n.startswith("a8::") or "a8::" in n for n in kernels), sorted(kernels)
