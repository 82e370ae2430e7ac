"""The continuous-batching loop's scheduling logic on the CPU, over a fake engine that follows FastEngine's slot
semantics (serve/engine_worker.py:1105-1250): lowest free slots, the bucket covering the highest busy slot, the
first tick of a row dropped (its audio is the silence frame), EOS or the frame cap ending a row, slots reused."""
import importlib

import numpy as np
import pytest
import torch

from conftest import REPO  # noqa: F401


@pytest.fixture(scope="module")
def serving(a8):
    return importlib.import_module(a8.__name__ + ".serving")


class FakeEngine:
    """B slots; a row consumes EOS on its `eos_at`-th tick after admission (never if 0); audio = tick count."""

    def __init__(self, B=8, buckets=(1, 2, 4, 8), eos=99):
        self.B, self.eos, self.up, self.sr = B, eos, 4, 4 * 100        # 10 ms frames
        self.buckets = sorted(buckets)
        self.tok_in = torch.zeros(B, dtype=torch.int64)
        self.audio = torch.zeros(B, self.up)
        self.n = [0] * B
        self.eos_at = [0] * B
        self.replays, self.admitted = [], []

    def bucket_for(self, n):
        return next((b for b in self.buckets if b >= n), self.buckets[-1])

    def admit(self, slots, reqs):
        out = []
        for s, r in zip(slots, reqs):
            if r["text"] == "too long":
                out.append(-1)
                continue
            self.n[s], self.eos_at[s] = 0, int(r["item"])
            out.append(10)
        self.admitted.append(list(slots))
        return out

    def replay(self, b):
        self.replays.append(b)
        for s in range(b):
            self.n[s] += 1
            self.tok_in[s] = self.eos if self.n[s] == self.eos_at[s] else 7
            self.audio[s].fill_(self.n[s])


class FakeClock:
    """Wall clock advanced by the loop itself: 1 ms per poll, plus what `sleep` asks for."""

    def __init__(self):
        self.t = 0.0

    def __call__(self):
        self.t += 1e-3
        return self.t

    def sleep(self, d):
        self.t += d


def _req(serving, rid, arrival, cap, eos_at=0, text=None):
    return serving.Request(rid=rid, arrival=arrival, text=text or f"r{rid}", item=eos_at, key="v", cap=cap)


def test_frames_caps_and_eos(serving):
    fe = FakeEngine()
    reqs = [_req(serving, 0, 0.0, cap=5), _req(serving, 1, 0.0, cap=50, eos_at=8), _req(serving, 2, 0.0, cap=3)]
    clk = FakeClock()
    st = serving.ContinuousBatcher(fe, admit_every=1).run(reqs, clock=clk, sleep=clk.sleep)
    assert [r.frames for r in reqs] == [5, 7, 3]        # EOS consumed on tick 8: frames of ticks 2..8
    assert [r.eos for r in reqs] == [False, True, False]
    assert all(r.t_first is not None and r.t_done >= r.t_first >= r.arrival for r in reqs)
    assert [r.slot for r in reqs] == [0, 1, 2]
    assert fe.admitted == [[0, 1, 2]]                     # one packed admission
    assert st.summary()["finished"] == 3
    # the bucket always covers the highest busy slot; busy rows shrink as requests end
    assert max(fe.replays) == 4 and fe.replays[-1] == 2


def test_audio_first_tick_dropped(serving):
    fe = FakeEngine()
    got = []
    b = serving.ContinuousBatcher(fe)
    b.on_audio = lambda r, a: got.append(float(a[0]))
    clk = FakeClock()
    b.run([_req(serving, 0, 0.0, cap=4)], clock=clk, sleep=clk.sleep)
    assert got == [2.0, 3.0, 4.0, 5.0]                    # tick 1 (the silence frame) is not delivered


def test_slots_reused_lowest_first(serving):
    fe = FakeEngine(B=2, buckets=(1, 2))
    reqs = [_req(serving, i, 0.0, cap=c) for i, c in enumerate((3, 9, 4, 2))]
    clk = FakeClock()
    serving.ContinuousBatcher(fe, admit_every=1).run(reqs, clock=clk, sleep=clk.sleep)
    assert all(r.t_done is not None for r in reqs)
    assert [r.slot for r in reqs] == [0, 1, 0, 0]         # slot 0 frees first and is taken by each next request
    assert [r.frames for r in reqs] == [3, 9, 4, 2]
    # a request never starts before the one it replaces in its slot has ended
    assert reqs[2].t_admit >= reqs[0].t_done and reqs[3].t_admit >= reqs[2].t_done


def test_rejected_prompt_frees_slot(serving):
    fe = FakeEngine(B=2, buckets=(2,))
    reqs = [_req(serving, 0, 0.0, cap=3, text="too long"), _req(serving, 1, 0.0, cap=3)]
    clk = FakeClock()
    st = serving.ContinuousBatcher(fe).run(reqs, clock=clk, sleep=clk.sleep)
    assert reqs[0].rejected and reqs[0].t_done is None
    assert reqs[1].slot == 1 and reqs[1].frames == 3
    assert st.summary()["rejected"] == 1


def test_arrivals_wait_and_admission_cadence(serving):
    fe = FakeEngine(B=8)
    reqs = [_req(serving, 0, 0.0, cap=40)] + [_req(serving, i, 0.005 + 1e-4 * i, cap=5) for i in range(1, 4)]
    clk = FakeClock()
    serving.ContinuousBatcher(fe, admit_every=4, admit_batch=32).run(reqs, clock=clk, sleep=clk.sleep)
    assert fe.admitted[0] == [0]
    # later arrivals join running ticks only every admit_every ticks, batched into one admission
    assert len(fe.admitted) <= 3 and sorted(s for a in fe.admitted[1:] for s in a) == [1, 2, 3]
    assert all(r.t_first - r.arrival < 0.05 for r in reqs)


def test_idle_gap_sleeps_until_arrival(serving):
    fe = FakeEngine()
    reqs = [_req(serving, 0, 0.0, cap=2), _req(serving, 1, 5.0, cap=2)]
    clk = FakeClock()
    st = serving.ContinuousBatcher(fe).run(reqs, clock=clk, sleep=clk.sleep)
    assert reqs[1].t_admit >= 5.0 and st.wall >= 5.0
    assert st.ticks == 8      # 4 ticks each: silence frame, 2 frames, and one launched before the end is read


def test_closed_loop_users(serving):
    fe = FakeEngine(B=4, buckets=(4,))
    cl = serving.ClosedLoop(streams=3, seconds=0.5, seed=0, ncb=10, n_voices=2, voice_frames=4, ramp=0.01,
                            mean_frames=10.0, cap=20)
    for r in cl.initial:
        r.item = 0                                        # the fake's EOS knob: never
    orig = cl.follow

    def follow(r, t):
        n = orig(r, t)
        if n is not None:
            n.item = 0
        return n
    clk = FakeClock()
    st = serving.ContinuousBatcher(fe, admit_every=1).run(cl.initial, follow=follow, clock=clk, sleep=clk.sleep)
    users = {}
    for r in st.requests:
        users.setdefault(r.user, []).append(r)
    assert sorted(users) == [0, 1, 2]
    for rs in users.values():
        for a, b in zip(rs, rs[1:]):
            assert b.arrival == pytest.approx(a.t_done)   # the next utterance is asked for when one ends
        assert rs[-1].arrival < 0.5
    assert all(r.t_done is not None for r in st.requests)
    s = st.summary()
    assert 0 < s["mean_streams"] <= 3.0


def test_poisson_trace_shape(serving):
    reqs, voices = serving.poisson_trace(40.0, 60.0, seed=0, ncb=10)
    assert len(voices) == 8 and all(v.ref_code.shape == (150, 10) for _, v in voices)
    n = len(reqs)
    assert 2100 < n < 2700                                # 40 req/s x 60 s
    gaps = np.diff([r.arrival for r in reqs])
    assert abs(gaps.mean() - 1 / 40) < 0.003
    caps = np.array([r.cap for r in reqs])
    assert caps.max() <= 1024 and caps.min() >= 1 and 270 < caps.mean() < 330
    nt = np.array([len(r.text.split()) for r in reqs])
    assert nt.min() >= 20 and nt.max() <= 200
    assert {r.key for r in reqs} <= {k for k, _ in voices}
    again, _ = serving.poisson_trace(40.0, 60.0, seed=0, ncb=10)
    assert [(r.arrival, r.cap, r.text) for r in again] == [(r.arrival, r.cap, r.text) for r in reqs]


def test_least_loaded_assignment(serving):
    reqs, _ = serving.poisson_trace(320.0, 5.0, seed=3, ncb=10)
    k = serving.assign_least_loaded(reqs, 8)
    assert len(k) == len(reqs) and set(k) == set(range(8))
    # each request went to a replica with the fewest (estimated) streams in flight at its arrival
    ends = [[] for _ in range(8)]
    for r, kk in zip(reqs, k):
        live = [sum(e > r.arrival for e in h) for h in ends]
        assert live[kk] == min(live)
        ends[kk].append(r.arrival + r.cap * serving.FRAME_S * 0.5)
    frames = np.bincount(k, weights=[r.cap for r in reqs], minlength=8)
    assert frames.max() - frames.min() <= 0.2 * frames.mean()
    # first arrivals fan out over the replicas in index order
    first = sorted(range(len(reqs)), key=lambda i: reqs[i].arrival)[:8]
    assert [k[i] for i in first] == list(range(8))
    assert serving.assign_least_loaded(reqs, 8) == k      # deterministic: every rank computes the same split


def _assign_worker(rank, world, port, out):
    import torch.distributed as dist
    import importlib as il
    from __graft_entry__ import load_package
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    serving = il.import_module(load_package().__name__ + ".serving")
    reqs, _ = serving.poisson_trace(80.0, 3.0, seed=5, ncb=10)
    k = serving.assign_least_loaded(reqs, world)
    mine = [r.rid for r, kk in zip(reqs, k) if kk == rank]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        out.put((gathered, [r.rid for r in reqs]))
    dist.destroy_process_group()


def test_replica_split_two_ranks():
    """Two gloo ranks each take their share of one global trace: disjoint, and together the whole trace."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    ps = [ctx.Process(target=_assign_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(120)
    assert all(p.exitcode == 0 for p in ps)
    gathered, rids = q.get()
    assert not set(gathered[0]) & set(gathered[1])
    assert sorted(gathered[0] + gathered[1]) == sorted(rids)
    assert abs(len(gathered[0]) - len(gathered[1])) <= 0.1 * len(rids)


def test_chunks_ramp_and_final(serving):
    """Chunks of 1, 2, 4, 6, 6, ... frames, the rest at the end (the worker's ramp), concatenating to every frame."""
    fe = FakeEngine()
    got = []
    b = serving.ContinuousBatcher(fe, first_chunk=1, chunk_frames=6)
    b.on_chunk = lambda r, y, final: got.append((len(y) // fe.up, final, y[::fe.up].tolist()))
    clk = FakeClock()
    b.run([_req(serving, 0, 0.0, cap=21)], clock=clk, sleep=clk.sleep)
    assert [n for n, _, _ in got] == [1, 2, 4, 6, 6, 2]
    assert [f for _, f, _ in got] == [False] * 5 + [True]
    assert [v for _, _, vs in got for v in vs] == [float(i) for i in range(2, 23)]   # ticks 2..22, in order


def test_pcm16(serving):
    y = np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 3.0], dtype=np.float32)
    out = np.frombuffer(serving.pcm16(y), dtype="<i2")
    assert out.tolist() == [-32767, -32767, -16383, 0, 16383, 32767, 32767]


class FakeResampler:
    """The device resampler's per-slot contract on the CPU: the first frame of a stream dropped, 2 samples a frame
    (value = the frame's audio), 3 more (-1) when the frame is the stream's last (EOS consumed or cap reached)."""

    out_max = 8

    def __init__(self, B):
        self.skip, self.left, self.done = [False] * B, [0] * B, [True] * B
        self.pcm = torch.zeros(B, self.out_max, dtype=torch.int16)
        self.cnt = torch.zeros(B, dtype=torch.int32)
        self.resets = []

    def reset(self, slots, caps):
        self.resets.append(list(slots))
        for s, c in zip(slots, caps):
            self.skip[s], self.left[s], self.done[s] = True, c, False

    def step(self, audio, tok_in, eos, b):
        self.cnt.zero_()
        for r in range(b):
            end = int(tok_in[r]) == eos
            if self.done[r]:
                continue
            if self.skip[r]:
                self.skip[r], self.done[r] = False, end
                continue
            self.left[r] -= 1
            last = end or self.left[r] <= 0
            n = 5 if last else 2
            self.pcm[r, :2] = int(audio[r, 0])
            self.pcm[r, 2:5] = -1
            self.cnt[r] = n
            self.done[r] = last
        return self.pcm[:b], self.cnt[:b]


def test_resampled_chunks(serving):
    """With a resampler the loop resets a slot's stream on admission, steps it every tick and delivers int16 chunks
    whose samples are exactly the resampler's rows: the silence frame gives none, the last frame carries the tail."""
    fe = FakeEngine()
    rs = FakeResampler(fe.B)
    got = {}
    b = serving.ContinuousBatcher(fe, resampler=rs, copy_audio=False, first_chunk=1, chunk_frames=2)
    b.on_chunk = lambda r, y, final: got.setdefault(r.rid, []).append((y.dtype, y.tolist(), final))
    clk = FakeClock()
    reqs = [_req(serving, 0, 0.0, cap=4), _req(serving, 1, 0.0, cap=9, eos_at=3), _req(serving, 2, 0.0, cap=5, eos_at=1)]
    b.run(reqs, clock=clk, sleep=clk.sleep)
    assert rs.resets == [[0, 1, 2]]
    assert all(d == np.int16 for c in got.values() for d, _, _ in c)
    flat = lambda rid: [v for _, vs, _ in got[rid] for v in vs]
    assert flat(0) == [2, 2, 3, 3, 4, 4, 5, 5, -1, -1, -1]            # ticks 2-5, the tail on the capped frame
    assert [f for _, _, f in got[0]] == [False, False, True]           # chunks of 1, 2, then the rest
    assert flat(1) == [2, 2, 3, 3, -1, -1, -1]                         # EOS consumed on tick 3
    assert got[2] == [(np.int16, [], True)]                            # EOS on the silence tick: an empty final chunk


def test_cancel_running_and_waiting(serving):
    """A client that goes away (the worker's ("__cancel__", rid)): a running request ends with an empty final chunk and
    frees its slot for the next request; a waiting one is never admitted; ids that are unknown or already ended are
    ignored; cancelled requests are counted apart from the finished ones."""
    fe = FakeEngine(B=1, buckets=(1,))
    reqs = [_req(serving, 0, 0.0, cap=50), _req(serving, 1, 0.0, cap=3), _req(serving, 2, 0.0, cap=4)]
    loop = serving.ContinuousBatcher(fe, admit_every=1)
    got = {}

    def on_chunk(r, y, final):
        got.setdefault(r.rid, []).append((len(y), final))
        if r.rid == 0 and r.frames >= 5 and not got.get("sent"):
            got["sent"] = True
            loop.cancel(0)          # running: ends at the next iteration
            loop.cancel(2)          # waiting behind it: dropped
            loop.cancel(99)         # unknown: ignored
    loop.on_chunk = on_chunk
    clk = FakeClock()
    st = loop.run(reqs, clock=clk, sleep=clk.sleep)
    r0, r1, r2 = reqs
    assert r0.cancelled and 5 <= r0.frames < 50 and got[0][-1] == (0, True)
    assert r2.cancelled and r2.slot == -1 and r2.frames == 0 and got[2] == [(0, True)]
    assert not r1.cancelled and r1.frames == 3 and r1.slot == 0 and r1.t_admit >= r0.t_done
    s = st.summary()
    assert s["cancelled"] == 2 and s["finished"] == 1
    loop.cancel(1)                  # already ended: nothing happens on a later run
    loop.run([], clock=clk, sleep=clk.sleep)
    assert not r1.cancelled


def test_cancel_last_pending_ends_run(serving):
    """Cancelling the only request not yet arrived ends the run instead of waiting for it."""
    fe = FakeEngine()
    loop = serving.ContinuousBatcher(fe)
    reqs = [_req(serving, 0, 0.0, cap=2), _req(serving, 1, 100.0, cap=2)]
    loop.on_audio = lambda r, a: loop.cancel(1)
    clk = FakeClock()
    st = loop.run(reqs, clock=clk, sleep=clk.sleep)
    assert reqs[1].cancelled and reqs[1].t_admit is None and st.wall < 100.0


class FlakyEngine(FakeEngine):
    """Raises on the admissions / ticks whose (1-based) call numbers are listed."""

    def __init__(self, bad_admits=(), bad_ticks=(), **kw):
        super().__init__(**kw)
        self.bad_admits, self.bad_ticks, self.n_admit, self.n_tick = set(bad_admits), set(bad_ticks), 0, 0

    def admit(self, slots, reqs):
        self.n_admit += 1
        if self.n_admit in self.bad_admits:
            raise RuntimeError("admit failed")
        return super().admit(slots, reqs)

    def replay(self, b):
        self.n_tick += 1
        if self.n_tick in self.bad_ticks:
            raise RuntimeError("tick failed")
        super().replay(b)


def _run_flaky(serving, fe, reqs, **kw):
    loop = serving.ContinuousBatcher(fe, **kw)
    errs, finals = {}, {}
    loop.on_error = lambda r, m: errs.setdefault(r.rid, []).append(m)
    loop.on_chunk = lambda r, y, final: finals.__setitem__(r.rid, finals.get(r.rid, 0) + int(final))
    clk = FakeClock()
    return loop.run(reqs, clock=clk, sleep=clk.sleep), errs, finals


def test_admit_failure_frees_slots_and_continues(serving):
    """A failed admission (engine_worker.py:828-832): each of its requests gets "engine error" and its end of stream,
    its slots are free again, and later requests are served."""
    fe = FlakyEngine(bad_admits=(1,), B=2, buckets=(1, 2))
    reqs = [_req(serving, 0, 0.0, cap=3), _req(serving, 1, 0.0, cap=3), _req(serving, 2, 0.5, cap=4)]
    st, errs, finals = _run_flaky(serving, fe, reqs, admit_every=1)
    assert errs == {0: ["engine error"], 1: ["engine error"]} and finals[0] == finals[1] == 1
    assert reqs[0].slot == -1 and reqs[2].frames == 4 and reqs[2].slot == 0 and reqs[2].error is None
    s = st.summary()
    assert s["failed"] == 2 and s["finished"] == 1


def test_tick_failure_ends_running_rows(serving):
    """A failed tick (engine_worker.py:1186-1190) ends every running row with "engine error"; reads in flight are
    dropped; the loop goes on with the requests that arrive later."""
    fe = FlakyEngine(bad_ticks=(3,), B=4, buckets=(4,))
    reqs = [_req(serving, 0, 0.0, cap=9), _req(serving, 1, 0.0, cap=9), _req(serving, 2, 1.0, cap=3)]
    st, errs, finals = _run_flaky(serving, fe, reqs, admit_every=1)
    assert errs == {0: ["engine error"], 1: ["engine error"]} and finals[0] == finals[1] == 1
    assert reqs[0].frames <= 2 and reqs[0].t_done is not None
    assert reqs[2].error is None and reqs[2].frames == 3
    assert st.summary()["failed"] == 2


def test_too_long_prompt_reports_error(serving):
    fe = FakeEngine(B=2, buckets=(2,))
    reqs = [_req(serving, 0, 0.0, cap=3, text="too long"), _req(serving, 1, 0.0, cap=3)]
    st, errs, finals = _run_flaky(serving, fe, reqs)
    assert errs == {0: ["text too long for TTS_MAX_SEQ"]} and finals[0] == 1 and reqs[0].rejected
    assert st.summary()["failed"] == 0 and st.summary()["rejected"] == 1


# ------------------------------------------------------------------------------------------------ code-switch chains
class ChainEngine:
    """FastEngine's slot semantics for chains: a row admitted with text T plays the next script queued for T (a list
    of loud / silent frames, then EOS); tick m after admission generates frame m-1 (frame_prev = [admission id, frame
    index, 0]) and delivers frame m-2's audio (0.5 loud, 0 silent; tick 1 the silence frame). `too_long`: texts whose
    prompt does not fit with a context."""

    def __init__(self, scripts, B=4, eos=99, too_long=()):
        self.B, self.eos, self.up, self.sr = B, eos, 400, 4000          # 0.1 s frames
        self.scripts = {k: list(v) for k, v in scripts.items()}
        self.too_long = set(too_long)
        self.tok_in = torch.zeros(B, dtype=torch.int64)
        self.audio = torch.zeros(B, self.up)
        self.frame_prev = torch.zeros(B, 3, dtype=torch.int64)
        self.row = [None] * B                                             # (admission id, script, tick)
        self.admissions = []                                              # (slot, admission dict, id)

    def bucket_for(self, n):
        return self.B

    def admit(self, slots, reqs):
        out = []
        for s, q in zip(slots, reqs):
            if q["text"] in self.too_long and q.get("ctx_codes") is not None:
                out.append(-1)
                continue
            aid = len(self.admissions)
            self.admissions.append((s, dict(q), aid))
            self.row[s] = [aid, self.scripts[q["text"]].pop(0), 0]
            out.append(10)
        return out

    def replay(self, b):
        for s in range(b):
            if self.row[s] is None:
                continue
            aid, sc, m = self.row[s]
            m += 1
            self.row[s][2] = m
            if m - 1 < len(sc):
                self.tok_in[s] = 7
                self.frame_prev[s] = torch.tensor([aid, m - 1, 0])
            else:
                self.tok_in[s] = self.eos
            self.audio[s].fill_(0.5 if 2 <= m <= len(sc) + 1 and sc[m - 2] else 0.0)


def _chain(serving, segs, mode="prev", cap=64, rid=0):
    ch = serving.Chain(segs=[serving.Segment(text=t, key="v", item=None) for t in segs], mode=mode)
    return serving.Request(rid=rid, arrival=0.0, text=segs[0], item=None, key="v", cap=cap, chain=ch)


def _run_chain(serving, fe, reqs, **kw):
    got = {}
    b = serving.ContinuousBatcher(fe, admit_every=1, **kw)
    b.on_chunk = lambda r, y, final: got.setdefault(r.rid, []).append((y.copy(), final))
    clk = FakeClock()
    st = b.run(reqs, clock=clk, sleep=clk.sleep)
    return b, st, got


@pytest.mark.parametrize("mode", ["prev", "full", "none"])
def test_chain_segments_share_slot_and_context(serving, mode):
    """Each next segment goes into the line's own slot with the codec state kept and, as its context, the codes the
    earlier segments generated: the last one ("prev"), all of them ("full") or none; one stream of chunks, final once."""
    fe = ChainEngine({"one.": [[1, 1, 1]], "two,": [[1, 1]], "three": [[1, 1, 1, 1]]})
    r = _chain(serving, ["one.", "two,", "three"], mode=mode)
    _, st, got = _run_chain(serving, fe, [r])
    assert [a[0] for a in fe.admissions] == [0, 0, 0]
    assert [a[1].get("keep_voc", False) for a in fe.admissions] == [False, True, True]
    c1 = np.array([[0, i, 0] for i in range(3)])
    c2 = np.array([[1, i, 0] for i in range(2)])
    ctx = [a[1].get("ctx_codes") for a in fe.admissions]
    txt = [a[1].get("ctx_text") for a in fe.admissions]
    assert ctx[0] is None
    if mode == "none":
        assert ctx[1] is None and ctx[2] is None
    else:
        np.testing.assert_array_equal(ctx[1], c1)
        assert txt[1] == "one."
        np.testing.assert_array_equal(ctx[2], c2 if mode == "prev" else np.concatenate([c1, c2]))
        assert txt[2] == ("two," if mode == "prev" else "one. two,")
    y = np.concatenate([c for c, _ in got[0]])
    assert [f for _, f in got[0]].count(True) == 1 and got[0][-1][1]
    assert r.frames == 9 and r.eos and r.t_done is not None and st.summary()["finished"] == 1
    # every voiced frame went out; the switch "one." -> "two," padded the sentence end to 0.24 s of silence
    assert int((y == 0.5).sum()) == 9 * 400
    assert int((y == 0).sum()) >= int(0.24 * 4000) - 40


def test_chain_gates_lead_and_tail_silence(serving):
    """A segment's trailing silence is cut to its punctuation's tail (0.24 s after a sentence end, faded) and the
    codes kept as context stop that far after its last voiced frame; a continuation's silent lead is cut to the
    lead (0.16 s) and the frames dropped with it are not context."""
    fe = ChainEngine({"a.": [[1, 1, 1, 0, 0, 0, 0, 0]], "b": [[0, 0, 0, 0, 1, 1, 0]], "c": [[1]]})
    r = _chain(serving, ["a.", "b", "c"], mode="prev")
    _, _, got = _run_chain(serving, fe, [r])
    y = np.concatenate([c for c, _ in got[0]])
    loud = np.flatnonzero(y > 0.49)
    # 3 loud frames, the 0.24 s tail (960 samples, fading to 0 at its end), 0.16 s lead of b, 2 loud frames, b's
    # trailing silence cut to 0.06 s (no punctuation), then c
    assert loud[0] == 0 and np.all(y[:1200] == 0.5)
    assert np.all(y[1200:1200 + 960 + 640] == 0)
    assert np.all(y[2800:3600] == 0.5)
    assert np.all(y[3600:3600 + 240] == 0) and np.all(y[3840:4240] == 0.5) and y.size == 4240 + 0
    ctx_b = fe.admissions[1][1]["ctx_codes"]
    np.testing.assert_array_equal(ctx_b[:, 1], np.arange(6))          # 3 voiced + ceil(0.24 / 0.1) = 3 tail frames
    ctx_c = fe.admissions[2][1]["ctx_codes"]
    # lead of 4 silent frames: 2 kept (0.16 s), 2 dropped; voiced 4, 5; tail ceil(0.06 / 0.1) = 1 frame
    np.testing.assert_array_equal(ctx_c[:, 1], [2, 3, 4, 5, 6])


def test_chain_silent_continuation_sampled_again(serving):
    """A continuation silent past LEAD_MAX frames is sampled again into the same slot; from CTX_DROP_TRY on without
    the context; after TRIES_MAX tries the line goes on with what it has. Nothing of a discarded try is sent."""
    quiet = [0] * (serving.LEAD_MAX + 3)
    fe = ChainEngine({"x.": [[1, 1]], "y": [quiet, quiet, [0, 1, 1]]})
    r = _chain(serving, ["x.", "y"])
    _, _, got = _run_chain(serving, fe, [r])
    adm = fe.admissions
    assert [a[1]["text"] for a in adm] == ["x.", "y", "y", "y"] and all(a[0] == 0 for a in adm)
    assert [a[1].get("ctx_codes") is not None for a in adm] == [False, True, True, False]
    assert r.chain.tries == 2 and r.eos
    y = np.concatenate([c for c, _ in got[0]])
    assert int((y == 0.5).sum()) == 4 * 400                             # 2 + 2 voiced frames, no discarded audio


def test_chain_context_too_long_goes_on_without(serving):
    fe = ChainEngine({"p.": [[1, 1]], "q": [[1]]}, too_long={"q"})
    r = _chain(serving, ["p.", "q"])
    _run_chain(serving, fe, [r])
    assert [a[1]["text"] for a in fe.admissions] == ["p.", "q"]
    assert fe.admissions[1][1].get("ctx_codes") is None and fe.admissions[1][1]["keep_voc"]
    assert r.eos and r.error is None


def test_chain_cancel_between_segments(serving):
    """A line cancelled while its next segment waits for admission ends with an empty final chunk and frees the slot."""
    fe = ChainEngine({"m.": [[1, 1]], "n": [[1]]}, B=1)
    r = _chain(serving, ["m.", "n"])
    b = serving.ContinuousBatcher(fe, admit_every=10 ** 6)
    finals = []
    b.on_chunk = lambda q, y, final: finals.append(final)

    class Clock(FakeClock):
        def __call__(self):
            if r.chain.k == 1 and not r.cancelled:
                b.cancel(r.rid)
            return super().__call__()

    clk = Clock()
    b.run([r], clock=clk, sleep=clk.sleep)
    assert r.cancelled and finals[-1] and len(fe.admissions) <= 2
