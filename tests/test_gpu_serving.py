"""The continuous-batching loop over a real FastEngine on the GPU (the tiny stand-in: real widths, 2 slow layers):
requests arrive while others run, are admitted in packed prefills into the lowest free slots, tick in CUDA graphs of
the covering bucket, deliver one frame of audio a tick after their silence frame, and end at their cap; every slot is
reused. Checks the delivered audio against the engine's own audio rows and the bookkeeping of every request."""
import importlib

import numpy as np
import pytest
import torch

from oracle.standin import StubTokenizer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def serving(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return importlib.import_module(a8.__name__ + ".serving")


def test_serving_loop_on_engine(a8, serving, tiny_model):
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=6, max_seq=512, buckets=[2, 4, 6],
                        seq_from_env=False, seed=5)
    eng.capture(log=lambda *a: None)
    ncb = int(tiny_model.config.num_codebooks)
    voices = serving.voice_items(2, 12, ncb, seed=3)
    serving.warm_voices(eng, voices)
    caps = [5, 9, 3, 12, 7, 4, 6, 8, 10, 2]
    reqs = [serving.Request(rid=i, arrival=0.01 * i, text=" ".join(str(100 + i + k) for k in range(8 + i)),
                            item=voices[i % 2][1], key=voices[i % 2][0], cap=c) for i, c in enumerate(caps)]
    loop = serving.ContinuousBatcher(eng, admit_every=1, admit_batch=4)
    got = {}
    loop.on_audio = lambda r, pcm: got.setdefault(r.rid, []).append(pcm.clone())
    st = loop.run(reqs)
    assert a8.device_error()[0] == 0
    s = st.summary()
    assert s["rejected"] == 0 and s["finished"] + s["eos"] >= 1
    for r in reqs:
        assert r.t_done is not None and 0 <= r.slot < 6
        assert (r.frames == r.cap) or r.eos                  # the cap, or EOS drawn earlier
        assert len(got.get(r.rid, [])) == r.frames
        for pcm in got.get(r.rid, []):                       # one frame of fp32 PCM in [-1, 1] (tanh output)
            assert pcm.shape == (eng.up,) and torch.isfinite(pcm).all() and float(pcm.abs().max()) <= 1.0
        assert r.t_first is None or r.t_first >= r.arrival
    # more requests than slots: slots were reused, and at most 6 rows were ever busy
    assert max(st.buckets) <= 6 and len({r.slot for r in reqs}) <= 6
    assert sum(r.frames for r in reqs) == s["frames"]


def test_serving_loop_resampled(a8, serving, tiny_model):
    """out_sr=16000: every request's chunks are int16 at 16 kHz, ceil(frames x 2048 x 160 / 441) samples in all (its
    stream flushed on its last frame), and the first chunk is ready after one frame."""
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=6, max_seq=512, buckets=[2, 4, 6],
                        seq_from_env=False, seed=6)
    eng.capture(log=lambda *a: None)
    ncb = int(tiny_model.config.num_codebooks)
    voices = serving.voice_items(2, 12, ncb, seed=4)
    serving.warm_voices(eng, voices)
    caps = [5, 9, 3, 12, 7, 4, 6, 8]
    reqs = [serving.Request(rid=i, arrival=0.01 * i, text=" ".join(str(200 + i + k) for k in range(8 + i)),
                            item=voices[i % 2][1], key=voices[i % 2][0], cap=c) for i, c in enumerate(caps)]
    loop = serving.ContinuousBatcher(eng, admit_every=1, admit_batch=4, copy_audio=False, out_sr=16000)
    got = {}
    loop.on_chunk = lambda r, y, final: got.setdefault(r.rid, []).append((y.copy(), final))
    loop.run(reqs)
    assert a8.device_error()[0] == 0
    for r in reqs:
        chunks = got[r.rid]
        assert all(y.dtype == np.int16 for y, _ in chunks) and [f for _, f in chunks][-1]
        n = sum(len(y) for y, _ in chunks)
        assert n == -(-r.frames * eng.up * 160 // 441), (r.rid, r.frames, n)
        if r.frames:
            assert len(chunks[0][0]) <= 743 + 90 and np.abs(np.concatenate([y for y, _ in chunks])).max() > 0


def test_serving_chain_on_engine(a8, serving, tiny_model):
    """A code-switch line of three segments (two voices) beside plain requests: every segment of the line runs in the
    line's one slot, continuations keep the codec state, and each continuation's context is exactly the codes the
    engine generated for the previous segment in that slot (read back by the loop every tick), from its first kept
    frame on -- checked against frame_prev recorded after every replay."""
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=6, max_seq=512, buckets=[2, 4, 6],
                        seq_from_env=False, seed=7)
    eng.capture(log=lambda *a: None)
    ncb = int(tiny_model.config.num_codebooks)
    voices = serving.voice_items(2, 12, ncb, seed=5)
    serving.warm_voices(eng, voices)
    rec, adm = [], []
    replay0, admit0 = eng.replay, eng.admit

    def replay(b, *a):
        replay0(b, *a)
        torch.cuda.synchronize()
        rec.append(eng.frame_prev[:b].cpu().clone())

    def admit(slots, reqs):
        adm.append((len(rec), list(slots), [dict(q) for q in reqs]))
        return admit0(slots, reqs)

    eng.replay, eng.admit = replay, admit
    segs = [serving.Segment(text="11 12 13 14 15.", key=voices[0][0], item=voices[0][1], cap=6),
            serving.Segment(text="21 22 23", key=voices[1][0], item=voices[1][1], cap=5),
            serving.Segment(text="31 32 33 34", key=voices[0][0], item=voices[0][1], cap=4)]
    line = serving.Request(rid=100, arrival=0.0, text=segs[0].text, item=segs[0].item, key=segs[0].key, cap=64,
                           chain=serving.Chain(segs=segs, mode="prev"))
    plain = [serving.Request(rid=i, arrival=0.002 * i, text=" ".join(str(300 + i + k) for k in range(6 + i)),
                             item=voices[i % 2][1], key=voices[i % 2][0], cap=4 + i) for i in range(3)]
    loop = serving.ContinuousBatcher(eng, admit_every=1, admit_batch=4)
    got = []
    loop.on_chunk = lambda r, y, final: got.append((y.copy(), final)) if r.rid == 100 else None
    loop.run([line] + plain)
    assert a8.device_error()[0] == 0
    assert line.t_done is not None and line.error is None and got[-1][1]
    mine = [(t, s[i], q[i]) for t, s, q in adm for i in range(len(s)) if q[i]["text"] in {g.text for g in segs}]
    assert len({s for _, s, _ in mine}) == 1                       # one slot for the whole line
    slot = mine[0][1]
    assert [q.get("keep_voc", False) for _, _, q in mine][:1] == [False] and all(q["keep_voc"] for _, _, q in mine[1:])
    hist = line.chain.hist
    assert len(hist) == 2 and [h[1] for h in hist] == [segs[0].text, segs[1].text]
    for k, (codes, _) in enumerate(hist):
        t_adm = [t for t, _, q in mine if q["text"] == segs[k].text][-1]          # the try whose codes were kept
        gen = torch.stack([rec[t_adm + i][slot] for i in range(segs[k].cap)]).numpy()
        lo = next(o for o in range(len(gen)) if np.array_equal(gen[o], codes[0]))  # leading silence not kept
        np.testing.assert_array_equal(codes, gen[lo:lo + len(codes)])
        nxt = [q for _, _, q in mine if q["text"] == segs[k + 1].text][-1]
        np.testing.assert_array_equal(np.asarray(nxt["ctx_codes"]), codes)      # "prev": the last segment only
        assert nxt["ctx_text"] == segs[k].text
    y = np.concatenate([c for c, _ in got])
    assert y.size > 0 and np.isfinite(y).all() and np.abs(y).max() <= 1.0
    assert all(r.t_done is not None and r.error is None for r in plain)
