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
