"""Code-switch continuation and voice priming on the GPU (tiny stand-in: real widths, 2 slow layers), against the CPU
oracle engine and the oracle codec.

Continuation (serve/fast_engine.py:970-980 and :1134-1156): a request's `ctx_text` is prepended to its text and its
`ctx_codes` appended as audio positions; its prompt length, cache rows and last hidden equal the oracle's, and the
first tick after it matches the oracle teacher-forced. A `keep_voc` row keeps its codec state untouched and decodes the
silence frame first, so its audio continues the previous utterance's stream; a fresh row starts clean.

Priming (TTS_VOC_PRIME=1, serve/fast_engine.py:994-1033): each voice's last `TTS_VOC_PRIME_FRAMES` reference frames
decode through the codec, the row is snapshotted after the second-to-last frame, and an admitted row starts from that
snapshot with the last reference frame as the frame it decodes first: its first audio frame equals (SNR bar of the
codec tests) the oracle codec streaming those reference frames from a clean row.
"""
import pytest
import torch

from oracle import ref_cpu as R
from oracle.standin import StubTokenizer
from test_gpu_engine import _near_tie, _requests, _resync, rel
from test_gpu_vocoder import snr_db

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return torch.device("cuda", 0)


def _blob(eng, row):
    return eng.voc.snapshot(row)[0].cpu()


def test_continuation_matches_oracle(a8, dev, tiny_model):
    from audio8_b200.codec import StreamingVocoder
    gp = dict(do_sample=False, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, buckets=[1, 2, 3],
                        seq_from_env=False, seed=31)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, seed=31, with_voc=False)
    first = _requests(4)
    eng.admit([0, 1], first)
    for _ in range(3):                                   # the rows' codecs carry a few frames of state
        eng.tick(2)
    torch.cuda.synchronize()
    before = [_blob(eng, r) for r in range(2)]
    assert before[0].any() and before[1].any()
    g = torch.Generator().manual_seed(8)
    cc = torch.randint(0, 4096, (6, eng.ncg), generator=g)
    cont = [dict(first[0], ctx_text="12 34 56", ctx_codes=cc, keep_voc=True),
            dict(first[1], ctx_text="78 90")]
    plain = [dict(first[0]), dict(first[1])]
    n_plain = [p.shape[0] + r.shape[0] for _, p, r in eng.build_prompts(plain)]
    lens = eng.admit([0, 1], cont)
    assert lens == ora.admit([0, 1], cont)
    assert lens[0] >= n_plain[0] + len(cc) + 1 and lens[1] > n_plain[1]   # ctx text and codes are in the prompt
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    assert torch.equal(eng.cpos[:2].cpu(), ora.cpos[:2]) and torch.equal(eng.cpos[:2].cpu(), torch.tensor(lens))
    assert rel(eng.hid[:2], ora.hid[:2]) < 2e-2
    for s in range(2):
        n = lens[s]
        assert rel(eng.slow.kc[:, s, :, :n], ora.slow.kc[:, s, :, :n]) < 2e-2, s
        assert rel(eng.slow.vc[:, s, :, :n], ora.slow.vc[:, s, :, :n]) < 2e-2, s
    # codec rows: kept as they were (keep_voc) or cleared, and both decode the silence frame first
    assert torch.equal(_blob(eng, 0), before[0])
    assert not _blob(eng, 1).any()
    sil = eng.sil_frame.cpu()
    assert torch.equal(eng.frame_prev[:2].cpu(), sil.expand(2, -1))
    assert torch.equal(ora.frame_prev[:2], sil.expand(2, -1))
    # the first tick: the keep row's audio continues its stream (a standalone codec loaded with the pre-admission
    # state, bit-identical); the slow/fast AR matches the oracle teacher-forced
    voc = StreamingVocoder(tiny_model.load_codec(device="cpu"), 3, dev)
    voc.load_many([0], [before[0].pin_memory()])
    voc.clear_many([1])
    want_audio = voc.step(eng.frame_prev[:2].clone(), 2).clone()
    _resync(ora, eng)
    ora.record = {}
    eng.tick(2)
    codes_o = ora.tick(2)
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    assert torch.equal(eng.audio[:2], want_audio)
    codes_e = eng.codes[:2].cpu()
    for r in range(2):
        diff = (codes_e[r] != codes_o[r]).nonzero()
        if len(diff):
            k = int(diff[0])
            ok, why = _near_tie(ora.record["fast_logits"][k - 1][r], int(codes_e[r, k]), int(codes_o[r, k]))
            assert ok, (r, k, why)
            continue
        assert rel(eng.logits[r, :eng.nh], ora.record["logits"][-1][r]) < 2e-2, r
        assert int(eng.cpos[r]) == int(ora.cpos[r]) and torch.equal(eng.frame_prev[r].cpu(), ora.frame_prev[r])


def test_voice_priming(a8, dev, tiny_model, monkeypatch):
    from types import SimpleNamespace
    monkeypatch.setenv("TTS_VOC_PRIME", "1")
    monkeypatch.setenv("TTS_VOC_PRIME_FRAMES", "4")
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=3, max_seq=512, buckets=[3],
                        seq_from_env=False, seed=41)
    assert eng.voc_prime and eng.prime_frames == 4
    g = torch.Generator().manual_seed(21)
    ref0 = torch.randint(0, 4096, (20, eng.ncg), generator=g)          # truncated to its last 4 frames
    ref1 = torch.randint(0, 4096, (1, eng.ncg), generator=g)           # one frame: the snapshot is a clean row
    it0 = SimpleNamespace(ref_code=ref0, ref_text="12 34")
    it1 = SimpleNamespace(ref_code=ref1, ref_text="56 78")
    it2 = SimpleNamespace(ref_code=ref0[:5], ref_text="90")
    eng.prime_speakers([("v0", it0), ("v1", it1), ("v0", it0)])
    torch.cuda.synchronize()
    assert sorted(eng.voc_snaps) == ["v0", "v1"]
    assert torch.equal(eng.voc_snaps["v0"][1], ref0[-1]) and torch.equal(eng.voc_snaps["v1"][1], ref1[-1])
    assert eng.voc_snaps["v0"][0][0].any() and not eng.voc_snaps["v1"][0][0].any()
    t = " ".join(str(100 + k) for k in range(10))
    reqs = [dict(text=t, item=it0, key="v0"), dict(text=t, item=it1, key="v1"), dict(text=t, item=it2, key="v2")]
    assert min(eng.admit([0, 1, 2], reqs)) > 0
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    assert torch.equal(_blob(eng, 0), eng.voc_snaps["v0"][0][0])
    assert not _blob(eng, 1).any() and not _blob(eng, 2).any()        # v2 was never primed: a clean row
    sil = eng.sil_frame.cpu()
    assert torch.equal(eng.frame_prev[0].cpu(), ref0[-1]) and torch.equal(eng.frame_prev[1].cpu(), ref1[-1])
    assert torch.equal(eng.frame_prev[2].cpu(), sil)
    eng.tick(3)
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    audio = eng.audio[:3].cpu()
    # the oracle codec streams each row's frames from a clean row: the primed frames, then the first decoded one
    streams = [ref0[-4:], ref1[-1:], sil[None]]
    for r, frames in enumerate(streams):
        ov = R.Vocoder(tiny_model.load_codec(device="cpu"), 1)
        for f in frames:
            w = ov.step(f[None].long(), 1)
        s = snr_db(audio[r], w[0])
        print(f"row {r}: first audio frame after {len(frames) - 1} primed frames, SNR {s:.1f} dB")
        assert s >= 38.0, (r, s)


def test_voice_snapshots_on_disk(a8, dev, tiny_model, monkeypatch, tmp_path):
    """A disk-backed store (the worker's TTS_SNAP_DIR): priming writes one file a voice; a second engine on the same
    directory primes nothing, reads the snapshot back on the voice's first admission, and starts the row from it."""
    from types import SimpleNamespace
    from audio8_b200.snapstore import SnapStore
    monkeypatch.setenv("TTS_VOC_PRIME", "1")
    monkeypatch.setenv("TTS_VOC_PRIME_FRAMES", "4")
    gp = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)
    g = torch.Generator().manual_seed(23)
    items = [(f"v{k}", SimpleNamespace(ref_code=torch.randint(0, 4096, (9, 10), generator=g), ref_text="12 34"))
             for k in range(2)]
    engs = []
    for _ in range(2):
        eng = a8.FastEngine(tiny_model, StubTokenizer(), gp, max_slots=2, max_seq=512, buckets=[2],
                            seq_from_env=False, seed=43)
        eng.voc_snaps = SnapStore(str(tmp_path), ram=1)
        eng.prime_speakers(items)
        torch.cuda.synchronize()
        engs.append(eng)
    first, second = engs
    assert first.voc_snaps.on_disk() == 2 and second.voc_snaps.loads == 0 and len(second.voc_snaps) == 0
    reqs = [dict(text="10 11 12 13", item=items[1][1], key="v1"), dict(text="14 15", item=items[0][1], key="v0")]
    second.admit([0, 1], reqs)
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0 and second.voc_snaps.loads == 2
    assert torch.equal(_blob(second, 0), _blob_of(first, "v1")) and torch.equal(_blob(second, 1), _blob_of(first, "v0"))
    assert torch.equal(second.frame_prev[0].cpu(), items[1][1].ref_code[-1])


def _blob_of(eng, key):
    return eng.voc_snaps[key][0][0].reshape(1, -1).cpu()
