"""Edge cases of the drop-in on the GPU against the CPU oracle engine (tiny stand-in: real widths, 2 slow layers).

Admission (serve/fast_engine.py:1050-1071, :1089-1133): an empty call; a prompt longer than min(S - 32, prefill
tokens) rejected with -1 while the others of the same call are admitted and the rejected slot is left as it was;
packed prefill run in pieces of TTS_PREFILL_ROWS rows, one request spanning several pieces and the voice prefix's KV
computed in pieces too -- lengths, cache rows and last hidden as the oracle's (which prefills each request whole).
Tick (serve/fast_engine.py:757-769): a row consuming EOS keeps EOS (sticky) and queues the silence frame; a row at
position S - 1 stays there (cpos = min(pos + 1, S - 1)).
"""
from types import SimpleNamespace

import pytest
import torch

from oracle import ref_cpu as R
from oracle.standin import StubTokenizer
from test_gpu_engine import _near_tie, _resync, rel

pytestmark = pytest.mark.gpu
GREEDY = dict(do_sample=False, temperature=0.8, top_k=50, top_p=0.95, max_new_tokens=64)


@pytest.fixture(scope="module")
def dev(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return torch.device("cuda", 0)


def _words(g, n):
    return " ".join(str(int(t)) for t in torch.randint(0, 151643, (n,), generator=g))


def test_admission_edges(a8, dev, tiny_model, monkeypatch):
    monkeypatch.setenv("TTS_PREFILL_ROWS", "64")
    eng = a8.FastEngine(tiny_model, StubTokenizer(), GREEDY, max_slots=4, max_seq=256, buckets=[4],
                        seq_from_env=False, seed=13)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), GREEDY, max_slots=4, max_seq=256, seed=13, with_voc=False)
    assert eng.pf_rows == 64
    assert eng.admit([], []) == []
    g = torch.Generator().manual_seed(5)
    item = SimpleNamespace(ref_code=torch.randint(0, 4096, (70, 10), generator=g), ref_text=_words(g, 6))
    reqs = [dict(text=_words(g, 120), item=item, key="v"),       # its rest spans two 64-row pieces
            dict(text=_words(g, 400), item=item, key="v"),       # longer than S - 32: rejected
            dict(text=_words(g, 5), item=item, key="v"),
            dict(text=_words(g, 30), item=item, key="v")]
    lens = eng.admit([0, 1, 2, 3], reqs)
    assert lens == ora.admit([0, 1, 2, 3], reqs), lens
    torch.cuda.synchronize()
    assert a8.device_error()[0] == 0
    assert lens[1] == -1 and min(lens[0], lens[2], lens[3]) > 0
    assert lens[0] == eng.S - 32                                  # exactly at the limit: still admitted
    assert eng.build_prompts([reqs[0]])[0][2].shape[0] > 64 and eng.build_prompts([reqs[0]])[0][1].shape[0] > 64
    ok = [0, 2, 3]
    assert int(eng.cpos[1]) == 0                                  # the rejected slot was not touched
    assert torch.equal(eng.cpos[ok].cpu(), ora.cpos[ok])
    assert rel(eng.hid[ok], ora.hid[ok]) < 2e-2
    for s in ok:
        n = lens[s]
        assert rel(eng.slow.kc[:, s, :, :n], ora.slow.kc[:, s, :, :n]) < 2e-2, s
        assert rel(eng.slow.vc[:, s, :, :n], ora.slow.vc[:, s, :, :n]) < 2e-2, s


def test_sticky_eos_and_position_clamp(a8, dev, tiny_model):
    eng = a8.FastEngine(tiny_model, StubTokenizer(), GREEDY, max_slots=3, max_seq=256, buckets=[3],
                        seq_from_env=False, seed=17)
    ora = R.OracleEngine(tiny_model, StubTokenizer(), GREEDY, max_slots=3, max_seq=256, seed=17, with_voc=False)
    g = torch.Generator().manual_seed(6)
    item = SimpleNamespace(ref_code=torch.randint(0, 4096, (10, 10), generator=g), ref_text="12 34")
    reqs = [dict(text=_words(g, 6 + i), item=item, key="v") for i in range(3)]
    eng.admit([0, 1, 2], reqs)
    torch.cuda.synchronize()
    S = eng.S
    eng.tok[0] = eng.eos                                          # row 0 consumes EOS on this tick
    eng.cpos[1] = S - 1                                           # row 1 sits at the last position
    for t in range(2):
        _resync(ora, eng)
        ora.record = {}
        t_in = eng.tok[:3].cpu().clone()
        eng.tick(3)
        codes_o = ora.tick(3)
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        assert int(eng.tok_in[0]) == eng.eos and int(eng.tok[0]) == eng.eos        # sticky
        assert torch.equal(eng.frame_prev[0].cpu(), eng.sil_frame.cpu())
        assert int(eng.cpos[1]) == S - 1 == int(ora.cpos[1])
        assert torch.equal(eng.cpos[:3].cpu(), ora.cpos[:3]) and torch.equal(eng.nstep[:3].cpu(), ora.nstep[:3])
        assert torch.equal(eng.prev[:3].cpu(), ora.prev[:3])
        codes_e = eng.codes[:3].cpu()
        for r in range(3):
            diff = (codes_e[r] != codes_o[r]).nonzero()
            if len(diff):
                k = int(diff[0])
                okk, why = _near_tie(ora.record["fast_logits"][k - 1][r], int(codes_e[r, k]), int(codes_o[r, k]))
                assert okk, (t, r, k, why)
                continue
            assert rel(eng.logits[r, :eng.nh], ora.record["logits"][-1][r]) < 2e-2, (t, r)
            if int(t_in[r]) != eng.eos:
                assert torch.equal(eng.frame_prev[r].cpu(), codes_e[r])
