"""The per-slot streaming resampler (a8_resample_reset / a8_resample_step, 44.1 -> 16 kHz) on the GPU against the
CPU oracle (oracle/resample_ref.py, pinned to scipy.signal.resample_poly over the same FIR).

Bars: the per-step output counts are exact; the fp32 samples within 2e-5 of the oracle's float64 sums (431-tap fp32
dot products); PCM16 within one step of the oracle's _pcm16 and equal wherever the oracle's scaled sample is more
than 0.02 from an integer (fp32 rounding can only move a truncation across a boundary that close)."""
import importlib

import numpy as np
import pytest
import torch

from oracle import resample_ref as RR

pytestmark = pytest.mark.gpu
EOS = 4096


@pytest.fixture(scope="module")
def dev(a8):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    a8.load()
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def rsm(a8):
    return importlib.import_module(a8.__name__ + ".resample")


def _frames(g, b, n=2048, loud=()):
    """Speech-band test signals: a few tones and a little noise a row; rows in `loud` exceed [-1, 1] (clipped)."""
    t = np.arange(n) / 44100.0
    x = np.zeros((b, n))
    for r in range(b):
        for _ in range(3):
            x[r] += 0.25 * np.sin(2 * np.pi * g.uniform(80, 7000) * t + g.uniform(0, 6.3))
        x[r] += 0.02 * g.standard_normal(n)
        if r in loud:
            x[r] *= 2.0
    return x.astype(np.float32)


def _check(r, got_f, got_p, want):
    assert len(got_f) == len(want), (r, len(got_f), len(want))
    if not len(want):
        return
    assert np.abs(got_f - want).max() < 2e-5, (r, np.abs(got_f - want).max())
    pw = RR.pcm16(want)
    d = np.abs(got_p.astype(np.int32) - pw.astype(np.int32))
    assert d.max() <= 1, r
    s = np.clip(want.astype(np.float32), -1, 1) * np.float32(32767.0)
    far = np.abs(s - np.round(s)) > 0.02
    assert (d[far] == 0).all(), r


def test_resample_slots_match_oracle(a8, dev, rsm):
    """Six slots over 12 ticks: dropped first frames, caps, EOS (also on the dropped frame), rows that end while the
    bucket keeps ticking, slots restarted mid-run, clipped rows."""
    rs = rsm.Resampler(6, 44100, 16000, 2048, dev, f32_out=True)
    ora = RR.SlotStreams(6, rs.h, rs.up, rs.down)
    g = np.random.default_rng(3)
    caps = [1, 3, 5, 12, 4, 7]
    eos_at = {4: 2, 5: 0, 3: 9}                 # row -> tick on which it consumes EOS
    rs.reset(list(range(6)), caps)
    ora.reset(list(range(6)), caps)
    restart = {6: ([0, 1], [4, 2])}
    total = [0] * 6
    for tick in range(12):
        if tick in restart:
            s, c = restart[tick]
            rs.reset(s, c)
            ora.reset(s, c)
        b = 6 if tick < 10 else 4
        audio = _frames(g, 6, loud=(2,))
        tok = np.full(6, 7, dtype=np.int64)
        for r, t in eos_at.items():
            if t == tick:
                tok[r] = EOS
        A, T = torch.from_numpy(audio).to(dev), torch.from_numpy(tok).to(dev)
        pcm, cnt = rs.step(A, T, EOS, b)
        want = ora.step(audio, tok, EOS, b)
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        cnt = cnt.cpu().numpy()
        pcm, f32 = pcm.cpu().numpy(), rs.f32[:b].cpu().numpy()
        for r in range(b):
            n = int(cnt[r])
            _check((tick, r), f32[r, :n], pcm[r, :n], want[r])
            total[r] += n
    full = lambda f: -(-f * 2048 * rs.up // rs.down)
    assert total[5] == 0                        # EOS on its dropped first frame: no audio at all
    assert total[4] == full(2)                  # frames of ticks 1-2, EOS consumed on tick 2
    assert total[2] == full(5)


@pytest.mark.parametrize("b", [192, 600])
def test_resample_full_bucket(a8, dev, rsm, b):
    """The cfg2 bucket (192 slots: each row's taps split over a 2-CTA cluster) and 600 slots (one CTA a row), 5
    ticks: a sample of rows against the oracle, and the per-row counts equal for all rows (every row at the same
    stream position). The 6-slot test above runs 4-CTA clusters."""
    rs = rsm.Resampler(b, 44100, 16000, 2048, dev, f32_out=True)
    rows = [0, 1, 77, 147, 148, b - 1]
    ora = RR.SlotStreams(len(rows), rs.h, rs.up, rs.down)
    rs.reset(list(range(b)), [4] * b)
    ora.reset(list(range(len(rows))), [4] * len(rows))
    g = np.random.default_rng(9)
    tok = np.full(b, 7, dtype=np.int64)
    T = torch.from_numpy(tok).to(dev)
    for tick in range(5):
        audio = _frames(g, b)
        pcm, cnt = rs.step(torch.from_numpy(audio).to(dev), T, EOS, b)
        want = ora.step(audio[rows], tok[rows], EOS, len(rows))
        torch.cuda.synchronize()
        assert a8.device_error()[0] == 0
        cnt = cnt.cpu().numpy()
        assert (cnt == cnt[0]).all()
        pcm, f32 = pcm.cpu().numpy(), rs.f32[:b].cpu().numpy()
        for k, r in enumerate(rows):
            n = int(cnt[r])
            _check((tick, r), f32[r, :n], pcm[r, :n], want[k])
