"""The streaming resampler's host side on the CPU: the filter design (band edges, attenuation, unit gain), the
polyphase table, the oracle pinned against scipy.signal.resample_poly over the same FIR, the oracle's streaming
contract (chunking does not change the stream; ceil(N up / down) samples in all; delay-compensated), the per-slot
state machine, and the launch geometry the host derives for several rate pairs."""
import importlib
import math

import numpy as np
import pytest
import scipy.signal as ss

from oracle import resample_ref as RR


@pytest.fixture(scope="module")
def rsm(a8):
    return importlib.import_module(a8.__name__ + ".resample")


def test_design_band_edges(rsm):
    up, down, h = rsm.design_filter(44100, 16000)
    assert (up, down) == (160, 441) and len(h) % 2 == 1
    assert abs(h.sum() - 1.0) < 1e-12 and np.allclose(h, h[::-1])          # unit DC gain, linear phase
    n = 1 << 21
    f = np.fft.rfftfreq(n, 1.0 / (44100 * up))
    mag = 20 * np.log10(np.abs(np.fft.rfft(h, n)) + 1e-300)
    assert np.abs(mag[f <= 7200]).max() < 1e-3                              # passband flat to 90 % of 8 kHz
    assert mag[f >= 8000].max() < -115.0                                    # stopband from the output Nyquist


def test_polyphase_table(rsm):
    up, down, h = rsm.design_filter(44100, 16000)
    t = rsm.polyphase_table(h, up)
    assert t.shape == (-(-len(h) // up), up) and t.dtype == np.float32
    k, p = 7, 33
    assert t[k, p] == np.float32(up * h[p + k * up]) and t[-1, -1] == 0.0
    t32 = rsm.polyphase_table(h, up, 32)                  # padded with zero taps for the kernel's staged chunks
    assert t32.shape == (448, up) and np.array_equal(t32[:t.shape[0]], t) and not t32[t.shape[0]:].any()


@pytest.mark.parametrize("rates", [(44100, 16000), (48000, 16000), (44100, 48000)])
def test_oracle_pinned_to_resample_poly(rsm, rates):
    up, down, h = rsm.design_filter(*rates)
    g = np.random.default_rng(0)
    x = g.standard_normal(9000) * 0.3
    want = ss.resample_poly(x, up, down, window=h)
    rs = RR.StreamResampler(h, up, down)
    cuts = np.sort(g.choice(np.arange(1, len(x)), 6, replace=False))
    parts = np.split(x, cuts)
    got = np.concatenate([rs.resample_chunk(c, last=(i == len(parts) - 1)) for i, c in enumerate(parts)])
    assert len(got) == len(want) == -(-len(x) * up // down)
    assert np.abs(got - want).max() < 1e-12


def test_oracle_sine_is_delay_compensated(rsm):
    """A 1 kHz tone at 44.1 kHz comes out as the same tone at 16 kHz, in phase, amplitude within 1e-5."""
    up, down, h = rsm.design_filter(44100, 16000)
    t_in = np.arange(44100) / 44100.0
    rs = RR.StreamResampler(h, up, down)
    y = np.concatenate([rs.resample_chunk(c) for c in np.split(0.5 * np.sin(2 * np.pi * 1000 * t_in), 20)]
                       + [rs.resample_chunk(np.zeros(0), last=True)])
    assert len(y) == 16000
    ref = 0.5 * np.sin(2 * np.pi * 1000 * np.arange(16000) / 16000.0)
    mid = slice(500, 15500)                                        # away from the zero-padded ends
    assert np.abs(y[mid] - ref[mid]).max() < 1e-5


def test_oracle_streaming_counts(rsm):
    """Before the flush a stream has given every output whose window lies in its input; the flush gives the rest."""
    up, down, h = rsm.design_filter(44100, 16000)
    rs = RR.StreamResampler(h, up, down)
    half = (len(h) - 1) // 2
    total = 0
    for k in range(1, 5):
        total += len(rs.resample_chunk(np.ones(2048)))
        N = 2048 * k
        assert total == (N * up - 1 - half) // down + 1
        assert ((total - 1) * down + half) // up <= N - 1 < (total * down + half) // up
    total += len(rs.resample_chunk(np.zeros(0), last=True))
    assert total == math.ceil(4 * 2048 * up / down)


def test_slot_streams_state_machine(rsm):
    up, down, h = rsm.design_filter(44100, 16000)
    S = RR.SlotStreams(4, h, up, down)
    S.reset([0, 1, 2, 3], [2, 5, 1, 4])
    eos = 99
    g = np.random.default_rng(1)
    got = [[] for _ in range(4)]
    toks = [[7, 7, 7, 7, 7], [7, 7, 99, 7, 7], [7, 7, 7, 7, 7], [99, 7, 7, 7, 7]]
    for t in range(5):
        out = S.step(g.standard_normal((4, 2048)) * 0.1, np.array([toks[r][t] for r in range(4)]), eos, 4)
        for r in range(4):
            got[r].append(len(out[r]))
    full = lambda f: -(-f * 2048 * up // down)
    assert got[0][0] == 0 and sum(got[0]) == full(2)          # silence frame dropped, cap 2: ticks 2-3
    assert sum(got[1]) == full(2) and got[1][3:] == [0, 0]    # EOS consumed on tick 3: its frame is the last
    assert sum(got[2]) == full(1)
    assert sum(got[3]) == 0                                    # EOS on the silence tick: nothing at all


@pytest.mark.parametrize("rates", [(44100, 16000), (48000, 16000), (44100, 48000), (24000, 16000), (44100, 22050)])
def test_launch_geometry(rsm, rates):
    """hist / zero tail / output rows / threads cover every access the kernel makes (the bounds csrc/resample.cu
    checks on the host before a launch)."""
    r = rsm.Resampler(2, rates[0], rates[1], 2048, "cpu")
    assert r.hist_len >= r.taps + r.down // r.up + 2 and r.zpad >= r.half // r.up + r.down // r.up + 2
    assert r.period % r.up == 0 and r.period <= 512 and r.period * rsm.RS_PT >= r.out_max
    assert r.taps % rsm.RS_KC == 0 and r.taps * r.up >= len(r.h)
    per_frame = 2048 * r.up // r.down + 1
    tail = (r.half + 1) // r.down + 2
    assert r.out_max >= per_frame + tail
    smem = 4 * (2 * rsm.RS_KC * r.up + r.hist_len + 2048 + r.zpad)
    assert smem <= 200 * 1024
