"""Per-slot streaming rate conversion and PCM16 of the engine's audio on the GPU.

The reference worker converts each request's audio on the host: one soxr.ResampleStream(native_sr, out_sr, 1,
dtype="float32", quality=TTS_RESAMPLE_QUALITY) per request, fed each emitted chunk with resample_chunk(y,
last=final), then _pcm16 (serve/engine_worker.py:443-449, :460-461, :423-424, :699; out_sr from TTS_OUT_SR, default
16000, serve/config.py:111). Here every slot of the engine has a stream on the device and one launch a tick converts
the frame each row just decoded (`a8_resample_step`), so the host receives int16 samples at the output rate.

The filter is a linear-phase low-pass FIR at the up-sampled rate (in_sr x up), designed by Kaiser's window method
(J. F. Kaiser, "Nonrecursive digital filter design using the I0-sinh window function", 1974): stopband attenuation
A dB needs beta = 0.1102 (A - 8.7) and N - 1 = (A - 7.95) / (2.285 dw) taps for a transition width dw (radians per
sample). The default band: pass to 90 % of the lower Nyquist, stop from 100 % of it, A = 120 dB (the 20-bit class of
soxr's HQ recipe). Output sample n is centred on input time n down / up (delay compensated), like
scipy.signal.resample_poly with the same FIR.
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Sequence

import numpy as np
import torch

from . import _lib as L

RS_PT = 8          # outputs a thread of k_resample at most (csrc/resample.cu)
RS_KC = 32         # taps a table chunk k_resample stages in shared memory: the table's taps are a multiple of it


def design_filter(in_sr: int, out_sr: int, atten_db: float = 120.0, pass_frac: float = 0.9):
    """(up, down, h): the rational factors of out_sr / in_sr and a unit-DC-gain FIR h (float64, odd length) at the
    up-sampled rate in_sr * up, passband to pass_frac x and stopband from 1.0 x the lower of the two Nyquist rates."""
    g = math.gcd(int(in_sr), int(out_sr))
    up, down = int(out_sr) // g, int(in_sr) // g
    nyq = min(in_sr, out_sr) / 2.0
    f_pass, f_stop = pass_frac * nyq, nyq
    fs_up = float(in_sr) * up
    dw = 2.0 * math.pi * (f_stop - f_pass) / fs_up
    n = int(math.ceil((atten_db - 7.95) / (2.285 * dw))) + 1
    length = n | 1
    beta = 0.1102 * (atten_db - 8.7) if atten_db > 50 else 0.5842 * (atten_db - 21) ** 0.4 + 0.07886 * (atten_db - 21)
    half = (length - 1) // 2
    fc = 0.5 * (f_pass + f_stop) / fs_up            # cutoff, cycles per up-sampled sample
    j = np.arange(length, dtype=np.float64) - half
    h = 2.0 * fc * np.sinc(2.0 * fc * j) * np.kaiser(length, beta)
    return up, down, h / h.sum()


def polyphase_table(h: np.ndarray, up: int, multiple: int = 1) -> np.ndarray:
    """[taps, up] float32: table[k][p] = up * h[p + k up] (0 past the filter), taps rounded up to `multiple`."""
    taps = -(-(-(-len(h) // up)) // multiple) * multiple
    hp = np.zeros(taps * up, dtype=np.float64)
    hp[:len(h)] = h * up
    return hp.reshape(taps, up).astype(np.float32)


class Resampler:
    """Streaming in_sr -> out_sr conversion for `rows` slots on the device, one frame of `frame` samples a slot a
    step. A slot's stream starts at reset(slots, caps) (its first frame dropped when drop_first: the silence frame a
    fresh row decodes) and ends, flushed, with the frame of the tick on which the row consumed EOS or took its last
    capped frame -- the serving loop's own end rule, so nothing past a row's end reaches its stream."""

    def __init__(self, rows: int, in_sr: int, out_sr: int, frame: int, dev, atten_db: float = 120.0,
                 pass_frac: float = 0.9, f32_out: bool = False):
        self.rows, self.in_sr, self.out_sr, self.frame, self.dev = int(rows), int(in_sr), int(out_sr), int(frame), dev
        up, down, h = design_filter(in_sr, out_sr, atten_db, pass_frac)
        self.up, self.down, self.h = up, down, h
        self.half = (len(h) - 1) // 2
        tab = polyphase_table(h, up, RS_KC)
        self.taps = tab.shape[0]
        self.table = torch.from_numpy(tab).to(dev)
        r32 = lambda n: -(-n // 32) * 32
        self.hist_len = r32(self.taps + down // up + 2)
        self.zpad = r32(self.half // up + down // up + 2)
        # outputs a step: a frame's (at most frame up / down + 1) plus a flush's tail (at most (half + 1) / down + 2)
        self.out_max = -(-(frame * up // down + 1 + self.half // down + 3) // 16) * 16
        per = max(128, -(-self.out_max // RS_PT))
        self.period = -(-per // up) * up
        if self.period > 512:
            raise ValueError(f"{in_sr} -> {out_sr} Hz: {self.period} threads a row would be needed")
        self.hist = torch.zeros(rows, self.hist_len, dtype=torch.float32, device=dev)
        self.n_in = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.n_out = torch.zeros(rows, dtype=torch.int64, device=dev)
        self.left = torch.zeros(rows, dtype=torch.int32, device=dev)
        self.flags = torch.full((rows,), 2, dtype=torch.int32, device=dev)    # no stream until a reset
        self.pcm = torch.zeros(rows, self.out_max, dtype=torch.int16, device=dev)
        self.f32 = torch.zeros(rows, self.out_max, dtype=torch.float32, device=dev) if f32_out else None
        self.counts = torch.zeros(rows, dtype=torch.int32, device=dev)
        self._args = torch.zeros(2, rows, dtype=torch.int32, device=dev)
        self.desc = L.A8Resample(
            table=L.ptr(self.table), hist=L.ptr(self.hist), n_in=L.ptr(self.n_in), n_out=L.ptr(self.n_out),
            left=L.ptr(self.left), flags=L.ptr(self.flags), up=up, down=down, taps=self.taps,
            hist_len=self.hist_len, zpad=self.zpad, frame=self.frame, rows=self.rows, out_max=self.out_max,
            period=self.period, half=self.half)

    def reset(self, slots: Sequence[int], caps: Sequence[int], drop_first: bool = True):
        n = len(slots)
        if n == 0:
            return
        assert n <= self.rows and len(caps) == n
        self._args[:, :n].copy_(torch.tensor([list(slots), [max(1, int(c)) for c in caps]], dtype=torch.int32),
                                non_blocking=True)
        L.call("a8_resample_reset", C.byref(self.desc), L.ptr(self._args[0]), L.ptr(self._args[1]), n,
               int(bool(drop_first)), L.stream_handle())

    def step(self, audio: torch.Tensor, tok_in: torch.Tensor, eos: int, b: int):
        """Rows [0, b): audio fp32 [>= b, frame], tok_in int64 [>= b]. Returns (pcm int16 [b, out_max], counts int32
        [b]) -- views overwritten by the next step; row r's new samples are pcm[r, :counts[r]]."""
        assert audio.dtype == torch.float32 and audio.shape[1] >= self.frame and tok_in.dtype == torch.int64
        L.call("a8_resample_step", C.byref(self.desc), L.ptr(audio), audio.stride(0), L.ptr(tok_in), int(eos), int(b),
               L.ptr(self.pcm), L.ptr(self.f32), self.out_max, L.ptr(self.counts), L.stream_handle())
        return self.pcm[:b], self.counts[:b]

    @staticmethod
    def total_outputs(n_in: int, up: int, down: int) -> int:
        return -(-n_in * up // down)

