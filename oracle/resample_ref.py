"""CPU oracle of the per-slot streaming resampler -- TEST INFRASTRUCTURE ONLY (imported by tests/, never by the
product path).

What it restates. The reference converts each request's audio from the codec's rate to out_sr on the host with
python-soxr (`soxr.ResampleStream(native_sr, out_sr, 1, dtype="float32", quality=...)`, fed chunk by chunk with
`resample_chunk(y, last=final)`, serve/engine_worker.py:443-449, :460-461) and sends `_pcm16(y)`
(serve/engine_worker.py:423-424: clip to [-1, 1], x 32767, cast to int16). python-soxr (libsoxr) is a third-party
dependency that is not installed in this image, so soxr's own filters cannot be reproduced here: this oracle keeps
soxr's streaming contract (state carried across chunks, a flush on the last chunk, ceil(N out_sr / in_sr) samples
in all, delay-compensated output) over an explicit linear-phase FIR h at the up-sampled rate:

    y[n] = sum_j up h[j] u[n down + half - j],   u[i] = x[i / up] if up divides i else 0,   half = (len(h) - 1) / 2

evaluated per output in polyphase form, x zero outside [0, N). It is pinned against scipy.signal.resample_poly
(an independent implementation of the same sum, window=h) in tests/test_resample.py; parity with soxr's own output
is not pinned.

`SlotStreams` mirrors the device's per-slot state machine (csrc/resample.cu): a stream per slot, the first frame
dropped, the last frame the one on which the row consumed EOS or took its last capped frame -- the serving loop's
rule (serve/engine_worker.py:1146-1251).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np


def pcm16(y: np.ndarray) -> np.ndarray:
    """serve/engine_worker.py:423-424 on float32 samples, as int16 values."""
    return (np.clip(np.asarray(y, dtype=np.float32), -1.0, 1.0) * 32767.0).astype("<i2")


class StreamResampler:
    """soxr.ResampleStream's chunked contract over the FIR h (float64), rate change up / down."""

    def __init__(self, h: np.ndarray, up: int, down: int):
        self.h = np.asarray(h, dtype=np.float64) * up
        self.up, self.down = int(up), int(down)
        self.half = (len(h) - 1) // 2
        self.taps = -(-len(h) // up)
        hp = np.zeros(self.taps * up)
        hp[:len(h)] = self.h
        self.table = hp.reshape(self.taps, up)          # table[k, p] = up h[p + k up]
        self.x = np.zeros(0)
        self.n_out = 0
        self.ended = False

    def _outputs(self, n0: int, n1: int) -> np.ndarray:
        if n1 <= n0:
            return np.zeros(0)
        n = np.arange(n0, n1, dtype=np.int64)
        q = n * self.down + self.half
        m, p = q // self.up, q % self.up
        idx = m[:, None] - np.arange(self.taps)[None, :]
        ok = (idx >= 0) & (idx < len(self.x))
        xs = np.where(ok, self.x[np.clip(idx, 0, max(0, len(self.x) - 1))] if len(self.x) else 0.0, 0.0)
        return (self.table[:, p].T * xs).sum(1)

    def resample_chunk(self, x: np.ndarray, last: bool = False) -> np.ndarray:
        assert not self.ended
        self.x = np.concatenate([self.x, np.asarray(x, dtype=np.float64)])
        N = len(self.x)
        if last:
            n_end = -(-N * self.up // self.down)
            self.ended = True
        else:
            n_end = max(self.n_out, (N * self.up - 1 - self.half) // self.down + 1)
        y = self._outputs(self.n_out, n_end)
        self.n_out = n_end
        return y


class SlotStreams:
    """The device resampler's slots: reset(slots, caps, drop_first), step(audio, tok_in, eos, b) -> per row the
    new samples (float64)."""

    def __init__(self, rows: int, h: np.ndarray, up: int, down: int):
        self.h, self.up, self.down = h, up, down
        self.rs: List[Optional[StreamResampler]] = [None] * rows
        self.skip = [False] * rows
        self.left = [0] * rows

    def reset(self, slots, caps, drop_first=True):
        for s, c in zip(slots, caps):
            self.rs[s] = StreamResampler(self.h, self.up, self.down)
            self.skip[s] = bool(drop_first)
            self.left[s] = max(1, int(c))

    def step(self, audio: np.ndarray, tok_in: np.ndarray, eos: int, b: int) -> List[np.ndarray]:
        out = []
        for r in range(b):
            rs = self.rs[r]
            if rs is None or rs.ended:
                out.append(np.zeros(0))
                continue
            end = int(tok_in[r]) == int(eos)
            if self.skip[r]:
                self.skip[r] = False
                if end:
                    rs.ended = True
                out.append(np.zeros(0))
                continue
            self.left[r] -= 1
            out.append(rs.resample_chunk(np.asarray(audio[r], dtype=np.float32), last=end or self.left[r] <= 0))
        return out
