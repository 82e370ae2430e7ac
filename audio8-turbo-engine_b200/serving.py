"""Continuous batching over a FastEngine: the fixed-slot serving loop of serve/engine_worker.py:590-1251 (fast_main),
without its process plumbing, text segmentation and audio post-processing -- the part that decides what the GPU runs.

Per iteration: requests that have arrived wait in a queue; every `admit_every` ticks (or as soon as `admit_batch`
wait, or when nothing runs) they are admitted into the lowest free slots in ONE packed prefill (``FastEngine.admit``,
engine_worker.py:1105-1140); then the tick of the bucket covering the highest busy slot is replayed
(``FastEngine.replay(fe.bucket_for(busy[-1] + 1))``, engine_worker.py:1168-1172) and its consumed tokens and audio are
copied to pinned host buffers asynchronously and read one tick later (engine_worker.py:1180-1215). The vocoder runs
one frame behind the AR: a row's first tick yields the audio of its silence frame, which is dropped. Frames go out as
chunks of 1, 2, 4, then 6 frames (the worker's ramp), the rest when the row ends; `pcm16` is the worker's int16
conversion. A row ends on EOS or at its frame cap, and its slot is free for the next admission.

Timing is wall clock, as the reference's serving numbers (README "Results": RTF = wall time / audio duration, TTFA
included): TTFA = first audio frame on the host - arrival; RTF = (last frame on the host - arrival) / audio length.

Three drivers use the loop: an open-loop trace (Poisson arrivals, ``poisson_trace``), closed-loop "N streams
sustained" users that ask again as soon as their utterance ends (``ClosedLoop``), and the replica scale-out, where a
host scheduler assigns each request of one global trace to the least-loaded replica (``assign_least_loaded``).
"""
from __future__ import annotations

import heapq
import time
from collections import deque
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

FRAME_S = 2048 / 44100          # one codec frame of audio (2048 samples at 44.1 kHz)


@dataclass
class Request:
    rid: int
    arrival: float                # seconds after the start of the run
    text: str
    item: object                  # the voice reference (ref_code [T, ncb], ref_text)
    key: str                      # the voice's prefix-cache key
    cap: int                      # frames to generate (the request ends earlier on EOS)
    user: int = -1                # closed-loop user that issued it
    slot: int = -1
    started: bool = False
    frames: int = 0
    t_admit: Optional[float] = None
    t_first: Optional[float] = None
    t_done: Optional[float] = None
    eos: bool = False
    rejected: bool = False
    cancelled: bool = False       # the client went away (engine_worker.py:1125-1143): ended without its audio
    error: Optional[str] = None   # why it failed (engine_worker.py:828-832, :883, :893, :1186-1190)
    pend: list = field(default_factory=list)   # frames not yet emitted as a chunk
    target: int = 0                            # frames the next chunk waits for
    chunks: int = 0

    def as_admit(self):
        return dict(text=self.text, item=self.item, key=self.key)


@dataclass
class RunStats:
    requests: List[Request] = field(default_factory=list)
    ticks: int = 0
    rows_ticked: int = 0
    busy_time: float = 0.0        # sum over ticks of (rows busy x tick wall time): time-averaged concurrency
    admits: int = 0
    wall: float = 0.0
    frame_s: float = FRAME_S
    buckets: Dict[int, int] = field(default_factory=dict)

    def finished(self):
        return [r for r in self.requests if r.t_done is not None and r.frames > 0 and not r.cancelled
                and r.error is None]

    def summary(self):
        done = self.finished()
        ttfa = np.array([r.t_first - r.arrival for r in done]) * 1000.0
        rtf = np.array([(r.t_done - r.arrival) / (r.frames * self.frame_s) for r in done])
        pct = lambda a, q: float(np.percentile(a, q)) if len(a) else float("nan")
        frames = sum(r.frames for r in done)
        return {
            "requests": len(self.requests), "finished": len(done),
            "rejected": sum(r.rejected for r in self.requests), "eos": sum(r.eos for r in done),
            "cancelled": sum(r.cancelled for r in self.requests),
            "failed": sum(r.error is not None and not r.rejected for r in self.requests),
            "ttfa_ms_p50": round(pct(ttfa, 50), 1), "ttfa_ms_p95": round(pct(ttfa, 95), 1),
            "rtf_p50": round(pct(rtf, 50), 4), "rtf_p95": round(pct(rtf, 95), 4),
            "mean_streams": round(self.busy_time / max(1e-9, self.wall), 1),
            "peak_streams": max((b for b in self.buckets), default=0),
            "ticks": self.ticks, "admissions": self.admits, "wall_s": round(self.wall, 2),
            "frames": frames, "frames_per_s": round(frames / max(1e-9, self.wall), 1),
        }


class _HostEvent:
    """Stands in for a CUDA event when the engine's tensors live on the CPU (tests of the scheduling logic)."""

    def record(self):
        pass

    def synchronize(self):
        pass


class ContinuousBatcher:
    """The serving loop over one engine (one GPU).

    `engine` provides B, eos, up, sr, tok_in [B] and audio [B, up] (device tensors the tick writes), bucket_for(n),
    admit(slots, reqs) -> prompt lengths (-1: rejected) and replay(b)."""

    def __init__(self, engine, admit_every: int = 2, admit_batch: int = 8, max_admit: int = 64, nbuf: int = 4,
                 copy_audio: bool = True, first_chunk: int = 1, chunk_frames: int = 6, out_sr: Optional[int] = None,
                 resampler=None):
        self.fe = engine
        # streamed chunks (engine_worker.py:696-697, :1246-1248): the first after `first_chunk` frames (the
        # reference's TTS_FIRST_CHUNK_FRAMES), then doubling up to `chunk_frames` (TTS_FRAMES_PER_CHUNK); the rest
        # when the row ends
        self.first_chunk, self.chunk_frames = max(1, first_chunk), max(1, chunk_frames)
        self.admit_every, self.admit_batch, self.max_admit = admit_every, admit_batch, max_admit
        self.nbuf = max(2, nbuf)
        self.copy_audio = copy_audio
        cuda = engine.tok_in.is_cuda
        pin = (lambda t: t.pin_memory()) if cuda else (lambda t: t)
        B = engine.B
        self.tok_h = pin(torch.empty(self.nbuf, B, dtype=torch.int64))
        self.aud_h = pin(torch.empty(self.nbuf, B, engine.up, dtype=torch.float32)) if copy_audio else None
        # out_sr: each slot's audio converted to out_sr and PCM16 on the device, one launch a tick after the replay
        # (the worker's per-request soxr stream + _pcm16, engine_worker.py:443-461); the host reads int16 rows
        if resampler is None and out_sr is not None and int(out_sr) > 0:
            from .resample import Resampler
            resampler = Resampler(B, engine.sr, int(out_sr), engine.up, engine.audio.device)
        self.rs = resampler
        if self.rs is not None:
            self.pcm_h = pin(torch.empty(self.nbuf, B, self.rs.out_max, dtype=torch.int16))
            self.cnt_h = pin(torch.empty(self.nbuf, B, dtype=torch.int32))
        self.events = [torch.cuda.Event() if cuda else _HostEvent() for _ in range(self.nbuf)]
        # on_audio(request, frame): fp32 [up] at the native rate (copy_audio), or with a resampler its int16 samples
        self.on_audio: Optional[Callable[[Request, torch.Tensor], None]] = None
        # on_chunk(request, pcm as numpy, final): a chunk of consecutive frames, as the worker emits -- fp32 [n * up]
        # at the native rate, or with a resampler int16 at out_sr (the last chunk carries the flushed tail)
        self.on_chunk: Optional[Callable[[Request, np.ndarray, bool], None]] = None
        # on_error(request, message): the worker's ("__error__", message), followed by the request's final chunk
        self.on_error: Optional[Callable[[Request, str], None]] = None
        self._cancels: deque = deque()

    def cancel(self, rid: int):
        """The client of request `rid` went away (the worker's ("__cancel__", rid) message): a running request ends
        at the next iteration and frees its slot, a waiting one is dropped; either gets an empty final chunk (the
        worker's end-of-stream). Safe to call from callbacks or another thread; unknown or ended ids are ignored."""
        self._cancels.append(rid)

    def run(self, requests: List[Request], follow: Optional[Callable[[Request, float], Optional[Request]]] = None,
            clock=time.perf_counter, sleep=time.sleep) -> RunStats:
        """Serve `requests` (each admitted once its arrival time has passed) until all have ended. `follow(r, t)`
        may return the next request of r's user when r ends at time t (closed loop); it is queued at once."""
        fe = self.fe
        eos = int(fe.eos)
        st = RunStats(requests=list(requests), frame_s=fe.up / fe.sr)
        pending = deque(sorted(requests, key=lambda r: r.arrival))
        waiting: deque = deque()
        free = list(range(fe.B))
        heapq.heapify(free)
        rows: Dict[int, Request] = {}
        inflight: deque = deque()
        tick, last_admit = 0, -10 ** 9
        t0 = clock()
        now = lambda: clock() - t0
        t_prev = None
        def end_stream(r):
            if self.on_chunk is not None:
                self.on_chunk(r, np.zeros(0, np.float32 if self.rs is None else np.int16), True)

        def end_cancelled(r, t):
            r.cancelled, r.t_done, r.pend = True, t, []
            end_stream(r)

        def end_failed(r, msg, t):
            r.error, r.pend = msg, []
            if t is not None:
                r.t_done = t
            if self.on_error is not None:
                self.on_error(r, msg)
            end_stream(r)

        while pending or waiting or rows or inflight:
            t = now()
            while self._cancels:
                rid = self._cancels.popleft()
                s_run = next((s for s, r in rows.items() if r.rid == rid), None)
                if s_run is not None:
                    r = rows.pop(s_run)
                    heapq.heappush(free, s_run)
                    end_cancelled(r, t)
                    continue
                for q in (waiting, pending):
                    r = next((r for r in q if r.rid == rid), None)
                    if r is not None:
                        q.remove(r)
                        end_cancelled(r, t)
                        break
            while pending and pending[0].arrival <= t:
                waiting.append(pending.popleft())
            if not rows and not waiting and not inflight:
                if pending:                                   # idle until the next arrival (none left: done)
                    sleep(max(0.0, min(0.05, pending[0].arrival - t)))
                t_prev = None
                continue
            if waiting and free and (not rows or tick - last_admit >= self.admit_every
                                     or len(waiting) >= self.admit_batch):
                take = min(len(waiting), len(free), self.max_admit)
                slots = [heapq.heappop(free) for _ in range(take)]
                reqs = [waiting.popleft() for _ in range(take)]
                try:
                    lens = fe.admit(slots, [r.as_admit() for r in reqs])
                except Exception:                             # the whole admission fails; its slots are freed
                    lens = None
                st.admits += 1
                ta = now()
                if lens is None:
                    for r, s in zip(reqs, slots):
                        heapq.heappush(free, s)
                        end_failed(r, "engine error", ta)
                else:
                    for r, s, n in zip(reqs, slots, lens):
                        if n < 0:                             # prompt too long for the engine
                            r.rejected = True
                            heapq.heappush(free, s)
                            end_failed(r, "text too long for TTS_MAX_SEQ", None)
                        else:
                            r.slot, r.t_admit = s, ta
                            rows[s] = r
                    if self.rs is not None:
                        ok = [r for r in reqs if not r.rejected]
                        self.rs.reset([r.slot for r in ok], [r.cap for r in ok])
                last_admit = tick
            busy = sorted(rows)
            if busy:
                b = fe.bucket_for(busy[-1] + 1)
                try:
                    fe.replay(b)
                except Exception:                             # a failed tick ends every running row
                    tf = now()
                    for s in busy:
                        heapq.heappush(free, s)
                        end_failed(rows.pop(s), "engine error", tf)
                    inflight.clear()
                    t_prev = None
                    continue
                j = tick % self.nbuf
                self.tok_h[j, :b].copy_(fe.tok_in[:b], non_blocking=True)
                if self.copy_audio:
                    self.aud_h[j, :b].copy_(fe.audio[:b], non_blocking=True)
                if self.rs is not None:
                    pcm, cnt = self.rs.step(fe.audio, fe.tok_in, eos, b)
                    self.pcm_h[j, :b].copy_(pcm, non_blocking=True)
                    self.cnt_h[j, :b].copy_(cnt, non_blocking=True)
                self.events[j].record()
                inflight.append((j, [(s, rows[s]) for s in busy]))
                tick += 1
                st.ticks += 1
                st.rows_ticked += len(busy)
                st.buckets[len(busy)] = st.buckets.get(len(busy), 0) + 1
            while inflight and (len(inflight) > 1 or not busy):
                j, snap = inflight.popleft()
                self.events[j].synchronize()
                t = now()
                if t_prev is not None:
                    st.busy_time += len(snap) * (t - t_prev)
                t_prev = t
                toks = self.tok_h[j].tolist()
                cnts = self.cnt_h[j].tolist() if self.rs is not None else None
                for s, r in snap:
                    if rows.get(s) is not r:
                        continue
                    if r.started:
                        r.frames += 1
                        if r.frames == 1:
                            r.t_first = t
                        out = self.aud_h[j, s] if self.rs is None else self.pcm_h[j, s, :cnts[s]]
                        if self.on_audio is not None:
                            self.on_audio(r, out)
                        if self.on_chunk is not None:
                            r.pend.append(out.numpy().copy())
                    else:
                        r.started = True                      # the first tick decodes the silence frame
                        r.target = self.first_chunk
                    end = toks[s] == eos or r.frames >= r.cap
                    if self.on_chunk is not None and r.pend and (end or len(r.pend) >= r.target):
                        self.on_chunk(r, np.concatenate(r.pend), end)
                        r.pend, r.chunks = [], r.chunks + 1
                        r.target = min(self.chunk_frames, r.target * 2)
                    elif self.on_chunk is not None and end:
                        self.on_chunk(r, np.zeros(0, np.float32 if self.rs is None else np.int16), True)
                    if end:
                        r.eos = toks[s] == eos
                        r.t_done = t
                        del rows[s]
                        heapq.heappush(free, s)
                        if follow is not None:
                            nxt = follow(r, t)
                            if nxt is not None:
                                st.requests.append(nxt)
                                waiting.append(nxt)
        st.wall = now()
        return st


# ------------------------------------------------------------------------------------------------ traces
def pcm16(y: np.ndarray) -> bytes:
    """fp32 PCM in [-1, 1] to little-endian int16 bytes, as the worker sends it (engine_worker.py:423-424)."""
    return (np.clip(y, -1.0, 1.0) * 32767.0).astype("<i2").tobytes()


def voice_items(n_voices: int, frames: int, ncb: int, seed: int):
    """n_voices cached voices, each a reference of `frames` uniform-random code frames and a short transcript."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for v in range(n_voices):
        codes = torch.randint(0, 4096, (frames, ncb), generator=g)
        text = " ".join(str(int(x)) for x in torch.randint(0, 151643, (12,), generator=g))
        out.append((f"voice{v}", SimpleNamespace(ref_code=codes, ref_text=text)))
    return out


class _Draw:
    """One request's text, voice and length: U[text_lo, text_hi] random token ids (the stand-in tokenizer takes an
    integer word as its id), one of the cached voices, geometric output length with mean `mean_frames`, capped."""

    def __init__(self, rng, voices, text_lo=20, text_hi=200, mean_frames=300.0, cap=1024):
        self.rng, self.voices = rng, voices
        self.text_lo, self.text_hi, self.p, self.cap = text_lo, text_hi, 1.0 / mean_frames, cap
        self.n = 0

    def __call__(self, arrival, user=-1):
        rng = self.rng
        n = int(rng.integers(self.text_lo, self.text_hi + 1))
        key, item = self.voices[int(rng.integers(0, len(self.voices)))]
        frames = min(self.cap, int(rng.geometric(self.p)))
        r = Request(rid=self.n, arrival=float(arrival), text=" ".join(str(int(x)) for x in rng.integers(0, 151643, n)),
                    item=item, key=key, cap=frames, user=user)
        self.n += 1
        return r


def poisson_trace(rate: float, seconds: float, seed: int, ncb: int, n_voices: int = 8, voice_frames: int = 150,
                  **draw):
    """Open-loop trace: Poisson arrivals at `rate` req/s for `seconds`; returns (requests, voices)."""
    rng = np.random.default_rng(seed)
    voices = voice_items(n_voices, voice_frames, ncb, seed + 1)
    d = _Draw(rng, voices, **draw)
    reqs, t = [], 0.0
    while True:
        t += rng.exponential(1.0 / rate)
        if t >= seconds:
            break
        reqs.append(d(t))
    return reqs, voices


class ClosedLoop:
    """`streams` users for `seconds`: each starts within the first `ramp` seconds and asks for its next utterance as
    soon as the previous one has been delivered (the reference's "N streams, sustained 60 s" load)."""

    def __init__(self, streams: int, seconds: float, seed: int, ncb: int, n_voices: int = 8, voice_frames: int = 150,
                 ramp: float = 2.0, **draw):
        rng = np.random.default_rng(seed)
        self.voices = voice_items(n_voices, voice_frames, ncb, seed + 1)
        self.draw = _Draw(rng, self.voices, **draw)
        self.seconds = seconds
        self.initial = [self.draw(float(rng.uniform(0, ramp)), user=u) for u in range(streams)]

    def follow(self, r: Request, t: float) -> Optional[Request]:
        return self.draw(t, user=r.user) if t < self.seconds else None


def assign_least_loaded(reqs: List[Request], replicas: int, frame_s: float = FRAME_S, est_rtf: float = 0.5):
    """Host scheduler of the replica scale-out: each request of the global trace, in arrival order, goes to the
    replica with the fewest streams in flight (ties: lowest index). In-flight counts are the scheduler's own
    estimate -- a stream occupies its replica for `cap` frames at `est_rtf` x real time -- so every rank computes
    the same assignment from the same trace without exchanging anything. Returns one replica index per request."""
    ends = [[] for _ in range(replicas)]
    out = []
    for r in sorted(reqs, key=lambda q: q.arrival):
        for h in ends:
            while h and h[0] <= r.arrival:
                heapq.heappop(h)
        k = min(range(replicas), key=lambda i: (len(ends[i]), i))
        heapq.heappush(ends[k], r.arrival + r.cap * frame_s * est_rtf)
        out.append((r.rid, k))
    order = dict(out)
    return [order[r.rid] for r in reqs]


@torch.inference_mode()
def warm_voices(engine, voices):
    """The voices are cached before the trace starts: prefix prompt embeddings and prefix K/V per key
    (engine_worker.py keeps them across requests), plus the codec snapshot when the engine primes voices."""
    if engine._parts is None:
        engine._parts_init()
    for key, item in voices:
        engine._prefix_kv(key, engine._speaker_prefix(key, item))
    engine.prime_speakers(voices)
