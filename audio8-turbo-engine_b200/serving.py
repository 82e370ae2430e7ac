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

Code-switch chains (engine_worker.py:925-1117): a request may carry a ``Chain`` of segments -- a line voiced piece by
piece, each its own generation with its own text and voice. The line holds ONE slot throughout: when a segment ends,
the next is admitted into the same slot with ``keep_voc`` (the codec's state goes on, so the audio is continuous) and
the earlier segments' generated codes and text as the prompt's context (all of them, the last one, or none: the line's
``mode``, overridable per segment). Every tick's frame codes are read back for that context. Between segments the
audio is gated as the worker does: a continuation's leading silence is held and only the last `lead` seconds of it
(by the punctuation ending the previous segment) are sent; a segment's trailing silence is cut to `tail` seconds and
the codes kept as context stop that far after its last voiced frame. A continuation that stays silent for LEAD_MAX
frames, or ends without a voiced frame, is sampled again (at most TRIES_MAX times; from CTX_DROP_TRY on without the
context); one whose prompt no longer fits with its context is admitted without it. Not carried over from the worker:
segments held whole (short texts, drawn-out words, stressed words, sound effects and their post-processing), guided
groups, and a per-line resampler stream -- with ``out_sr`` each segment is its own resampled stream, flushed at the
switch.

Timing is wall clock, as the reference's serving numbers (README "Results": RTF = wall time / audio duration, TTFA
included): TTFA = first audio frame on the host - arrival; RTF = (last frame on the host - arrival) / audio length.

Three drivers use the loop: an open-loop trace (Poisson arrivals, ``poisson_trace``), closed-loop "N streams
sustained" users that ask again as soon as their utterance ends (``ClosedLoop``), and the replica scale-out, where a
host scheduler assigns each request of one global trace to the least-loaded replica (``assign_least_loaded``).
"""
from __future__ import annotations

import heapq
import math
import time
from collections import deque
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

FRAME_S = 2048 / 44100          # one codec frame of audio (2048 samples at 44.1 kHz)

# code-switch chains (engine_worker.py:50-57)
SIL_AMP = 10 ** (-45 / 20)      # a frame whose RMS is below this is silence
LEAD_MAX = 12                   # a continuation silent for longer than this many frames is sampled again ...
TRIES_MAX = 3                   # ... at most this many times
CTX_DROP_TRY = 2                # from this retry on, without the previous segments as context
_SENT_END = set(".!?\u2026\u3002\uff01\uff1f")
_CLAUSE_END = set(",;:\uff0c\u3001\uff1b\uff1a")
_CLOSERS = "\"'\u201d\u2019\u00bb)\uff09]\u300d\u300f"


def text_units(text: str) -> int:
    """Speech length of `text` in Latin letters (engine_worker.py:207-220): a Han character or Hangul block counts
    3, a kana 2, anything else 1."""
    n = 0
    for c in text:
        o = ord(c)
        if 0x4E00 <= o <= 0x9FFF or 0x3400 <= o <= 0x4DBF or 0xF900 <= o <= 0xFAFF or 0xAC00 <= o <= 0xD7AF:
            n += 3
        elif 0x3040 <= o <= 0x30FF:
            n += 2
        else:
            n += 1
    return n


def seg_cap(text: str) -> int:
    """Frame cap of a chain segment, about 3x a normal speech rate (engine_worker.py:222-225)."""
    return 12 + 2 * text_units(text)


def keep_seconds(text: str):
    """(tail, lead): seconds of silence kept at a switch after a segment ending in `text` -- after its last voiced
    frame / before the next segment's first -- by its closing punctuation (engine_worker.py:244-251)."""
    t = text.rstrip().rstrip(_CLOSERS)[-1:]
    return (0.24, 0.16) if t in _SENT_END else (0.16, 0.08) if t in _CLAUSE_END else (0.06, 0.04)


def cut_silence(frames: List[np.ndarray], seconds: float, sr: int, keep_end: bool) -> np.ndarray:
    """`seconds` of the concatenated silent frames -- the head, or the tail with keep_end -- with a 5 ms linear fade
    at the cut (engine_worker.py:390-402). Works on fp32 or int16 samples (returned in the same type)."""
    dt = frames[0].dtype if frames else np.float32
    y = np.concatenate(frames).astype(np.float32) if frames else np.zeros(0, np.float32)
    n = min(y.size, int(round(seconds * sr)))
    y = (y[y.size - n:] if keep_end else y[:n]).copy()
    f = min(n, int(0.005 * sr))
    if f:
        ramp = np.linspace(0.0, 1.0, f, dtype=np.float32)
        if keep_end:
            y[:f] *= ramp
        else:
            y[n - f:] *= ramp[::-1]
    return y.astype(dt) if dt != np.float32 else y


@dataclass
class Segment:
    """One piece of a code-switch line: its text and voice, an optional frame cap (0: seg_cap(text)) and an
    optional context mode of its own ("full" | "prev" | "none")."""
    text: str
    key: str
    item: object
    cap: int = 0
    ctx: Optional[str] = None


@dataclass
class Chain:
    """A line voiced segment by segment in one slot. `mode`: the context each continuation gets -- every finished
    segment ("full"), the last one ("prev", the worker's default) or none. State: the segment running (k), the
    finished segments' (codes [n, ncb] int64, text) in `hist`, and the tries of the current segment."""
    segs: List[Segment]
    mode: str = "prev"
    k: int = 0
    hist: list = field(default_factory=list)
    tries: int = 0


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
    chain: Optional[Chain] = None              # a code-switch line (text / item / key are then its first segment's)
    gen: int = 0                               # admissions so far: ticks replayed for an earlier one are ignored
    seg_frames: int = 0                        # chain rows: frames of the segment running
    codes: list = field(default_factory=list)  # chain rows: the segment's generated frame codes
    vflags: list = field(default_factory=list) # chain rows: whether frame i of the segment sounds
    hold: list = field(default_factory=list)   # chain rows: silent frames held back (a continuation's lead, a tail)
    voiced: bool = False                       # chain rows: the segment has sounded
    lead_drop: int = 0                         # chain rows: leading silent frames of the segment not sent

    def as_admit(self):
        return dict(text=self.text, item=self.item, key=self.key)

    def seg_admit(self):
        """The admission of the chain's current segment: the first as a plain request, a continuation with the
        codec state kept and the context its mode asks for (engine_worker.py:926-945)."""
        ch = self.chain
        seg = ch.segs[ch.k]
        if ch.k == 0:
            return dict(text=seg.text, item=seg.item, key=seg.key)
        mode = seg.ctx or ch.mode
        hist = ch.hist if mode == "full" else ch.hist[-1:] if mode == "prev" else []
        if ch.tries >= CTX_DROP_TRY:
            hist = []
        q = dict(text=seg.text, item=seg.item, key=seg.key, keep_voc=True)
        if hist:
            q["ctx_codes"] = np.concatenate([c for c, _ in hist])
            q["ctx_text"] = " ".join(t for _, t in hist)
        return q

    def seg_cap(self):
        seg = self.chain.segs[self.chain.k]
        return seg.cap if seg.cap > 0 else min(self.cap, seg_cap(seg.text))


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
        self.fr_h = None                          # pinned [nbuf, B, ncb] frame codes, once a chain runs

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
        cont: deque = deque()                 # chain lines between two segments: (request, its reserved slot)
        free = list(range(fe.B))
        heapq.heapify(free)
        rows: Dict[int, Request] = {}
        inflight: deque = deque()
        tick, last_admit = 0, -10 ** 9
        t0 = clock()
        now = lambda: clock() - t0
        t_prev = None
        out_sr = getattr(self.rs, "out_sr", fe.sr)     # rate of the audio the loop delivers
        frame_sec = fe.up / fe.sr
        empty = lambda: np.zeros(0, np.float32 if self.rs is None else np.int16)

        def end_stream(r):
            if self.on_chunk is not None:
                self.on_chunk(r, empty(), True)

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

        def emit(r, final):
            """The pending frames as one chunk (final: the stream's last, possibly empty)."""
            if self.on_chunk is None:
                return
            if r.pend:
                self.on_chunk(r, np.concatenate(r.pend), final)
                r.pend, r.chunks = [], r.chunks + 1
                r.target = min(self.chunk_frames, r.target * 2)
            elif final:
                self.on_chunk(r, empty(), True)

        def finish(r, s, is_eos, t):
            r.eos = is_eos
            r.t_done = t
            del rows[s]
            heapq.heappush(free, s)
            if follow is not None:
                nxt = follow(r, t)
                if nxt is not None:
                    st.requests.append(nxt)
                    waiting.append(nxt)

        # ---- code-switch chains (engine_worker.py:925-1117) ----
        def release(r, a, t):
            """Audio of a chain line that passed the gate goes out."""
            if r.t_first is None:
                r.t_first = t
            if self.on_audio is not None:
                self.on_audio(r, torch.from_numpy(a))
            if self.on_chunk is not None:
                r.pend.append(a)

        def queue_segment(r, s):
            """Segment chain.k of r's line (again, on a retry) into r's slot, which stays reserved."""
            rows.pop(s, None)
            cont.append((r, s))

        def retry_segment(r, s):
            r.chain.tries += 1
            queue_segment(r, s)

        def chain_audio(r, a, v, t):
            """Gate one frame of a chain segment (v: whether it sounds); True if the segment is to be sampled again
            (a continuation silent for too long)."""
            ch = r.chain
            r.vflags.append(v)
            if not r.voiced:
                if v:
                    r.voiced = True
                    if ch.k > 0 and r.hold:         # only the last `lead` seconds of the continuation's silent lead
                        lead = keep_seconds(ch.segs[ch.k - 1].text)[1]
                        r.lead_drop = max(0, len(r.hold) - math.ceil(lead / frame_sec))
                        y = cut_silence(r.hold, lead, out_sr, keep_end=True)
                        if y.size:
                            release(r, y, t)
                    else:
                        for h in r.hold:
                            release(r, h, t)
                    r.hold = []
                    release(r, a, t)
                elif ch.k == 0:                     # the line's first segment is never gated (TTFA)
                    release(r, a, t)
                else:
                    r.hold.append(a)
                    if len(r.hold) > LEAD_MAX and ch.tries < TRIES_MAX:
                        return True
            elif v:
                for h in r.hold:                    # a pause inside the segment: it goes out after all
                    release(r, h, t)
                r.hold = []
                release(r, a, t)
            elif ch.k == len(ch.segs) - 1:
                release(r, a, t)
            else:
                r.hold.append(a)                    # maybe the segment's trailing silence
            return False

        def end_segment(r, s, runaway, t):
            """Segment over (EOS, or its frame cap): sampled again if a continuation never sounded; the line ends
            after its last segment; otherwise the tail is cut, the segment's codes join the context, and the next
            segment is queued into the slot."""
            ch = r.chain
            k = ch.k
            if not r.voiced and k > 0 and ch.tries < TRIES_MAX:
                retry_segment(r, s)
                return
            if k == len(ch.segs) - 1:
                for h in r.hold:
                    release(r, h, t)
                r.hold = []
                emit(r, True)
                finish(r, s, not runaway, t)
                return
            text = ch.segs[k].text
            tail = keep_seconds(text)[0]
            y = cut_silence(r.hold, tail, out_sr, keep_end=False) if r.hold else empty()
            end_ch = text.rstrip().rstrip(_CLOSERS)[-1:]
            pad = int(round(tail * out_sr)) - y.size if end_ch in _SENT_END | _CLAUSE_END else 0
            if pad > 0:                             # a comma / sentence end the voice ran on through
                y = np.concatenate([y, np.zeros(pad, y.dtype)])
            if y.size:
                release(r, y, t)
            r.hold = []
            emit(r, False)
            n = min(len(r.codes), len(r.vflags))
            vi = [i for i in range(n) if r.vflags[i]]
            end = min(n, vi[-1] + 1 + math.ceil(tail / frame_sec)) if vi else n
            if end > r.lead_drop:
                ch.hist.append((np.stack(r.codes[r.lead_drop:end]), text))
            ch.k += 1
            ch.tries = 0
            queue_segment(r, s)

        while pending or waiting or rows or inflight or cont:
            t = now()
            while self._cancels:
                rid = self._cancels.popleft()
                s_run = next((s for s, r in rows.items() if r.rid == rid), None)
                if s_run is not None:
                    r = rows.pop(s_run)
                    heapq.heappush(free, s_run)
                    end_cancelled(r, t)
                    continue
                c = next((c for c in cont if c[0].rid == rid), None)
                if c is not None:                     # between two segments of a line
                    cont.remove(c)
                    heapq.heappush(free, c[1])
                    end_cancelled(c[0], t)
                    continue
                for q in (waiting, pending):
                    r = next((r for r in q if r.rid == rid), None)
                    if r is not None:
                        q.remove(r)
                        end_cancelled(r, t)
                        break
            while pending and pending[0].arrival <= t:
                waiting.append(pending.popleft())
            if not rows and not waiting and not inflight and not cont:
                if pending:                                   # idle until the next arrival (none left: done)
                    sleep(max(0.0, min(0.05, pending[0].arrival - t)))
                t_prev = None
                continue
            if (cont or (waiting and free)) and (not rows or tick - last_admit >= self.admit_every
                                                 or len(waiting) + len(cont) >= self.admit_batch):
                # a line's next segment first (its listener is mid-line), then new requests into the lowest slots
                items = []                                    # (request, slot, admission, continuation)
                while cont and len(items) < self.max_admit:
                    r, s = cont.popleft()
                    items.append((r, s, r.seg_admit(), True))
                take = min(len(waiting), len(free), self.max_admit - len(items))
                for _ in range(max(0, take)):
                    r = waiting.popleft()
                    items.append((r, heapq.heappop(free), r.seg_admit() if r.chain is not None else r.as_admit(),
                                  False))
                try:
                    lens = fe.admit([it[1] for it in items], [it[2] for it in items])
                except Exception:                             # the whole admission fails; its slots are freed
                    lens = None
                if lens is not None:
                    # a continuation whose prompt no longer fits with its context goes on without it
                    redo = [i for i, it in enumerate(items) if lens[i] < 0 and "ctx_codes" in it[2]]
                    if redo:
                        for i in redo:
                            r, s, q, c = items[i]
                            items[i] = (r, s, {k: v for k, v in q.items() if k not in ("ctx_codes", "ctx_text")}, c)
                        lens = list(lens)
                        try:
                            again = fe.admit([items[i][1] for i in redo], [items[i][2] for i in redo])
                        except Exception:
                            again = None
                        for n_i, i in enumerate(redo):
                            lens[i] = again[n_i] if again is not None else None
                st.admits += 1
                ta = now()
                if lens is None:
                    for r, s, _, _ in items:
                        heapq.heappush(free, s)
                        end_failed(r, "engine error", ta)
                else:
                    ok = []
                    for (r, s, _, c), n in zip(items, lens):
                        if n is None:
                            heapq.heappush(free, s)
                            end_failed(r, "engine error", ta)
                        elif n < 0:                           # prompt too long for the engine
                            heapq.heappush(free, s)
                            if c:                             # a line that can't go on
                                end_failed(r, "text too long for TTS_MAX_SEQ", ta)
                            else:
                                r.rejected = True
                                end_failed(r, "text too long for TTS_MAX_SEQ", None)
                        else:
                            r.slot, r.gen, r.started = s, r.gen + 1, False
                            if r.t_admit is None:
                                r.t_admit = ta
                            if r.chain is not None:
                                r.seg_frames, r.codes, r.vflags, r.hold, r.voiced, r.lead_drop = 0, [], [], [], \
                                    False, 0
                            rows[s] = r
                            ok.append(r)
                    if self.rs is not None:
                        self.rs.reset([r.slot for r in ok], [r.seg_cap() if r.chain is not None else r.cap for r in ok])
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
                chained = any(rows[s].chain is not None for s in busy)
                if chained:                                   # the frame codes chain lines keep as context
                    if self.fr_h is None:
                        self.fr_h = torch.empty(self.nbuf, fe.B, fe.frame_prev.shape[1], dtype=torch.int64)
                        if fe.tok_in.is_cuda:
                            self.fr_h = self.fr_h.pin_memory()
                    self.fr_h[j, :b].copy_(fe.frame_prev[:b], non_blocking=True)
                self.events[j].record()
                inflight.append((j, chained, [(s, rows[s], rows[s].gen) for s in busy]))
                tick += 1
                st.ticks += 1
                st.rows_ticked += len(busy)
                st.buckets[len(busy)] = st.buckets.get(len(busy), 0) + 1
            while inflight and (len(inflight) > 1 or not busy):
                j, chained, snap = inflight.popleft()
                self.events[j].synchronize()
                t = now()
                if t_prev is not None:
                    st.busy_time += len(snap) * (t - t_prev)
                t_prev = t
                toks = self.tok_h[j].tolist()
                cnts = self.cnt_h[j].tolist() if self.rs is not None else None
                frs = self.fr_h[j].numpy() if chained else None
                for s, r, g in snap:
                    if rows.get(s) is not r or r.gen != g:    # ended, or an earlier segment's tick
                        continue
                    if r.chain is not None:
                        if r.started:
                            r.frames += 1
                            r.seg_frames += 1
                            if self.rs is None:
                                a = self.aud_h[j, s].numpy().copy()
                                v = float(np.sqrt(np.mean(a * a))) > SIL_AMP
                            else:
                                a = self.pcm_h[j, s, :cnts[s]].numpy().copy()
                                v = a.size > 0 and float(np.sqrt(np.mean((a / 32767.0) ** 2))) > SIL_AMP
                            if chain_audio(r, a, v, t):
                                retry_segment(r, s)
                                continue
                        else:
                            r.started = True                  # the first tick decodes the silence frame
                            r.target = self.first_chunk
                        if toks[s] != eos:
                            r.codes.append(frs[s].copy())
                        if toks[s] == eos or r.seg_frames >= r.seg_cap():
                            end_segment(r, s, toks[s] != eos, t)
                        elif r.pend and len(r.pend) >= r.target:
                            emit(r, False)
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
                    if end or len(r.pend) >= r.target:
                        emit(r, end)
                    if end:
                        finish(r, s, toks[s] == eos, t)
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
