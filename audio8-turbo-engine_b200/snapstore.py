"""The voices' codec snapshots (FastEngine.voc_snaps): key -> ([state blobs], last reference frame).

Drop-in for the reference's SnapStore and ref_fp (serve/fast_engine.py:495-564), which the worker installs as
`fe.voc_snaps` with TTS_SNAP_DIR / TTS_SNAP_RAM (serve/engine_worker.py:643-670). Without a path every snapshot stays
in host memory (the engine's default). With a path every snapshot is also a file `<path>/<key>.<fp:08x>.snap`, fp a
CRC-32 of the voice's reference codes, made once and reused across restarts (a voice rebuilt from other codes gets
another file); host memory keeps the `resident` keys (the pinned voices) plus the `ram` most recently used others,
and a miss is read back from its file. The state blobs are this engine's (one uint8 blob of every codec state
segment of a row, `StreamingVocoder.snapshot`), so the files are not interchangeable with the reference's.
"""
from __future__ import annotations

import hashlib
import os
import re
import zlib
from collections import OrderedDict
from typing import Dict, Optional

import numpy as np
import torch


def ref_fp(item) -> int:
    """CRC-32 of a voice's reference codes as int32 (0 without codes): names the file its snapshot is kept in."""
    rc = getattr(item, "ref_code", None)
    if rc is None:
        return 0
    return zlib.crc32(np.ascontiguousarray(torch.as_tensor(rc).detach().cpu().numpy().astype(np.int32)).tobytes())


class SnapStore:
    """Residents (the pinned voices) live in their own map and are never evicted; every other snapshot sits in an LRU
    of at most `ram` entries (only with a path: without one nothing could be read back, so nothing is dropped)."""

    def __init__(self, path: Optional[str] = None, ram: int = 2048):
        self.path, self.ram = path, int(ram)
        self._pinned: Dict[str, tuple] = {}
        self._lru: "OrderedDict[str, tuple]" = OrderedDict()
        self._resident: set = set()
        self.fp: Dict[str, int] = {}
        self.loads = 0                                  # snapshots read back from disk (misses)
        if path:
            os.makedirs(path, exist_ok=True)

    # the pinned keys: assigning moves their snapshots out of (or back into) the LRU
    @property
    def resident(self) -> set:
        return self._resident

    @resident.setter
    def resident(self, keys):
        self._resident = set(keys)
        for k in [k for k in self._pinned if k not in self._resident]:
            self._lru[k] = self._pinned.pop(k)
        for k in [k for k in self._lru if k in self._resident]:
            self._pinned[k] = self._lru.pop(k)
        self._trim()

    _PLAIN = re.compile(r"[A-Za-z0-9_][A-Za-z0-9_.-]{0,127}")

    def _file(self, key: str) -> Optional[str]:
        """`<key>.<fp:08x>.snap` inside the directory. Voice keys come from clients: a key that is not a plain file
        name (a path separator, `..`, a leading dot, other characters) is named by its SHA-1 instead, so no key
        reaches outside the directory."""
        if not self.path or key not in self.fp:
            return None
        k = str(key)
        if not self._PLAIN.fullmatch(k) or ".." in k:
            k = "_h" + hashlib.sha1(k.encode("utf-8", "surrogatepass")).hexdigest()[:24]
        return os.path.join(self.path, f"{k}.{self.fp[key]:08x}.snap")

    def set_fp(self, key: str, fp: int):
        """The fingerprint of the codes `key`'s snapshot is (to be) made from; another one drops the stale copy."""
        if key in self.fp and self.fp[key] != int(fp):
            self._pinned.pop(key, None)
            self._lru.pop(key, None)
        self.fp[key] = int(fp)

    def _cached(self, key):
        if key in self._pinned:
            return self._pinned[key]
        v = self._lru.get(key)
        if v is not None:
            self._lru.move_to_end(key)
        return v

    def __contains__(self, key) -> bool:
        if key in self._pinned or key in self._lru:
            return True
        f = self._file(key)
        return f is not None and os.path.exists(f)

    def __len__(self) -> int:
        return len(self._pinned) + len(self._lru)

    def get(self, key, default=None):
        v = self._cached(key)
        if v is not None:
            return v
        f = self._file(key)
        if f is None or not os.path.exists(f):
            return default
        blobs, last = torch.load(f, map_location="cpu", weights_only=True)
        if torch.cuda.is_available():
            blobs = [t.pin_memory() for t in blobs]
        self.loads += 1
        v = (blobs, last)
        self._put(key, v)
        return v

    def __getitem__(self, key):
        v = self.get(key)
        if v is None:
            raise KeyError(key)
        return v

    def __setitem__(self, key, v):
        f = self._file(key)
        if f is not None:                               # written whole, then renamed: a reader never sees half
            torch.save(([t.cpu() for t in v[0]], v[1].cpu()), f + ".part")
            os.replace(f + ".part", f)
        self._put(key, v)

    def _put(self, key, v):
        if key in self._resident:
            self._pinned[key] = v
            return
        self._lru[key] = v
        self._lru.move_to_end(key)
        self._trim()

    def _trim(self):
        while self.path and len(self._lru) > self.ram:
            self._lru.popitem(last=False)

    def values(self):
        return list(self._pinned.values()) + list(self._lru.values())

    def keys(self):
        return list(self._pinned) + list(self._lru)

    def __iter__(self):
        return iter(self.keys())

    def on_disk(self) -> int:
        return len(os.listdir(self.path)) if self.path else 0
