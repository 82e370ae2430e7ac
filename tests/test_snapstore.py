"""The codec-snapshot store (FastEngine.voc_snaps; the reference's SnapStore, serve/fast_engine.py:495-564) on the CPU:
memory-only by default; with a directory every snapshot is a file named by its voice's reference-code fingerprint,
kept across restarts, read back on a miss; residents never leave memory, the others are an LRU of `ram`."""
import importlib
from types import SimpleNamespace

import pytest
import torch


@pytest.fixture(scope="module")
def ss(a8):
    return importlib.import_module(a8.__name__ + ".snapstore")


def _snap(v):
    return ([torch.full((1, 64), v, dtype=torch.uint8)], torch.arange(10) + v)


def _same(a, b):
    return all(torch.equal(x, y) for x, y in zip(a[0], b[0])) and torch.equal(a[1], b[1])


def test_ref_fp(ss):
    a = SimpleNamespace(ref_code=torch.arange(40).reshape(4, 10))
    b = SimpleNamespace(ref_code=torch.arange(40).reshape(4, 10) + 1)
    assert ss.ref_fp(a) == ss.ref_fp(SimpleNamespace(ref_code=torch.arange(40).reshape(4, 10)))
    assert ss.ref_fp(a) != ss.ref_fp(b) and ss.ref_fp(SimpleNamespace()) == 0


def test_memory_only_keeps_everything(ss):
    st = ss.SnapStore(ram=1)
    for k in range(5):
        st[f"v{k}"] = _snap(k)
    assert len(st) == 5 and all(f"v{k}" in st for k in range(5)) and st.on_disk() == 0
    assert _same(st["v3"], _snap(3)) and st.get("nope") is None and st.loads == 0


def test_disk_lru_residents_and_restart(ss, tmp_path):
    st = ss.SnapStore(str(tmp_path), ram=2)
    for k in range(4):
        st.set_fp(f"v{k}", 100 + k)
    st.resident = {"v0"}
    for k in range(4):
        st[f"v{k}"] = _snap(k)
    assert st.on_disk() == 4 and len(st) == 3                 # v0 pinned + the 2 most recent others (v2, v3)
    assert sorted(st.keys()) == ["v0", "v2", "v3"]
    assert "v1" in st                                         # on disk
    got = st.get("v1")
    assert _same(got, _snap(1)) and st.loads == 1            # read back: now v3, v1 are the LRU's two
    assert sorted(st.keys()) == ["v0", "v1", "v3"]
    st.get("v3")
    st.set_fp("v4", 7)
    st["v4"] = _snap(4)
    assert sorted(st.keys()) == ["v0", "v3", "v4"]            # v1 was least recently used
    # a new process on the same directory finds every snapshot by key + fingerprint
    st2 = ss.SnapStore(str(tmp_path), ram=8)
    assert "v2" not in st2                                    # no fingerprint known yet
    st2.set_fp("v2", 102)
    assert "v2" in st2 and _same(st2["v2"], _snap(2)) and st2.loads == 1


def test_fingerprint_change_drops_stale(ss, tmp_path):
    st = ss.SnapStore(str(tmp_path))
    st.set_fp("v", 1)
    st["v"] = _snap(1)
    st.set_fp("v", 2)                                          # the voice was rebuilt from other codes
    assert "v" not in st and st.get("v") is None
    st["v"] = _snap(2)
    assert st.on_disk() == 2 and _same(st["v"], _snap(2))


def test_keys_stay_inside_the_directory(ss, tmp_path):
    """Client-chosen voice keys with path separators or `..` are stored under a hashed name inside the directory."""
    d = tmp_path / "snaps"
    st = ss.SnapStore(str(d), ram=1)
    for i, key in enumerate(("../escape", "a/b", "/abs", "..", ".hidden", "ok-key_1.v2")):
        st.set_fp(key, 7 + i)
        st[key] = _snap(i)
    names = sorted(p.name for p in d.iterdir())
    assert len(names) == 6 and all(p.parent == d for p in d.iterdir())
    assert not (tmp_path / "escape.00000007.snap").exists()
    assert "ok-key_1.v2.0000000c.snap" in names
    st2 = ss.SnapStore(str(d), ram=1)
    for i, key in enumerate(("../escape", "a/b", "/abs", "..", ".hidden", "ok-key_1.v2")):
        st2.set_fp(key, 7 + i)
        assert key in st2 and _same(st2[key], _snap(i))
