"""audio8-turbo-engine_b200: the Audio8 decode tick on B200 (sm_100a).

``FastEngine`` is the drop-in for the reference's serve/fast_engine.py FastEngine; ``_lib`` binds the C ABI of
libaudio8_b200.so (include/audio8_b200.h). The directory name is not a Python identifier, so the package is loaded
by path (``__graft_entry__.load_package()``) under the module name ``audio8_b200``.
"""
from . import _lib  # noqa: F401
from ._lib import A8Error, device_error, load  # noqa: F401


def __getattr__(name):
    if name in ("FastEngine", "PackedStack", "Scratch", "permute_qk", "rope_tables", "interleave_w13"):
        from . import engine
        return getattr(engine, name)
    raise AttributeError(name)
