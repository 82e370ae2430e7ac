"""The C ABI library loads and exports every function include/audio8_b200.h declares (no compute calls: CPU only)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "audio8_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|long long)\s+(a8_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for must in ("a8_gemm", "a8_attention", "a8_rmsnorm", "a8_sample", "a8_stack_forward", "a8_tick",
                 "a8_prefill_finish", "a8_get_error"):
        assert must in names


def test_library_exports_every_declared_symbol(a8):
    lib = ctypes.CDLL(a8._lib.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_signatures_cover_header(a8):
    assert set(declared()) <= set(a8._lib.SIGNATURES), set(declared()) - set(a8._lib.SIGNATURES)


def test_struct_layouts_match_header(a8):
    """ctypes structs mirror the C structs: field order as declared in the header."""
    L = a8._lib
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for cname, cls in (("A8Epilogue", L.A8Epilogue), ("A8Scratch", L.A8Scratch), ("A8StackDesc", L.A8StackDesc),
                       ("A8StackRun", L.A8StackRun), ("A8Engine", L.A8Engine), ("A8ConvOp", L.A8ConvOp),
                       ("A8Upsample", L.A8Upsample), ("A8Vocoder", L.A8Vocoder), ("A8StateSeg", L.A8StateSeg),
                       ("A8ConvRun", L.A8ConvRun), ("A8CtxShift", L.A8CtxShift), ("A8Resample", L.A8Resample)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), src, flags=re.S).group(1)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            decl = re.sub(r"\[[^\]]*\]", "", decl)                      # arrays: the field name only
            decl = re.sub(r"^(const\s+)?[\w\s]+?[\s\*]+(?=\w+(\s*,|$))", "", decl, count=1)
            fields += [f.strip().lstrip("*") for f in decl.split(",") if f.strip()]
        # a C field named like a Python keyword is bound with a trailing underscore ("in" -> "in_")
        assert fields == [f[0].rstrip("_") for f in cls._fields_], (cname, fields)


def test_no_cpu_fallback_without_gpu(a8):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(a8.A8Error):
        a8.FastEngine(None, None, {})


def test_struct_sizes_match_c_compiler(a8, tmp_path):
    """sizeof and the offset of every field of each struct, from the C compiler, equal the ctypes layout."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    L = a8._lib
    structs = {"A8Epilogue": L.A8Epilogue, "A8Scratch": L.A8Scratch, "A8StackDesc": L.A8StackDesc,
               "A8StackRun": L.A8StackRun, "A8Engine": L.A8Engine, "A8ConvOp": L.A8ConvOp,
               "A8Upsample": L.A8Upsample, "A8Vocoder": L.A8Vocoder, "A8StateSeg": L.A8StateSeg,
               "A8ConvRun": L.A8ConvRun, "A8CtxShift": L.A8CtxShift, "A8Resample": L.A8Resample}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "audio8_b200.h"', 'int main(void) {']
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for f in cls._fields_:
            cf = f[0].rstrip("_")
            lines.append(f'printf("{cname} {f[0]} %zu\\n", offsetof({cname}, {cf}));')
    lines.append("return 0; }")
    src = tmp_path / "abi.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for f in cls._fields_:
            assert got[(cname, f[0])] == getattr(cls, f[0]).offset, (cname, f[0])
