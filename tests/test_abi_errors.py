"""The C ABI's argument checks on the CPU (no device work is reached): null pointers, out-of-range sizes and
inconsistent descriptors return A8_ERR_ARG; a zero-row resampler step is a no-op; the attention workspace query
(host arithmetic only) sizes the split scratch by the split rule -- enough (row, head, part) blocks to fill 2 x 148
SMs, parts of at least 64 keys, at most 16."""
import ctypes as C

import pytest

ARG, OK = 1, 0


@pytest.fixture(scope="module")
def lib(a8):
    return a8._lib.load()


def test_null_pointers_rejected(lib):
    N = None
    assert lib.a8_gemm(N, 896, N, 896, 896, 4, N, 896, N, 0, N) == ARG
    assert lib.a8_attention(N, 896, N, N, 1, 1, 14, 2, 64, 64, 0, N, N, 1, 64, 0.0, N, 896, N, 0, N, 0, N) == ARG
    assert lib.a8_prefill_attention(N, 896, N, N, 1, 1, 14, 2, 64, 64, 0, N, 1, 1, 0.0, N, 896, N) == ARG
    assert lib.a8_rmsnorm(N, 896, N, 0, N, N, 896, 4, 896, 1e-6, N) == ARG
    assert lib.a8_embed_frame(N, N, 10, 4096, N, N, N, 896, 4, 896, 151680, N) == ARG
    assert lib.a8_gather_rows(N, 896, N, N, 896, 4, 896, N) == ARG
    assert lib.a8_sample(N, 4097, 4097, 4, 1, 50, 0.95, 0.8, 1, 16, N, N, N) == ARG
    assert lib.a8_conv(N, N) == ARG
    assert lib.a8_ctx_shift(N, 1, 1, N) == ARG
    assert lib.a8_conv_input(N, 1, 0, 4, 1024, N, 6, N, N, 1, N) == ARG
    assert lib.a8_ups_dwln(N, 2, 1024, N, 0, 7, N, N, N, N, 1e-6, N, 1, N) == ARG
    assert lib.a8_codec_embed(N, 10, N, 4096, N, 1024, 1024, N, N, N, N, 8192, 128, 1, N) == ARG
    assert lib.a8_voc_step(N, N, 1, N) == ARG
    assert lib.a8_voc_decode(N, N, 1, N) == ARG
    assert lib.a8_state_rows(N, 1, N, 1, 0, N, N) == ARG
    assert lib.a8_stack_forward(N, N, N) == ARG
    assert lib.a8_tick(N, 1, N) == ARG
    assert lib.a8_slow_step(N, 1, N) == ARG
    assert lib.a8_prefill_finish(N, N, 1, N, N, N, N) == ARG
    assert lib.a8_resample_reset(N, N, N, 1, 1, N) == ARG
    assert lib.a8_resample_step(N, N, 2048, N, 0, 1, N, N, 832, N, N) == ARG


def test_sizes_and_descriptors_rejected(a8, lib):
    L = a8._lib
    e = L.A8Engine()
    e.B = 4
    assert lib.a8_tick(C.byref(e), 5, None) == ARG                 # more rows than slots
    assert lib.a8_tick(C.byref(e), 0, None) == ARG
    assert lib.a8_slow_step(C.byref(e), 5, None) == ARG
    assert lib.a8_rmsnorm(C.c_void_p(16), 896, None, 0, C.c_void_p(16), C.c_void_p(16), 896, 4, 1030, 1e-6,
                          None) == ARG                             # N over 1024
    seg = (L.A8StateSeg * 1)()
    assert lib.a8_state_rows(seg, 1, C.c_void_p(16), 1, 3, None, None) == ARG      # no such op
    assert lib.a8_state_rows(seg, 1, C.c_void_p(16), 1, L.STATE_LOAD, None, None) == ARG   # a load needs a blob


def test_resampler_descriptor_checks(a8, lib):
    import importlib
    RS = importlib.import_module(a8.__name__ + ".resample")
    L = a8._lib
    r = RS.Resampler(2, 44100, 16000, 2048, "cpu")
    p = C.c_void_p(16)
    ok = dict(audio=p, ld=2048, tok=p, b=2, pcm=p, ld_out=r.out_max, counts=p)

    def step(desc, **kw):
        a = dict(ok, **kw)
        return lib.a8_resample_step(C.byref(desc), a["audio"], a["ld"], a["tok"], 0, a["b"], a["pcm"], None,
                                    a["ld_out"], a["counts"], None)
    assert step(r.desc, b=0) == OK                                 # nothing to do, nothing launched
    assert step(r.desc, b=3, ld=2048) == ARG                       # more rows than slots
    assert step(r.desc, ld=2047) == ARG                            # a frame row shorter than a frame
    assert step(r.desc, ld_out=r.out_max - 1) == ARG               # output rows too short
    for field, bad in (("period", r.period + 1), ("taps", r.taps - 1), ("hist_len", r.taps - 1), ("zpad", 0),
                       ("period", 2048)):
        d = L.A8Resample.from_buffer_copy(r.desc)
        setattr(d, field, bad)
        assert step(d, b=0) == ARG, field                          # checked before anything else
    assert lib.a8_resample_reset(C.byref(r.desc), p, p, 0, 1, None) == OK


def _splits(rows, nkv, max_len):
    want = -(-296 // (rows * nkv))
    return max(1, min(want, -(-max_len // 64), 16))


@pytest.mark.parametrize("rows,nkv,hd,max_len", [(192, 2, 64, 2048), (64, 2, 64, 1500), (8, 8, 128, 128),
                                                 (1, 2, 64, 40)])
def test_attention_workspace_query(lib, rows, nkv, hd, max_len):
    n, t = C.c_longlong(), C.c_int()
    assert lib.a8_attention_workspace(rows, nkv, hd, max_len, C.byref(n), C.byref(t)) == OK
    split = [(r, _splits(r, nkv, max_len)) for r in range(1, rows + 1)]
    need = max((r * nkv * s * (16 * hd + 32) for r, s in split if s > 1), default=0)
    tickets = max((r * nkv for r, s in split if s > 1), default=0)
    assert (n.value, t.value) == (need, tickets)
    assert lib.a8_attention_workspace(0, nkv, hd, max_len, C.byref(n), C.byref(t)) == ARG
    assert lib.a8_attention_workspace(rows, nkv, 96, max_len, C.byref(n), C.byref(t)) == ARG


NOALLOC_FLOATS = 5 << 18          # A8_ATTENTION_NOALLOC_FLOATS (include/audio8_b200.h)


def test_noalloc_array_holds_every_valid_call(lib):
    """The allocation-free attention's fixed array covers the split workspace + tickets of every call the split rule
    allows (host arithmetic only: any rows x kv heads, hd 64 and 128, long rows)."""
    worst = 0
    for hd in (64, 128):
        for x in range(1, 400):                      # x = rows * nkv
            s = _splits(x, 1, 1 << 16)
            if s > 1:
                worst = max(worst, x * s * (16 * hd + 32) + x)
    assert worst == 1227495 and worst <= NOALLOC_FLOATS
    for rows, nkv in ((36, 8), (147, 2), (295, 1)):
        n, t = C.c_longlong(), C.c_int()
        assert lib.a8_attention_workspace(rows, nkv, 128, 2048, C.byref(n), C.byref(t)) == OK
        assert n.value + t.value <= NOALLOC_FLOATS


def test_noalloc_rejects_before_touching_its_array(lib):
    """Bad arguments come back as A8_ERR_ARG from the checks that run before the shared array is used (no device
    work: every pointer here is null or the shape is unsupported)."""
    N = None
    assert lib.a8_attention_noalloc(N, 896, N, N, 1, 1, 14, 2, 64, 64, 0, N, N, 1, 64, 0.0, N, 896, N) == ARG
    p = C.c_void_p(256)
    assert lib.a8_attention_noalloc(p, 896, p, p, 1, 1, 14, 2, 96, 64, 0, p, N, 1, 64, 0.0, p, 896, N) == ARG  # hd
    assert lib.a8_attention_noalloc(p, 896, p, p, 1, 1, 14, 2, 64, 64, 1, p, N, 1, 64, 0.0, p, 896, N) == ARG  # layer
    assert lib.a8_attention_noalloc(p, 896, p, p, 1, 1, 14, 2, 64, 64, 0, p, N, 1, 65, 0.0, p, 896, N) == ARG  # len


def test_prefill_attention_shape_checks(lib):
    """The tensor-core prefill attention takes hd 64 and groups of at most 8 query heads; rows need 16-byte alignment
    (they are TMA tiles); all checked before any device work."""
    p, N = C.c_void_p(256), None
    assert lib.a8_prefill_attention(p, 1024, p, p, 1, 1, 8, 8, 128, 64, 0, p, 1, 1, 0.0, p, 1024, N) == ARG   # hd
    assert lib.a8_prefill_attention(p, 896, p, p, 1, 1, 14, 1, 64, 64, 0, p, 1, 1, 0.0, p, 896, N) == ARG   # group 14
    assert lib.a8_prefill_attention(p, 896, p, p, 1, 1, 14, 2, 64, 64, 0, p, 0, 1, 0.0, p, 896, N) == ARG   # no blocks
    assert lib.a8_prefill_attention(p, 900, p, p, 1, 1, 14, 2, 64, 64, 0, p, 1, 1, 0.0, p, 896, N) == 3     # stride
    assert lib.a8_prefill_attention(C.c_void_p(258), 896, p, p, 1, 1, 14, 2, 64, 64, 0, p, 1, 1, 0.0, p, 896,
                                    N) == 3                                                                 # q align
